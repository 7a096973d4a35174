"""Sequence-sharded parallel mode on the CPU: the protocol of
prlstm_b200.sequence_parallel (chunk maps, their composition across ranks,
each chunk's scan from its composed carry) checked against the
whole-sequence float64 oracle, in one process over R chunks and with two
gloo ranks exchanging the maps by all_gather.  The chunk maps and the chunk
scans here are the oracle's; the composition is the product's."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import hs_oracle as O
from prlstm_b200.sequence_parallel import compose_backward, compose_forward, fold_initial

EPS = 1e-6


def _problem(T, B, D, H, seed, with_c0):
    g = torch.Generator().manual_seed(seed)
    W_ih, _, b_ih, _, _ = O.init_params(D, H, a_init=0.0, generator=g, dtype=torch.float64)
    b_ih[0:2 * H].uniform_(-4, 4, generator=g)
    x = torch.randn(T, B, D, generator=g, dtype=torch.float64)
    G = torch.randn(T, B, H, generator=g, dtype=torch.float64)
    c0 = torch.rand(B, H, generator=g, dtype=torch.float64) if with_c0 else None
    if c0 is not None:
        c0[:, :2] = 0.0
    Gh = torch.randn(B, H, generator=g, dtype=torch.float64)
    Gc = torch.randn(B, H, generator=g, dtype=torch.float64)
    return W_ih, b_ih, x, G, c0, Gh, Gc


def _full(W_ih, b_ih, x, G, c0, Gh, Gc):
    B, H = x.shape[1], W_ih.shape[0] // 4
    c0z = c0 if c0 is not None else torch.zeros(B, H, dtype=torch.float64)
    out, h_n, c_n, saved = O.par_forward_linear(x, c0z, W_ih, b_ih)
    dx, dW, db, dc0, _ = O.par_backward_linear(saved, G, Gh, Gc)
    return out, dx, dW, db, dc0


def _bounds(T, R):
    b = [T * r // R for r in range(R + 1)]
    return [(b[r], b[r + 1]) for r in range(R)]


def _chunk_forward_maps(W_ih, b_ih, xr):
    Z = torch.nn.functional.linear(xr, W_ih, b_ih)
    return Z, O.par_chunk_maps(Z)


def _chunk_run(W_ih, b_ih, xr, Gr, c_in, dh_last, e_in, B, H):
    cz = c_in if c_in is not None else torch.zeros(B, H, dtype=torch.float64)
    out, h_l, c_l, saved = O.par_forward_linear(xr, cz, W_ih, b_ih)
    dx, dW, db, dc0, _ = O.par_backward_linear(saved, Gr, dh_last, e_in)
    return out, dx, dW, db, dc0, saved


@pytest.mark.parametrize("R,with_c0", [(2, False), (3, True), (5, True)])
def test_sequence_sharded_protocol_matches_whole_sequence(R, with_c0):
    T, B, D, H = 37, 3, 5, 6
    W_ih, b_ih, x, G, c0, Gh, Gc = _problem(T, B, D, H, seed=R, with_c0=with_c0)
    ref_out, ref_dx, ref_dW, ref_db, ref_dc0 = _full(W_ih, b_ih, x, G, c0, Gh, Gc)
    bnd = _bounds(T, R)
    A, C, Z = [], [], []
    for t0, t1 in bnd:
        z, (a, cc) = _chunk_forward_maps(W_ih, b_ih, x[t0:t1])
        Z.append(z); A.append(a); C.append(cc)
    c_in = compose_forward(A, C, c0, EPS)
    # forward per chunk, then backward maps from each chunk's states
    fw = []
    for r, (t0, t1) in enumerate(bnd):
        cz = c_in[r] if c_in[r] is not None else torch.zeros(B, H, dtype=torch.float64)
        out, h_l, c_l, saved = O.par_forward_linear(x[t0:t1], cz, W_ih, b_ih)
        fw.append((out, saved))
    dh_last = [None] * (R - 1) + [Gh]
    dc_last = [None] * (R - 1) + [Gc]
    D = []
    for r, (t0, t1) in enumerate(bnd):
        _, d = O.par_chunk_maps(Z[r], fw[r][1]["c"], G[t0:t1], dh_last[r], backward=True)
        D.append(d)
    e_in = compose_backward(A, D, dc_last)
    outs, dxs, dW, db = [], [], 0, 0
    for r, (t0, t1) in enumerate(bnd):
        dx, dw, dbb, dc0, _ = O.par_backward_linear(fw[r][1], G[t0:t1], dh_last[r], e_in[r])
        outs.append(fw[r][0]); dxs.append(dx); dW = dW + dw; db = db + dbb
        if r == 0:
            got_dc0 = dc0
    rel = lambda a, b: ((a - b).abs().max() / b.abs().max()).item()
    assert rel(torch.cat(outs), ref_out) < 1e-12
    assert rel(torch.cat(dxs), ref_dx) < 1e-12
    assert rel(dW, ref_dW) < 1e-12 and rel(db, ref_db) < 1e-12
    if with_c0:
        assert rel(got_dc0, ref_dc0) < 1e-12


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, B, D, H = 29, 2, 4, 5
        W_ih, b_ih, x, G, c0, Gh, Gc = _problem(T, B, D, H, seed=7, with_c0=True)
        ref_out, ref_dx, ref_dW, ref_db, _ = _full(W_ih, b_ih, x, G, c0, Gh, Gc)
        t0, t1 = _bounds(T, world)[rank]
        z, (a, cc) = _chunk_forward_maps(W_ih, b_ih, x[t0:t1])
        a_own = a
        if rank == 0:  # only rank 0 holds c0: it publishes its map with c0 folded in
            a, cc = fold_initial(a, cc, c0, EPS)
        A = [torch.empty_like(a) for _ in range(world)]
        C = [torch.empty_like(cc) for _ in range(world)]
        dist.all_gather(A, a)
        dist.all_gather(C, cc)
        c_in = compose_forward(A, C, c0 if rank == 0 else None, EPS)[rank]
        A[rank] = a_own  # the backward composes the chunks' own maps
        cz = c_in if c_in is not None else torch.zeros(B, H, dtype=torch.float64)
        out, _, _, saved = O.par_forward_linear(x[t0:t1], cz, W_ih, b_ih)
        last = rank == world - 1
        dh_l = Gh if last else None
        dc_l = Gc if last else torch.zeros(B, H, dtype=torch.float64)
        _, d = O.par_chunk_maps(z, saved["c"], G[t0:t1], dh_l, backward=True)
        Dl = [torch.empty_like(d) for _ in range(world)]
        Ll = [torch.empty_like(dc_l) for _ in range(world)]
        dist.all_gather(Dl, d)
        dist.all_gather(Ll, dc_l)
        e_in = compose_backward(A, Dl, Ll)[rank]
        dx, dW, db, _, _ = O.par_backward_linear(saved, G[t0:t1], dh_l, e_in)
        dist.all_reduce(dW)
        dist.all_reduce(db)
        rel = lambda u, v: ((u - v).abs().max() / v.abs().max()).item()
        errs = [rel(out, ref_out[t0:t1]), rel(dx, ref_dx[t0:t1]), rel(dW, ref_dW), rel(db, ref_db)]
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(2, _free_port(), q), nprocs=2, join=True, start_method="spawn")
    res = {}
    while not q.empty():
        r, e = q.get()
        res[r] = e
    assert set(res) == {0, 1}
    assert max(res.values()) < 1e-12, res
