"""Sequence-sharded parallel mode on the GPU (prlstm_b200.sequence_parallel).

* hs_scan_chunk_maps against the float64 oracle's chunk maps, both
  directions, with the configs[4] forget-gate spread.
* The whole protocol on one GPU: a sequence cut into three chunks, each
  chunk's projection, maps, scan from its composed carry and backward from
  its composed incoming gradient, run in phases in one process, against the
  whole sequence in float64, within the parallel-mode bound of every parity
  test: max(1e-5, 2 x the reference float32 path's own error on the inputs).
* Two GPUs: SeqParallelFn over NCCL, each rank holding half the time steps,
  against one GPU's whole-sequence module (skipped with one GPU).
"""

import os
import socket

import pytest
import torch

from oracle import hs_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).abs().max() / b.abs().max()).item()


def _problem(T, B, D, H, seed, with_c0=True):
    g = torch.Generator().manual_seed(seed)
    W_ih, _, b_ih, _, _ = O.init_params(D, H, a_init=0.0, generator=g)
    b_ih[0:2 * H].uniform_(-8, 8, generator=g)
    x = torch.randn(T, B, D, generator=g)
    G = torch.randn(T, B, H, generator=g)
    c0 = torch.rand(B, H, generator=g) if with_c0 else None
    Gh = torch.randn(B, H, generator=g)
    Gc = torch.randn(B, H, generator=g)
    return W_ih, b_ih, x, G, c0, Gh, Gc


def _truth(W_ih, b_ih, x, G, c0, Gh, Gc):
    B, H = x.shape[1], W_ih.shape[0] // 4
    c0d = c0.double() if c0 is not None else torch.zeros(B, H, dtype=torch.float64)
    out, h_n, c_n, saved = O.par_forward_linear(x.double(), c0d, W_ih.double(), b_ih.double())
    dx, dW, db, dc0, _ = O.par_backward_linear(saved, G.double(), Gh.double(), Gc.double())
    return dict(out=out, h_n=h_n, c_n=c_n, dx=dx, dW=dW, db=db, dc0=dc0)


def _tolerances(W_ih, b_ih, x, G, c0, Gh, Gc, truth):
    """The parallel-mode bound of every parity test: max(1e-5, 2 x the error
    of the reference's float32 log-domain path (_parallel.py:21-74, the
    oracle's par_forward) on the same inputs, against float64)."""
    xg = x.clone().requires_grad_(True)
    Wg = W_ih.clone().requires_grad_(True)
    bg = b_ih.clone().requires_grad_(True)
    cg = c0.clone().requires_grad_(True)
    out, h_n, c_n = O.par_forward(xg, cg, Wg, bg)
    ((out * G).sum() + (h_n * Gh).sum() + (c_n * Gc).sum()).backward()
    ref = dict(out=out.detach(), h_n=h_n.detach(), c_n=c_n.detach(), dx=xg.grad, dW=Wg.grad, db=bg.grad,
               dc0=cg.grad)
    return {k: max(TOL, 2 * _rel(ref[k], truth[k])) for k in truth}


def test_chunk_maps_match_oracle():
    from prlstm_b200 import sequence_parallel as S

    dev = torch.device("cuda", 0)
    T, B, D, H = 300, 4, 32, 96
    W_ih, b_ih, x, G, c0, Gh, Gc = _problem(T, B, D, H, seed=1)
    Z = torch.nn.functional.linear(x.double(), W_ih.double(), b_ih.double())
    A_ref, C_ref = O.par_chunk_maps(Z)
    _, _, _, saved = O.par_forward_linear(x.double(), c0.double(), W_ih.double(), b_ih.double())
    _, D_ref = O.par_chunk_maps(Z, saved["c"], G.double(), Gh.double(), backward=True)
    z = Z.float().to(dev)
    A, C = S.chunk_maps(z)
    A2, Dm = S.chunk_maps(z, saved["c"].float().to(dev), G.to(dev), Gh.to(dev), backward=True)
    torch.cuda.synchronize()
    assert _rel(A, A_ref) < TOL and _rel(A2, A_ref) < TOL
    assert _rel(C, C_ref) < TOL
    assert _rel(Dm, D_ref) < TOL


@pytest.mark.parametrize("T,B,D,H,R", [(600, 4, 64, 128, 3), (2048, 8, 64, 256, 2)])
def test_three_chunks_on_one_gpu_match_whole_sequence(T, B, D, H, R):
    from prlstm_b200 import sequence_parallel as S

    dev = torch.device("cuda", 0)
    W_ih, b_ih, x, G, c0, Gh, Gc = _problem(T, B, D, H, seed=T + R)
    truth = _truth(W_ih, b_ih, x, G, c0, Gh, Gc)
    Wd, bd = W_ih.to(dev), b_ih.to(dev)
    bnd = [T * r // R for r in range(R + 1)]
    xs = [x[bnd[r]:bnd[r + 1]].to(dev).contiguous() for r in range(R)]
    Gs = [G[bnd[r]:bnd[r + 1]].to(dev).contiguous() for r in range(R)]
    c0d = c0.to(dev)
    # forward: every chunk's maps (rank 0 folds c0 in), composed carries, scans
    Z, A_own, A_pub, C_pub = [], [], [], []
    for r in range(R):
        z = S.chunk_project(xs[r], Wd, bd)
        a, cc = S.chunk_maps(z)
        Z.append(z)
        A_own.append(a)
        if r == 0:
            a, cc = S.fold_initial(a, cc, c0d)
        A_pub.append(a)
        C_pub.append(cc)
    fw = []
    for r in range(R):
        c_in = S.compose_forward(A_pub, C_pub, c0d if r == 0 else None)[r]
        fw.append((c_in,) + S.chunk_scan_forward(Z[r], c_in))
    # backward: every chunk's maps, composed incoming gradients, backward
    dh_last = [None] * (R - 1) + [Gh.to(dev)]
    dc_last = [torch.zeros(B, H, device=dev)] * (R - 1) + [Gc.to(dev)]
    Dm = [S.chunk_maps(Z[r], fw[r][2], Gs[r], dh_last[r], backward=True)[1] for r in range(R)]
    e_in = S.compose_backward(A_own, Dm, dc_last)
    outs, dxs, dW, db, dc0 = [], [], 0, 0, None
    for r in range(R):
        c_in, out, c, h_l, c_l, kf = fw[r]
        dx, dw, dbb, d0 = S.chunk_backward(xs[r], Wd, Z[r], c, c_in, Gs[r], dh_last[r], e_in[r], kf,
                                           want_dc0=(r == 0))
        outs.append(out)
        dxs.append(dx)
        dW = dW + dw
        db = db + dbb
        if r == 0:
            dc0 = d0
    torch.cuda.synchronize()
    from prlstm_b200 import _lib

    _lib.check_device_status(dev)
    # fw[r] = (c_in, out, c, h_last, c_last, kf): the last chunk's are the sequence's h_n, c_n
    got = dict(out=torch.cat(outs), h_n=fw[-1][3], c_n=fw[-1][4], dx=torch.cat(dxs), dW=dW, db=db, dc0=dc0)
    tol = _tolerances(W_ih, b_ih, x, G, c0, Gh, Gc, truth)
    for k in truth:
        e = _rel(got[k], truth[k])
        print(f"SEQPAR R={R} {k} {e:.3e} tol {tol[k]:.3e}")
        assert e < tol[k], f"{k}: {e:.3e} > {tol[k]:.3e}"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path):
    import datetime

    import torch.distributed as dist

    from prlstm_b200.sequence_parallel import headstartlstm_parallel_seqsharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        T, B, D, H = 4096, 4, 64, 256
        W_ih, b_ih, x, G, c0, Gh, Gc = _problem(T, B, D, H, seed=11)
        t0, t1 = T * rank // world, T * (rank + 1) // world
        W = W_ih.to(dev).requires_grad_(True)
        b = b_ih.to(dev).requires_grad_(True)
        c0d = c0.to(dev).requires_grad_(True)
        xd = x[t0:t1].to(dev).contiguous().requires_grad_(True)
        out, h_l, c_l = headstartlstm_parallel_seqsharded(xd, c0d, W, b)
        loss = (out * G[t0:t1].to(dev)).sum()
        if rank == world - 1:
            loss = loss + (h_l * Gh.to(dev)).sum() + (c_l * Gc.to(dev)).sum()
        loss.backward()
        dist.all_reduce(W.grad)
        dist.all_reduce(b.grad)
        torch.cuda.synchronize(dev)
        torch.save(dict(out=out.detach().cpu(), dx=xd.grad.cpu(), dW=W.grad.cpu(), db=b.grad.cpu(),
                        dc0=None if c0d.grad is None else c0d.grad.cpu(), h_n=h_l.detach().cpu(),
                        c_n=c_l.detach().cpu()), f"{path}.{rank}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_sequence_sharded_matches_whole_sequence(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    path = str(tmp_path / "seq")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    r0, r1 = torch.load(f"{path}.0"), torch.load(f"{path}.1")
    T, B, D, H = 4096, 4, 64, 256
    prob = _problem(T, B, D, H, seed=11)
    truth = _truth(*prob)
    tol = _tolerances(*prob, truth)
    got = dict(out=torch.cat([r0["out"], r1["out"]]), dx=torch.cat([r0["dx"], r1["dx"]]), dW=r0["dW"], db=r0["db"],
               dc0=r0["dc0"], h_n=r1["h_n"], c_n=r1["c_n"])
    assert r1["dc0"] is None
    for k in truth:
        e = _rel(got[k], truth[k])
        print(f"SEQPAR 2GPU {k} {e:.3e} tol {tol[k]:.3e}")
        assert e < tol[k], f"{k}: {e:.3e} > {tol[k]:.3e}"
