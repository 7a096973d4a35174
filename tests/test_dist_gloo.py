"""Batch data parallelism on CPU with two gloo ranks.

Each rank runs the float64 oracle on its shard of the batch (the same
arithmetic the GPU path reproduces), the gradients are summed with
prlstm_b200.data_parallel.GradAllReducer, and the result must equal the
single-process full-batch gradients.  Covers both modes, an uneven split and
a non-zero initial state sharded alongside the batch."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import hs_oracle as O
from prlstm_b200.data_parallel import GradAllReducer, shard_batch, shard_range

GRADS = ("dW_ih", "dW_hh", "db_ih", "db_hh", "da")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(parallel, T, B, D, H, with_hx):
    g = torch.Generator().manual_seed(1000 * T + 10 * B + int(parallel))
    params = O.init_params(D, H, a_init=0.3, generator=g, dtype=torch.float64)
    x = torch.randn(T, B, D, generator=g, dtype=torch.float64)
    G = torch.randn(T, B, H, generator=g, dtype=torch.float64)
    hx = None
    if with_hx:
        hx = (torch.randn(B, H, generator=g, dtype=torch.float64),
              torch.rand(B, H, generator=g, dtype=torch.float64))
    return params, x, G, hx


def _worker(rank, world, port, case, errq):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        parallel, T, B, D, H, with_hx = case
        params, x, G, hx = _problem(parallel, T, B, D, H, with_hx)
        xs = shard_batch(x, rank, world)
        Gs = shard_batch(G, rank, world)
        hxs = None
        if hx is not None:
            # the module takes hx as [1, B, H]; the oracle as [B, H]
            hxs = tuple(shard_batch(t.unsqueeze(0), rank, world)[0] for t in hx)
        mine = O.module_forward_backward(params, xs, Gs, parallel, hx=hxs, linear_truth=True)
        grads = [mine[k] for k in GRADS]
        GradAllReducer()(grads)
        full = O.module_forward_backward(params, x, G, parallel, hx=hx, linear_truth=True)
        s, e = shard_range(B, rank, world)
        msgs = []
        for k, got in zip(GRADS, grads):
            want = full[k]
            if want is None:
                if got is not None:
                    msgs.append(f"{k}: expected None")
                continue
            err = ((got - want).abs().max() / want.abs().max().clamp_min(1e-300)).item()
            if err > 1e-12:
                msgs.append(f"{k}: rel err {err:.3e}")
        # the per-sequence outputs of the shard are the full run's rows
        for k in ("out", "dx"):
            err = (mine[k] - full[k][:, s:e]).abs().max().item()
            if err > 1e-12:
                msgs.append(f"{k}: shard rows differ by {err:.3e}")
        if msgs:
            errq.put(f"rank {rank}: " + "; ".join(msgs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [
    (True, 24, 4, 6, 5, False),   # parallel mode, even split
    (True, 17, 5, 3, 4, True),    # parallel mode, 3+2 split, c0 sharded
    (False, 12, 4, 5, 6, False),  # recurrent mode, even split
    (False, 9, 3, 4, 3, True),    # recurrent mode, 2+1 split, h0/c0 sharded
])
def test_sharded_sum_equals_full_batch(case):
    world = 2
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), case, errq), nprocs=world,
                       join=True, start_method="spawn")
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, "\n".join(errs)


def test_shard_range_partitions_the_batch():
    for B in range(0, 11):
        for world in range(1, 5):
            rs = [shard_range(B, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == B
            for (s0, e0), (s1, e1) in zip(rs, rs[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in rs]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_shard_batch_layouts():
    x = torch.arange(2 * 5 * 3).reshape(2, 5, 3)
    assert torch.equal(shard_batch(x, 1, 2), x[:, 3:5])
    assert torch.equal(shard_batch(x.transpose(0, 1), 0, 2, batch_first=True), x.transpose(0, 1)[0:3])
