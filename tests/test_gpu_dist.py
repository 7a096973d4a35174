"""Batch data parallelism on two GPUs over NCCL (skipped with fewer GPUs).

Two ranks each run the module forward/backward on their contiguous shard of
the batch and sum the gradients with prlstm_b200.data_parallel; the result
must equal one full-batch run on a single GPU to float32 rounding: the sum
of per-sequence gradients is the same sum, but the order of its additions
depends on each run's batch extent (the recurrent cluster kernels size their
sequence blocks to the batch group, the FFMA GEMMs split their reduction by
its length), so the bound is the recurrent parity bound, 1e-5 of the
largest gradient entry (measured differences reach 1.3e-6)."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

NAMES = ("weight_ih_l0", "weight_hh_l0", "bias_ih_l0", "bias_hh_l0", "a")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(parallel, T, B, D, H):
    from _cases import make_inputs

    return make_inputs(T, B, D, H, a=0.0 if parallel else 0.2, seed=3 + int(parallel))


def _run(params, x, G, parallel, dev):
    import prlstm_b200

    D, H = params[0].shape[1], params[1].shape[1]
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=parallel).to(dev)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    out, _ = m(x.to(dev))
    (out * G.to(dev)).sum().backward()
    return m


def _worker(rank, world, port, case, path):
    import torch.distributed as dist

    from prlstm_b200.data_parallel import allreduce_grads, shard_batch

    import datetime

    # NVLS off; a short process-group timeout with asynchronous error
    # handling, so that if one rank fails before the all-reduce the other's
    # collective gives up with an error instead of waiting on the GPU
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        parallel, T, B, D, H = case
        params, x, G = _inputs(parallel, T, B, D, H)
        m = _run(params, shard_batch(x, rank, world), shard_batch(G, rank, world), parallel, dev)
        allreduce_grads(m.parameters())
        torch.cuda.synchronize(dev)
        if rank == 0:  # a file, not a queue: the parent reads only after join
            torch.save({n: (None if p.grad is None else p.grad.cpu()) for n, p in m.named_parameters()}, path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(True, 256, 8, 64, 128), (False, 32, 6, 48, 64)])
def test_two_gpu_sharded_gradients_equal_full_batch(case, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    path = str(tmp_path / "grads.pt")
    mp.start_processes(_worker, args=(2, _free_port(), case, path), nprocs=2, join=True,
                       start_method="spawn")
    got = torch.load(path)
    parallel, T, B, D, H = case
    params, x, G = _inputs(parallel, T, B, D, H)
    ref = _run(params, x, G, parallel, torch.device("cuda", 0))
    for n, p in ref.named_parameters():
        if p.grad is None:
            assert got[n] is None, n
            continue
        g = got[n]
        err = ((g - p.grad.cpu()).abs().max() / p.grad.abs().max().cpu()).item()
        assert err < 1e-5, f"{n}: {err:.3e}"
