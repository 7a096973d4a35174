"""Batch data parallelism for HeadStartLSTM: one process per GPU.

Sequences of a batch are independent in both modes (the recurrence and the
scan run along time, separately per sequence), so the batch is split into
contiguous shards, each rank runs the unchanged forward/backward on its
shard, and the only exchange is one all-reduce of the parameter gradients.
The reduction is a SUM, not a mean: the reference's training objective is a
sum over sequences (``tests/test_parallel.py:92-95`` differentiates
``out.sum()``), so the summed shard gradients equal the
gradients of the full batch in one process.

The reference itself has no multi-process code; this module is the plumbing
the batch-sharded benchmark and multi-GPU users need.  It is backend
agnostic: NCCL on GPUs, gloo for the CPU tests.
"""

from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Tuple

import torch

__all__ = ["shard_range", "shard_batch", "GradAllReducer", "allreduce_grads"]


def shard_range(batch: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of ``rank``'s sequences when ``batch`` sequences are split
    over ``world`` ranks: contiguous, sizes differing by at most one (the
    first ``batch % world`` ranks take one extra).  A rank may get an empty
    shard when ``batch < world``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if batch < 0:
        raise ValueError(f"batch must be >= 0, got {batch}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(x: torch.Tensor, rank: int, world: int, batch_first: bool = False) -> torch.Tensor:
    """This rank's slice of ``x`` along the batch dimension (dim 1 for the
    module's default ``[T, B, ...]`` layout, dim 0 with ``batch_first``); a
    view, no copy."""
    dim = 0 if batch_first else 1
    s, e = shard_range(x.shape[dim], rank, world)
    return x.narrow(dim, s, e - s)


class GradAllReducer:
    """Sums gradients over the process group with one collective per dtype.

    The gradients are packed into a persistent flat buffer (allocated on the
    first call, reused afterwards), reduced in place with ``all_reduce(SUM)``
    and unpacked, so a step costs one NCCL launch instead of one per tensor
    (five tensors in recurrent mode, two in parallel mode).  Tensors that are
    ``None`` are skipped; every rank must pass the same sequence of shapes,
    since the collectives pair up by position.
    """

    def __init__(self, group=None):
        self.group = group
        self._flat = {}

    def __call__(self, tensors: Sequence[Optional[torch.Tensor]]) -> None:
        import torch.distributed as dist

        live = [t for t in tensors if t is not None]
        if not live or not dist.is_available() or not dist.is_initialized():
            return
        if dist.get_world_size(self.group) == 1:
            return
        by_dtype: dict = {}
        for t in live:
            by_dtype.setdefault((t.dtype, t.device), []).append(t)
        for key in sorted(by_dtype, key=str):
            ts = by_dtype[key]
            n = sum(t.numel() for t in ts)
            flat = self._flat.get(key)
            if flat is None or flat.numel() < n:
                flat = torch.empty(n, dtype=key[0], device=key[1])
                self._flat[key] = flat
            buf = flat[:n]
            off = 0
            for t in ts:
                buf[off:off + t.numel()].copy_(t.reshape(-1))
                off += t.numel()
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
            off = 0
            for t in ts:
                t.copy_(buf[off:off + t.numel()].view_as(t))
                off += t.numel()


def allreduce_grads(params: Iterable[torch.nn.Parameter], group=None,
                    reducer: Optional[GradAllReducer] = None) -> None:
    """Sum ``p.grad`` over the group for every parameter that has one (in
    parallel mode W_hh, b_hh and a have no gradient and are skipped on every
    rank alike)."""
    r = reducer if reducer is not None else GradAllReducer(group)
    grads: List[Optional[torch.Tensor]] = [p.grad for p in params]
    r(grads)
