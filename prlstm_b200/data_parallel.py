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

__all__ = ["shard_range", "shard_batch", "GradAllReducer", "PendingReduction", "allreduce_grads",
           "PeerMonitor", "PeerFailure"]


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


class PeerFailure(RuntimeError):
    """A rank did not reach a step within the heartbeat timeout."""

    def __init__(self, step: int, missing: Sequence[int]):
        self.step = step
        self.missing = list(missing)
        super().__init__(f"ranks {self.missing} did not reach step {step}: presumed failed")


class PeerMonitor:
    """Host-side heartbeat through a ``torch.distributed`` store, checked
    before each step's collective.

    Every rank records the step it has reached (``beat``) and then waits, up
    to ``timeout_s``, for every other rank's record of the same step
    (``wait``).  A rank that raised or exited between steps never writes its
    record, so the others learn of it on the host, with ``PeerFailure``
    naming it, before they launch a collective that could not complete.  A
    rank leaves only between steps, with nothing of its own in flight.
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "hs_hb"):
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = float(timeout_s)
        self.prefix = prefix

    def _key(self, rank: int, step: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank, step), "1")

    def wait(self, step: int) -> None:
        import time

        others = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        pending = list(others)
        while pending:
            pending = [r for r in pending if not self.store.check([self._key(r, step)])]
            if not pending:
                return
            if time.monotonic() > deadline:
                raise PeerFailure(step, pending)
            time.sleep(0.01)

    def step(self, step: int) -> None:
        self.beat(step)
        self.wait(step)


class GradAllReducer:
    """Sums gradients over the process group with one collective per dtype.

    With a ``PeerMonitor`` every call first checks, on the host, that all
    ranks reached the same call (a failed rank raises ``PeerFailure`` on the
    others instead of leaving them in a collective).

    The gradients are packed into a persistent flat buffer (allocated on the
    first call, reused afterwards), reduced in place with ``all_reduce(SUM)``
    and unpacked, so a step costs one NCCL launch instead of one per tensor
    (five tensors in recurrent mode, two in parallel mode).  Tensors that are
    ``None`` are skipped; every rank must pass the same sequence of shapes,
    since the collectives pair up by position.
    """

    def __init__(self, group=None, monitor: Optional[PeerMonitor] = None):
        self.group = group
        self.monitor = monitor
        self.calls = 0
        self._flat = {}

    def __call__(self, tensors: Sequence[Optional[torch.Tensor]]) -> None:
        self.start(tensors).finish()

    def start(self, tensors: Sequence[Optional[torch.Tensor]]) -> "PendingReduction":
        """Pack the gradients and launch the all-reduce without waiting for
        it: with NCCL the collective runs on the process group's own stream,
        so work the caller queues next on its stream (the input-gradient GEMM
        of a backward, say) overlaps with it.  ``finish()`` on the result
        makes the caller's stream wait for the reduction and unpacks it."""
        import torch.distributed as dist

        live = [t for t in tensors if t is not None]
        if not live or not dist.is_available() or not dist.is_initialized():
            return PendingReduction([])
        if dist.get_world_size(self.group) == 1:
            return PendingReduction([])
        if self.monitor is not None:
            # every peer must have reached this reduction before it launches
            self.monitor.step(self.calls)
        self.calls += 1
        by_dtype: dict = {}
        for t in live:
            by_dtype.setdefault((t.dtype, t.device), []).append(t)
        parts = []
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
            work = dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
            parts.append((work, buf, ts))
        return PendingReduction(parts)


class PendingReduction:
    """An all-reduce launched by ``GradAllReducer.start``."""

    def __init__(self, parts):
        self.parts = parts

    def finish(self) -> None:
        for work, buf, ts in self.parts:
            work.wait()
            off = 0
            for t in ts:
                t.copy_(buf[off:off + t.numel()].view_as(t))
                off += t.numel()
        self.parts = []


def allreduce_grads(params: Iterable[torch.nn.Parameter], group=None,
                    reducer: Optional[GradAllReducer] = None) -> None:
    """Sum ``p.grad`` over the group for every parameter that has one (in
    parallel mode W_hh, b_hh and a have no gradient and are skipped on every
    rank alike)."""
    r = reducer if reducer is not None else GradAllReducer(group)
    grads: List[Optional[torch.Tensor]] = [p.grad for p in params]
    r(grads)
