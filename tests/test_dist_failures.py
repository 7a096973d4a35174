"""Failure detection on the collective side, with two gloo ranks on the CPU.

Failures are made on the host only: a rank that raises, a rank that exits
between steps, a rank that never joins.  Each case checks that the surviving
rank ends with a clean error (an exception it can catch) within its
timeout, rather than waiting for good:

  * a rank raises before the gradient all-reduce: the survivor's all-reduce
    fails (the peer's connection closes, or the process group times out);
  * a rank exits between steps: with a PeerMonitor the survivor learns of it
    on the host, as PeerFailure naming the rank, before it launches the next
    collective; without one, the collective itself fails;
  * a rank never joins: init_process_group(timeout=...) expires.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from prlstm_b200.data_parallel import GradAllReducer, PeerFailure, PeerMonitor

PG_TIMEOUT = datetime.timedelta(seconds=5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=PG_TIMEOUT)


def _grads():
    return [torch.ones(64, 8, dtype=torch.float64), torch.ones(64, dtype=torch.float64)]


def _report(q, rank, exc=None, **extra):
    if exc is None:
        q.put((rank, "ok", "", "", extra))
    else:
        q.put((rank, "error", type(exc).__name__, str(exc)[:300], extra))


def _w_raise_before_allreduce(rank, world, port, _port2, q):
    _init(rank, world, port)
    if rank == 1:
        raise RuntimeError("rank 1 fails before its all-reduce (planted)")
    try:
        t0 = time.monotonic()
        GradAllReducer()(_grads())
        _report(q, rank)
    except Exception as e:  # noqa: BLE001 - the survivor's error is the result
        _report(q, rank, e, seconds=time.monotonic() - t0)


def _w_exit_between_steps(rank, world, port, port2, q, use_monitor):
    _init(rank, world, port)
    monitor = None
    if use_monitor:
        store = dist.TCPStore("127.0.0.1", port2, world, is_master=(rank == 0),
                              timeout=datetime.timedelta(seconds=10), wait_for_workers=False)
        monitor = PeerMonitor(store, rank, world, timeout_s=3.0)
    red = GradAllReducer(monitor=monitor)
    g = _grads()
    red(g)  # step 0: both ranks
    ok0 = bool(torch.all(g[0] == 2.0))
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        t0 = time.monotonic()
        red(_grads())  # step 1: the peer is gone
        _report(q, rank, ok0=ok0)
    except PeerFailure as e:
        _report(q, rank, e, ok0=ok0, missing=e.missing, step=e.step, seconds=time.monotonic() - t0)
    except Exception as e:  # noqa: BLE001
        _report(q, rank, e, ok0=ok0, seconds=time.monotonic() - t0)


def _w_never_joined(rank, world, port, _port2, q):
    t0 = time.monotonic()
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=2))
        _report(q, rank)
    except Exception as e:  # noqa: BLE001
        _report(q, rank, e, seconds=time.monotonic() - t0)


def _run(fn, nprocs, world, *extra, limit_s=60):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port, port2 = _free_port(), _free_port()
    pc = mp.start_processes(fn, args=(world, port, port2, q, *extra), nprocs=nprocs, join=False,
                            start_method="spawn")
    deadline = time.monotonic() + limit_s
    for p in pc.processes:
        p.join(max(0.1, deadline - time.monotonic()))
    hung = [p.pid for p in pc.processes if p.is_alive()]
    for p in pc.processes:  # only our own children, by their own handles
        if p.is_alive():
            p.kill()
            p.join(5)
    res = {}
    while not q.empty():
        rank, status, kind, msg, extra_ = q.get()
        res[rank] = dict(status=status, kind=kind, msg=msg, **extra_)
    return res, hung, [p.exitcode for p in pc.processes]


def test_rank_raises_before_allreduce():
    res, hung, codes = _run(_w_raise_before_allreduce, 2, 2)
    assert not hung, "a rank was still waiting at the test's limit"
    assert codes[1] != 0  # the planted exception ended rank 1
    assert res[0]["status"] == "error", res
    assert res[0]["seconds"] < PG_TIMEOUT.total_seconds() + 30


def test_rank_exits_between_steps_peer_monitor():
    res, hung, codes = _run(_w_exit_between_steps, 2, 2, True)
    assert not hung
    r = res[0]
    assert r["ok0"], "step 0 all-reduce must have summed both ranks"
    assert r["status"] == "error" and r["kind"] == "PeerFailure", r
    assert r["missing"] == [1] and r["step"] == 1
    assert r["seconds"] < 10


def test_rank_exits_between_steps_collective_errors():
    res, hung, codes = _run(_w_exit_between_steps, 2, 2, False)
    assert not hung
    r = res[0]
    assert r["ok0"]
    assert r["status"] == "error", r
    assert r["seconds"] < PG_TIMEOUT.total_seconds() + 30


def test_init_timeout_when_a_rank_never_joins():
    # world of two, only rank 0 is started
    res, hung, codes = _run(_w_never_joined, 1, 2)
    assert not hung
    assert res[0]["status"] == "error", res
    assert res[0]["seconds"] < 30


def test_peer_monitor_single_process_store():
    """PeerMonitor on a HashStore: a step every rank reached passes, a step
    one rank never reached raises PeerFailure naming it."""
    store = dist.HashStore()
    a = PeerMonitor(store, 0, 3, timeout_s=0.2)
    b = PeerMonitor(store, 1, 3, timeout_s=0.2)
    c = PeerMonitor(store, 2, 3, timeout_s=0.2)
    for m in (a, b, c):
        m.beat(0)
    a.wait(0)
    a.beat(1)
    b.beat(1)
    with pytest.raises(PeerFailure) as ei:
        a.wait(1)
    assert ei.value.missing == [2] and ei.value.step == 1
