"""The allocation-free scan entry point, for callers that cannot allocate
device memory (a host framework that gives the library only its input and
output buffers, or a latency-critical path that must not pay cudaMalloc's
implicit synchronisation).

hs_scan_forward_noalloc keeps its look-back scratch in a fixed device array
inside the library.  Called twice in a row through the C ABI (different
inputs, so the second call must not see the first call's leftovers), it must
agree with hs_scan_forward, which runs the same kernel on a caller-owned
workspace.  Both scan paths are forced in turn (HS_SCAN_PATH), and both ways
of reporting device-side failures are checked: the caller's status word, and
the library's own word (dev_status NULL) read back with
hs_scan_noalloc_status.  Kept in its own file, collected last, so a failure
here leaves every other test already run.
"""

import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

# Same bound as the parity tests' float32 scan checks (normwise).
TOL = 1e-6


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max()).item()


class _path:
    """Force one scan implementation for the duration of a block."""

    def __init__(self, path):
        self.path = path

    def __enter__(self):
        self.old = os.environ.get("HS_SCAN_PATH")
        if self.path:
            os.environ["HS_SCAN_PATH"] = self.path
        else:
            os.environ.pop("HS_SCAN_PATH", None)

    def __exit__(self, *exc):
        if self.old is None:
            os.environ.pop("HS_SCAN_PATH", None)
        else:
            os.environ["HS_SCAN_PATH"] = self.old


def _library_status(L, dev):
    v = ctypes.c_int(-1)
    L.call("hs_scan_noalloc_status", ctypes.byref(v), L.stream_ptr(dev))
    return v.value


def _call_pair(L, dev, T, B, H, seed, own_status):
    P = L.ptr
    g = torch.Generator(device=dev).manual_seed(seed)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    c0 = torch.rand(B, H, device=dev, generator=g)
    outs = {}
    for kind in ("workspace", "noalloc"):
        out = torch.full((T, B, H), float("nan"), device=dev)
        c = torch.full((T, B, H), float("nan"), device=dev)
        h_n = torch.full((B, H), float("nan"), device=dev)
        c_n = torch.full((B, H), float("nan"), device=dev)
        st = L.stream_ptr(dev)
        if kind == "workspace":
            lib = L.load()
            ws = L.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
            L.call("hs_scan_forward", P(z), P(c0), P(out), P(c), P(h_n), P(c_n), T, B, H, 1e-6,
                   P(ws), ws.numel(), P(L.status_word(dev)), st)
        else:
            status = None if own_status else L.status_word(dev)
            L.call("hs_scan_forward_noalloc", P(z), P(c0), P(out), P(c), P(h_n), P(c_n), T, B, H,
                   1e-6, P(status), st)
        torch.cuda.synchronize(dev)
        outs[kind] = (out, c, h_n, c_n)
    return outs


@pytest.mark.parametrize("own_status", [True, False], ids=["library_status", "caller_status"])
@pytest.mark.parametrize("path", ["chain", "lookback", None])
@pytest.mark.parametrize("T,B,H", [(128, 32, 256), (1000, 3, 24)])
def test_noalloc_matches_workspace_entry_point_twice(T, B, H, path, own_status):
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with _path(path):
        for seed in (1, 2):  # two calls in a row on the shared scratch array
            outs = _call_pair(L, dev, T, B, H, seed, own_status)
            for a, b in zip(outs["noalloc"], outs["workspace"]):
                assert _rel(a, b) <= TOL
            if own_status:
                assert _library_status(L, dev) == L.HS_OK
    L.check_device_status(dev)  # the caller's word (used by both entry points above)


@pytest.mark.parametrize("path", ["chain", "lookback"])
def test_noalloc_library_status_reports_and_does_not_go_stale(path):
    """A timeout planted in the library's own word (the bounded-wait self test
    aimed at it, no device fault) is reported by hs_scan_noalloc_status, and a
    later NULL-status call still runs: it clears the word before its kernels
    read it."""
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    st = L.stream_ptr(dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)  # nothing ever sets it
    _library_status(L, dev)  # start from a clear word
    L.call("hs_selftest_bounded_wait", L.ptr(flag), None, 2_000_000, st)
    assert _library_status(L, dev) == L.HS_ERR_DEVICE_TIMEOUT
    assert _library_status(L, dev) == L.HS_OK  # read-and-clear

    L.call("hs_selftest_bounded_wait", L.ptr(flag), None, 2_000_000, st)  # stale failure
    with _path(path):
        outs = _call_pair(L, dev, 256, 32, 256, 3, own_status=True)
    for a, b in zip(outs["noalloc"], outs["workspace"]):
        assert _rel(a, b) <= TOL
    assert _library_status(L, dev) == L.HS_OK


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from prlstm_b200 import _lib as L

    lib = L.load()
    P = ctypes.c_void_p
    # 16384 x 32 x 1024 on the look-back path needs 512 MiB of scratch:
    # rejected on the host, before any launch
    with _path("lookback"):
        rc = lib.hs_scan_forward_noalloc(P(256), None, P(256), P(256), None, None, 16384, 32, 1024,
                                         1e-6, None, None)
    assert rc == 3
    assert b"fixed" in lib.hs_last_error_message()


def test_noalloc_chain_path_needs_no_scratch():
    """The same shape on the chain kernels (the default for it: 1024 columns)
    uses no scratch and runs, matching the workspace entry point."""
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with _path(None):
        outs = _call_pair(L, dev, 2048, 32, 1024, 4, own_status=True)
    for a, b in zip(outs["noalloc"], outs["workspace"]):
        assert _rel(a, b) <= TOL
    assert _library_status(L, dev) == L.HS_OK
