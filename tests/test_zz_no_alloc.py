"""The allocation-free scan entry point, for callers that cannot allocate
device memory (a host framework that gives the library only its input and
output buffers, or a latency-critical path that must not pay cudaMalloc's
implicit synchronisation).

hs_scan_forward_noalloc keeps its look-back scratch in a fixed device array
inside the library.  Called twice in a row through the C ABI (different
inputs, so the second call must not see the first call's leftovers), it must
agree with hs_scan_forward, which runs the same kernel on a caller-owned
workspace.  Kept in its own file, collected last, so a failure here leaves
every other test already run.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

# Same bound as the parity tests' float32 scan checks (normwise).
TOL = 1e-6


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max()).item()


def _call_pair(L, dev, T, B, H, seed):
    P = L.ptr
    g = torch.Generator(device=dev).manual_seed(seed)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    c0 = torch.rand(B, H, device=dev, generator=g)
    outs = {}
    for kind in ("workspace", "noalloc"):
        out = torch.empty(T, B, H, device=dev)
        c = torch.empty(T, B, H, device=dev)
        h_n = torch.empty(B, H, device=dev)
        c_n = torch.empty(B, H, device=dev)
        st = L.stream_ptr(dev)
        if kind == "workspace":
            lib = L.load()
            ws = L.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
            L.call("hs_scan_forward", P(z), P(c0), P(out), P(c), P(h_n), P(c_n), T, B, H, 1e-6,
                   P(ws), ws.numel(), P(L.status_word(dev)), st)
        else:
            L.call("hs_scan_forward_noalloc", P(z), P(c0), P(out), P(c), P(h_n), P(c_n), T, B, H,
                   1e-6, None, st)
        torch.cuda.synchronize(dev)
        outs[kind] = (out, c, h_n, c_n)
    return outs


@pytest.mark.parametrize("T,B,H", [(128, 32, 256), (1000, 3, 24)])
def test_noalloc_matches_workspace_entry_point_twice(T, B, H):
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for seed in (1, 2):  # two calls in a row on the shared scratch array
        outs = _call_pair(L, dev, T, B, H, seed)
        for a, b in zip(outs["noalloc"], outs["workspace"]):
            assert _rel(a, b) <= TOL
    L.check_device_status(dev)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from prlstm_b200 import _lib as L

    lib = L.load()
    P = ctypes.c_void_p
    # 16384 x 32 x 1024 needs 512 MiB of look-back scratch: rejected on the host
    rc = lib.hs_scan_forward_noalloc(P(256), None, P(256), P(256), None, None, 16384, 32, 1024,
                                     1e-6, None, None)
    assert rc == 3
    assert b"fixed" in lib.hs_last_error_message()
