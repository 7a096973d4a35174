"""The three linear-layer GEMMs through the C ABI against a float64 product.

Shapes are chosen so the tensor-core path takes them: aligned and ragged
extents, bias, beta (accumulate), split-K with and without scratch.  By
default that path is the fp16 split (three fp16 tcgen05 products of
power-of-two-scaled hi/lo parts, the pair kernel on SM pairs); without
scratch for the split, the 3xTF32 kernels run.  Bound: normwise 2e-6 (the
fp16 split with promoted accumulation measures 2e-7 to 1.4e-6; a single
16-bit product would be ~1e-3, so the bound also proves the lo-part
products run)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-6


def _rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    e = ((a - b).abs().max() / b.abs().max()).item()
    print(f"GEMMERR {e:.3e}")
    return e


def _lib():
    from prlstm_b200 import _lib as L

    return L


def _ws(L, M, N, K, dev, use=True):
    if not use:
        return None, 0
    n = L.load().hs_linear_workspace_bytes(M, N, K)
    t = L.workspace(n, dev)
    return t, t.numel()


@pytest.mark.parametrize("M,N,K,bias", [(4096, 1024, 256, True), (1000, 520, 132, True),
                                        (8192, 2048, 100, False), (2048, 8192, 1024, True)])
def test_linear_forward(M, N, K, bias):
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    x = torch.randn(M, K, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g) / K ** 0.5
    b = torch.randn(N, device=dev, generator=g) if bias else None
    y = torch.empty(M, N, device=dev)
    ws, n = _ws(L, M, N, K, dev)
    P = L.ptr
    L.call("hs_linear_forward", P(x), P(w), P(b), P(y), M, N, K, P(ws), n, P(L.status_word(dev)),
           L.stream_ptr(dev))
    ref = x.double().cpu() @ w.double().cpu().t()
    if bias:
        ref += b.double().cpu()
    assert _rel(y, ref) < TOL
    L.check_device_status(dev)


@pytest.mark.parametrize("M,N,K", [(4096, 1024, 256), (8192, 2048, 512), (999, 96, 40)])
def test_linear_dgrad(M, N, K):
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7 + M)
    dy = torch.randn(M, N, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g) / N ** 0.5
    dx = torch.empty(M, K, device=dev)
    ws, n = _ws(L, M, N, K, dev)
    P = L.ptr
    L.call("hs_linear_dgrad", P(dy), P(w), P(dx), M, N, K, P(ws), n, P(L.status_word(dev)),
           L.stream_ptr(dev))
    assert _rel(dx, dy.double().cpu() @ w.double().cpu()) < TOL
    L.check_device_status(dev)


@pytest.mark.parametrize("M,N,K,beta,use_ws", [(8192, 2048, 512, 0, True), (8192, 2048, 512, 1, True),
                                               (8192, 2048, 512, 1, False), (65536, 4096, 512, 0, True),
                                               (2000, 1024, 256, 0, True), (2000, 1000, 260, 1, True)])
def test_linear_wgrad(M, N, K, beta, use_ws):
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11 + M + beta)
    dy = torch.randn(M, N, device=dev, generator=g) * 0.1
    x = torch.randn(M, K, device=dev, generator=g)
    dw = torch.randn(N, K, device=dev, generator=g) if beta else torch.empty(N, K, device=dev)
    ref = dy.double().cpu().t() @ x.double().cpu()
    if beta:
        ref += dw.double().cpu()
    ws, n = _ws(L, M, N, K, dev, use_ws)
    P = L.ptr
    L.call("hs_linear_wgrad", P(dy), P(x), P(dw), M, N, K, beta, P(ws), n, P(L.status_word(dev)),
           L.stream_ptr(dev))
    assert _rel(dw, ref) < TOL
    L.check_device_status(dev)


def test_colsum_matches():
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    dy = torch.randn(5000, 1000, device=dev, generator=g)
    db = torch.empty(1000, device=dev)
    P = L.ptr
    L.call("hs_colsum", P(dy), P(db), 5000, 1000, 0, L.stream_ptr(dev))
    assert _rel(db, dy.double().cpu().sum(0)) < 1e-6


def test_both_tensor_core_kernels_agree():
    """K-major-A products run on the TMEM-A kernel by default; HS_TC_TMEM_A=0
    selects the shared-memory-A kernel.  Run the forward and the input
    gradient once each way (the switch is read once per process, so the
    second run is a child process) and compare both with float64."""
    import os
    import subprocess
    import sys

    code = r'''
import sys, torch
sys.path.insert(0, ".")
from prlstm_b200 import _lib as L
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev).manual_seed(7)
M, N, K = 4096, 1024, 512
x = torch.randn(M, K, device=dev, generator=g)
w = torch.randn(N, K, device=dev, generator=g) / K ** 0.5
b = torch.randn(N, device=dev, generator=g)
dy = torch.randn(M, N, device=dev, generator=g)
y = torch.empty(M, N, device=dev)
dx = torch.empty(M, K, device=dev)
lib = L.load()
ws = L.workspace(lib.hs_linear_workspace_bytes(M, N, K), dev)
P = L.ptr
st = L.stream_ptr(dev)
L.call("hs_linear_forward", P(x), P(w), P(b), P(y), M, N, K, P(ws), ws.numel(), P(L.status_word(dev)), st)
L.call("hs_linear_dgrad", P(dy), P(w), P(dx), M, N, K, P(ws), ws.numel(), P(L.status_word(dev)), st)
torch.cuda.synchronize()
L.check_device_status(dev)
ry = x.double().cpu() @ w.double().cpu().t() + b.double().cpu()
rx = dy.double().cpu() @ w.double().cpu()
ey = ((y.double().cpu() - ry).abs().max() / ry.abs().max()).item()
ex = ((dx.double().cpu() - rx).abs().max() / rx.abs().max()).item()
print(f"{ey:.3e} {ex:.3e}")
'''
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    errs = {}
    for v in ("1", "0"):
        env = dict(os.environ, HS_TC_TMEM_A=v)
        out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True,
                             text=True, timeout=300)
        assert out.returncode == 0, out.stderr[-2000:]
        errs[v] = [float(t) for t in out.stdout.split()[-2:]]
        print(f"GEMMERR HS_TC_TMEM_A={v}: forward {errs[v][0]:.3e} dgrad {errs[v][1]:.3e}")
    for v, (ey, ex) in errs.items():
        assert ey < TOL and ex < TOL, (v, ey, ex)


@pytest.mark.parametrize("M,N,K,beta,with_dx", [(8192, 1024, 256, 0, True), (4096, 2048, 512, 1, True),
                                               (3000, 520, 132, 0, False), (5000, 520, 40, 1, True)])
def test_linear_backward(M, N, K, beta, with_dx):
    """dx = dy.w and dw = beta*dw + dy^T.x in one call (the fp16-split path
    shares one conversion of dy between the two products)."""
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + K + beta)
    dy = torch.randn(M, N, device=dev, generator=g)
    x = torch.randn(M, K, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g) / K ** 0.5
    dx = torch.empty(M, K, device=dev) if with_dx else None
    dw0 = torch.randn(N, K, device=dev, generator=g)
    dw = dw0.clone()
    ws, n = _ws(L, M, N, K, dev)
    P = L.ptr
    L.call("hs_linear_backward", P(dy), P(x), P(w), P(dx), P(dw), M, N, K, beta, P(ws), n,
           P(L.status_word(dev)), L.stream_ptr(dev))
    dy64, x64, w64 = dy.double().cpu(), x.double().cpu(), w.double().cpu()
    ref_dw = dy64.t() @ x64 + (dw0.double().cpu() if beta else 0)
    assert _rel(dw, ref_dw) < TOL
    if with_dx:
        assert _rel(dx, dy64 @ w64) < TOL
    L.check_device_status(dev)


@pytest.mark.parametrize("M,N,K,beta", [(8192, 1024, 256, 0), (3000, 520, 132, 1)])
def test_linear_backward_with_known_absmax(M, N, K, beta):
    """hs_linear_backward_absmax with the exact max |dy| gives the same bits
    as hs_linear_backward (which measures it itself); a looser upper bound
    (4x) still meets the tolerance."""
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + K)
    dy = torch.randn(M, N, device=dev, generator=g)
    x = torch.randn(M, K, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g) / K ** 0.5
    dw0 = torch.randn(N, K, device=dev, generator=g)
    ws, n = _ws(L, M, N, K, dev)
    P, st, status = L.ptr, L.stream_ptr(dev), L.status_word(dev)
    res = {}
    for name, bound in (("own", None), ("exact", 1.0), ("loose", 4.0)):
        dx = torch.empty(M, K, device=dev)
        dw = dw0.clone()
        if bound is None:
            L.call("hs_linear_backward", P(dy), P(x), P(w), P(dx), P(dw), M, N, K, beta, P(ws), n, P(status), st)
        else:
            am = (dy.abs().max() * bound).reshape(1).view(torch.int32).clone()
            L.call("hs_linear_backward_absmax", P(dy), P(x), P(w), P(dx), P(dw), M, N, K, beta, P(am), P(ws), n,
                   P(status), st)
        res[name] = (dx, dw)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    assert torch.equal(res["own"][0], res["exact"][0]) and torch.equal(res["own"][1], res["exact"][1])
    dy64, x64, w64 = dy.double().cpu(), x.double().cpu(), w.double().cpu()
    ref_dw = dy64.t() @ x64 + (dw0.double().cpu() if beta else 0)
    assert _rel(res["loose"][1], ref_dw) < TOL
    assert _rel(res["loose"][0], dy64 @ w64) < TOL


@pytest.mark.parametrize("scale", [1e-30, 1e30])
def test_linear_backward_extreme_magnitudes(scale):
    """dy of magnitude 1e-30 or 1e30: the operand scales of the fp16 split
    reach 2^114 / 2^-85, so the descale is applied one operand at a time
    (their product would leave float range)."""
    L = _lib()
    dev = torch.device("cuda", 0)
    M, N, K = 4096, 1024, 256
    g = torch.Generator(device=dev).manual_seed(11)
    dy = torch.randn(M, N, device=dev, generator=g) * scale
    x = torch.randn(M, K, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g) / K ** 0.5
    dx = torch.empty(M, K, device=dev)
    dw = torch.empty(N, K, device=dev)
    ws, n = _ws(L, M, N, K, dev)
    P = L.ptr
    L.call("hs_linear_backward", P(dy), P(x), P(w), P(dx), P(dw), M, N, K, 0, P(ws), n, P(L.status_word(dev)),
           L.stream_ptr(dev))
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    dy64, x64, w64 = dy.double().cpu(), x.double().cpu(), w.double().cpu()
    assert _rel(dx, dy64 @ w64) < TOL
    assert _rel(dw, dy64.t() @ x64) < TOL


@pytest.mark.parametrize("M,N,K,beta,use_ws", [(4096, 64, 32, 0, True), (4096, 64, 32, 1, True),
                                               (512, 512, 64, 1, True), (3000, 100, 20, 0, True),
                                               (4096, 64, 32, 1, False)])
def test_small_products_split_k(M, N, K, beta, use_ws):
    """Products below the tensor-core threshold run on the FFMA kernel; with
    few output tiles and a long reduction (the gradient products of a short
    recurrent sequence) it splits the reduction into partial tiles added in a
    fixed order, and runs unsplit without scratch.  wgrad reduces over M,
    dgrad over N, the forward over K (with bias)."""
    L = _lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + K + beta)
    dy = torch.randn(M, N, device=dev, generator=g)
    x = torch.randn(M, K, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g)
    b = torch.randn(N, device=dev, generator=g)
    ws, n = _ws(L, M, N, K, dev, use_ws)
    P, st, sw = L.ptr, L.stream_ptr(dev), L.status_word(dev)
    dw = torch.randn(N, K, device=dev, generator=g) if beta else torch.empty(N, K, device=dev)
    ref_dw = dy.double().t() @ x.double() + (dw.double() if beta else 0)
    L.call("hs_linear_wgrad", P(dy), P(x), P(dw), M, N, K, beta, P(ws), n, P(sw), st)
    dx = torch.empty(M, K, device=dev)
    L.call("hs_linear_dgrad", P(dy), P(w), P(dx), M, N, K, P(ws), n, P(sw), st)
    y = torch.empty(M, N, device=dev)
    L.call("hs_linear_forward", P(x), P(w), P(b), P(y), M, N, K, P(ws), n, P(sw), st)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    assert _rel(dw, ref_dw) < TOL
    assert _rel(dx, dy.double() @ w.double()) < TOL
    assert _rel(y, x.double() @ w.double().t() + b.double()) < TOL
