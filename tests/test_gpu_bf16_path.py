"""The bf16 arithmetic path of a bfloat16 module (parallel mode).

A bf16 x bf16 product is exact in float32, so the linear-layer products of
a bf16 module run as one bf16 tensor-core MMA per k-step
(hs_linear_forward_bf16 / hs_linear_backward_bf16) instead of widening the
operands to float32 and running the three-product fp16 split, and its saved
activations (Z, c) are stored in bf16 (hs_scan_forward_bf16 /
hs_scan_backward_bf16; the scan backward writes dZ directly as the bf16
operand of the gradient GEMMs).  Checked here:

* the bf16 GEMMs against float64 products of the same bf16 values
  (normwise 3e-5: exact products, float32 accumulation on the tensor core
  folded into float32 registers every 512 k; measured 6e-8 to 7e-7),
  including the benchmark's weight-gradient shape (K = 524,288, split-K);
* the bf16-storage scans (Z, c, out, dout, dZ in bf16; float32 arithmetic
  and state) against the float32 per-column scans fed the same bf16
  values: every stored value must equal the float32 result rounded to bf16
  bit for bit (same arithmetic in the same order), h_n, c_n, dc0, db
  identical; shapes without the per-column kernels are refused;
* hs_parallel_forward_bf16 against its parts (bf16 GEMM writing bf16 Z,
  then the bf16 scan), bit for bit;
* a bf16 module's full configs[4] micro-batch (T=16384, B=32, D=512,
  H=1024) forward and backward against float64 at the bf16 variant's 2e-2
  (Z rounded to bf16 costs about 1.3e-3 on out at this T with the forget
  gate spread over [-8, 8]).
"""

import math

import pytest
import torch

from _cases import make_inputs
from oracle import hs_oracle as O

pytestmark = pytest.mark.gpu
TOL_GEMM = 3e-5


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max()).item()


def _L():
    from prlstm_b200 import _lib as L

    return L


def _bf(t):
    return t.to(torch.bfloat16).contiguous()


@pytest.mark.parametrize("M,N,K,bias", [(4096, 1024, 256, True), (1000, 520, 136, True), (2048, 8192, 1024, False),
                                        (300, 64, 8, True), (16384, 4096, 512, True)])
def test_linear_forward_bf16(M, N, K, bias):
    L = _L()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    x = _bf(torch.randn(M, K, device=dev, generator=g))
    w = _bf(torch.randn(N, K, device=dev, generator=g) / math.sqrt(K))
    b = torch.randn(N, device=dev, generator=g) if bias else None
    y = torch.empty(M, N, device=dev)
    ws = L.workspace(L.load().hs_linear_bf16_workspace_bytes(M, N, K), dev)
    P = L.ptr
    L.call("hs_linear_forward_bf16", P(x), P(w), P(b), P(y), M, N, K, P(ws), ws.numel(), P(L.status_word(dev)),
           L.stream_ptr(dev))
    ref = x.double() @ w.double().t()
    if bias:
        ref += b.double()
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    e = _rel(y, ref)
    print(f"BF16GEMM fwd {M}x{N}x{K} {e:.3e}")
    assert e < TOL_GEMM


@pytest.mark.parametrize("M,N,K,beta,with_dx", [(4096, 1024, 256, 0, True), (1000, 520, 136, 1, True),
                                                (8192, 2048, 64, 0, False), (2048, 256, 1024, 1, True)])
def test_linear_backward_bf16(M, N, K, beta, with_dx):
    L = _L()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + 3 * N + K)
    dy = _bf(torch.randn(M, N, device=dev, generator=g))
    x = _bf(torch.randn(M, K, device=dev, generator=g))
    w = _bf(torch.randn(N, K, device=dev, generator=g) / math.sqrt(K))
    dw0 = torch.randn(N, K, device=dev, generator=g)
    dw = dw0.clone()
    dx = torch.empty(M, K, device=dev) if with_dx else None
    ws = L.workspace(L.load().hs_linear_bf16_workspace_bytes(M, N, K), dev)
    P = L.ptr
    L.call("hs_linear_backward_bf16", P(dy), P(x), P(w), P(dx), P(dw), M, N, K, beta, P(ws), ws.numel(),
           P(L.status_word(dev)), L.stream_ptr(dev))
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    ref_dw = dy.double().t() @ x.double() + (dw0.double() if beta else 0)
    e = _rel(dw, ref_dw)
    print(f"BF16GEMM wgrad {M}x{N}x{K} {e:.3e}")
    assert e < TOL_GEMM
    if with_dx:
        e = _rel(dx, dy.double() @ w.double())
        print(f"BF16GEMM dgrad {M}x{N}x{K} {e:.3e}")
        assert e < TOL_GEMM


def test_linear_backward_bf16_at_benchmark_k():
    """dW_ih = dZ^T x over M = T*B = 524,288 rows (split-K) and dX = dZ W_ih
    at the configs[4] micro-batch shape, checked on sampled rows."""
    L = _L()
    dev = torch.device("cuda", 0)
    M, N, K = 16384 * 32, 4096, 512
    g = torch.Generator(device=dev).manual_seed(46)
    dz = torch.randn(M, N, device=dev, generator=g)
    dz.mul_(torch.rand(1, N, device=dev, generator=g).pow_(4))
    dz = _bf(dz)
    x = _bf(torch.randn(M, K, device=dev, generator=g))
    w = _bf(torch.randn(N, K, device=dev, generator=g) / math.sqrt(K))
    dx = torch.empty(M, K, device=dev)
    dw = torch.empty(N, K, device=dev)
    ws = L.workspace(L.load().hs_linear_bf16_workspace_bytes(M, N, K), dev)
    P = L.ptr
    L.call("hs_linear_backward_bf16", P(dz), P(x), P(w), P(dx), P(dw), M, N, K, 0, P(ws), ws.numel(),
           P(L.status_word(dev)), L.stream_ptr(dev))
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    del ws
    rows = torch.randperm(N, generator=torch.Generator().manual_seed(1))[:512].to(dev)
    e = _rel(dw[rows], dz[:, rows].double().t() @ x.double())
    print(f"BF16GEMM wgrad K=524288 {e:.3e}")
    assert e < TOL_GEMM
    mrows = torch.randperm(M, generator=torch.Generator().manual_seed(2))[:16384].to(dev)
    e = _rel(dx[mrows], dz[mrows].double() @ w.double())
    print(f"BF16GEMM dgrad M=524288 {e:.3e}")
    assert e < TOL_GEMM
    del dz, x, dx, dw
    torch.cuda.empty_cache()


def _scan_inputs(T, B, H, dev):
    g = torch.Generator(device=dev).manual_seed(T + B + H)
    z = (torch.randn(T, B, 4 * H, device=dev, generator=g) * 3)
    z[..., H:2 * H] += 4.0
    c0 = torch.rand(B, H, device=dev, generator=g)
    dout = torch.randn(T, B, H, device=dev, generator=g)
    dh_n = torch.randn(B, H, device=dev, generator=g)
    dc_n = torch.randn(B, H, device=dev, generator=g)
    return _bf(z), c0, _bf(dout), dh_n, dc_n


@pytest.mark.parametrize("T,B,H", [(2048, 32, 1024), (100, 24, 1024), (577, 64, 328)])
def test_bf16_scans_equal_float32_scans_on_the_same_values(T, B, H):
    """hs_scan_forward_bf16 / hs_scan_backward_bf16 (bf16 z, c, out, dout,
    dZ) against the float32 per-column scans fed the same bf16 values: the
    arithmetic is the same, so every stored value must equal the float32
    result rounded to bf16, and h_n, c_n, dc0, db must be identical."""
    L = _L()
    lib = L.load()
    dev = torch.device("cuda", 0)
    assert lib.hs_scan_uses_column_kernels(T, B, H) == 1
    z, c0, dout, dh_n, dc_n = _scan_inputs(T, B, H, dev)
    P, st, sw = L.ptr, L.stream_ptr(dev), L.status_word(dev)
    bf = torch.bfloat16
    # bf16 storage
    out_b, c_b = torch.empty(T, B, H, device=dev, dtype=bf), torch.empty(T, B, H, device=dev, dtype=bf)
    hn_b, cn_b = torch.empty(B, H, device=dev), torch.empty(B, H, device=dev)
    L.call("hs_scan_forward_bf16", P(z), P(c0), P(out_b), P(c_b), P(hn_b), P(cn_b), T, B, H, 1e-6, P(sw), st)
    dz_b = torch.empty(T, B, 4 * H, device=dev, dtype=bf)
    dc0_b, db_b = torch.empty(B, H, device=dev), torch.empty(4 * H, device=dev)
    wsb = L.workspace(lib.hs_scan_bf16_workspace_bytes(T, B, H), dev)
    L.call("hs_scan_backward_bf16", P(z), P(c_b), P(c0), P(dout), P(dh_n), P(dc_n), P(dz_b), P(dc0_b), P(db_b),
           T, B, H, 1e-6, P(wsb), wsb.numel(), P(sw), st)
    # float32 storage of the same values
    z32 = z.float()
    out32, c32 = torch.empty(T, B, H, device=dev), torch.empty(T, B, H, device=dev)
    hn32, cn32 = torch.empty(B, H, device=dev), torch.empty(B, H, device=dev)
    ws = L.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
    L.call("hs_scan_forward", P(z32), P(c0), P(out32), P(c32), P(hn32), P(cn32), T, B, H, 1e-6, P(ws), ws.numel(),
           P(sw), st)
    dz32, dc0_32, db32 = torch.empty_like(z32), torch.empty(B, H, device=dev), torch.empty(4 * H, device=dev)
    cb32 = c_b.float()  # the backward reads the bf16-stored c in both runs
    d32 = dout.float()
    L.call("hs_scan_backward", P(z32), P(cb32), P(c0), P(d32), P(dh_n), P(dc_n), P(dz32), P(dc0_32),
           P(db32), T, B, H, 1e-6, P(ws), ws.numel(), P(sw), st)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    assert torch.equal(out_b, out32.to(bf)) and torch.equal(c_b, c32.to(bf))
    assert torch.equal(hn_b, hn32) and torch.equal(cn_b, cn32)
    assert torch.equal(dz_b, dz32.to(bf))
    assert torch.equal(dc0_b, dc0_32) and torch.equal(db_b, db32)


def test_bf16_scan_refuses_shapes_without_column_kernels():
    L = _L()
    lib = L.load()
    dev = torch.device("cuda", 0)
    T, B, H = 64, 2, 64
    assert lib.hs_scan_uses_column_kernels(T, B, H) == 0
    assert lib.hs_parallel_bf16_supported(T, B, 64, H) == 0
    z, c0, _, _, _ = _scan_inputs(T, B, H, dev)
    out = torch.empty(T, B, H, device=dev, dtype=torch.bfloat16)
    c = torch.empty_like(out)
    P = L.ptr
    rc = lib.hs_scan_forward_bf16(P(z), P(c0), P(out), P(c), None, None, T, B, H, 1e-6, P(L.status_word(dev)),
                                  L.stream_ptr(dev))
    assert rc == 3  # HS_ERR_UNSUPPORTED


def test_parallel_forward_bf16_is_its_parts():
    """hs_parallel_forward_bf16's bf16 Z equals the bf16 GEMM's float32
    result rounded to bf16 (same MMAs, same accumulation order), and its out,
    c, h_n, c_n equal the bf16 scan's on that Z."""
    L = _L()
    lib = L.load()
    dev = torch.device("cuda", 0)
    T, B, D, H = 512, 32, 512, 1024
    assert lib.hs_parallel_bf16_supported(T, B, D, H) == 1
    g = torch.Generator(device=dev).manual_seed(9)
    x = _bf(torch.randn(T, B, D, device=dev, generator=g))
    W = _bf(torch.randn(4 * H, D, device=dev, generator=g) / math.sqrt(D))
    b = torch.randn(4 * H, device=dev, generator=g)
    b[H:2 * H] += 3.0
    bf = torch.bfloat16
    P, st, sw = L.ptr, L.stream_ptr(dev), L.status_word(dev)
    z = torch.empty(T, B, 4 * H, device=dev, dtype=bf)
    out, c = torch.empty(T, B, H, device=dev, dtype=bf), torch.empty(T, B, H, device=dev, dtype=bf)
    hn, cn = torch.empty(B, H, device=dev), torch.empty(B, H, device=dev)
    ws = L.workspace(lib.hs_parallel_bf16_workspace_bytes(T, B, D, H), dev)
    L.call("hs_parallel_forward_bf16", P(x), None, P(W), P(b), P(z), P(out), P(c), P(hn), P(cn), T, B, D, H, 1e-6,
           P(ws), ws.numel(), P(sw), st)
    y = torch.empty(T, B, 4 * H, device=dev)
    wl = L.workspace(lib.hs_linear_bf16_workspace_bytes(T * B, 4 * H, D), dev)
    L.call("hs_linear_forward_bf16", P(x), P(W), P(b), P(y), T * B, 4 * H, D, P(wl), wl.numel(), P(sw), st)
    out2, c2 = torch.empty_like(out), torch.empty_like(c)
    hn2, cn2 = torch.empty_like(hn), torch.empty_like(cn)
    L.call("hs_scan_forward_bf16", P(z), None, P(out2), P(c2), P(hn2), P(cn2), T, B, H, 1e-6, P(sw), st)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    assert torch.equal(z, y.to(bf))
    assert torch.equal(out, out2) and torch.equal(c, c2) and torch.equal(hn, hn2) and torch.equal(cn, cn2)
    e = _rel(y, (x.double().reshape(-1, D) @ W.double().t() + b.double()).reshape(T, B, 4 * H))
    assert e < TOL_GEMM


def _module(D, H, params, dev, dtype):
    import prlstm_b200

    m = prlstm_b200.HeadStartLSTM(D, H, parallel=True).to(dev, dtype)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    return m


def test_bf16_cfg4_micro_batch_full_size_vs_float64():
    """One configs[4] micro-batch in bf16 through the module: forward and
    sum(out*G) backward against float64 on the same bf16-valued inputs and
    weights (time-chunked float64 checker on the GPU), at 2e-2."""
    import prlstm_b200

    dev = torch.device("cuda", 0)
    T, B, D, H = 16384, 32, 512, 1024
    params, _, _ = make_inputs(8, 1, D, H, a=0.0, bias_spread=8.0, seed=0)
    params = tuple(p.to(torch.bfloat16) for p in params)
    W_ih, _, b_ih, _, _ = params
    g = torch.Generator(device=dev).manual_seed(47)
    x = torch.randn(T, B, D, device=dev, generator=g).to(torch.bfloat16)
    G = torch.randn(T, B, H, device=dev, generator=g).to(torch.bfloat16)
    m = _module(D, H, params, dev, torch.bfloat16)
    xd = x.clone().requires_grad_(True)
    out, (h_n, c_n) = m(xd)
    (out.float() * G.float()).sum().backward()
    torch.cuda.synchronize(dev)
    prlstm_b200.check_device_status(dev)
    ours = dict(out=out.detach(), h_n=h_n[0].detach(), c_n=c_n[0].detach(), dx=xd.grad,
                dW_ih=m.weight_ih_l0.grad, db_ih=m.bias_ih_l0.grad)
    assert all(v.dtype == torch.bfloat16 for v in ours.values())
    del xd, out
    W64, b64 = W_ih.double().to(dev), b_ih.double().to(dev)
    x64 = x.double()
    dx64 = torch.empty_like(x64)
    dW64 = torch.zeros_like(W64)

    def zchunk(t0, t1):
        return torch.nn.functional.linear(x64[t0:t1], W64, b64)

    def on_dz(t0, t1, dz):
        dx64[t0:t1] = dz @ W64
        dW64.add_(dz.reshape(-1, 4 * H).t() @ x64[t0:t1].reshape(-1, D))

    c0 = torch.zeros(B, H, dtype=torch.float64, device=dev)
    r = O.par_linear_chunked(zchunk, T, c0, G.double(), chunk=256, on_dz=on_dz)
    truth = dict(out=r["out"], h_n=r["h_n"], c_n=r["c_n"], dx=dx64, dW_ih=dW64, db_ih=r["db"])
    errs = {k: _rel(ours[k], truth[k]) for k in truth}
    print("BF16 cfg4 micro-batch:", {k: f"{e:.3e}" for k, e in errs.items()})
    for k, e in errs.items():
        assert e < 2e-2, f"{k}: {e:.3e}"
    del ours, truth, r, x64, dx64
    torch.cuda.empty_cache()
