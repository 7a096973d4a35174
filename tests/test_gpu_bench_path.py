"""Parity on the benchmark's own kernel path at the benchmark's own size.

configs[4] runs every 32-sequence micro-batch (T=16384, D=512, H=1024)
through: the split of x and the f16x3 pair-GEMM projection, the per-column
chain scan forward (B * H/32 = 1024 columns: the chain kernels are the
default), the split-writing chain scan backward that hands dZ to the
gradient GEMMs as its fp16 split, and dX / dW_ih on the pair GEMM with
split-K over K = T*B = 524,288.  These tests run exactly that, through the
module API and through the C ABI, against a float64 checker evaluated in
time chunks on the GPU (oracle.hs_oracle.par_linear_chunked: the clamped
linear recurrence and its hand-derived gradient, pinned on the CPU against
the whole-sequence oracle).

Bounds (normwise max|diff| / max|ref|): 1e-5 for the module's outputs and
gradients and for the scans' outputs and dZ, as for every parallel-mode
config; 2e-6 for the GEMM products, as in tests/test_gpu_gemm.py.
"""

import math
import os

import pytest
import torch

from _cases import make_inputs
from oracle import hs_oracle as O

pytestmark = pytest.mark.gpu

T4, B4, D4, H4 = 16384, 32, 512, 1024


def _rel(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()


def test_cfg4_micro_batch_full_size_vs_float64():
    """One configs[4] micro-batch through prlstm_b200.HeadStartLSTM, forward
    and sum(out*G) backward, against float64."""
    import prlstm_b200

    dev = torch.device("cuda", 0)
    params, _, _ = make_inputs(8, 1, D4, H4, a=0.0, bias_spread=8.0, seed=0)
    W_ih, _, b_ih, _, _ = params
    g = torch.Generator(device=dev).manual_seed(44)
    x = torch.randn(T4, B4, D4, device=dev, generator=g)
    G = torch.randn(T4, B4, H4, device=dev, generator=g)
    m = prlstm_b200.HeadStartLSTM(D4, H4, parallel=True).to(dev)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    xd = x.clone().requires_grad_(True)
    out, (h_n, c_n) = m(xd)
    (out * G).sum().backward()
    torch.cuda.synchronize(dev)
    prlstm_b200.check_device_status(dev)
    ours = dict(out=out.detach(), h_n=h_n[0].detach(), c_n=c_n[0].detach(), dx=xd.grad,
                dW_ih=m.weight_ih_l0.grad, db_ih=m.bias_ih_l0.grad)
    del xd, out
    assert m.weight_hh_l0.grad is None and m.a.grad is None

    # float64 truth, time-chunked on the GPU
    W64 = W_ih.double().to(dev)
    b64 = b_ih.double().to(dev)
    x64 = x.double()
    dx64 = torch.empty_like(x64)
    dW64 = torch.zeros_like(W64)

    def zchunk(t0, t1):
        return torch.nn.functional.linear(x64[t0:t1], W64, b64)

    def on_dz(t0, t1, dz):
        dx64[t0:t1] = dz @ W64
        dW64.add_(dz.reshape(-1, 4 * H4).t() @ x64[t0:t1].reshape(-1, D4))

    c0 = torch.zeros(B4, H4, dtype=torch.float64, device=dev)
    r = O.par_linear_chunked(zchunk, T4, c0, G.double(), chunk=256, on_dz=on_dz)
    truth = dict(out=r["out"], h_n=r["h_n"], c_n=r["c_n"], dx=dx64, dW_ih=dW64, db_ih=r["db"])
    errs = {k: _rel(ours[k], truth[k]) for k in truth}
    for k, e in errs.items():
        assert e <= 1e-5, f"{k}: rel err {e:.3e} (all: {errs})"
    del ours, truth, r, x64, dx64
    torch.cuda.empty_cache()


def test_fused_projection_scan_full_size_vs_float64():
    """The projection with the scan forward in its epilogue
    (hs_projection_scan_forward, the bench's `fused_projection_scan_step`)
    on one configs[4] micro-batch at full size, with c0: Z, out, c, h_n, c_n
    against float64 (Z from float64 products of the same x, W_ih, b_ih; the
    scan from that Z), 512 chains of 128 time tiles each."""
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    params, _, _ = make_inputs(8, 1, D4, H4, a=0.0, bias_spread=8.0, seed=0)
    W_ih, _, b_ih, _, _ = (t.to(dev) for t in params)
    g = torch.Generator(device=dev).manual_seed(46)
    x = torch.randn(T4, B4, D4, device=dev, generator=g)
    c0 = torch.rand(B4, H4, device=dev, generator=g)
    lib = L.load()
    P, st = L.ptr, L.stream_ptr(dev)
    M = T4 * B4
    words = torch.zeros(64, dtype=torch.int32, device=dev)
    xs = torch.empty(lib.hs_split_bytes(M, D4), dtype=torch.uint8, device=dev)
    L.call("hs_split", P(x), M, D4, P(xs), P(words[0:]), st)
    ws = L.workspace(lib.hs_projection_scan_workspace_bytes(T4, B4, D4, H4), dev)
    z = torch.empty(T4, B4, 4 * H4, device=dev)
    out = torch.empty(T4, B4, H4, device=dev)
    c = torch.empty(T4, B4, H4, device=dev)
    h_n = torch.empty(B4, H4, device=dev)
    c_n = torch.empty(B4, H4, device=dev)
    L.call("hs_projection_scan_forward", P(xs), P(words[0:]), P(W_ih), P(b_ih), P(c0), P(z), P(out), P(c),
           P(h_n), P(c_n), T4, B4, D4, H4, 1e-6, P(ws), ws.numel(), P(words[16:]), P(L.status_word(dev)), st)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    del xs, ws
    W64, b64, x64 = W_ih.double(), b_ih.double(), x.double()
    ez = 0.0
    for t0 in range(0, T4, 1024):
        ez = max(ez, _rel(z[t0:t0 + 1024], torch.nn.functional.linear(x64[t0:t0 + 1024], W64, b64)))
    assert ez < 2e-6, f"z: {ez:.3e}"
    del x64
    zero = torch.zeros(1, B4, H4, dtype=torch.float64, device=dev).expand(T4, B4, H4)
    r = O.par_linear_chunked(lambda t0, t1: z[t0:t1].double(), T4, c0.double(), zero, chunk=256)
    errs = {k: _rel(v, r[k]) for k, v in dict(out=out, c=c, h_n=h_n, c_n=c_n).items()}
    for k, e in errs.items():
        assert e <= 1e-5, f"{k}: rel err {e:.3e} (all: {errs})"
    del z, out, c, r
    torch.cuda.empty_cache()


def test_weight_gradient_split_k_at_benchmark_k():
    """dW_ih = dZ^T x and dX = dZ W_ih at the benchmark's micro-batch shape
    (M = T*B = 524,288 rows, N = 4H = 4096, K = D = 512) through
    hs_linear_backward_presplit with dZ given as its fp16 split (hs_split of
    a float32 dZ) and x as its split: the weight gradient reduces over
    524,288 rows with split-K.  Checked against float64 products on a
    sample of output rows (all of dW_ih's reduction length is covered)."""
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    M, N, K = T4 * B4, 4 * H4, D4
    g = torch.Generator(device=dev).manual_seed(45)
    # dZ like the scan's: mostly small, heavy-tailed columns
    dz = torch.randn(M, N, device=dev, generator=g)
    dz.mul_(torch.rand(1, N, device=dev, generator=g).pow_(4))
    x = torch.randn(M, K, device=dev, generator=g)
    w = torch.randn(N, K, device=dev, generator=g) / math.sqrt(K)
    lib = L.load()
    P, st = L.ptr, L.stream_ptr(dev)
    words = torch.zeros(64, dtype=torch.int32, device=dev)
    dz_split = torch.empty(lib.hs_split_bytes(M, N), dtype=torch.uint8, device=dev)
    x_split = torch.empty(lib.hs_split_bytes(M, K), dtype=torch.uint8, device=dev)
    L.call("hs_split", P(dz), M, N, P(dz_split), P(words[0:]), st)
    L.call("hs_split", P(x), M, K, P(x_split), P(words[16:]), st)
    ws = L.workspace(lib.hs_linear_presplit_workspace_bytes(M, N, K), dev)
    dx = torch.empty(M, K, device=dev)
    dw = torch.empty(N, K, device=dev)
    L.call("hs_linear_backward_presplit", P(dz_split), P(words[0:]), None, P(x_split), P(words[16:]), P(w),
           P(dx), P(dw), M, N, K, 0, P(ws), ws.numel(), P(L.status_word(dev)), st)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    del dz_split, x_split, ws
    rows = torch.randperm(N, generator=torch.Generator().manual_seed(1))[:512].to(dev)
    ref_dw = dz[:, rows].double().t() @ x.double()
    assert _rel(dw[rows], ref_dw) < 2e-6
    mrows = torch.randperm(M, generator=torch.Generator().manual_seed(2))[:16384].to(dev)
    ref_dx = dz[mrows].double() @ w.double()
    assert _rel(dx[mrows], ref_dx) < 2e-6
    del dz, x, dx, dw
    torch.cuda.empty_cache()


@pytest.mark.parametrize("H", [256, 1024])
def test_chain_scan_full_T_fp32_and_split(H):
    """The chain scan kernels at T=16384 through the C ABI (forced with
    HS_SCAN_PATH=chain, as the benchmark's shape takes them by default):
    hs_scan_forward_kf, then both backward forms, float32 dZ
    (hs_scan_backward, what the bench's scan_alone times) and the fp16 split
    (hs_scan_backward_split, what the step runs), with c0, dh_n and dc_n,
    against float64.  The forget pre-activations are spread over [-8, 8]
    as in configs[4]."""
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    T, B = T4, 8
    g = torch.Generator(device=dev).manual_seed(46 + H)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    z[..., 0:2 * H] += 16.0 * torch.rand(2 * H, device=dev, generator=g) - 8.0
    c0 = torch.rand(B, H, device=dev, generator=g)
    G = torch.randn(T, B, H, device=dev, generator=g)
    dh_n = torch.randn(B, H, device=dev, generator=g)
    dc_n = torch.randn(B, H, device=dev, generator=g)
    old = os.environ.get("HS_SCAN_PATH")
    os.environ["HS_SCAN_PATH"] = "chain"
    try:
        lib = L.load()
        P, st = L.ptr, L.stream_ptr(dev)
        ws = L.workspace(max(lib.hs_scan_workspace_bytes(T, B, H), lib.hs_scan_split_workspace_bytes(T, B, H)),
                         dev)
        words = torch.zeros(64, dtype=torch.int32, device=dev)
        out = torch.empty(T, B, H, device=dev)
        c = torch.empty(T, B, H, device=dev)
        h_n = torch.empty(B, H, device=dev)
        c_n = torch.empty(B, H, device=dev)
        status = P(L.status_word(dev))
        L.call("hs_scan_forward_kf", P(z), P(c0), P(out), P(c), P(h_n), P(c_n), T, B, H, 1e-6, P(ws), ws.numel(),
               P(words[0:]), status, st)
        dz = torch.empty_like(z)
        dc0 = torch.empty(B, H, device=dev)
        db = torch.empty(4 * H, device=dev)
        L.call("hs_scan_backward", P(z), P(c), P(c0), P(G), P(dh_n), P(dc_n), P(dz), P(dc0), P(db), T, B, H,
               1e-6, P(ws), ws.numel(), status, st)
        zc = z.clone()
        split = torch.empty(lib.hs_split_bytes(T * B, 4 * H), dtype=torch.uint8, device=dev)
        dc0s = torch.empty(B, H, device=dev)
        dbs = torch.empty(4 * H, device=dev)
        L.call("hs_scan_backward_split", P(zc), P(c), P(c0), P(G), P(dh_n), P(dc_n), P(words[0:]), P(split),
               P(words[16:]), P(dc0s), P(dbs), T, B, H, 1e-6, P(ws), ws.numel(), status, st)
        torch.cuda.synchronize(dev)
        L.check_device_status(dev)
    finally:
        if old is None:
            os.environ.pop("HS_SCAN_PATH", None)
        else:
            os.environ["HS_SCAN_PATH"] = old
    n = T * B * 4 * H
    m = torch.tensor([int(words[16].item())], dtype=torch.int32).view(torch.float32).item()
    s = 2.0 ** (14 - math.floor(math.log2(m)))
    dz_from_split = ((split[: 2 * n].view(torch.float16).double() + split[2 * n: 4 * n].view(torch.float16).double())
                     / s).view(T, B, 4 * H)
    del split, zc

    z64 = z.double()
    err = {"dz": [0.0, 0.0], "dz_split": [0.0, 0.0]}

    def on_dz(t0, t1, d):
        for k, got in (("dz", dz[t0:t1]), ("dz_split", dz_from_split[t0:t1])):
            err[k][0] = max(err[k][0], (got.double() - d).abs().max().item())
            err[k][1] = max(err[k][1], d.abs().max().item())

    r = O.par_linear_chunked(lambda t0, t1: z64[t0:t1], T, c0.double(), G.double(), dh_n.double(),
                             dc_n.double(), chunk=1024, on_dz=on_dz)
    assert m >= err["dz"][1]  # the split's scale word bounds max |dZ|
    for k, got in (("out", out), ("c", c), ("h_n", h_n), ("c_n", c_n), ("dc0", dc0), ("db", db),
                   ("dc0_split", dc0s), ("db_split", dbs)):
        e = _rel(got, r[k.replace("_split", "")])
        assert e < 1e-5, f"H={H} {k}: rel err {e:.3e}"
    for k, (num, den) in err.items():
        assert num / den < 1e-5, f"H={H} {k}: rel err {num / den:.3e}"
