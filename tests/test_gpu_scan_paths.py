"""Both scan implementations through the C ABI (hs_scan_forward /
hs_scan_backward), forced with HS_SCAN_PATH: the one-warp-per-chain kernels
and the decoupled look-back kernels.  Each is checked against the float64
oracle (clamped linear recurrence and its hand-derived gradient), including
c0, dh_n/dc_n, dc0 and the bias sums, on ragged H (partial 32-unit chains,
H not a multiple of 4)."""

import math
import os

import pytest
import torch

from oracle import hs_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return ((a - b).abs().max() / b.abs().max()).item()


def _run(path, z, c0, G, dh_n, dc_n):
    from prlstm_b200 import _lib as L

    T, B, H4 = z.shape
    H = H4 // 4
    dev = z.device
    old = os.environ.get("HS_SCAN_PATH")
    os.environ["HS_SCAN_PATH"] = path
    try:
        lib = L.load()
        ws = L.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
        st = L.stream_ptr(dev)
        P = L.ptr
        out = torch.empty(T, B, H, device=dev)
        c = torch.empty(T, B, H, device=dev)
        h_n = torch.empty(B, H, device=dev)
        c_n = torch.empty(B, H, device=dev)
        L.call("hs_scan_forward", P(z), P(c0), P(out), P(c), P(h_n), P(c_n), T, B, H, 1e-6, P(ws),
               ws.numel(), P(L.status_word(dev)), st)
        dz = torch.empty_like(z)
        dc0 = torch.empty(B, H, device=dev)
        db = torch.empty(4 * H, device=dev)
        L.call("hs_scan_backward", P(z), P(c), P(c0), P(G), P(dh_n), P(dc_n), P(dz), P(dc0), P(db), T,
               B, H, 1e-6, P(ws), ws.numel(), P(L.status_word(dev)), st)
        torch.cuda.synchronize(dev)
        L.check_device_status(dev)
    finally:
        if old is None:
            del os.environ["HS_SCAN_PATH"]
        else:
            os.environ["HS_SCAN_PATH"] = old
    return dict(out=out, c=c, h_n=h_n, c_n=c_n, dz=dz, dc0=dc0, db=db)


def _truth(z, c0, G, dh_n, dc_n, eps=1e-6):
    """float64: forward by the linear recurrence, backward by its gradient."""
    z = z.double().cpu()
    c0 = c0.double().cpu()
    i, f, g, o = torch.sigmoid(z).chunk(4, dim=-1)
    fp = torch.clamp(f, min=eps)
    bp = torch.clamp(i * g, min=eps)
    T = z.shape[0]
    c = torch.empty_like(fp)
    cp = torch.clamp(c0, min=eps)
    for t in range(T):
        cp = fp[t] * cp + bp[t]
        c[t] = cp
    out = o * torch.tanh(c)
    saved = dict(x=torch.zeros(T, z.shape[1], 1, dtype=torch.float64), Z=z, c=c, c0=c0,
                 W_ih=torch.zeros(z.shape[2], 1, dtype=torch.float64), eps=eps)
    _, _, db, dc0, dz = O.par_backward_linear(saved, G.double().cpu(), dh_n.double().cpu(),
                                             dc_n.double().cpu())
    return dict(out=out, c=c, h_n=out[-1], c_n=c[-1], dz=dz, dc0=dc0, db=db)


@pytest.mark.parametrize("T,B,H", [(1000, 5, 96), (700, 3, 100), (300, 2, 70)])
def test_scan_paths_match_float64(T, B, H):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(T + H)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    z[..., H:2 * H] += 3.0  # long memory in part of the units
    c0 = torch.rand(B, H, device=dev, generator=g)
    c0[:, :5] = 0.0
    G = torch.randn(T, B, H, device=dev, generator=g)
    dh_n = torch.randn(B, H, device=dev, generator=g)
    dc_n = torch.randn(B, H, device=dev, generator=g)
    truth = _truth(z, c0, G, dh_n, dc_n)
    res = {p: _run(p, z, c0, G, dh_n, dc_n) for p in ("chain", "lookback")}
    for p, r in res.items():
        for k in truth:
            e = _rel(r[k], truth[k])
            assert e < TOL, f"{p}:{k} rel err {e:.3e}"
    for k in truth:
        assert _rel(res["chain"][k], res["lookback"][k]) < TOL


@pytest.mark.parametrize("path", ["chain", "lookback"])
def test_scan_backward_absmax(path):
    """hs_scan_backward_absmax writes the same dz as hs_scan_backward (the
    same bits on the column-chain path; the look-back path may combine a
    carry from a tile's aggregate or from its inclusive prefix, whichever is
    published first, so its bits may differ in rounding) and the exact
    max |dz| of its own dz (as float bits) into its word."""
    from prlstm_b200 import _lib as L

    T, B, H = 512, 4, 100
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    c0 = torch.rand(B, H, device=dev, generator=g)
    G = torch.randn(T, B, H, device=dev, generator=g)
    dh_n = torch.randn(B, H, device=dev, generator=g)
    dc_n = torch.randn(B, H, device=dev, generator=g)
    ref = _run(path, z, c0, G, dh_n, dc_n)
    old = os.environ.get("HS_SCAN_PATH")
    os.environ["HS_SCAN_PATH"] = path
    try:
        lib = L.load()
        ws = L.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
        P, st = L.ptr, L.stream_ptr(dev)
        dz = torch.empty_like(z)
        dc0 = torch.empty(B, H, device=dev)
        db = torch.empty(4 * H, device=dev)
        am = torch.full((4,), -1, dtype=torch.int32, device=dev)  # the call zeroes it first
        L.call("hs_scan_backward_absmax", P(z), P(ref["c"]), P(c0), P(G), P(dh_n), P(dc_n), P(dz), P(dc0),
               P(db), T, B, H, 1e-6, P(ws), ws.numel(), P(am), P(L.status_word(dev)), st)
        torch.cuda.synchronize(dev)
        L.check_device_status(dev)
    finally:
        if old is None:
            del os.environ["HS_SCAN_PATH"]
        else:
            os.environ["HS_SCAN_PATH"] = old
    for k, v in (("dz", dz), ("db", db), ("dc0", dc0)):
        if path == "chain":
            assert torch.equal(v, ref[k]), k
        else:
            assert _rel(v, ref[k]) < TOL, k
    assert am[0].item() == dz.abs().max().reshape(1).view(torch.int32).item()


def _split_run(path, z, c0, G, dh_n, dc_n, T, B, H):
    """hs_scan_forward_kf + hs_scan_backward_split on copies of the
    inputs; returns (dz rebuilt from the split, scale word, db, dc0)."""
    from prlstm_b200 import _lib as L

    dev = z.device
    old = os.environ.get("HS_SCAN_PATH")
    os.environ["HS_SCAN_PATH"] = path
    try:
        lib = L.load()
        P, st = L.ptr, L.stream_ptr(dev)
        ws = L.workspace(max(lib.hs_scan_workspace_bytes(T, B, H), lib.hs_scan_split_workspace_bytes(T, B, H)), dev)
        words = torch.zeros(64, dtype=torch.int32, device=dev)
        out = torch.empty(T, B, H, device=dev)
        c = torch.empty(T, B, H, device=dev)
        L.call("hs_scan_forward_kf", P(z), P(c0), P(out), P(c), None, None, T, B, H, 1e-6, P(ws), ws.numel(),
               P(words[0:]), P(L.status_word(dev)), st)
        zc = z.clone()
        split = torch.empty(lib.hs_split_bytes(T * B, 4 * H), dtype=torch.uint8, device=dev)
        dc0 = torch.empty(B, H, device=dev)
        db = torch.empty(4 * H, device=dev)
        L.call("hs_scan_backward_split", P(zc), P(c), P(c0), P(G), P(dh_n), P(dc_n), P(words[0:]), P(split),
               P(words[16:]), P(dc0), P(db), T, B, H, 1e-6, P(ws), ws.numel(), P(L.status_word(dev)), st)
        torch.cuda.synchronize(dev)
        L.check_device_status(dev)
    finally:
        if old is None:
            del os.environ["HS_SCAN_PATH"]
        else:
            os.environ["HS_SCAN_PATH"] = old
    n = T * B * 4 * H
    scale_bits = int(words[16].item())
    m = torch.tensor([scale_bits], dtype=torch.int32).view(torch.float32).item()
    s = 2.0 ** (14 - math.floor(math.log2(m))) if 0 < m < 3e38 else 1.0
    hi = split[: 2 * n].view(torch.float16).double()
    lo = split[2 * n: 4 * n].view(torch.float16).double()
    dz = ((hi + lo) / s).view(T, B, 4 * H)
    return dz, m, db, dc0, split, words


@pytest.mark.parametrize("path,T,B,H,saturate", [("chain", 700, 3, 96, False), ("chain", 300, 2, 128, True),
                                                 ("lookback", 500, 3, 100, False)])
def test_scan_backward_split(path, T, B, H, saturate):
    """hs_scan_backward_split: dZ rebuilt from its fp16 split (hi + lo, over
    the scale) equals the float32 dZ of hs_scan_backward to 1e-6 normwise,
    the scale word bounds max |dZ|, and the bias and c0 gradients are the
    same.  saturate: output gates near zero make dZ tiny against the bound
    from sum |dout|, which exercises the exact-maximum re-run."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(T + H)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    if saturate:
        z[..., 3 * H:] = -60.0  # o ~ 1e-26
        z[..., 0:H] = -60.0     # i*g below eps: only the clamp feeds c
    c0 = torch.rand(B, H, device=dev, generator=g)
    G = torch.randn(T, B, H, device=dev, generator=g)
    dh_n = torch.randn(B, H, device=dev, generator=g)
    dc_n = torch.randn(B, H, device=dev, generator=g)
    ref = _run(path, z, c0, G, dh_n, dc_n)
    dz, m, db, dc0, _, _ = _split_run(path, z, c0, G, dh_n, dc_n, T, B, H)
    ref_dz = ref["dz"].double().cpu()
    amax = ref_dz.abs().max().item()
    assert m >= amax, (m, amax)
    if amax > 0:
        e = ((dz.cpu() - ref_dz).abs().max() / amax).item()
        assert e < 1e-6, e
    assert _rel(db, ref["db"]) < TOL and _rel(dc0, ref["dc0"]) < TOL


@pytest.mark.parametrize("path", ["chain", "lookback"])
def test_linear_backward_from_split(path):
    """The scan backward's fp16 split of dZ fed to hs_linear_backward_presplit
    gives dX = dZ.W_ih and dW_ih = dZ^T.x (beta 0 and 1, x as float32 or as
    its hs_split) within 2e-6 of float64 products of the float32 dZ; and
    hs_linear_forward_presplit from the same split of x gives x.W^T + b."""
    from prlstm_b200 import _lib as L

    T, B, H, D = 640, 4, 128, 96
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    c0 = torch.rand(B, H, device=dev, generator=g)
    G = torch.randn(T, B, H, device=dev, generator=g)
    ref = _run(path, z, c0, G, None, None)
    _, _, _, _, split, words = _split_run(path, z, c0, G, None, None, T, B, H)
    x = torch.randn(T * B, D, device=dev, generator=g)
    w = torch.randn(4 * H, D, device=dev, generator=g) / D ** 0.5
    dw0 = torch.randn(4 * H, D, device=dev, generator=g)
    lib = L.load()
    M, N = T * B, 4 * H
    ws = L.workspace(lib.hs_linear_presplit_workspace_bytes(M, N, D), dev)
    P, st = L.ptr, L.stream_ptr(dev)
    dz64 = ref["dz"].double().cpu().reshape(M, N)
    xsplit = torch.empty(lib.hs_split_bytes(M, D), dtype=torch.uint8, device=dev)
    L.call("hs_split", P(x), M, D, P(xsplit), P(words[32:]), st)
    for beta, given in ((0, "x"), (1, "x"), (0, "split"), (1, "split")):
        dx = torch.empty(M, D, device=dev)
        dw = dw0.clone()
        xa, xs, xsc = (P(x), None, None) if given == "x" else (None, P(xsplit), P(words[32:]))
        L.call("hs_linear_backward_presplit", P(split), P(words[16:]), xa, xs, xsc, P(w), P(dx), P(dw), M, N, D,
               beta, P(ws), ws.numel(), P(L.status_word(dev)), st)
        torch.cuda.synchronize(dev)
        L.check_device_status(dev)
        ref_dw = dz64.t() @ x.double().cpu() + (dw0.double().cpu() if beta else 0)
        assert _rel(dw, ref_dw) < 2e-6
        assert _rel(dx, dz64 @ w.double().cpu()) < 2e-6

    y = torch.empty(M, N, device=dev)
    bias = torch.randn(N, device=dev, generator=g)
    wf = torch.randn(N, D, device=dev, generator=g) / D ** 0.5
    L.call("hs_linear_forward_presplit", P(xsplit), P(words[32:]), P(wf), P(bias), P(y), M, N, D, P(ws), ws.numel(),
           P(L.status_word(dev)), st)
    torch.cuda.synchronize(dev)
    assert _rel(y, x.double().cpu() @ wf.double().cpu().t() + bias.double().cpu()) < 2e-6


def test_scan_wave_sequences_sizing_hint():
    """hs_scan_wave_sequences(H): the sequences whose per-column scan CTAs
    (one per sequence x 64 units) are all resident at once, i.e. resident
    CTAs per SM x SMs / columns per sequence."""
    from prlstm_b200 import _lib as L

    lib = L.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    w64 = lib.hs_scan_wave_sequences(64)
    assert w64 > 0 and w64 % sms == 0 and 1 <= w64 // sms <= 16, (w64, sms)
    assert lib.hs_scan_wave_sequences(1024) == w64 // 16
    assert lib.hs_scan_wave_sequences(1000) == w64 // 16  # 16 columns of 64 units
    assert lib.hs_scan_wave_sequences(0) == 0
