"""The projection and the scan forward as one kernel
(hs_projection_scan_forward) through the C ABI, against the float64 oracle
(Z = x W_ih^T + b_ih, then the clamped linear recurrence of
_parallel.py:21-74) and against the two calls it replaces
(hs_linear_forward_presplit + hs_scan_forward_kf).

Shapes: a partial last time tile (T not a multiple of 128), odd B (the
second CTA of the last pair has no sequence), D not a multiple of 64 (a
zero-filled k tail) or of 8 (padded split rows), the smallest H (one
32-unit block), no bias, c0 given or not, several time tiles per chain
(carries handed between tiles), one time tile (no carries), a configs[4]
micro-batch width (512 chains of 2 sequences x 32 units), and configs[4]'s
full T = 16384 on a few chains (128 tiles per chain)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

# (T, B, D, H, with c0, with bias)
CASES = [
    (256, 4, 128, 256, True, True),
    (300, 5, 96, 128, True, False),
    (1000, 8, 512, 256, False, True),
    (128, 32, 256, 256, True, True),
    (512, 32, 512, 1024, True, True),
    (16384, 4, 64, 128, True, True),
    (300, 9, 100, 32, True, True),   # D % 8 != 0 (padded split rows), H = 32 (one unit block)
    (130, 7, 520, 64, False, True),  # T just past one tile, K tail of 8 in the last k-block
]
EPS = 1e-6


def _rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return ((a - b).abs().max() / b.abs().max()).item()


def _inputs(T, B, D, H, with_c0, with_bias, dev):
    g = torch.Generator().manual_seed(T * 7 + B * 3 + D + H)
    x = torch.randn(T, B, D, generator=g)
    W = torch.randn(4 * H, D, generator=g) / D ** 0.5
    b = torch.randn(4 * H, generator=g) * 2.0 if with_bias else None
    c0 = torch.rand(B, H, generator=g) if with_c0 else None
    to = (lambda t: None if t is None else t.to(dev))
    return x, W, b, c0, to(x), to(W), to(b), to(c0)


def _fused(x, W, b, c0, T, B, D, H):
    from prlstm_b200 import _lib as L

    dev = x.device
    lib = L.load()
    P, st = L.ptr, L.stream_ptr(dev)
    M = T * B
    xs = torch.empty(lib.hs_split_bytes(M, D), dtype=torch.uint8, device=dev)
    words = torch.zeros(64, dtype=torch.int32, device=dev)  # [0] x scale, [16] kf
    L.call("hs_split", P(x), M, D, P(xs), P(words[0:]), st)
    ws = L.workspace(lib.hs_projection_scan_workspace_bytes(T, B, D, H), dev)
    r = dict(z=torch.empty(T, B, 4 * H, device=dev), out=torch.empty(T, B, H, device=dev),
             c=torch.empty(T, B, H, device=dev), h_n=torch.empty(B, H, device=dev),
             c_n=torch.empty(B, H, device=dev))
    L.call("hs_projection_scan_forward", P(xs), P(words[0:]), P(W), P(b), P(c0), P(r["z"]), P(r["out"]),
           P(r["c"]), P(r["h_n"]), P(r["c_n"]), T, B, D, H, EPS, P(ws), ws.numel(), P(words[16:]),
           P(L.status_word(dev)), st)
    # the two-call path on the same split
    u = {k: torch.empty_like(v) for k, v in r.items()}
    ws2 = L.workspace(lib.hs_parallel_workspace_bytes(T, B, D, H), dev)
    L.call("hs_linear_forward_presplit", P(xs), P(words[0:]), P(W), P(b), P(u["z"]), M, 4 * H, D, P(ws2),
           ws2.numel(), P(L.status_word(dev)), st)
    L.call("hs_scan_forward_kf", P(u["z"]), P(c0), P(u["out"]), P(u["c"]), P(u["h_n"]), P(u["c_n"]), T, B, H,
           EPS, P(ws2), ws2.numel(), P(words[32:]), P(L.status_word(dev)), st)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    kf = words[16:17].view(torch.float32).item()
    kf2 = words[32:33].view(torch.float32).item()
    return r, u, kf, kf2


def _scan64(z, c0, eps=EPS):
    """float64 linear recurrence of the clamped gates (and max c_{t-1} f'(1-f'))."""
    z = z.double().cpu()
    i, f, g, o = torch.sigmoid(z).chunk(4, dim=-1)
    fp = torch.clamp(f, min=eps)
    bp = torch.clamp(i * g, min=eps)
    cp = torch.clamp(c0.double().cpu() if c0 is not None else torch.zeros_like(fp[0]), min=eps)
    c = torch.empty_like(fp)
    kf = 0.0
    for t in range(z.shape[0]):
        kf = max(kf, (cp * fp[t] * (1 - fp[t])).max().item())
        cp = fp[t] * cp + bp[t]
        c[t] = cp
    out = o * torch.tanh(c)
    return dict(out=out, c=c, h_n=out[-1], c_n=c[-1]), kf


@pytest.mark.parametrize("case", CASES, ids=[f"T{c[0]}_B{c[1]}_D{c[2]}_H{c[3]}" for c in CASES])
def test_projection_scan_matches_oracle_and_two_call_path(case):
    from prlstm_b200 import _lib as L

    T, B, D, H, with_c0, with_bias = case
    dev = torch.device("cuda", 0)
    x, W, b, c0, xd, Wd, bd, c0d = _inputs(T, B, D, H, with_c0, with_bias, dev)
    if not L.load().hs_projection_scan_workspace_bytes(T, B, D, H):
        pytest.fail("no workspace size for a valid shape")
    r, u, kf, kf2 = _fused(xd, Wd, bd, c0d, T, B, D, H)
    # Z: the pair GEMM's arithmetic (same split, same accumulation groups)
    z64 = x.double().reshape(T * B, D) @ W.double().t()
    if b is not None:
        z64 = z64 + b.double()
    ez = _rel(r["z"].reshape(T * B, 4 * H), z64)
    ezu = _rel(r["z"], u["z"])
    print(f"PROJSCAN T={T} B={B} D={D} H={H}: z vs fp64 {ez:.2e}, vs two-call {ezu:.2e}")
    assert ez < 2e-6, f"z vs fp64 {ez:.3e}"
    assert ezu < 1e-6, f"z vs the pair GEMM {ezu:.3e}"
    # the scan from this z, in float64
    truth, kf64 = _scan64(r["z"], c0)
    for k in ("out", "c", "h_n", "c_n"):
        e = _rel(r[k], truth[k])
        e2 = _rel(r[k], u[k])
        print(f"  {k}: vs fp64 {e:.2e}, vs two-call {e2:.2e}")
        assert e < 1e-5, f"{k} vs fp64 {e:.3e}"
        assert e2 < 1e-5, f"{k} vs two-call {e2:.3e}"
    assert abs(kf - kf64) <= 1e-5 * kf64 + 1e-12, (kf, kf64)
    assert abs(kf - kf2) <= 1e-5 * kf2 + 1e-12, (kf, kf2)


def test_projection_scan_policy_and_errors():
    """The default policy takes the fused kernel when T fills most of one
    128-step time tile, not for short T (a tile would be mostly
    padding) nor over longer T (configs[4], where the two calls are faster
    in the step); shapes it cannot run are refused with an error."""
    from prlstm_b200 import _lib as L

    lib = L.load()
    assert lib.hs_projection_scan_supported(128, 32, 256, 256) == 1
    assert lib.hs_projection_scan_supported(112, 32, 256, 256) == 1
    assert lib.hs_projection_scan_supported(8, 2048, 512, 1024) == 0
    assert lib.hs_projection_scan_supported(100, 32, 256, 256) == 0
    assert lib.hs_projection_scan_supported(16384, 32, 512, 1024) == 0
    assert lib.hs_projection_scan_supported(16384, 2, 512, 1024) == 0
    assert lib.hs_projection_scan_supported(256, 32, 512, 1000) == 0  # H % 32
    dev = torch.device("cuda", 0)
    z = torch.empty(16, device=dev)
    with pytest.raises(RuntimeError):
        L.call("hs_projection_scan_forward", L.ptr(z), L.ptr(z), L.ptr(z), None, None, L.ptr(z), L.ptr(z),
               L.ptr(z), None, None, 256, 32, 512, 1000, EPS, None, 0, None, L.ptr(L.status_word(dev)),
               L.stream_ptr(dev))
