"""GPU parity of the CUDA library against the reference (golden vectors) and
the CPU oracle.  Every call goes through the C ABI (prlstm_b200 -> ctypes ->
libhsb200.so).

Tolerances (normwise max|diff| / max|ref|, float32 runs):
  * recurrent mode: 1e-5 against the reference torch backend in float32
    and against float64;
  * parallel mode: judged against float64 truth, tol = max(1e-5, 2 x the
    reference float32 path's own error vs float64) -- the reference's float32
    log-domain scan is itself off float64 at long T; the raw difference to the
    reference float32 result is also bounded.
"""

import pytest
import torch

from _cases import case_tensors, golden_expect, golden_names, load_golden, make_inputs, rel_err
from oracle import hs_oracle as O

pytestmark = pytest.mark.gpu

KEYS = ("out", "h_n", "c_n", "dx", "dW_ih", "dW_hh", "db_ih", "db_hh", "da")
REC_TOL = 1e-5


def run_ours(params, x, G, parallel, hx=None, batch_first=False, dev="cuda"):
    """One fwd + sum(out*G).backward() through prlstm_b200.HeadStartLSTM."""
    import prlstm_b200

    W_ih, W_hh, b_ih, b_hh, a = params
    D = W_ih.shape[1]
    H = W_hh.shape[1]
    m = prlstm_b200.HeadStartLSTM(D, H, batch_first=batch_first, parallel=parallel).to(dev)
    with torch.no_grad():
        for p, v in zip(m.parameters(), (W_ih, W_hh, b_ih, b_hh, a)):
            p.copy_(v.float())
    xx = x.float()
    GG = G.float()
    if batch_first:
        xx = xx.transpose(0, 1).contiguous()
        GG = GG.transpose(0, 1).contiguous()
    xd = xx.to(dev).requires_grad_(True)
    hxd = None
    if hx is not None:
        hxd = (hx[0].float().to(dev).unsqueeze(0), hx[1].float().to(dev).unsqueeze(0))
    out, (h_n, c_n) = m(xd, hxd)
    (out * GG.to(dev)).sum().backward()
    torch.cuda.synchronize()
    prlstm_b200.check_device_status()
    o = out.detach()
    dx = xd.grad
    if batch_first:
        o = o.transpose(0, 1)
        dx = dx.transpose(0, 1)
    res = dict(out=o.cpu(), h_n=h_n[0].detach().cpu(), c_n=c_n[0].detach().cpu(), dx=dx.cpu())
    for name, key in zip(("weight_ih_l0", "weight_hh_l0", "bias_ih_l0", "bias_hh_l0", "a"),
                         ("dW_ih", "dW_hh", "db_ih", "db_hh", "da")):
        g = getattr(m, name).grad
        res[key] = None if g is None else g.cpu()
    return res


def assert_close(got, ref, tol, tag):
    for k in KEYS:
        if k not in ref:
            continue
        if ref[k] is None:
            assert got[k] is None, f"{tag}:{k} must have no gradient"
            continue
        e = rel_err(got[k], ref[k])
        assert e <= tol, f"{tag}:{k} rel err {e:.3e} > {tol:.1e}"


# ------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("name", golden_names("rec_"))
def test_recurrent_matches_reference_golden(name):
    g = load_golden(name)
    params, x, G, hx = case_tensors(g)
    ours = run_ours(params, x, G, parallel=False, hx=hx)
    exp = golden_expect(g)
    assert_close(ours, exp, REC_TOL, name)


@pytest.mark.parametrize("name", golden_names("par_"))
def test_parallel_matches_reference_golden(name):
    g = load_golden(name)
    params, x, G, hx = case_tensors(g)
    ref32 = golden_expect(g)
    p64, x64, G64, hx64 = case_tensors(g, dtype=torch.float64)
    truth = O.module_forward_backward(p64, x64, G64, parallel=True, hx=hx64, linear_truth=True)
    ours = run_ours(params, x, G, parallel=True, hx=hx)
    for k in ("out", "h_n", "c_n", "dx", "dW_ih", "db_ih"):
        ref_err = rel_err(ref32[k], truth[k]) if str(g["dtype"]) == "float32" else 0.0
        tol = max(1e-5, 2 * ref_err)
        e = rel_err(ours[k], truth[k])
        assert e <= tol, f"{name}:{k} vs fp64 {e:.3e} > {tol:.1e}"
        raw = rel_err(ours[k], ref32[k])
        assert raw <= tol + max(ref_err, 1e-5), f"{name}:{k} vs reference {raw:.3e}"
    for k in ("dW_hh", "db_hh", "da"):
        assert ours[k] is None


# ------------------------------------------------------------ benchmark configs
CONFIGS = {
    "cfg0": dict(T=32, B=16, D=64, H=128, a=1e-4, parallel=False),
    "cfg1": dict(T=128, B=32, D=256, H=256, a=0.0, parallel=True),
    "cfg2": dict(T=256, B=32, D=256, H=512, a=1e-4, parallel=False),
    "cfg3": dict(T=64, B=32, D=1024, H=2048, a_uniform=(0.0, 0.5), parallel=False),
    # configs[4] at full T on a 2-sequence batch slice
    "cfg4_slice": dict(T=16384, B=2, D=512, H=1024, a=0.0, bias_spread=8.0, parallel=True),
    # configs[4]'s 32-sequence micro-batch at short T: enough columns for the
    # per-column scan, so the backward hands dZ to the GEMMs as its fp16 split
    "cfg4_columns": dict(T=256, B=32, D=512, H=1024, a=0.0, bias_spread=8.0, parallel=True),
}


@pytest.mark.parametrize("cfg", list(CONFIGS))
def test_config_parity_vs_oracle(cfg):
    c = dict(CONFIGS[cfg])
    parallel = c.pop("parallel")
    T, B, D, H = c.pop("T"), c.pop("B"), c.pop("D"), c.pop("H")
    params, x, G = make_inputs(T, B, D, H, seed=0, **c)
    ours = run_ours(params, x, G, parallel=parallel)
    p64 = tuple(t.double() for t in params)
    truth = O.module_forward_backward(p64, x.double(), G.double(), parallel=parallel,
                                      linear_truth=parallel)
    if not parallel:
        ref32 = O.module_forward_backward(params, x, G, parallel=False)
        assert_close(ours, ref32, REC_TOL, cfg + " vs ref fp32")
        assert_close(ours, truth, REC_TOL, cfg + " vs fp64")
    else:
        assert_close(ours, truth, 1e-5, cfg + " vs fp64")


def test_split_handoff_rerun_through_module():
    """Output and input gates saturated shut (biases -60): dZ is some 2^40
    below the bound from sum |dout|, so the module's backward takes the
    exact-maximum re-run of the split handoff; gradients still match the
    float64 oracle."""
    T, B, D, H = 64, 32, 64, 1024
    params, x, G = make_inputs(T, B, D, H, a=0.0, seed=4)
    b_ih = params[2].clone()
    b_ih[0:H] = -60.0
    b_ih[3 * H:4 * H] = -60.0
    params = (params[0], params[1], b_ih, params[3], params[4])
    ours = run_ours(params, x, G, parallel=True)
    truth = O.module_forward_backward(tuple(t.double() for t in params), x.double(), G.double(),
                                      parallel=True, linear_truth=True)
    assert_close(ours, truth, 1e-5, "saturated gates vs fp64")


def test_scan_forward_kf_value():
    """hs_scan_forward_kf's word equals max over steps of c_{t-1} f'(1 - f')
    (float64 of the same inputs, relative 1e-5), on both scan paths."""
    import os
    from prlstm_b200 import _lib as L

    T, B, H = 300, 24, 256
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(8)
    z = 2.0 * torch.randn(T, B, 4 * H, device=dev, generator=g)
    c0 = torch.rand(B, H, device=dev, generator=g)
    eps = 1e-6
    zd, c0d = z.double().cpu(), c0.double().cpu()
    i, f, gg, o = torch.sigmoid(zd).chunk(4, dim=-1)
    fp, bp = f.clamp(min=eps), (i * gg).clamp(min=eps)
    cprev = c0d.clamp(min=eps)
    kf = 0.0
    for t in range(T):
        kf = max(kf, (cprev * fp[t] * (1 - fp[t])).max().item())
        cprev = fp[t] * cprev + bp[t]
    lib = L.load()
    for path in ("chain", "lookback"):
        old = os.environ.get("HS_SCAN_PATH")
        os.environ["HS_SCAN_PATH"] = path
        try:
            ws = L.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
            words = torch.zeros(4, dtype=torch.int32, device=dev)
            out = torch.empty(T, B, H, device=dev)
            c = torch.empty(T, B, H, device=dev)
            L.call("hs_scan_forward_kf", L.ptr(z), L.ptr(c0), L.ptr(out), L.ptr(c), None, None, T, B, H, eps,
                   L.ptr(ws), ws.numel(), L.ptr(words), L.ptr(L.status_word(dev)), L.stream_ptr(dev))
            torch.cuda.synchronize(dev)
        finally:
            if old is None:
                del os.environ["HS_SCAN_PATH"]
            else:
                os.environ["HS_SCAN_PATH"] = old
        got = words[:1].cpu().view(torch.float32).item()
        assert abs(got - kf) <= 1e-5 * kf, (path, got, kf)


# ------------------------------------------------------------ reference test suite, ported
def test_parallel_equals_recurrent_at_zero_a():
    """tests/test_parallel.py:47-60 of the reference."""
    params, x, G = make_inputs(12, 3, 16, 24, a=0.0, seed=4)
    rec = run_ours(params, x, G, parallel=False)
    par = run_ours(params, x, G, parallel=True)
    for k in ("out", "h_n", "c_n"):
        assert (rec[k] - par[k]).abs().max().item() < 1e-4


def test_divergence_grows_with_a():
    """tests/test_parallel.py:63-81 of the reference."""
    params, x, G = make_inputs(12, 3, 16, 24, a=0.0, seed=5)
    diffs = []
    for a_val in (0.0, 1e-4, 1e-2, 1e-1, 1.0):
        p = list(params)
        p[4] = torch.full((4,), a_val)
        rec = run_ours(p, x, G, parallel=False)
        par = run_ours(p, x, G, parallel=True)
        diffs.append((rec["out"] - par["out"]).abs().max().item())
    assert diffs[0] < 1e-4
    assert diffs[-1] > diffs[0] * 100


def test_backward_parity_at_zero_a():
    """tests/test_parallel.py:84-122: input-path grads agree at a=0; the
    recurrent-only parameters get no gradient in parallel mode."""
    params, x, G = make_inputs(10, 3, 8, 12, a=0.0, seed=6)
    rec = run_ours(params, x, G, parallel=False)
    par = run_ours(params, x, G, parallel=True)
    for k in ("dW_ih", "db_ih", "dx"):
        assert (rec[k] - par[k]).abs().max().item() < 1e-4
    assert par["dW_hh"] is None and par["db_hh"] is None and par["da"] is None
    assert rec["dW_hh"] is not None and rec["da"] is not None


@pytest.mark.parametrize("parallel", [False, True])
def test_sgd_training_step_matches_oracle(parallel):
    """tests/test_cpp.py:110-147: one SGD step with an MSE loss."""
    import prlstm_b200

    T, B, D, H, lr = 12, 4, 8, 12, 1e-2
    params, x, target = make_inputs(T, B, D, H, a=0.0 if parallel else 1e-4, seed=8)
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=parallel).cuda()
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    opt = torch.optim.SGD(m.parameters(), lr=lr)
    opt.zero_grad()
    out, _ = m(x.cuda())
    ((out - target.cuda()) ** 2).mean().backward()
    opt.step()
    # oracle step in float64
    p64 = [t.double().clone().requires_grad_(True) for t in params]
    if parallel:
        o, _, _ = O.par_forward(x.double(), torch.zeros(B, H, dtype=torch.float64), p64[0], p64[2])
    else:
        o = _rec_autograd(x.double(), p64)
    ((o - target.double()) ** 2).mean().backward()
    for (n, p), q in zip(m.named_parameters(), p64):
        ref = q.detach() - lr * (q.grad if q.grad is not None else torch.zeros_like(q))
        assert (p.detach().cpu().double() - ref).abs().max().item() < 1e-6, n


def _rec_autograd(x, p):
    """Step-by-step recurrent forward with autograd (tests/test_cpp.py:25-48)."""
    W_ih, W_hh, b_ih, b_hh, a = p
    T, B, _ = x.shape
    H = W_hh.shape[1]
    ae = a.repeat_interleave(H)
    h = x.new_zeros(B, H)
    c = x.new_zeros(B, H)
    outs = []
    for t in range(T):
        gates = torch.nn.functional.linear(x[t], W_ih, b_ih) + torch.nn.functional.linear(
            h, ae.unsqueeze(1) * W_hh, ae * b_hh)
        i, f, g, o = torch.sigmoid(gates).chunk(4, dim=1)
        c = f * c + i * g
        h = o * torch.tanh(c)
        outs.append(h)
    return torch.stack(outs)


# ------------------------------------------------------------ edge cases
@pytest.mark.parametrize("parallel", [False, True])
@pytest.mark.parametrize("T,B,D,H", [(1, 1, 3, 5), (7, 2, 5, 6), (33, 5, 9, 130), (5, 40, 16, 24)])
def test_ragged_shapes(parallel, T, B, D, H):
    params, x, G = make_inputs(T, B, D, H, a=0.0 if parallel else 0.2, seed=T + B)
    ours = run_ours(params, x, G, parallel=parallel)
    p64 = tuple(t.double() for t in params)
    truth = O.module_forward_backward(p64, x.double(), G.double(), parallel=parallel,
                                      linear_truth=parallel)
    assert_close(ours, truth, 1e-5, f"ragged {T},{B},{D},{H} parallel={parallel}")


@pytest.mark.parametrize("parallel", [False, True])
def test_loss_through_final_state(parallel):
    """Gradients arriving through h_n and c_n (not only through out)."""
    import prlstm_b200

    T, B, D, H = 9, 3, 7, 16
    params, x, G = make_inputs(T, B, D, H, a=0.0 if parallel else 0.3, seed=12)
    gh = torch.randn(B, H, generator=torch.Generator().manual_seed(1))
    gc = torch.randn(B, H, generator=torch.Generator().manual_seed(2))
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=parallel).cuda()
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    xd = x.cuda().requires_grad_(True)
    out, (h_n, c_n) = m(xd)
    ((out * G.cuda()).sum() + (h_n[0] * gh.cuda()).sum() + (c_n[0] * gc.cuda()).sum()).backward()
    # oracle in float64 with autograd through the reference formulation
    x64 = x.double().requires_grad_(True)
    p64 = [t.double().clone().requires_grad_(True) for t in params]
    if parallel:
        o, hn, cn = O.par_forward(x64, torch.zeros(B, H, dtype=torch.float64), p64[0], p64[2])
    else:
        ae = p64[4].repeat_interleave(H)
        h = torch.zeros(B, H, dtype=torch.float64)
        c = torch.zeros(B, H, dtype=torch.float64)
        outs = []
        for t in range(T):
            gates = torch.nn.functional.linear(x64[t], p64[0], p64[2]) + torch.nn.functional.linear(
                h, ae.unsqueeze(1) * p64[1], ae * p64[3])
            i, f, g, o_ = torch.sigmoid(gates).chunk(4, dim=1)
            c = f * c + i * g
            h = o_ * torch.tanh(c)
            outs.append(h)
        o, hn, cn = torch.stack(outs), h, c
    ((o * G.double()).sum() + (hn * gh.double()).sum() + (cn * gc.double()).sum()).backward()
    assert rel_err(xd.grad.cpu(), x64.grad) < 1e-5
    for (n, p), q in zip(m.named_parameters(), p64):
        if q.grad is None:
            assert p.grad is None, n
        else:
            assert rel_err(p.grad.cpu(), q.grad) < 1e-5, n


def test_batch_first_and_hx_golden():
    g = load_golden("rec_hx_bf_t6_b5_d10_h20_f32")
    params, x, G, hx = case_tensors(g)
    # case_tensors gives [T,B,*]; run_ours feeds the module [B,T,*] when batch_first
    ours = run_ours(params, x, G, parallel=False, hx=hx, batch_first=True)
    exp = golden_expect(g)
    assert_close(ours, exp, REC_TOL, "batch_first+hx")


def test_fused_projection_scan_through_module_with_hx_batch_first():
    """The module's parallel forward at a shape the library runs as one
    fused projection + scan kernel (T <= 128 and the tensor-core GEMM size;
    hs_projection_scan_supported), with hx (its c0 enters the kernel's first
    time tile, and gets a gradient) and batch_first, against float64."""
    from prlstm_b200 import _lib as L

    T, B, D, H = 128, 24, 256, 256
    assert L.load().hs_projection_scan_supported(T, B, D, H) == 1
    params, x, G = make_inputs(T, B, D, H, a=0.0, bias_spread=8.0, seed=31)
    g = torch.Generator().manual_seed(32)
    hx = (torch.randn(B, H, generator=g) * 0.3, torch.rand(B, H, generator=g))
    ours = run_ours(params, x, G, parallel=True, hx=hx, batch_first=True)
    p64 = tuple(t.double() for t in params)
    truth = O.module_forward_backward(p64, x.double(), G.double(), parallel=True,
                                      hx=(hx[0].double(), hx[1].double()), linear_truth=True)
    assert_close(ours, truth, 1e-5, "fused+hx+batch_first")


# ------------------------------------------------------------ size-independent properties
def test_parallel_batch_independence():
    """Each sequence's result does not depend on the others in the batch (up
    to the rounding of the look-back, whose combine order depends on timing)."""
    import prlstm_b200

    T, B, D, H = 4096, 8, 64, 256
    params, x, G = make_inputs(T, B, D, H, a=0.0, bias_spread=8.0, seed=21)
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=True).cuda()
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    out_all, (hn, cn) = m(x.cuda())
    for b in (0, 5):
        out_b, (hb, cb) = m(x[:, b:b + 1].cuda())
        assert rel_err(out_b, out_all[:, b:b + 1]) < 1e-6
        assert rel_err(cb, cn[:, b:b + 1]) < 1e-6


def test_parallel_backward_linear_in_dout():
    """The backward is linear in the incoming gradient: g(G1+G2) = g(G1)+g(G2)."""
    T, B, D, H = 2048, 4, 32, 128
    params, x, G1 = make_inputs(T, B, D, H, a=0.0, bias_spread=8.0, seed=31)
    G2 = torch.randn(T, B, H, generator=torch.Generator().manual_seed(32))
    r1 = run_ours(params, x, G1, parallel=True)
    r2 = run_ours(params, x, G2, parallel=True)
    r12 = run_ours(params, x, G1 + G2, parallel=True)
    for k in ("dx", "dW_ih", "db_ih"):
        assert rel_err(r12[k], r1[k] + r2[k]) < 1e-5, k


def test_final_state_equals_last_step():
    import prlstm_b200

    for parallel in (False, True):
        params, x, _ = make_inputs(64, 4, 16, 32, a=0.0 if parallel else 0.1, seed=41)
        m = prlstm_b200.HeadStartLSTM(16, 32, parallel=parallel).cuda()
        with torch.no_grad():
            for p, v in zip(m.parameters(), params):
                p.copy_(v)
        out, (h_n, c_n) = m(x.cuda())
        assert torch.equal(out[-1], h_n[0])


# ------------------------------------------------------------ errors and failure detection
def test_cpu_tensors_rejected():
    import prlstm_b200

    m = prlstm_b200.HeadStartLSTM(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(3, 2, 4))


def test_bounded_wait_gives_up_and_context_survives():
    """A device wait on a flag nothing sets gives up after its limit, records
    HS_ERR_DEVICE_TIMEOUT in the status word, and the context stays usable."""
    import prlstm_b200
    from prlstm_b200 import _lib

    dev = torch.device("cuda", 0)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call("hs_selftest_bounded_wait", _lib.ptr(flag), _lib.ptr(status), 50_000_000,
              _lib.stream_ptr(dev))
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.HS_ERR_DEVICE_TIMEOUT
    # context still usable: a normal call afterwards is correct
    params, x, G = make_inputs(8, 2, 4, 8, a=0.0, seed=51)
    ours = run_ours(params, x, G, parallel=True)
    truth = O.module_forward_backward(tuple(t.double() for t in params), x.double(), G.double(),
                                      parallel=True, linear_truth=True)
    assert rel_err(ours["out"], truth["out"]) < 1e-5
    prlstm_b200.check_device_status()
