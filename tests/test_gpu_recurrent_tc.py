"""The recurrent path's tensor-core kernels (csrc/recurrent_tc.cu) against the
float64 oracle and against the FFMA kernels (HS_REC_PATH=ffma), through the
module API.

Shapes cover: a resident weight tile with 32 units per CTA (H=128, 256,
384), 16 units per CTA with the upper half of the 128-row tile unused
(H=512), the streamed weight ring (H=2048 forward, and every backward),
batches padded to 16 or 32, several batch groups side by side (B=40, 70),
T=1, a non-zero initial state, gradients entering through h_n and c_n, and
H=96 (tensor-core forward, FFMA backward: H is not a multiple of 128).
Bound: 1e-5 normwise, the recurrent-mode bound of every parity test.
"""

import os

import pytest
import torch

from oracle import hs_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-300)).item()


def _problem(T, B, D, H, a, seed):
    g = torch.Generator().manual_seed(seed)
    params = list(O.init_params(D, H, a_init=0.0 if a is None else a, generator=g))
    if a is None:
        params[4].uniform_(0.0, 0.5, generator=g)
    x = torch.randn(T, B, D, generator=g)
    G = torch.randn(T, B, H, generator=g)
    h0 = 0.5 * torch.randn(B, H, generator=g)
    c0 = torch.randn(B, H, generator=g)
    Gh = torch.randn(B, H, generator=g)
    Gc = torch.randn(B, H, generator=g)
    return params, x, G, h0, c0, Gh, Gc


def _ours(params, x, G, h0, c0, Gh, Gc, path):
    import prlstm_b200

    old = os.environ.get("HS_REC_PATH")
    os.environ["HS_REC_PATH"] = path
    try:
        D, H = params[0].shape[1], params[1].shape[1]
        m = prlstm_b200.HeadStartLSTM(D, H).cuda()
        with torch.no_grad():
            for p, v in zip(m.parameters(), params):
                p.copy_(v)
        xd = x.cuda().requires_grad_(True)
        out, (h_n, c_n) = m(xd, (h0.cuda().unsqueeze(0), c0.cuda().unsqueeze(0)))
        loss = (out * G.cuda()).sum() + (h_n[0] * Gh.cuda()).sum() + (c_n[0] * Gc.cuda()).sum()
        loss.backward()
        torch.cuda.synchronize()
        prlstm_b200.check_device_status()
    finally:
        if old is None:
            os.environ.pop("HS_REC_PATH", None)
        else:
            os.environ["HS_REC_PATH"] = old
    return dict(out=out.detach(), h_n=h_n[0].detach(), c_n=c_n[0].detach(), dx=xd.grad,
                dW_ih=m.weight_ih_l0.grad, dW_hh=m.weight_hh_l0.grad, db_ih=m.bias_ih_l0.grad,
                db_hh=m.bias_hh_l0.grad, da=m.a.grad)


def _truth(params, x, G, h0, c0, Gh, Gc):
    p64 = [t.double() for t in params]
    out, h_n, c_n, saved = O.rec_forward(x.double(), h0.double(), c0.double(), *p64)
    dx, dW_ih, dW_hh, db_ih, db_hh, da = O.rec_backward(saved, G.double(), Gh.double(), Gc.double())
    return dict(out=out, h_n=h_n, c_n=c_n, dx=dx, dW_ih=dW_ih, dW_hh=dW_hh, db_ih=db_ih, db_hh=db_hh, da=da)


CASES = [
    (17, 5, 24, 128, 0.3),
    (9, 40, 16, 256, 0.5),
    (1, 3, 8, 128, 0.2),
    (33, 32, 64, 512, None),
    (12, 70, 32, 384, 0.4),
    (20, 16, 32, 96, 0.3),
    (6, 8, 32, 2048, None),
]


@pytest.mark.parametrize("T,B,D,H,a", CASES)
def test_tensor_core_recurrence_matches_float64_and_ffma(T, B, D, H, a):
    prob = _problem(T, B, D, H, a, seed=T * 1000 + B * 10 + H)
    truth = _truth(*prob)
    tc = _ours(*prob, path="tc")
    ff = _ours(*prob, path="ffma")
    for k in truth:
        e = _rel(tc[k], truth[k])
        assert e <= TOL, f"{k}: tensor-core path vs float64 {e:.3e}"
        e2 = _rel(tc[k], ff[k])
        assert e2 <= TOL, f"{k}: tensor-core path vs FFMA path {e2:.3e}"
