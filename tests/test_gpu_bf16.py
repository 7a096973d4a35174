"""Reduced-precision variant: a bfloat16 module fed bfloat16 inputs.

The reference runs the same module in bfloat16 end to end and checks its
backends against each other at 1e-2 absolute (tests/test_parallel.py:24,
tests/test_triton.py:22).  A recurrent bf16 module whose step runs on the
tensor cores multiplies bf16 a*W_hh by the bf16-rounded state each step
(configs[3], and H=512 forced onto the tensor cores); parallel bf16 modules
of the per-column scan's shapes run bf16 products with bf16 saved
activations.  Here the variant is checked against the float64
oracle fed the same bf16-rounded inputs and weights, with the stated
tolerance of 2e-2 normwise (outputs and gradients are returned in bfloat16,
whose rounding alone is 2^-9 relative).  Output and gradient dtypes must be
the module's."""

import os

import pytest
import torch

from oracle import hs_oracle as O
from _cases import make_inputs, rel_err

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2


@pytest.mark.parametrize("parallel,T,B,D,H,a", [
    (False, 64, 8, 64, 128, 1e-4),
    (False, 32, 4, 96, 256, 0.3),
    (True, 256, 8, 64, 128, 0.0),
    # configs[3], "fp32 and bf16-input fwd+bwd": a ~ U(0, 0.5), tensor-core recurrence
    (False, 64, 32, 1024, 2048, "U(0,0.5)"),
    # configs[4]'s micro-batch at short T: pair GEMMs, per-column scan, split handoff
    (True, 256, 32, 512, 1024, "spread"),
    # the bf16 step product on the tensor cores with resident weights, both directions
    (False, 48, 20, 128, 512, "tc"),
])
def test_bf16_module_against_float64_oracle(parallel, T, B, D, H, a, monkeypatch):
    import prlstm_b200

    dev = torch.device("cuda", 0)
    if a == "tc":
        monkeypatch.setenv("HS_REC_PATH", "tc")
        a = 0.3
    if a == "U(0,0.5)":
        params, x, G = make_inputs(T, B, D, H, a_uniform=(0.0, 0.5), seed=T + H)
    elif a == "spread":
        params, x, G = make_inputs(T, B, D, H, a=0.0, bias_spread=8.0, seed=T + H)
    else:
        params, x, G = make_inputs(T, B, D, H, a=a, seed=T + H)
    params = tuple(p.to(torch.bfloat16) for p in params)
    x = x.to(torch.bfloat16)
    G = G.to(torch.bfloat16)
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=parallel).to(dev, torch.bfloat16)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    xd = x.to(dev).requires_grad_(True)
    out, (h_n, c_n) = m(xd)
    assert out.dtype == h_n.dtype == c_n.dtype == torch.bfloat16
    (out.float() * G.to(dev).float()).sum().backward()
    torch.cuda.synchronize()
    prlstm_b200.check_device_status()
    truth = O.module_forward_backward(tuple(p.double() for p in params), x.double(), G.double(),
                                      parallel=parallel, linear_truth=True)
    got = dict(out=out, h_n=h_n[0], c_n=c_n[0], dx=xd.grad)
    for name, key in zip(("weight_ih_l0", "weight_hh_l0", "bias_ih_l0", "bias_hh_l0", "a"),
                         ("dW_ih", "dW_hh", "db_ih", "db_hh", "da")):
        g = dict(m.named_parameters())[name].grad
        if truth[key] is None:
            assert g is None, name
            continue
        assert g.dtype == torch.bfloat16, name
        got[key] = g
    assert xd.grad.dtype == torch.bfloat16
    for k, v in got.items():
        e = rel_err(v.float().cpu(), truth[k])
        print(f"BF16ERR parallel={parallel} {k} {e:.3e}")
        assert e < TOL_BF16, f"{k}: {e:.3e}"


def test_float64_is_refused():
    import prlstm_b200

    m = prlstm_b200.HeadStartLSTM(8, 16).cuda().double()
    with pytest.raises(TypeError):
        m(torch.zeros(4, 2, 8, dtype=torch.float64, device="cuda"))
