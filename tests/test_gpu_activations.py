"""Accuracy of the scan kernels' activation functions on the device.

The scan evaluates the logistic sigmoid as a hardware exp followed by a
reciprocal refined by one Newton-Raphson step, and tanh of the (positive) cell
state as (1 - e^-2c)/(1 + e^-2c), with an odd Taylor polynomial below 0.25.
hs_selftest_activations measures both against double precision on the GPU;
the bounds below are what the parity tolerance of 1e-5 needs with a wide
margin, and what the methods give: a few float32 ulps plus the exp's
argument-rounding error, which grows like |x| * 2^-24 for the sigmoid."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("lim,sig_bound,tanh_bound", [(16.0, 1.5e-6, 1.0e-6), (4.0, 5.0e-7, 1.0e-6)])
def test_activation_errors_against_float64(lim, sig_bound, tanh_bound):
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    out = torch.empty(2, device=dev)
    L.call("hs_selftest_activations", L.ptr(out), 1 << 22, lim, L.stream_ptr(dev))
    torch.cuda.synchronize(dev)
    sig_err, tanh_err = out.tolist()
    print(f"ACTERR lim={lim} sigmoid {sig_err:.3e} tanh {tanh_err:.3e}")
    assert sig_err < sig_bound
    assert tanh_err < tanh_bound
