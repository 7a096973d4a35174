"""The module under CUDA-graph capture (torch.cuda.graph), as a user graphs a
launch-bound training step: forward and sum(out*G) backward captured once on
static inputs, replayed after new inputs are copied in.  Every library call
is stream-ordered (no host synchronisation, no allocation of its own), and
the status read-back stands aside while a stream is capturing, so replays
must equal eager runs on the same inputs bit for bit (same kernels, same
order), for configs[1]'s shape in float32 and a bf16 module.  The scans are
held on the per-column kernels (HS_SCAN_PATH=chain), whose order of
operations is fixed; the look-back kernels that configs[1]'s shape takes by
default compose carries in whichever order predecessors publish, so their
float32 results may differ in the last bits from run to run, graphed or
not."""

import os

import pytest
import torch

from _cases import make_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture
def chain_path():
    old = os.environ.get("HS_SCAN_PATH")
    os.environ["HS_SCAN_PATH"] = "chain"
    yield
    if old is None:
        del os.environ["HS_SCAN_PATH"]
    else:
        os.environ["HS_SCAN_PATH"] = old


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graphed_step_equals_eager(dtype, chain_path):
    import prlstm_b200

    dev = torch.device("cuda", 0)
    T, B, D, H = 128, 32, 256, 256
    params, _, _ = make_inputs(8, 1, D, H, a=0.0, seed=3)
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=True).to(dev, dtype)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    g = torch.Generator(device=dev).manual_seed(5)
    xs = [torch.randn(T, B, D, device=dev, generator=g).to(dtype) for _ in range(3)]
    Gs = [torch.randn(T, B, H, device=dev, generator=g).to(dtype) for _ in range(3)]

    def eager(x, G):
        m.zero_grad(set_to_none=True)
        xl = x.clone().requires_grad_(True)
        out, (h_n, c_n) = m(xl)
        (out * G).sum().backward()
        return [out.detach().clone(), h_n.detach().clone(), c_n.detach().clone(), xl.grad.clone()] + \
               [p.grad.clone() for p in (m.weight_ih_l0, m.bias_ih_l0)]

    want = [eager(x, G) for x, G in zip(xs, Gs)]
    sx, sG = xs[0].clone(), Gs[0].clone()
    xleaf = sx.detach().requires_grad_(True)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(2):
            m.zero_grad(set_to_none=True)
            out, _ = m(xleaf)
            (out * sG).sum().backward()
    torch.cuda.current_stream(dev).wait_stream(side)
    m.zero_grad(set_to_none=True)
    xleaf.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out, (h_n, c_n) = m(xleaf)
        (out * sG).sum().backward()
    for k, (x, G) in enumerate(zip(xs, Gs)):
        sx.copy_(x)
        sG.copy_(G)
        graph.replay()
        torch.cuda.synchronize(dev)
        got = [out, h_n, c_n, xleaf.grad, m.weight_ih_l0.grad, m.bias_ih_l0.grad]
        for i, (a, b) in enumerate(zip(got, want[k])):
            assert torch.equal(a, b), (k, i)
    prlstm_b200.check_device_status(dev)
    del graph


def test_graphed_recurrent_step_equals_eager():
    """configs[0]'s recurrent shape, whose recurrence runs on the cluster
    kernels (plain cluster launches, capturable; the FFMA and tensor-core
    recurrent kernels are cooperative launches and are not captured)."""
    import prlstm_b200
    from prlstm_b200 import _lib

    dev = torch.device("cuda", 0)
    T, B, D, H = 32, 16, 64, 128
    assert _lib.load().hs_recurrent_path(B, H, 0) == 2 and _lib.load().hs_recurrent_path(B, H, 1) == 2
    params, _, _ = make_inputs(8, 1, D, H, a=1e-4, seed=4)
    m = prlstm_b200.HeadStartLSTM(D, H).to(dev)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    g = torch.Generator(device=dev).manual_seed(6)
    xs = [torch.randn(T, B, D, device=dev, generator=g) for _ in range(3)]
    Gs = [torch.randn(T, B, H, device=dev, generator=g) for _ in range(3)]

    def eager(x, G):
        m.zero_grad(set_to_none=True)
        xl = x.clone().requires_grad_(True)
        out, (h_n, c_n) = m(xl)
        (out * G).sum().backward()
        return [out.detach().clone(), h_n.detach().clone(), c_n.detach().clone(), xl.grad.clone()] + \
               [p.grad.clone() for p in m.parameters()]

    want = [eager(x, G) for x, G in zip(xs, Gs)]
    sx, sG = xs[0].clone(), Gs[0].clone()
    xleaf = sx.detach().requires_grad_(True)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(2):
            m.zero_grad(set_to_none=True)
            out, _ = m(xleaf)
            (out * sG).sum().backward()
    torch.cuda.current_stream(dev).wait_stream(side)
    m.zero_grad(set_to_none=True)
    xleaf.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out, (h_n, c_n) = m(xleaf)
        (out * sG).sum().backward()
    for k, (x, G) in enumerate(zip(xs, Gs)):
        sx.copy_(x)
        sG.copy_(G)
        graph.replay()
        torch.cuda.synchronize(dev)
        got = [out, h_n, c_n, xleaf.grad] + [p.grad for p in m.parameters()]
        for i, (a, b) in enumerate(zip(got, want[k])):
            assert torch.equal(a, b), (k, i)
    prlstm_b200.check_device_status(dev)
    del graph
