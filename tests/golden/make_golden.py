"""Generate golden vectors by running the REFERENCE implementation itself.

Run in a container where the reference project is checked out (read-only is
fine):

    PYTHONDONTWRITEBYTECODE=1 PYTHONPATH=<reference>/src \
        python tests/golden/make_golden.py

It imports ``headstartlstm`` (m-j-tilley/prLSTM), drives the public module
API exactly as the reference's own tests do (``tests/test_cpp.py:55-107``,
``tests/test_parallel.py:47-122``): seeded construction, ``m(x)``,
``sum(out * G).backward()``, and stores inputs, outputs and every gradient as
``.npz`` fixtures next to this script.  The fixtures travel with the repo; the
reference does not.

Each case names the reference backend it ran: ``torch`` (recurrent,
``_torch.py``) or the ``parallel=True`` path (``_parallel.py``).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _run_case(name, T, B, D, H, *, parallel, dtype=torch.float32, a_value=None,
              a_uniform=None, seed=0, bias_spread=None, hx=False, batch_first=False,
              force_clamp=False):
    from headstartlstm import HeadStartLSTM  # the reference package

    torch.manual_seed(seed)
    m = HeadStartLSTM(D, H, batch_first=batch_first, backend="torch",
                      parallel=parallel).to(dtype)
    with torch.no_grad():
        if a_value is not None:
            m.a.fill_(a_value)
        if a_uniform is not None:
            m.a.uniform_(*a_uniform)
        if bias_spread is not None:
            # input- and forget-gate rows spread so log sigma(f) covers ~[-8, 0]
            m.bias_ih_l0[0:2 * H].uniform_(-bias_spread, bias_spread)
        if force_clamp:
            # drive some forget gates and some i*g products below eps=1e-6
            m.bias_ih_l0[H:H + H // 2] = -30.0
            m.bias_ih_l0[0:H // 3] = -30.0
    shape = (B, T, D) if batch_first else (T, B, D)
    x = torch.randn(*shape, dtype=dtype, requires_grad=True)
    G = torch.randn(*((B, T, H) if batch_first else (T, B, H)), dtype=dtype)
    h0 = c0 = None
    if hx:
        h0 = (0.5 * torch.randn(1, B, H, dtype=dtype))
        c0 = torch.rand(1, B, H, dtype=dtype)
        c0[..., : H // 4] = 0.0  # exercise clamp(c0, eps) in parallel mode
        out, (h_n, c_n) = m(x, (h0, c0))
    else:
        out, (h_n, c_n) = m(x)
    (out * G).sum().backward()

    rec = dict(T=T, B=B, D=D, H=H, parallel=int(parallel), batch_first=int(batch_first),
               hx=int(hx), dtype=str(dtype).replace("torch.", ""))
    for n, p in m.named_parameters():
        rec["p_" + n] = p.detach().numpy()
        rec["g_" + n] = (np.full(p.shape, np.nan) if p.grad is None
                         else p.grad.detach().numpy())
        rec["gnone_" + n] = int(p.grad is None)
    rec["x"] = x.detach().numpy()
    rec["G"] = G.numpy()
    if hx:
        rec["h0"] = h0.numpy()
        rec["c0"] = c0.numpy()
    rec["out"] = out.detach().numpy()
    rec["h_n"] = h_n.detach().numpy()
    rec["c_n"] = c_n.detach().numpy()
    rec["dx"] = x.grad.numpy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    print(f"{name}: T={T} B={B} D={D} H={H} parallel={parallel} dtype={dtype}")


CASES = [
    # recurrent, shapes of the reference's own tests (tests/test_cpp.py:55, :75)
    dict(name="rec_t10_b4_d16_h24_f32", T=10, B=4, D=16, H=24, parallel=False),
    dict(name="rec_t10_b4_d16_h24_f64", T=10, B=4, D=16, H=24, parallel=False,
         dtype=torch.float64),
    dict(name="rec_t8_b3_d8_h12_f32", T=8, B=3, D=8, H=12, parallel=False),
    # configs[0] of the benchmark (T=32,B=16,D=64,H=128, a=1e-4)
    dict(name="rec_cfg0_f32", T=32, B=16, D=64, H=128, parallel=False),
    # nonlinear regime (a ~ U(0, 0.5), as configs[3]) at a small shape
    dict(name="rec_anl_t16_b4_d32_h48_f32", T=16, B=4, D=32, H=48, parallel=False,
         a_uniform=(0.0, 0.5), seed=3),
    dict(name="rec_anl_t16_b4_d32_h48_f64", T=16, B=4, D=32, H=48, parallel=False,
         a_uniform=(0.0, 0.5), seed=3, dtype=torch.float64),
    # initial state given + batch_first (__init__.py:170-182, :230-231)
    dict(name="rec_hx_bf_t6_b5_d10_h20_f32", T=6, B=5, D=10, H=20, parallel=False,
         a_value=0.3, hx=True, batch_first=True, seed=5),
    # parallel, shapes of tests/test_parallel.py:47 and :84
    dict(name="par_t12_b3_d16_h24_f32", T=12, B=3, D=16, H=24, parallel=True, a_value=0.0),
    dict(name="par_t10_b3_d8_h12_f64", T=10, B=3, D=8, H=12, parallel=True, a_value=0.0,
         dtype=torch.float64),
    # parallel, configs[1] feature sizes on a short batch slice
    dict(name="par_t128_b2_d64_h64_f32", T=128, B=2, D=64, H=64, parallel=True, a_value=0.0,
         seed=1),
    # parallel, clamp active on f, i*g and c0
    dict(name="par_clamp_t20_b3_d8_h24_f32", T=20, B=3, D=8, H=24, parallel=True,
         a_value=0.0, force_clamp=True, hx=True, seed=7),
    dict(name="par_clamp_t20_b3_d8_h24_f64", T=20, B=3, D=8, H=24, parallel=True,
         a_value=0.0, force_clamp=True, hx=True, seed=7, dtype=torch.float64),
    # parallel, long sequence with forget spread (configs[4] distribution)
    dict(name="par_long_t2048_b1_d8_h16_f32", T=2048, B=1, D=8, H=16, parallel=True,
         a_value=0.0, bias_spread=8.0, seed=11),
    dict(name="par_long_t2048_b1_d8_h16_f64", T=2048, B=1, D=8, H=16, parallel=True,
         a_value=0.0, bias_spread=8.0, seed=11, dtype=torch.float64),
    # parallel, batch_first with nonzero a (a is ignored by parallel mode)
    dict(name="par_bf_t9_b4_d12_h16_f32", T=9, B=4, D=12, H=16, parallel=True,
         a_value=0.05, batch_first=True, seed=2),
]


def main():
    try:
        import headstartlstm  # noqa: F401
    except ImportError:
        sys.exit("set PYTHONPATH to the reference's src/ directory")
    torch.set_num_threads(1)
    for c in CASES:
        c = dict(c)
        _run_case(c.pop("name"), **c)


if __name__ == "__main__":
    main()
