"""The recurrent path at H = 512 on clusters of 16 CTAs with a few sequences
per cluster (csrc/recurrent_cluster.cu, rcw_* kernels: each CTA's 256 KB
weight slice split between registers and shared memory; the forward
all-gathers h in distributed shared memory, the backward reduce-scatters
its dh partial sums), against the float64 oracle and against the FFMA
kernels (HS_REC_PATH=ffma), through the module API.

Shapes: configs[2] (T=256, B=32, D=256, H=512); batches that give every
sequence count per cluster from 1 to 8 on a device running 7 or 8 such
clusters at once (B = 5, 13, 20, 28, 40, 49, 56), with a partial last
cluster; batches beyond 8 sequences per cluster, run as a second wave of
clusters (B = 64, 100; HS_REC_PATH=cluster, not the default there); T=1 and T=2 (the shortest barrier sequences); a
non-zero initial state and gradients entering through h_n and c_n.  Bound:
1e-5 normwise, the recurrent-mode bound of every parity test.
"""

import os

import pytest

from test_gpu_recurrent_tc import TOL, _ours, _problem, _rel, _truth

pytestmark = pytest.mark.gpu

CASES = [
    (256, 32, 256, 512, 1e-4),
    (17, 5, 24, 512, 0.3),
    (9, 13, 16, 512, 0.5),
    (6, 20, 32, 512, None),
    (5, 28, 32, 512, 0.2),
    (7, 40, 16, 512, 0.4),
    (4, 49, 16, 512, None),
    (12, 56, 32, 512, 0.4),
    (5, 64, 16, 512, 0.3),
    (3, 100, 16, 512, None),
    (1, 3, 8, 512, 0.2),
    (2, 7, 8, 512, 0.2),
]


@pytest.mark.parametrize("T,B,D,H,a", CASES)
def test_wide_cluster_recurrence_matches_float64_and_ffma(T, B, D, H, a):
    from prlstm_b200 import _lib

    lib = _lib.load()
    if B == 32:  # configs[2]: the default path
        assert lib.hs_recurrent_path(B, H, 0) == 2 and lib.hs_recurrent_path(B, H, 1) == 2
    old = os.environ.get("HS_REC_PATH")
    os.environ["HS_REC_PATH"] = "cluster"
    try:
        assert lib.hs_recurrent_path(B, H, 0) == 2 and lib.hs_recurrent_path(B, H, 1) == 2
    finally:
        if old is None:
            os.environ.pop("HS_REC_PATH", None)
        else:
            os.environ["HS_REC_PATH"] = old
    prob = _problem(T, B, D, H, a, seed=T * 1000 + B * 10 + H + 11)
    truth = _truth(*prob)
    cl = _ours(*prob, path="cluster")
    ff = _ours(*prob, path="ffma")
    for k in truth:
        e = _rel(cl[k], truth[k])
        e2 = _rel(cl[k], ff[k])
        print(f"WIDE T={T} B={B} {k}: vs float64 {e:.2e}, vs FFMA {e2:.2e}")
        assert e <= TOL, f"{k}: wide cluster path vs float64 {e:.3e}"
        assert e2 <= TOL, f"{k}: wide cluster path vs FFMA path {e2:.3e}"
