"""The recurrent path's cluster kernels (csrc/recurrent_cluster.cu: one
thread-block cluster per batch group of 32 sequences, the weights resident,
the state exchanged between the cluster's CTAs in distributed shared memory)
against the float64 oracle and against the FFMA kernels (HS_REC_PATH=ffma),
through the module API.

Shapes cover configs[0] (T=32, B=16, D=64, H=128), H=64 and H=32 (fewer
units per CTA), several batch groups side by side with a partial last one
(B=40, 70), T=1 and T=2 (the shortest barrier sequences), a non-zero
initial state and gradients entering through h_n and c_n, and both cluster
sizes (16 CTAs, and 8 with HS_RCL_CLUSTER=8).  Bound: 1e-5 normwise, the
recurrent-mode bound of every parity test.
"""

import os
import subprocess
import sys

import pytest
import torch

from test_gpu_recurrent_tc import TOL, _ours, _problem, _rel, _truth

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    (32, 16, 64, 128, 1e-4),
    (17, 5, 24, 128, 0.3),
    (9, 40, 16, 64, 0.5),
    (1, 3, 8, 128, 0.2),
    (2, 7, 8, 128, 0.2),
    (12, 70, 32, 32, None),
]


@pytest.mark.parametrize("T,B,D,H,a", CASES)
def test_cluster_recurrence_matches_float64_and_ffma(T, B, D, H, a):
    from prlstm_b200 import _lib

    lib = _lib.load()
    assert lib.hs_recurrent_path(B, H, 0) == 2 and lib.hs_recurrent_path(B, H, 1) == 2
    prob = _problem(T, B, D, H, a, seed=T * 1000 + B * 10 + H + 7)
    truth = _truth(*prob)
    cl = _ours(*prob, path="cluster")
    ff = _ours(*prob, path="ffma")
    for k in truth:
        e = _rel(cl[k], truth[k])
        assert e <= TOL, f"{k}: cluster path vs float64 {e:.3e}"
        e2 = _rel(cl[k], ff[k])
        assert e2 <= TOL, f"{k}: cluster path vs FFMA path {e2:.3e}"


def test_cluster_of_eight_ctas():
    """The same at configs[0]'s shape on clusters of 8 CTAs (16 units per
    CTA, two cells per thread), in a child process (the size is chosen once
    per process)."""
    code = (
        "import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "from test_gpu_recurrent_cluster import _check\n"
        "_check(32, 16, 64, 128, 1e-4)\n" % (HERE, os.path.dirname(HERE)))
    env = dict(os.environ, HS_RCL_CLUSTER="8")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr


def _check(T, B, D, H, a):
    prob = _problem(T, B, D, H, a, seed=99)
    truth = _truth(*prob)
    cl = _ours(*prob, path="cluster")
    for k in truth:
        e = _rel(cl[k], truth[k])
        assert e <= TOL, f"{k}: cluster path (8 CTAs) vs float64 {e:.3e}"
