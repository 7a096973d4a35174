"""The per-column scans with two hidden units per lane (the default) against
the one-unit kernels (HS_SCAN_UNITS=1): the same arithmetic in the same order
per unit, so every output must agree bit for bit: out, c, h_n, c_n, the
forward's kf bound, float32 dZ, dc0, db, the fp16 split of dZ with its
scale, and the bf16-storage scans.  Shapes cover H = 1024 (the benchmark's),
H not a multiple of 64 (a partial last pair column), ragged T, and c0,
dh_n, dc_n all present.  Each variant runs in its own child process (the
variable is read once per process)."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _run(units, path, T, B, H):
    env = dict(os.environ, HS_SCAN_UNITS=str(units), HS_SCAN_PATH="chain")
    env["PYTHONPATH"] = os.path.dirname(HERE) + os.pathsep + env.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, os.path.join(HERE, "scan_units_probe.py"), path, str(T), str(B), str(H)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.parametrize("T,B,H", [(1000, 32, 1024), (333, 24, 328), (64, 40, 96)])
def test_two_units_per_lane_equal_one(tmp_path, T, B, H):
    p1, p2 = str(tmp_path / "u1.pt"), str(tmp_path / "u2.pt")
    _run(1, p1, T, B, H)
    _run(2, p2, T, B, H)
    a, b = torch.load(p1), torch.load(p2)
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
