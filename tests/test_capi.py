"""The C ABI: the library loads, exports exactly what include/*.h declares,
and its host-side argument checks reject bad calls before any launch.  No
kernel runs here (CPU only)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "headstartlstm_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"HS_API\s+[\w\s\*]+?\b(hs_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from prlstm_b200 import _lib

    if not os.path.exists(_lib.LIB_PATH):
        from prlstm_b200 import build

        build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = _declared()
    for n in ("hs_parallel_forward", "hs_parallel_backward", "hs_recurrent_forward",
              "hs_recurrent_backward", "hs_scan_forward", "hs_scan_backward",
              "hs_linear_forward", "hs_linear_dgrad", "hs_linear_wgrad"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for n in _declared():
        assert hasattr(lib, n), f"{n} declared in the header but not exported"


def test_binding_covers_header():
    from prlstm_b200 import _lib

    assert sorted(_lib.SIGNATURES) == _declared()


def test_status_strings(lib):
    assert lib.hs_abi_version() == 1
    assert lib.hs_status_string(0) == b"ok"
    assert b"timed out" in lib.hs_status_string(5)
    assert lib.hs_status_string(99) == b"unknown status"


def test_workspace_queries(lib):
    assert lib.hs_linear_workspace_bytes(8192, 2048, 512) > 0      # small output: split-K scratch
    assert lib.hs_linear_workspace_bytes(0, 2048, 512) == 0
    assert lib.hs_parallel_workspace_bytes(128, 32, 256, 256) >= lib.hs_scan_workspace_bytes(128, 32, 256)
    assert lib.hs_scan_workspace_bytes(0, 1, 1) == 0
    n1 = lib.hs_scan_workspace_bytes(128, 32, 256)
    n2 = lib.hs_scan_workspace_bytes(16384, 32, 1024)
    assert 0 < n1 < n2
    assert lib.hs_recurrent_workspace_bytes(256, 32, 256, 512) > 4 * 2048 * 512
    assert lib.hs_recurrent_workspace_bytes(0, 32, 256, 512) == 0


@pytest.mark.parametrize("T,B,H", [(0, 2, 8), (4, 0, 8), (4, 2, -1)])
def test_scan_rejects_bad_shapes_before_launch(lib, T, B, H):
    P = ctypes.c_void_p
    rc = lib.hs_scan_forward(P(16), P(16), P(16), P(16), None, None, T, B, H, 1e-6, P(256), 1 << 20,
                             P(16), None)
    assert rc == 1
    assert b"positive" in lib.hs_last_error_message()


def test_recurrent_rejects_null_pointers(lib):
    rc = lib.hs_recurrent_forward(*([None] * 11), 4, 2, 3, 8, None, 0, None, None)
    assert rc == 1


def test_gemm_rejects_negative_extent(lib):
    P = ctypes.c_void_p
    assert lib.hs_linear_forward(P(16), P(16), None, P(16), -1, 4, 4, None, 0, None, None) == 1


def test_split_handoff_workspace_queries(lib):
    """Sizes of the split-handoff path: a split buffer holds hi and lo fp16
    rows padded to 8 columns; the parallel workspace covers the layout the
    backward uses for the handoff (dZ split + scale word + scan or GEMM
    scratch); non-positive extents give 0."""
    assert lib.hs_split_bytes(4, 8) == 256  # 4 * 4 * 8 bytes rounded up to 256
    assert lib.hs_split_bytes(1000, 6) >= 4 * 1000 * 8
    assert lib.hs_split_bytes(0, 8) == 0 and lib.hs_split_bytes(4, 0) == 0
    T, B, D, H = 16384, 32, 512, 1024
    M, N = T * B, 4 * H
    dz_split = lib.hs_split_bytes(M, N)
    need = dz_split + 256 + max(lib.hs_scan_split_workspace_bytes(T, B, H),
                                lib.hs_linear_presplit_workspace_bytes(M, N, D))
    assert lib.hs_parallel_workspace_bytes(T, B, D, H) >= need
    assert lib.hs_scan_split_workspace_bytes(T, B, H) > lib.hs_scan_workspace_bytes(T, B, H)
    assert lib.hs_scan_split_workspace_bytes(0, B, H) == 0
    assert lib.hs_linear_presplit_workspace_bytes(M, N, 0) == 0


def test_split_entry_points_reject_bad_arguments(lib):
    P = ctypes.c_void_p
    assert lib.hs_split(None, 4, 8, P(256), P(256), None) == 1
    assert lib.hs_split(P(256), 4, 8, P(8), P(256), None) == 1  # destination not 16-byte aligned
    assert lib.hs_linear_backward_presplit(None, P(256), P(256), None, None, P(256), P(256), P(256), 64, 64, 64,
                                           0, P(256), 1 << 20, P(16), None) == 1
    assert lib.hs_scan_forward_kf(P(16), None, P(16), P(16), None, None, 4, 2, 8, 1e-6, P(256), 1 << 20, None,
                                  P(16), None) == 1
