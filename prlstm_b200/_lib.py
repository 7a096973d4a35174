"""ctypes binding of ``libhsb200.so`` (the C ABI in include/headstartlstm_b200.h).

Loading is lazy and strict: a missing library is an ImportError-style
RuntimeError, never a silent fallback.  Every call checks the returned status
and raises ``RuntimeError`` with the library's message, mirroring the
``TORCH_CHECK`` errors of the reference's C++ entry point
(``src/headstartlstm/_csrc/lstm_cell.cpp:38-43``).
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
# HS_B200_LIB names another build of the library (e.g. one with different
# compile-time tile knobs); by default the in-tree build is loaded.
LIB_PATH = os.environ.get("HS_B200_LIB") or os.path.join(HERE, "libhsb200.so")

HS_OK = 0
HS_ERR_DEVICE_TIMEOUT = 5

_c_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/headstartlstm_b200.h
SIGNATURES = {
    "hs_abi_version": (_i32, []),
    "hs_status_string": (ctypes.c_char_p, [_i32]),
    "hs_last_error_message": (ctypes.c_char_p, []),
    "hs_read_status": (_i32, [_c_p, _c_p, _c_p]),
    "hs_clear_status": (_i32, [_c_p, _c_p]),
    "hs_selftest_bounded_wait": (_i32, [_c_p, _c_p, ctypes.c_uint64, _c_p]),
    "hs_selftest_activations": (_i32, [_c_p, _i32, _f32, _c_p]),
    "hs_linear_workspace_bytes": (_sz, [_i64] * 3),
    "hs_linear_forward": (_i32, [_c_p] * 4 + [_i64] * 3 + [_c_p, _sz, _c_p, _c_p]),
    "hs_linear_dgrad": (_i32, [_c_p] * 3 + [_i64] * 3 + [_c_p, _sz, _c_p, _c_p]),
    "hs_linear_wgrad": (_i32, [_c_p] * 3 + [_i64] * 3 + [_i32, _c_p, _sz, _c_p, _c_p]),
    "hs_linear_backward": (_i32, [_c_p] * 5 + [_i64] * 3 + [_i32, _c_p, _sz, _c_p, _c_p]),
    "hs_linear_backward_absmax": (_i32, [_c_p] * 5 + [_i64] * 3 + [_i32, _c_p, _c_p, _sz, _c_p, _c_p]),
    "hs_split_bytes": (_sz, [_i64] * 2),
    "hs_linear_presplit_workspace_bytes": (_sz, [_i64] * 3),
    "hs_split": (_i32, [_c_p, _i64, _i64, _c_p, _c_p, _c_p]),
    "hs_linear_forward_presplit": (_i32, [_c_p] * 5 + [_i64] * 3 + [_c_p, _sz, _c_p, _c_p]),
    "hs_linear_backward_presplit": (_i32, [_c_p] * 8 + [_i64] * 3 + [_i32, _c_p, _sz, _c_p, _c_p]),
    "hs_colsum": (_i32, [_c_p, _c_p, _i64, _i64, _i32, _c_p]),
    "hs_scan_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "hs_parallel_workspace_bytes": (_sz, [_i64] * 4),
    "hs_scan_forward": (_i32, [_c_p] * 6 + [_i64] * 3 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_scan_forward_noalloc": (_i32, [_c_p] * 6 + [_i64] * 3 + [_f32, _c_p, _c_p]),
    "hs_scan_noalloc_status": (_i32, [_c_p, _c_p]),
    "hs_scan_backward": (_i32, [_c_p] * 9 + [_i64] * 3 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_scan_backward_absmax": (_i32, [_c_p] * 9 + [_i64] * 3 + [_f32, _c_p, _sz, _c_p, _c_p, _c_p]),
    "hs_scan_forward_kf": (_i32, [_c_p] * 6 + [_i64] * 3 + [_f32, _c_p, _sz, _c_p, _c_p, _c_p]),
    "hs_projection_scan_workspace_bytes": (_sz, [_i64] * 4),
    "hs_projection_scan_supported": (_i32, [_i64] * 4),
    "hs_projection_scan_forward": (_i32, [_c_p] * 10 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p, _c_p]),
    "hs_scan_uses_column_kernels": (_i32, [_i64] * 3),
    "hs_scan_wave_sequences": (_i64, [_i64]),
    "hs_scan_split_workspace_bytes": (_sz, [_i64] * 3),
    "hs_scan_backward_split": (_i32, [_c_p] * 11 + [_i64] * 3 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_scan_chunk_maps": (_i32, [_c_p] * 4 + [_i64] * 3 + [_f32, _c_p, _c_p, _i32, _c_p]),
    "hs_parallel_forward": (_i32, [_c_p] * 9 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_parallel_backward": (_i32, [_c_p] * 12 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_parallel_forward_kf": (_i32, [_c_p] * 9 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p, _c_p]),
    "hs_parallel_backward_kf": (_i32, [_c_p] * 12 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p, _c_p]),
    "hs_linear_bf16_workspace_bytes": (_sz, [_i64] * 3),
    "hs_linear_forward_bf16": (_i32, [_c_p] * 4 + [_i64] * 3 + [_c_p, _sz, _c_p, _c_p]),
    "hs_linear_backward_bf16": (_i32, [_c_p] * 5 + [_i64] * 3 + [_i32, _c_p, _sz, _c_p, _c_p]),
    "hs_scan_forward_bf16": (_i32, [_c_p] * 6 + [_i64] * 3 + [_f32, _c_p, _c_p]),
    "hs_scan_bf16_workspace_bytes": (_sz, [_i64] * 3),
    "hs_scan_backward_bf16": (_i32, [_c_p] * 9 + [_i64] * 3 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_parallel_bf16_supported": (_i32, [_i64] * 4),
    "hs_parallel_bf16_workspace_bytes": (_sz, [_i64] * 4),
    "hs_parallel_forward_bf16": (_i32, [_c_p] * 9 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_parallel_backward_bf16": (_i32, [_c_p] * 12 + [_i64] * 4 + [_f32, _c_p, _sz, _c_p, _c_p]),
    "hs_recurrent_workspace_bytes": (_sz, [_i64] * 4),
    "hs_recurrent_uses_tensor_cores": (_i32, [_i64, _i64, _i32]),
    "hs_recurrent_path": (_i32, [_i64, _i64, _i32]),
    "hs_recurrent_forward": (_i32, [_c_p] * 11 + [_i64] * 4 + [_c_p, _sz, _c_p, _c_p]),
    "hs_recurrent_backward": (_i32, [_c_p] * 17 + [_i64] * 4 + [_c_p, _sz, _c_p, _c_p]),
    "hs_recurrent_forward_bf16": (_i32, [_c_p] * 11 + [_i64] * 4 + [_c_p, _sz, _c_p, _c_p]),
    "hs_recurrent_backward_bf16": (_i32, [_c_p] * 17 + [_i64] * 4 + [_c_p, _sz, _c_p, _c_p]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load the library (once) and declare every exported signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"prlstm_b200: CUDA library {path} is missing; build it with "
                "`python -m prlstm_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def ptr(t):
    """Device pointer of a tensor (or None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def call(name: str, *args):
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != HS_OK:
        msg = lib.hs_last_error_message().decode(errors="replace")
        what = lib.hs_status_string(rc).decode()
        raise RuntimeError(f"{name}: {what}: {msg}")
    return rc


# ---------------------------------------------------------------- status word
_status = {}
_pending = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device sticky device-status int the kernels report bounded-wait
    failures into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def note_launch(device: torch.device):
    """Queue an asynchronous read-back of the status word; the value is
    checked (without a sync) the next time the library is called.  Skipped
    while the stream is being captured into a CUDA graph (an event query is
    not allowed there): a graphed step reports through check_device_status."""
    if torch.cuda.is_current_stream_capturing():
        return
    idx = device.index if device.index is not None else torch.cuda.current_device()
    poll(device)
    host = torch.empty(1, dtype=torch.int32, pin_memory=True)
    host.copy_(status_word(device), non_blocking=True)
    ev = torch.cuda.Event()
    ev.record()
    _pending[idx] = (host, ev)


def _raise_status(code: int):
    lib = load()
    raise RuntimeError(f"prlstm_b200 device status: {lib.hs_status_string(code).decode()} "
                       f"(code {code}); clear it with prlstm_b200.clear_device_status()")


def poll(device: torch.device):
    if torch.cuda.is_current_stream_capturing():
        return
    idx = device.index if device.index is not None else torch.cuda.current_device()
    item = _pending.get(idx)
    if item is None:
        return
    host, ev = item
    if ev.query():
        del _pending[idx]
        if int(host.item()) != HS_OK:
            _raise_status(int(host.item()))


def check_device_status(device=None):
    """Synchronously read the device status word; raise if a kernel gave up."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_int(-1)
    call("hs_read_status", ptr(status_word(device)), ctypes.byref(out), stream_ptr(device))
    if out.value != HS_OK:
        _raise_status(out.value)


def clear_device_status(device=None):
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    call("hs_clear_status", ptr(status_word(device)), stream_ptr(device))
    idx = device.index if device.index is not None else torch.cuda.current_device()
    _pending.pop(idx, None)


def workspace(nbytes: int, device, min_bytes: int = 0) -> torch.Tensor:
    """Caller-owned scratch (the library never allocates); 256-byte aligned
    by the caching allocator.  If the full size does not fit in device
    memory and ``min_bytes`` is given, the smaller size is allocated instead:
    the library then takes the paths that need less scratch (same results,
    slower GEMMs)."""
    try:
        return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
    except torch.cuda.OutOfMemoryError:
        if not min_bytes or min_bytes >= nbytes:
            raise
        torch.cuda.empty_cache()
        return torch.empty(max(int(min_bytes), 256), dtype=torch.uint8, device=device)
