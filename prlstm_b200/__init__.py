"""prlstm_b200: B200-native (sm_100a) HeadStartLSTM.

Drop-in for ``headstartlstm.HeadStartLSTM`` (m-j-tilley/prLSTM,
``src/headstartlstm/__init__.py:99-233``): same constructor, parameter names
and order (``weight_ih_l0, weight_hh_l0, bias_ih_l0, bias_hh_l0, a``), same
initialisation, ``set_mode(parallel)``, ``batch_first``, ``hx`` handling and
return shapes.  The two hot paths run in ``libhsb200.so``:

* recurrent mode: input-projection GEMM, one persistent kernel for the T-step
  forward recurrence, one for the BPTT backward, then the gradient GEMMs;
* parallel mode: input-projection GEMM, a fused activation + chunked
  decoupled-look-back scan over T, and its reverse-time counterpart.

There is one implementation and no CPU fallback: tensors must live on a CUDA
device; ``backend`` and ``compile_cell`` are accepted for signature
compatibility and validated like the reference validates them.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _lib
from ._functions import EPS, headstartlstm_parallel, headstartlstm_recurrent
from ._lib import check_device_status, clear_device_status

__version__ = "0.1.0"

_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


class HeadStartLSTM(nn.Module):
    """LSTM with a sigmoid g-gate and a learnable per-gate recurrent scale
    ``a``; ``parallel=True`` drops the ``a * (W_hh h + b_hh)`` term and
    evaluates the cell state with the Heinsen scan.

    Parameters mirror the reference (``__init__.py:131-134``)."""

    _VALID_BACKENDS = ("auto", "torch", "cpp", "triton", "metal")

    def __init__(self, input_size: int, hidden_size: int, batch_first: bool = False,
                 a_init: float = 1e-4, backend: str = "auto", parallel: bool = False,
                 compile_cell: bool = False):
        super().__init__()
        assert backend in self._VALID_BACKENDS, (
            f"backend must be one of {self._VALID_BACKENDS}, got {backend!r}")
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.batch_first = batch_first
        self.a_init = a_init
        self.backend = backend
        self.parallel = parallel
        self.compile_cell = compile_cell
        # nn.LSTM names and layout, gate order [i, f, g, o] (__init__.py:147-152)
        self.weight_ih_l0 = nn.Parameter(torch.empty(4 * hidden_size, input_size))
        self.weight_hh_l0 = nn.Parameter(torch.empty(4 * hidden_size, hidden_size))
        self.bias_ih_l0 = nn.Parameter(torch.zeros(4 * hidden_size))
        self.bias_hh_l0 = nn.Parameter(torch.zeros(4 * hidden_size))
        self.a = nn.Parameter(torch.full((4,), float(a_init)))
        self.reset_parameters()

    def set_mode(self, parallel: bool):
        """Switch between recurrent (default) and parallel-scan mode."""
        self.parallel = parallel

    def reset_parameters(self):
        """nn.LSTM init, U(-1/sqrt(H), 1/sqrt(H)) on all four, then a = a_init
        (__init__.py:160-167)."""
        stdv = 1.0 / math.sqrt(self.hidden_size)
        for p in (self.weight_ih_l0, self.weight_hh_l0, self.bias_ih_l0, self.bias_hh_l0):
            nn.init.uniform_(p, -stdv, stdv)
        with torch.no_grad():
            self.a.fill_(self.a_init)

    def forward(self, x: torch.Tensor, hx=None):
        """``x`` [T, B, D] (or [B, T, D] with batch_first) -> ``(out, (h_n, c_n))``.

        float32 is the native precision.  bfloat16 and float16 modules and
        inputs are the reduced-precision variant: the kernels read the
        bf16-valued inputs and weights exactly (widened to float32), keep
        float32 accumulation and state, and the outputs come back in the
        input's dtype, as the reference returns them (its parameters, data and
        results share one dtype); parameter gradients arrive in the
        parameters' dtype.  float64 is refused: every kernel computes in
        float32, and silently returning float32-accurate results under a
        float64 dtype would misstate their precision."""
        if x.dim() != 3:
            raise RuntimeError("input must be [T, B, input_size]")
        if x.dtype not in _DTYPES:
            raise TypeError(f"prlstm_b200 computes in float32; got input dtype {x.dtype} "
                            "(use float32, bfloat16 or float16)")
        out_dtype = x.dtype
        if self.batch_first:
            x = x.transpose(0, 1).contiguous()
        T, B, D = x.shape
        if D != self.input_size:
            raise RuntimeError(f"input_size mismatch: expected {self.input_size}, got {D}")
        if hx is None:
            h0 = x.new_zeros(B, self.hidden_size)
            c0 = x.new_zeros(B, self.hidden_size)
        else:
            h0, c0 = hx
            if h0.dim() == 3:
                h0 = h0.squeeze(0)
            if c0.dim() == 3:
                c0 = c0.squeeze(0)
            if h0.dim() != 2 or c0.dim() != 2:
                raise RuntimeError("h0, c0 must be [B, hidden_size]")
        if self.parallel:
            output, h_n, c_n = headstartlstm_parallel(
                x, h0, c0, self.weight_ih_l0, self.weight_hh_l0,
                self.bias_ih_l0, self.bias_hh_l0, self.a)
        else:
            output, h_n, c_n = headstartlstm_recurrent(
                x, h0, c0, self.weight_ih_l0, self.weight_hh_l0,
                self.bias_ih_l0, self.bias_hh_l0, self.a)
        if out_dtype != torch.float32:
            output, h_n, c_n = output.to(out_dtype), h_n.to(out_dtype), c_n.to(out_dtype)
        if self.batch_first:
            output = output.transpose(0, 1).contiguous()
        return output, (h_n.unsqueeze(0), c_n.unsqueeze(0))


def library_path() -> str:
    return _lib.LIB_PATH


__all__ = ["HeadStartLSTM", "headstartlstm_recurrent", "headstartlstm_parallel",
           "check_device_status", "clear_device_status", "library_path", "EPS", "__version__"]
