"""autograd.Functions over the C ABI: the recurrent path and the parallel
(Heinsen) path.  Host code only allocates tensors and calls the library.

Reference counterparts:
  * ``RecurrentFn`` <- HeadStartLSTMTorchFn / HeadStartLSTMTritonFn
    (src/headstartlstm/_torch.py:78-176, _triton.py:327-470): same functional
    signature ``(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a) -> (out, h_n, c_n)``,
    same gradient outputs, including ``None`` for h0 and c0 (_torch.py:170).
  * ``ParallelFn`` <- headstartlstm_parallel (src/headstartlstm/_parallel.py:38-74):
    W_hh, b_hh, a and h0 are not inputs of the computation, so their
    gradients stay None exactly as with the reference's traced autograd.
"""

from __future__ import annotations

import torch

from . import _lib

EPS = 1e-6  # _parallel.py:21, :38


def _f32c(t):
    return t if (t.dtype == torch.float32 and t.is_contiguous()) else t.float().contiguous()


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("prlstm_b200 runs on CUDA devices (B200, sm_100a) only; "
                               f"got a tensor on {t.device}")


class RecurrentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, h0, c0, W_ih, W_hh, b_ih, b_hh, a):
        _check_cuda(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a)
        T, B, D = x.shape
        H = W_hh.shape[1]
        dev = x.device
        # a bf16 module: the step product in bf16 where it runs on the tensor cores
        bf = x.dtype == torch.bfloat16 and W_hh.dtype == torch.bfloat16
        x, h0, c0 = _f32c(x), _f32c(h0), _f32c(c0)
        W_ih, W_hh, b_ih, b_hh, a = (_f32c(t) for t in (W_ih, W_hh, b_ih, b_hh, a))
        _lib.poll(dev)
        h_save = torch.empty(T + 1, B, H, device=dev, dtype=torch.float32)
        c_save = torch.empty(T + 1, B, H, device=dev, dtype=torch.float32)
        acts = torch.empty(T, B, 4 * H, device=dev, dtype=torch.float32)
        lib = _lib.load()
        nws = lib.hs_recurrent_workspace_bytes(T, B, D, H)
        if nws == 0:
            raise RuntimeError(f"recurrent path: unsupported shape T={T} B={B} D={D} H={H}")
        ws = _lib.workspace(nws, dev)
        P = _lib.ptr
        _lib.call("hs_recurrent_forward_bf16" if bf else "hs_recurrent_forward", P(x), P(h0), P(c0), P(W_ih),
                  P(W_hh), P(b_ih), P(b_hh), P(a), P(h_save), P(c_save), P(acts), T, B, D, H, P(ws), ws.numel(),
                  P(_lib.status_word(dev)), _lib.stream_ptr(dev))
        ctx.save_for_backward(x, W_ih, W_hh, b_hh, a, h_save, c_save, acts)
        ctx.shape = (T, B, D, H)
        ctx.bf = bf
        ctx.consumed = False
        return h_save[1:], h_save[T], c_save[T]

    @staticmethod
    def backward(ctx, dout, dh_n, dc_n):
        if ctx.consumed:
            raise RuntimeError("Trying to backward through a prlstm_b200 recurrent graph a "
                               "second time: its saved activations were consumed")
        ctx.consumed = True
        x, W_ih, W_hh, b_hh, a, h_save, c_save, acts = ctx.saved_tensors
        T, B, D, H = ctx.shape
        dev = x.device
        dout = torch.zeros(T, B, H, device=dev) if dout is None else _f32c(dout)
        dh_n = None if dh_n is None else _f32c(dh_n)
        dc_n = None if dc_n is None else _f32c(dc_n)
        want_dx = ctx.needs_input_grad[0]
        dx = torch.empty(T, B, D, device=dev) if want_dx else None
        dW_ih = torch.empty_like(W_ih)
        dW_hh = torch.empty_like(W_hh)
        db_ih = torch.empty(4 * H, device=dev)
        db_hh = torch.empty(4 * H, device=dev)
        da = torch.empty(4, device=dev)
        lib = _lib.load()
        ws = _lib.workspace(lib.hs_recurrent_workspace_bytes(T, B, D, H), dev)
        P = _lib.ptr
        _lib.call("hs_recurrent_backward_bf16" if ctx.bf else "hs_recurrent_backward", P(x), P(W_ih), P(W_hh),
                  P(b_hh), P(a), P(h_save),
                  P(c_save), P(acts), P(dout), P(dh_n), P(dc_n), P(dx), P(dW_ih), P(dW_hh),
                  P(db_ih), P(db_hh), P(da), T, B, D, H, P(ws), ws.numel(),
                  P(_lib.status_word(dev)), _lib.stream_ptr(dev))
        _lib.note_launch(dev)
        return dx, None, None, dW_ih, dW_hh, db_ih, db_hh, da


def _bf16c(t):
    return t if (t.dtype == torch.bfloat16 and t.is_contiguous()) else t.to(torch.bfloat16).contiguous()


def _bf16_path(x, W_ih):
    """A bf16 module whose shape the bf16 path takes
    (hs_parallel_bf16_supported: D and H multiples of 8, a shape the
    per-column scan takes): its products run as one bf16 tensor-core MMA per
    k-step and its saved activations are stored in bf16, instead of widening
    everything to float32."""
    if x.dtype != torch.bfloat16 or W_ih.dtype != torch.bfloat16 or x.dim() != 3:
        return False
    T, B, D = x.shape
    H = W_ih.shape[0] // 4
    return (_lib.load().hs_parallel_bf16_supported(T, B, D, H) == 1
            and x.data_ptr() % 16 == 0 and W_ih.data_ptr() % 16 == 0)


class ParallelFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, c0, W_ih, b_ih, eps=EPS):
        _check_cuda(x, c0, W_ih, b_ih)
        T, B, D = x.shape
        H = W_ih.shape[0] // 4
        dev = x.device
        if _bf16_path(x, W_ih):
            return ParallelFn._forward_bf16(ctx, x.contiguous(), c0, W_ih.contiguous(), _f32c(b_ih), eps)
        ctx.bf16 = False
        x, W_ih, b_ih = _f32c(x), _f32c(W_ih), _f32c(b_ih)
        c0 = None if c0 is None else _f32c(c0)
        _lib.poll(dev)
        z = torch.empty(T, B, 4 * H, device=dev)
        out = torch.empty(T, B, H, device=dev)
        c = torch.empty(T, B, H, device=dev)
        h_n = torch.empty(B, H, device=dev)
        c_n = torch.empty(B, H, device=dev)
        lib = _lib.load()
        ws = _lib.workspace(lib.hs_parallel_workspace_bytes(T, B, D, H), dev,
                            min_bytes=lib.hs_scan_workspace_bytes(T, B, H))
        P = _lib.ptr
        # kf: the forward's max of c_{t-1} f'(1-f'), which lets the backward
        # hand dZ to the gradient GEMMs as its fp16 split
        kf = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.call("hs_parallel_forward_kf", P(x), P(c0), P(W_ih), P(b_ih), P(z), P(out), P(c),
                  P(h_n), P(c_n), T, B, D, H, float(eps), P(ws), ws.numel(), P(kf),
                  P(_lib.status_word(dev)), _lib.stream_ptr(dev))
        ctx.save_for_backward(x, c0, W_ih, z, c, kf)
        ctx.shape = (T, B, D, H)
        ctx.eps = float(eps)
        ctx.consumed = False
        return out, h_n, c_n

    @staticmethod
    def _forward_bf16(ctx, x, c0, W_ih, b_ih, eps):
        """bf16 storage: z, out, c (and, in the backward, dout, dZ, dx) are
        bf16; c0, h_n, c_n and the parameter gradients float32."""
        T, B, D = x.shape
        H = W_ih.shape[0] // 4
        dev = x.device
        c0 = None if c0 is None else _f32c(c0)
        _lib.poll(dev)
        bf = torch.bfloat16
        z = torch.empty(T, B, 4 * H, device=dev, dtype=bf)
        out = torch.empty(T, B, H, device=dev, dtype=bf)
        c = torch.empty(T, B, H, device=dev, dtype=bf)
        h_n = torch.empty(B, H, device=dev)
        c_n = torch.empty(B, H, device=dev)
        lib = _lib.load()
        ws = _lib.workspace(lib.hs_parallel_bf16_workspace_bytes(T, B, D, H), dev)
        P = _lib.ptr
        _lib.call("hs_parallel_forward_bf16", P(x), P(c0), P(W_ih), P(b_ih), P(z), P(out), P(c), P(h_n), P(c_n),
                  T, B, D, H, float(eps), P(ws), ws.numel(), P(_lib.status_word(dev)), _lib.stream_ptr(dev))
        ctx.save_for_backward(x, c0, W_ih, z, c, None)
        ctx.shape = (T, B, D, H)
        ctx.eps = float(eps)
        ctx.consumed = False
        ctx.bf16 = True
        return out, h_n, c_n

    @staticmethod
    def backward(ctx, dout, dh_n, dc_n):
        if ctx.consumed:
            raise RuntimeError("Trying to backward through a prlstm_b200 parallel graph a "
                               "second time: its saved activations were consumed")
        ctx.consumed = True
        x, c0, W_ih, z, c, kf = ctx.saved_tensors
        T, B, D, H = ctx.shape
        dev = x.device
        if ctx.bf16:
            return ParallelFn._backward_bf16(ctx, x, c0, W_ih, z, c, dout, dh_n, dc_n)
        dout = torch.zeros(T, B, H, device=dev) if dout is None else _f32c(dout)
        dh_n = None if dh_n is None else _f32c(dh_n)
        dc_n = None if dc_n is None else _f32c(dc_n)
        dx = torch.empty(T, B, D, device=dev) if ctx.needs_input_grad[0] else None
        dc0 = torch.empty(B, H, device=dev) if (c0 is not None and ctx.needs_input_grad[1]) else None
        dW_ih = torch.empty(W_ih.shape, device=dev)
        db_ih = torch.empty(4 * H, device=dev)
        lib = _lib.load()
        P = _lib.ptr
        ws = _lib.workspace(lib.hs_parallel_workspace_bytes(T, B, D, H), dev,
                            min_bytes=lib.hs_scan_workspace_bytes(T, B, H))
        _lib.call("hs_parallel_backward_kf", P(x), P(W_ih), P(z), P(c), P(c0), P(dout), P(dh_n),
                  P(dc_n), P(dx), P(dW_ih), P(db_ih), P(dc0), T, B, D, H, ctx.eps, P(ws),
                  ws.numel(), P(kf), P(_lib.status_word(dev)), _lib.stream_ptr(dev))
        _lib.note_launch(dev)
        return dx, dc0, dW_ih, db_ih, None

    @staticmethod
    def _backward_bf16(ctx, x, c0, W_ih, z, c, dout, dh_n, dc_n):
        T, B, D, H = ctx.shape
        dev = x.device
        bf = torch.bfloat16
        dout = torch.zeros(T, B, H, device=dev, dtype=bf) if dout is None else _bf16c(dout)
        dh_n = None if dh_n is None else _f32c(dh_n)
        dc_n = None if dc_n is None else _f32c(dc_n)
        dx = torch.empty(T, B, D, device=dev, dtype=bf) if ctx.needs_input_grad[0] else None
        dc0 = torch.empty(B, H, device=dev) if (c0 is not None and ctx.needs_input_grad[1]) else None
        dW_ih = torch.empty(W_ih.shape, device=dev)
        db_ih = torch.empty(4 * H, device=dev)
        lib = _lib.load()
        P = _lib.ptr
        ws = _lib.workspace(lib.hs_parallel_bf16_workspace_bytes(T, B, D, H), dev)
        _lib.call("hs_parallel_backward_bf16", P(x), P(W_ih), P(z), P(c), P(c0), P(dout), P(dh_n), P(dc_n),
                  P(dx), P(dW_ih), P(db_ih), P(dc0), T, B, D, H, ctx.eps, P(ws), ws.numel(),
                  P(_lib.status_word(dev)), _lib.stream_ptr(dev))
        _lib.note_launch(dev)
        return dx, dc0, dW_ih, db_ih, None


def headstartlstm_recurrent(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a):
    """Functional recurrent path: ``(out [T,B,H], h_n [B,H], c_n [B,H])``."""
    return RecurrentFn.apply(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a)


def headstartlstm_parallel(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a, eps: float = EPS):
    """Functional parallel path with the reference's signature
    (_parallel.py:38); W_hh, b_hh, a and h0 are accepted and unused."""
    del h0, W_hh, b_hh, a
    return ParallelFn.apply(x, c0, W_ih, b_ih, eps)
