"""Parallel (Heinsen-scan) mode with one long sequence split over time across
ranks: each rank holds a contiguous chunk of the time steps for every
sequence of the batch and runs the projection, the scan and the gradient
GEMMs on its chunk only.

The reference runs ``_log_parallel_scan`` (src/headstartlstm/_parallel.py:21-35)
on one device.  Its recurrence c_t = max(f_t,eps) c_{t-1} + max(i_t g_t,eps) is
affine in the carried state, so the ranks exchange only two [B, H] maps per
direction (``hs_scan_chunk_maps``):

* forward: chunk r maps the state entering it to its last state,
  c -> A_r c + C_r; with every rank's maps, rank r's entering state is
  c_in(r) = A_{r-1} c_in(r-1)' + C_{r-1} from c_in(0)' = max(c0, eps), and the
  rank runs the ordinary scan with c_in(r) as its c0;
* backward: chunk r maps the gradient arriving at its last state to the
  gradient it passes on, e -> A_r e + D_r, so the gradient entering rank r
  from the chunks after it is e_in(r) = A_{r+1} e_in(r+1) + D_{r+1} + dc_last_r,
  and the rank runs the ordinary scan backward with e_in(r) as its dc_n.

Parameter gradients stay per rank (each rank's chunk contributes a sum over
its steps); reduce them across ranks as for batch sharding
(``data_parallel.allreduce_grads``).  ``dc0`` reaches only rank 0.

The chunk steps are plain functions over device tensors so that one process
can drive several chunks in phases (tests on one GPU); ``SeqParallelFn``
chains them inside autograd with the exchange over ``torch.distributed``.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import _lib

EPS = 1e-6


# ---------------------------------------------------------------- composition
def compose_forward(A: Sequence[torch.Tensor], C: Sequence[torch.Tensor], c0: Optional[torch.Tensor],
                    eps: float = EPS) -> List[Optional[torch.Tensor]]:
    """Entering state of every chunk from all chunks' forward maps, in rank
    order.  Rank 0 gets ``c0`` as given (the scan clamps it); every later
    rank the state the chunks before it leave, always >= eps.  Ranks other
    than 0 do not hold c0: there rank 0's map comes folded (``fold_initial``)
    and c0 is passed as None."""
    R = len(A)
    out: List[Optional[torch.Tensor]] = [c0]
    c = torch.clamp(c0, min=eps) if c0 is not None else torch.full_like(A[0], eps)
    for r in range(R - 1):
        c = A[r] * c + C[r]
        out.append(c)
    return out


def fold_initial(A0: torch.Tensor, C0: torch.Tensor, c0: Optional[torch.Tensor], eps: float = EPS):
    """Rank 0's map with the sequence's initial state folded in (only rank 0
    holds c0): the constant map c -> A0 max(c0, eps) + C0, published as
    (0, A0 max(c0, eps) + C0) so that every rank composes the same carries."""
    c = torch.clamp(c0, min=eps) if c0 is not None else torch.full_like(A0, eps)
    return torch.zeros_like(A0), A0 * c + C0


def compose_backward(A: Sequence[torch.Tensor], D: Sequence[torch.Tensor],
                     dc_last: Sequence[Optional[torch.Tensor]]) -> List[Optional[torch.Tensor]]:
    """Gradient entering every chunk at its last state, from the chunks after
    it: e_in(R-1) = dc_last(R-1); e_in(r) = A(r+1) e_in(r+1) + D(r+1) + dc_last(r)."""
    R = len(A)
    out: List[Optional[torch.Tensor]] = [None] * R
    e = dc_last[R - 1]
    out[R - 1] = e
    for r in range(R - 2, -1, -1):
        nxt = D[r + 1] if e is None else A[r + 1] * e + D[r + 1]
        e = nxt if dc_last[r] is None else nxt + dc_last[r]
        out[r] = e
    return out


# ---------------------------------------------------------------- chunk steps
def _f32c(t):
    return None if t is None else (t if (t.dtype == torch.float32 and t.is_contiguous()) else t.float().contiguous())


def chunk_project(x, W_ih, b_ih):
    """z = x W_ih^T + b_ih for the chunk (x [Tr,B,D]) -> z [Tr,B,4H]."""
    T, B, D = x.shape
    N = W_ih.shape[0]
    dev = x.device
    z = torch.empty(T, B, N, device=dev)
    lib = _lib.load()
    ws = _lib.workspace(lib.hs_linear_workspace_bytes(T * B, N, D), dev)
    P = _lib.ptr
    _lib.call("hs_linear_forward", P(x), P(W_ih), P(b_ih), P(z), T * B, N, D, P(ws), ws.numel(),
              P(_lib.status_word(dev)), _lib.stream_ptr(dev))
    return z


def chunk_maps(z, c=None, dout=None, dh_last=None, backward=False, eps=EPS):
    """(A, C) of the chunk's forward, or (A, D) of its backward: [B,H] each."""
    T, B, H4 = z.shape
    H = H4 // 4
    A = torch.empty(B, H, device=z.device)
    CD = torch.empty(B, H, device=z.device)
    P = _lib.ptr
    _lib.call("hs_scan_chunk_maps", P(z), P(c), P(dout), P(dh_last), T, B, H, float(eps), P(A), P(CD),
              1 if backward else 0, _lib.stream_ptr(z.device))
    return A, CD


def chunk_scan_forward(z, c_in, eps=EPS):
    """The chunk's scan from entering state c_in (None = zeros): (out, c,
    h_last, c_last, kf)."""
    T, B, H4 = z.shape
    H = H4 // 4
    dev = z.device
    out = torch.empty(T, B, H, device=dev)
    c = torch.empty(T, B, H, device=dev)
    h_last = torch.empty(B, H, device=dev)
    c_last = torch.empty(B, H, device=dev)
    kf = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = _lib.workspace(lib.hs_scan_workspace_bytes(T, B, H), dev)
    P = _lib.ptr
    _lib.call("hs_scan_forward_kf", P(z), P(c_in), P(out), P(c), P(h_last), P(c_last), T, B, H, float(eps), P(ws),
              ws.numel(), P(kf), P(_lib.status_word(dev)), _lib.stream_ptr(dev))
    return out, c, h_last, c_last, kf


def chunk_backward(x, W_ih, z, c, c_in, dout, dh_last, e_in, kf, want_dx=True, want_dc0=False, eps=EPS):
    """The chunk's backward from the gradient e_in entering its last state:
    (dx, dW_ih, db_ih, dc_in).  z is overwritten (with dZ where the split
    handoff is not taken)."""
    T, B, D = x.shape
    H = c.shape[-1]
    dev = x.device
    dx = torch.empty(T, B, D, device=dev) if want_dx else None
    dW = torch.empty_like(W_ih)
    db = torch.empty(W_ih.shape[0], device=dev)
    dc0 = torch.empty(B, H, device=dev) if (want_dc0 and c_in is not None) else None
    lib = _lib.load()
    ws = _lib.workspace(lib.hs_parallel_workspace_bytes(T, B, D, H), dev,
                        min_bytes=lib.hs_scan_workspace_bytes(T, B, H))
    P = _lib.ptr
    _lib.call("hs_parallel_backward_kf", P(x), P(W_ih), P(z), P(c), P(c_in), P(dout), P(dh_last), P(e_in), P(dx),
              P(dW), P(db), P(dc0), T, B, D, H, float(eps), P(ws), ws.numel(), P(kf), P(_lib.status_word(dev)),
              _lib.stream_ptr(dev))
    return dx, dW, db, dc0


# ---------------------------------------------------------------- autograd
class SeqParallelFn(torch.autograd.Function):
    """One rank's chunk of a sequence split over time across the ranks of
    ``group``: inputs x [Tr,B,D] (this rank's steps), c0 [B,H] (used on rank
    0 only), W_ih, b_ih; outputs the chunk's out [Tr,B,H] and its last
    (h, c) (on the last rank, the module's h_n, c_n).  Both directions
    all-gather the chunk maps; parameter gradients are this rank's
    contribution."""

    @staticmethod
    def forward(ctx, x, c0, W_ih, b_ih, group=None, eps=EPS):
        import torch.distributed as dist

        x, W_ih, b_ih, c0 = _f32c(x), _f32c(W_ih), _f32c(b_ih), _f32c(c0)
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        z = chunk_project(x, W_ih, b_ih)
        A, C = chunk_maps(z, eps=eps)
        A_own = A
        if rank == 0:
            A, C = fold_initial(A, C, c0, eps)
        A_all = [torch.empty_like(A) for _ in range(world)]
        C_all = [torch.empty_like(C) for _ in range(world)]
        dist.all_gather(A_all, A, group=group)
        dist.all_gather(C_all, C, group=group)
        c_in = compose_forward(A_all, C_all, c0 if rank == 0 else None, eps)[rank]
        out, c, h_last, c_last, kf = chunk_scan_forward(z, c_in, eps)
        A_all[rank] = A_own
        ctx.save_for_backward(x, W_ih, z, c, c_in if c_in is not None else torch.empty(0, device=x.device), kf,
                              torch.stack(A_all))
        ctx.group, ctx.eps, ctx.rank, ctx.world = group, eps, rank, world
        ctx.has_c_in = c_in is not None
        return out, h_last, c_last

    @staticmethod
    def backward(ctx, dout, dh_last, dc_last):
        import torch.distributed as dist

        x, W_ih, z, c, c_in, kf, A_all = ctx.saved_tensors
        c_in = c_in if ctx.has_c_in else None
        group, eps, rank, world = ctx.group, ctx.eps, ctx.rank, ctx.world
        dev = x.device
        T, B, _ = x.shape
        H = c.shape[-1]
        dout = torch.zeros(T, B, H, device=dev) if dout is None else _f32c(dout)
        dh_last, dc_last = _f32c(dh_last), _f32c(dc_last)
        _, Dm = chunk_maps(z, c, dout, dh_last, backward=True, eps=eps)
        dcl = dc_last if dc_last is not None else torch.zeros(B, H, device=dev)
        D_all = [torch.empty_like(Dm) for _ in range(world)]
        L_all = [torch.empty_like(dcl) for _ in range(world)]
        dist.all_gather(D_all, Dm, group=group)
        dist.all_gather(L_all, dcl, group=group)
        e_in = compose_backward(list(A_all), D_all, L_all)[rank]
        dx, dW, db, dc0 = chunk_backward(x, W_ih, z, c, c_in, dout, dh_last, e_in, kf,
                                         want_dx=ctx.needs_input_grad[0],
                                         want_dc0=(rank == 0 and ctx.needs_input_grad[1]), eps=eps)
        return dx, dc0, dW, db, None, None


def headstartlstm_parallel_seqsharded(x_chunk, c0, W_ih, b_ih, group=None, eps: float = EPS):
    """Sequence-sharded parallel mode for this rank's chunk of time steps:
    ``(out_chunk, h_last, c_last)``; on the last rank (h_last, c_last) are
    the sequence's (h_n, c_n)."""
    return SeqParallelFn.apply(x_chunk, c0, W_ih, b_ih, group, eps)
