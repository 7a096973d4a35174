"""CPU oracle for the two HeadStartLSTM hot paths.  TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the arithmetic of the
reference implementation (m-j-tilley/prLSTM, package ``headstartlstm``).  It is
the checker the parity tests, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` compare the CUDA library against.  Nothing in the product
package ``prlstm_b200`` imports it, and the product never falls back to it.

Pinning: every function here is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py`` imports the
reference package and writes ``tests/golden/*.npz``); the not-gpu test
``tests/test_oracle_golden.py`` holds the oracle to those vectors.

Reference citations are ``path:line`` inside the reference project.

Recurrent path (``src/headstartlstm/_torch.py``):
  * ``rec_forward``  follows ``HeadStartLSTMTorchFn.forward``  (_torch.py:86-131)
  * ``rec_backward`` follows ``HeadStartLSTMTorchFn.backward`` (_torch.py:133-170)
  * the per-step cell math follows ``_cell_forward_step`` (_torch.py:27-36) and
    ``_cell_backward_step`` (_torch.py:39-53)

Parallel path (``src/headstartlstm/_parallel.py``):
  * ``par_forward`` follows ``headstartlstm_parallel`` (_parallel.py:38-74) and
    ``_log_parallel_scan`` (_parallel.py:21-35); gradients come from autograd
    through exactly those ops, as in the reference (_parallel.py:3-4).
  * ``par_forward_linear`` / ``par_backward_linear`` restate the same function
    as the clamped linear recurrence c_t = max(f_t,eps) c_{t-1} + max(i_t g_t,eps)
    with c_{-1} = max(c0,eps), and its hand-derived reverse-time gradient.  In
    float64 this is the "truth" the parallel-mode tolerances are judged against
    (the reference's float32 log-domain scan drifts from float64 at long T).
"""

from __future__ import annotations

import torch

EPS = 1e-6  # default clamp of _log_parallel_scan (_parallel.py:21, :38)


# --------------------------------------------------------------------------
# Recurrent path
# --------------------------------------------------------------------------
def a_expand(a: torch.Tensor, H: int) -> torch.Tensor:
    """Per-gate scale broadcast over the [4H] gate axis (_torch.py:91)."""
    return a.repeat_interleave(H)


def rec_forward(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a):
    """Recurrent forward (_torch.py:86-131).

    x [T,B,D], h0/c0 [B,H], W_ih [4H,D], W_hh [4H,H], b_* [4H], a [4].
    Returns (out [T,B,H], h_n [B,H], c_n [B,H], saved) where ``saved`` holds
    what the hand-written backward needs.
    """
    T, B, _ = x.shape
    H = h0.shape[-1]
    a_exp = a_expand(a, H)                                   # _torch.py:91
    W_hh_s = a_exp.unsqueeze(1) * W_hh                        # _torch.py:92
    b_hh_s = a_exp * b_hh                                     # _torch.py:93
    W_hh_T = W_hh_s.t().contiguous()                          # _torch.py:94
    Z = torch.nn.functional.linear(x, W_ih, b_ih)             # _torch.py:96

    h_save = x.new_zeros(T + 1, B, H)
    c_save = x.new_zeros(T + 1, B, H)
    acts = x.new_zeros(T, B, 4 * H)                           # i, f, g, o
    tanh_c = x.new_zeros(T, B, H)
    h_save[0] = h0
    c_save[0] = c0
    h, c = h0, c0
    for t in range(T):                                        # _torch.py:111-120
        gates = Z[t] + h @ W_hh_T + b_hh_s
        i_, f_, g_, o_ = gates.chunk(4, dim=1)                # _torch.py:28
        i_ = torch.sigmoid(i_)
        f_ = torch.sigmoid(f_)
        g_ = torch.sigmoid(g_)                                # sigmoid g (mod 1)
        o_ = torch.sigmoid(o_)
        c = f_ * c + i_ * g_                                  # _torch.py:33
        th = torch.tanh(c)
        h = o_ * th                                           # _torch.py:35
        h_save[t + 1] = h
        c_save[t + 1] = c
        acts[t] = torch.cat([i_, f_, g_, o_], dim=1)
        tanh_c[t] = th
    saved = dict(x=x, h_save=h_save, c_save=c_save, acts=acts, tanh_c=tanh_c,
                 W_ih=W_ih, W_hh=W_hh, b_hh=b_hh, a_exp=a_exp, W_hh_s=W_hh_s)
    return h_save[1:], h_save[T], c_save[T], saved


def rec_backward(saved, dout, dh_n=None, dc_n=None):
    """Hand-written BPTT (_torch.py:133-170).

    Returns (dx, dW_ih, dW_hh, db_ih, db_hh, da); like the reference no
    gradient is produced for h0 / c0 (_torch.py:170).
    """
    x = saved["x"]
    h_save, c_save = saved["h_save"], saved["c_save"]
    acts, tanh_c = saved["acts"], saved["tanh_c"]
    W_ih, W_hh, b_hh = saved["W_ih"], saved["W_hh"], saved["b_hh"]
    a_exp, W_hh_s = saved["a_exp"], saved["W_hh_s"]
    T, B, D = x.shape
    H = h_save.shape[-1]
    if dh_n is None:
        dh_n = x.new_zeros(B, H)
    if dc_n is None:
        dc_n = x.new_zeros(B, H)

    dG = x.new_zeros(T, B, 4 * H)
    dh = dh_n.clone()
    dc = dc_n.clone()
    for t in range(T - 1, -1, -1):                           # _torch.py:143-150
        dh = dh + dout[t]
        i_, f_, g_, o_ = acts[t].chunk(4, dim=1)
        th = tanh_c[t]
        do_act = dh * th                                      # _torch.py:41
        dc_tot = dc + dh * o_ * (1.0 - th * th)               # _torch.py:42
        df_act = dc_tot * c_save[t]
        dc = dc_tot * f_
        di_act = dc_tot * g_
        dg_act = dc_tot * i_
        dG[t] = torch.cat([di_act * i_ * (1.0 - i_),          # _torch.py:48-51
                           df_act * f_ * (1.0 - f_),
                           dg_act * g_ * (1.0 - g_),
                           do_act * o_ * (1.0 - o_)], dim=1)
        dh = dG[t] @ W_hh_s                                   # _torch.py:150

    dGf = dG.reshape(T * B, 4 * H)                            # _torch.py:153-162
    dW_hh_s = dGf.t() @ h_save[:-1].reshape(T * B, H)
    dW_ih = dGf.t() @ x.reshape(T * B, D)
    db = dGf.sum(dim=0)
    dx = (dGf @ W_ih).view(T, B, D)
    dW_hh = a_exp.unsqueeze(1) * dW_hh_s                      # _torch.py:165-168
    db_hh = a_exp * db
    da = ((W_hh * dW_hh_s).sum(dim=1) + b_hh * db).view(4, H).sum(dim=1)
    return dx, dW_ih, dW_hh, db.clone(), db_hh, da


# --------------------------------------------------------------------------
# Parallel (Heinsen) path
# --------------------------------------------------------------------------
def log_parallel_scan(f, c0, b, eps: float = EPS):
    """Heinsen log-domain scan over dim=1 of [B,T,H] (_parallel.py:21-35)."""
    log_f = torch.log(torch.clamp(f, min=eps))
    log_b = torch.log(torch.clamp(b, min=eps))
    log_c0 = torch.log(torch.clamp(c0, min=eps))
    a_star = torch.cumsum(log_f, dim=1)
    cats = torch.cat([log_c0, log_b - a_star], dim=1)
    tail = torch.logcumsumexp(cats, dim=1)[:, 1:]
    return torch.exp(a_star + tail)


def par_forward(x, c0, W_ih, b_ih, eps: float = EPS):
    """Parallel-mode forward exactly as the reference computes it
    (_parallel.py:52-74).  Differentiable through autograd, as the reference.
    Returns (out [T,B,H], h_n [B,H], c_n [B,H])."""
    gates = torch.nn.functional.linear(x, W_ih, b_ih)         # _parallel.py:56
    i_pre, f_pre, g_pre, o_pre = gates.chunk(4, dim=-1)
    i_act = torch.sigmoid(i_pre)
    f_act = torch.sigmoid(f_pre)
    g_act = torch.sigmoid(g_pre)
    o_act = torch.sigmoid(o_pre)
    b_act = i_act * g_act                                     # _parallel.py:63
    f_bt = f_act.transpose(0, 1).contiguous()                 # _parallel.py:66-68
    b_bt = b_act.transpose(0, 1).contiguous()
    c_bt = log_parallel_scan(f_bt, c0.unsqueeze(1), b_bt, eps=eps)
    c_seq = c_bt.transpose(0, 1).contiguous()                 # _parallel.py:71
    out = o_act * torch.tanh(c_seq)                           # _parallel.py:73
    return out, out[-1].contiguous(), c_seq[-1].contiguous()  # _parallel.py:74


def par_forward_linear(x, c0, W_ih, b_ih, eps: float = EPS):
    """The same function as ``par_forward`` written as the clamped linear
    recurrence (no log/exp round trip).  exp(a*_t + lcse_t) of
    _parallel.py:31-35 equals prod f' * (c0' + sum b'_s / prod_{r<=s} f'_r),
    which is this recurrence.  Returns (out, h_n, c_n, saved)."""
    T, B, _ = x.shape
    Z = torch.nn.functional.linear(x, W_ih, b_ih)
    i_, f_, g_, o_ = torch.sigmoid(Z).chunk(4, dim=-1)
    fp = torch.clamp(f_, min=eps)
    bp = torch.clamp(i_ * g_, min=eps)
    c_prev = torch.clamp(c0, min=eps)
    c = torch.empty_like(fp)
    for t in range(T):
        c_prev = fp[t] * c_prev + bp[t]
        c[t] = c_prev
    out = o_ * torch.tanh(c)
    saved = dict(x=x, Z=Z, c=c, c0=c0, W_ih=W_ih, eps=eps)
    return out, out[-1].clone(), c[-1].clone(), saved


def par_backward_linear(saved, dout, dh_n=None, dc_n=None):
    """Hand-derived reverse-time gradient of ``par_forward_linear``.

    Returns (dx, dW_ih, db_ih, dc0, dZ).  Clamp gradients pass where the
    clamped value is >= eps, matching torch.clamp's backward as used by
    _parallel.py:27-29.
    """
    x, Z, c, c0, W_ih, eps = (saved[k] for k in ("x", "Z", "c", "c0", "W_ih", "eps"))
    T, B, D = x.shape
    H = c.shape[-1]
    s = torch.sigmoid(Z)
    i_, f_, g_, o_ = s.chunk(4, dim=-1)
    fp = torch.clamp(f_, min=eps)
    b = i_ * g_
    th = torch.tanh(c)
    dout = dout.clone()
    if dh_n is not None:
        dout[-1] += dh_n
    dcd = dout * o_ * (1.0 - th * th)
    if dc_n is not None:
        dcd[-1] += dc_n
    c0p = torch.clamp(c0, min=eps)
    dc = torch.empty_like(c)
    e = torch.zeros_like(c0)
    for t in range(T - 1, -1, -1):
        dc[t] = dcd[t] + e
        e = fp[t] * dc[t]
    c_prev = torch.cat([c0p.unsqueeze(0), c[:-1]], dim=0)
    df = dc * c_prev * (f_ >= eps).to(c.dtype)
    db = dc * (b >= eps).to(c.dtype)
    do = dout * th
    dZ = torch.cat([db * g_ * i_ * (1 - i_), df * f_ * (1 - f_),
                    db * i_ * g_ * (1 - g_), do * o_ * (1 - o_)], dim=-1)
    dZf = dZ.reshape(T * B, 4 * H)
    dx = (dZf @ W_ih).view(T, B, D)
    dW_ih = dZf.t() @ x.reshape(T * B, D)
    db_ih = dZf.sum(0)
    dc0 = e * (c0 >= eps).to(c.dtype)
    return dx, dW_ih, db_ih, dc0, dZ


def par_linear_chunked(zchunk, T, c0, dout, dh_n=None, dc_n=None, eps: float = EPS, chunk: int = 512,
                       on_dz=None):
    """``par_forward_linear`` + ``par_backward_linear`` evaluated in chunks of
    time steps, so that no [T,B,4H] tensor is ever held: the checker for the
    benchmark's full sizes (T=16384, B=32, H=1024 is 17 GB of float64 Z),
    run on whatever device its inputs live on.

    ``zchunk(t0, t1)`` returns the gate pre-activations Z[t0:t1] ([n,B,4H]);
    it is called once per chunk forward and once backward.  ``on_dz(t0, t1,
    dZ)`` receives dZ[t0:t1] in reverse chunk order (to form dX and dW_ih).
    Returns dict(out [T,B,H], c [T,B,H], h_n, c_n, dc0, db (sum of dZ over
    t and b, [4H]))."""
    c_prev = torch.clamp(c0, min=eps)
    B, H = c0.shape
    out = c0.new_empty(T, B, H)
    c = c0.new_empty(T, B, H)
    for t0 in range(0, T, chunk):
        t1 = min(T, t0 + chunk)
        i_, f_, g_, o_ = torch.sigmoid(zchunk(t0, t1)).chunk(4, dim=-1)
        fp = torch.clamp(f_, min=eps)
        bp = torch.clamp(i_ * g_, min=eps)
        for t in range(t1 - t0):
            c_prev = fp[t] * c_prev + bp[t]
            c[t0 + t] = c_prev
        out[t0:t1] = o_ * torch.tanh(c[t0:t1])
    e = torch.zeros_like(c0)
    db = c0.new_zeros(4 * H)
    c0p = torch.clamp(c0, min=eps)
    starts = list(range(0, T, chunk))
    for t0 in reversed(starts):
        t1 = min(T, t0 + chunk)
        i_, f_, g_, o_ = torch.sigmoid(zchunk(t0, t1)).chunk(4, dim=-1)
        fp = torch.clamp(f_, min=eps)
        b = i_ * g_
        th = torch.tanh(c[t0:t1])
        dd = dout[t0:t1].clone()
        if dh_n is not None and t1 == T:
            dd[-1] += dh_n
        dcd = dd * o_ * (1.0 - th * th)
        if dc_n is not None and t1 == T:
            dcd[-1] += dc_n
        dc = torch.empty_like(dcd)
        for t in range(t1 - t0 - 1, -1, -1):
            dc[t] = dcd[t] + e
            e = fp[t] * dc[t]
        c_prev_c = torch.cat([(c0p if t0 == 0 else c[t0 - 1]).unsqueeze(0), c[t0:t1 - 1]], dim=0)
        df = dc * c_prev_c * (f_ >= eps).to(c.dtype)
        dbb = dc * (b >= eps).to(c.dtype)
        dZ = torch.cat([dbb * g_ * i_ * (1 - i_), df * f_ * (1 - f_),
                        dbb * i_ * g_ * (1 - g_), dd * th * o_ * (1 - o_)], dim=-1)
        db += dZ.sum(dim=(0, 1))
        if on_dz is not None:
            on_dz(t0, t1, dZ)
    dc0 = e * (c0 >= eps).to(c.dtype)
    return dict(out=out, c=c, h_n=out[-1].clone(), c_n=c[-1].clone(), dc0=dc0, db=db)


def par_chunk_maps(Z, c=None, dout=None, dh_last=None, backward=False, eps: float = EPS):
    """Affine maps of one chunk of time steps of the clamped linear
    recurrence (the checker of the sequence-sharded scan; _parallel.py:21-35
    restated as in ``par_forward_linear``).  Z [T,B,4H].  Forward: the chunk
    maps its entering state to its last state as c -> A c + C; returns (A, C)
    with A = prod max(f,eps) and C the last state from a zero carry.
    Backward: it maps the gradient arriving at its last state to the gradient
    leaving to the state before it as e -> A e + D; needs the chunk's states
    c and dout (dh_last added at the last step); returns (A, D)."""
    i_, f_, g_, o_ = torch.sigmoid(Z).chunk(4, dim=-1)
    fp = torch.clamp(f_, min=eps)
    T = Z.shape[0]
    A = torch.prod(fp, dim=0)
    if not backward:
        bp = torch.clamp(i_ * g_, min=eps)
        v = torch.zeros_like(A)
        for t in range(T):
            v = fp[t] * v + bp[t]
        return A, v
    d = dout.clone()
    if dh_last is not None:
        d[-1] += dh_last
    th = torch.tanh(c)
    dcd = d * o_ * (1.0 - th * th)
    v = torch.zeros_like(A)
    for t in range(T - 1, -1, -1):
        v = fp[t] * (dcd[t] + v)
    return A, v


# --------------------------------------------------------------------------
# Module-level helpers (HeadStartLSTM semantics, __init__.py:131-233)
# --------------------------------------------------------------------------
def init_params(D: int, H: int, a_init: float = 1e-4, generator=None, dtype=torch.float32):
    """Parameters in nn.LSTM order, drawn as reset_parameters does
    (__init__.py:147-152, :160-167): U(-1/sqrt(H), 1/sqrt(H)) on W_ih, W_hh,
    b_ih, b_hh in that order, then a = a_init."""
    stdv = 1.0 / (H ** 0.5)
    W_ih = torch.empty(4 * H, D, dtype=dtype).uniform_(-stdv, stdv, generator=generator)
    W_hh = torch.empty(4 * H, H, dtype=dtype).uniform_(-stdv, stdv, generator=generator)
    b_ih = torch.empty(4 * H, dtype=dtype).uniform_(-stdv, stdv, generator=generator)
    b_hh = torch.empty(4 * H, dtype=dtype).uniform_(-stdv, stdv, generator=generator)
    a = torch.full((4,), float(a_init), dtype=dtype)
    return W_ih, W_hh, b_ih, b_hh, a


def module_forward_backward(params, x, G, parallel: bool, hx=None, linear_truth=False):
    """One fwd + ``sum(out*G).backward()`` through the oracle, returning the
    outputs and every gradient the reference module would produce.

    ``params`` = (W_ih, W_hh, b_ih, b_hh, a).  Parallel mode yields None for
    W_hh, b_hh and a (_parallel.py:41-43 leaves them unused)."""
    W_ih, W_hh, b_ih, b_hh, a = params
    T, B, D = x.shape
    H = W_hh.shape[1]
    if hx is None:
        h0 = x.new_zeros(B, H)
        c0 = x.new_zeros(B, H)
    else:
        h0, c0 = hx
    if not parallel:
        out, h_n, c_n, saved = rec_forward(x, h0, c0, W_ih, W_hh, b_ih, b_hh, a)
        dx, dW_ih, dW_hh, db_ih, db_hh, da = rec_backward(saved, G)
        return dict(out=out, h_n=h_n, c_n=c_n, dx=dx, dW_ih=dW_ih, dW_hh=dW_hh,
                    db_ih=db_ih, db_hh=db_hh, da=da)
    if linear_truth:
        out, h_n, c_n, saved = par_forward_linear(x, c0, W_ih, b_ih)
        dx, dW_ih, db_ih, dc0, _ = par_backward_linear(saved, G)
        return dict(out=out, h_n=h_n, c_n=c_n, dx=dx, dW_ih=dW_ih, dW_hh=None,
                    db_ih=db_ih, db_hh=None, da=None, dc0=dc0)
    xg = x.detach().clone().requires_grad_(True)
    Wg = W_ih.detach().clone().requires_grad_(True)
    bg = b_ih.detach().clone().requires_grad_(True)
    out, h_n, c_n = par_forward(xg, c0, Wg, bg)
    (out * G).sum().backward()
    return dict(out=out.detach(), h_n=h_n.detach(), c_n=c_n.detach(), dx=xg.grad,
                dW_ih=Wg.grad, dW_hh=None, db_ih=bg.grad, db_hh=None, da=None)
