"""Shared helpers for the parity tests: golden fixtures, seeded inputs and
normwise error metrics.  Test infrastructure only."""

from __future__ import annotations

import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PARAM_NAMES = ("weight_ih_l0", "weight_hh_l0", "bias_ih_l0", "bias_hh_l0", "a")


def golden_names(prefix=""):
    return sorted(os.path.basename(p)[:-4]
                  for p in glob.glob(os.path.join(GOLDEN_DIR, prefix + "*.npz")))


def load_golden(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    return {k: z[k] for k in z.files}


def case_tensors(g, dtype=None):
    """Inputs of a golden case as torch tensors in [T,B,*] layout."""
    dt = dtype or (torch.float64 if str(g["dtype"]) == "float64" else torch.float32)
    params = tuple(torch.from_numpy(g["p_" + n]).to(dt) for n in PARAM_NAMES)
    x = torch.from_numpy(g["x"]).to(dt)
    G = torch.from_numpy(g["G"]).to(dt)
    if int(g["batch_first"]):
        x = x.transpose(0, 1).contiguous()
        G = G.transpose(0, 1).contiguous()
    hx = None
    if int(g["hx"]):
        hx = (torch.from_numpy(g["h0"]).to(dt)[0], torch.from_numpy(g["c0"]).to(dt)[0])
    return params, x, G, hx


def golden_expect(g):
    """Expected outputs/grads of a golden case in [T,B,*] layout."""
    bf = int(g["batch_first"])
    exp = {}
    for k in ("out", "dx"):
        v = torch.from_numpy(g[k])
        exp[k] = v.transpose(0, 1).contiguous() if bf else v
    exp["h_n"] = torch.from_numpy(g["h_n"])[0]
    exp["c_n"] = torch.from_numpy(g["c_n"])[0]
    names = dict(weight_ih_l0="dW_ih", weight_hh_l0="dW_hh", bias_ih_l0="db_ih",
                 bias_hh_l0="db_hh", a="da")
    for n, k in names.items():
        exp[k] = None if int(g["gnone_" + n]) else torch.from_numpy(g["g_" + n])
    return exp


def rel_err(got, ref):
    """Normwise relative error max|got-ref| / max|ref| (float64)."""
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    den = ref.abs().max().item()
    num = (got - ref).abs().max().item()
    return num / den if den > 0 else num


def make_inputs(T, B, D, H, *, a=1e-4, a_uniform=None, bias_spread=None, seed=0,
                dtype=torch.float32):
    """Seeded synthetic inputs in the order the benchmark configs define:
    params drawn as reset_parameters does, then a, then x ~ N(0,1), then
    G ~ N(0,1).  Returns (params, x, G) on the CPU."""
    from oracle.hs_oracle import init_params

    gen = torch.Generator().manual_seed(seed)
    W_ih, W_hh, b_ih, b_hh, a_t = init_params(D, H, a_init=a, generator=gen, dtype=dtype)
    if a_uniform is not None:
        a_t.uniform_(*a_uniform, generator=gen)
    if bias_spread is not None:
        b_ih[0:2 * H].uniform_(-bias_spread, bias_spread, generator=gen)
    x = torch.randn(T, B, D, generator=gen, dtype=dtype)
    G = torch.randn(T, B, H, generator=gen, dtype=dtype)
    return (W_ih, W_hh, b_ih, b_hh, a_t), x, G
