"""Benchmark of the HeadStartLSTM hot path on B200 (one JSON line on rank 0).

Default workload (``--config cfg4``): configs[4] of the benchmark, the
long-sequence parallel (Heinsen-scan) training step, T=16384, B=256 (global),
D=512, H=1024, a=0, fp32, fwd + backward of sum(out*G).  The batch is split
across ranks (strong scaling: the global batch is fixed) and each rank runs
its share as micro-batches sized to one wave of the scan kernels' columns
(micro_batches: 4 x 37 + 3 x 36 on one GPU, 32 at 2-8 GPUs) with gradients
accumulated, then one NCCL all-reduce SUM of the weight gradients.  Inputs
are seeded synthetic data with the config's distributions (no dataset
exists).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfgX]
    python bench.py --impl reference ...   # CPU reference arm (the stock reference package)

``value``: tokens/s (T*B per step, whole job) with inputs resident in HBM,
timed with CUDA events on the launching stream, max over ranks.
``e2e``: the same step through the public module API with the step's inputs
copied from pinned host memory and the loss read back, inside the timed
region.  ``roofline``: the dominant kernel of the step, from CUDA events
around each library call inside the timed region.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

CONFIGS = {
    "cfg0": dict(T=32, B=16, D=64, H=128, mode="recurrent", a=1e-4),
    "cfg1": dict(T=128, B=32, D=256, H=256, mode="parallel", a=0.0),
    "cfg2": dict(T=256, B=32, D=256, H=512, mode="recurrent", a=1e-4),
    "cfg3": dict(T=64, B=32, D=1024, H=2048, mode="recurrent", a_uniform=(0.0, 0.5)),
    "cfg4": dict(T=16384, B=256, D=512, H=1024, mode="parallel", a=0.0, bias_spread=8.0),
}
MICRO_BATCH = 32


def _peaks():
    """(HBM GB/s, bf16 TF/s burst, bf16 TF/s sustained, kind).  Kernels timed
    inside the multi-second training step are held to the sustained figure
    (the GEMM loop under the power cap); the burst one is reported beside."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        burst = float(d["bf16_tflops"])
        return float(d["hbm_gbs"]), burst, float(d.get("bf16_tflops_sustained", burst)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def _peaks_raw():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(p)) if os.path.exists(p) else {}


def _traffic(kernel: str, units: float):
    """DRAM bytes per launch of `kernel`, scaled from the committed ncu summary
    (profiles/traffic.json: bytes per element at a captured size)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p))
    e = d.get(kernel)
    if not e:
        return None
    return e["bytes_per_unit"] * units


# ------------------------------------------------------------------ inputs
def make_params(cfg, dtype=torch.float32):
    from oracle.hs_oracle import init_params  # parameter draw only (as reset_parameters)

    gen = torch.Generator().manual_seed(0)
    D, H = cfg["D"], cfg["H"]
    W_ih, W_hh, b_ih, b_hh, a = init_params(D, H, a_init=cfg.get("a", 1e-4), generator=gen,
                                            dtype=dtype)
    if "a_uniform" in cfg:
        a.uniform_(*cfg["a_uniform"], generator=gen)
    if "bias_spread" in cfg:
        s = cfg["bias_spread"]
        b_ih[0:2 * H].uniform_(-s, s, generator=gen)
    return W_ih, W_hh, b_ih, b_hh, a


def micro_batches(B_local, H):
    """Micro-batch sizes for a rank's B_local sequences: near-equal calls of
    at most the number of sequences whose per-column scans fill the GPU in
    one wave of columns (hs_scan_wave_sequences: 37 at H = 1024 on 148 SMs,
    so configs[4]'s 256 sequences run as 4 x 37 + 3 x 36); MICRO_BATCH
    where the library cannot say."""
    from prlstm_b200 import _lib
    cap = int(_lib.load().hs_scan_wave_sequences(H)) or MICRO_BATCH
    cap = max(1, min(cap, B_local))
    n = -(-B_local // cap)
    base, rem = divmod(B_local, n)
    return [base + 1] * rem + [base] * (n - rem)


def make_data(cfg, B_local, rank, dev, mb=None):
    """x ~ N(0,1) [T,B,D] and G ~ N(0,1) [T,B,H] for this rank.  With `mb`
    (a size, or a list of sizes summing to B_local), returned as lists of
    contiguous micro-batches."""
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    if mb is None:
        x = torch.randn(cfg["T"], B_local, cfg["D"], device=dev, generator=g)
        G = torch.randn(cfg["T"], B_local, cfg["H"], device=dev, generator=g)
        return x, G
    sizes = [mb] * (B_local // mb) if isinstance(mb, int) else list(mb)
    xs = [torch.randn(cfg["T"], n, cfg["D"], device=dev, generator=g) for n in sizes]
    Gs = [torch.randn(cfg["T"], n, cfg["H"], device=dev, generator=g) for n in sizes]
    return xs, Gs


# ------------------------------------------------------------------ clocks
def _gpu_id(dev):
    """nvidia-smi selector of this device (its UUID), robust to CUDA_VISIBLE_DEVICES."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index or 0)

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ our arm
class ParallelStep:
    """One parallel-mode training step on this rank through the C ABI, with
    CUDA events around every library call (the kernel breakdown)."""

    def __init__(self, cfg, params, B_local, dev, fused=None):
        from prlstm_b200 import _lib

        self.L = _lib
        self.cfg = cfg
        self.dev = dev
        T, D, H = cfg["T"], cfg["D"], cfg["H"]
        # micro-batches (micro_batches: one wave of scan columns each); the
        # buffers are sized for the largest, each call takes a contiguous
        # view of its own size
        self.sizes = micro_batches(B_local, H)
        self.mb = max(self.sizes)
        self.nmb = len(self.sizes)
        self.mb_mean = B_local / self.nmb
        self.W_ih = params[0].to(dev).contiguous()
        self.b_ih = params[2].to(dev).contiguous()
        mb = self.mb
        self.z = torch.empty(T, mb, 4 * H, device=dev)
        self.out = torch.empty(T, mb, H, device=dev)
        self.c = torch.empty(T, mb, H, device=dev)
        self.c0 = torch.zeros(mb, H, device=dev)
        self.h_n = torch.empty(mb, H, device=dev)
        self.c_n = torch.empty(mb, H, device=dev)
        self.dx = torch.empty(T, mb, D, device=dev)
        self.dW = torch.zeros(4 * H, D, device=dev)
        self.db = torch.zeros(4 * H, device=dev)
        self.dW_mb = torch.empty(4 * H, D, device=dev)
        self.db_mb = torch.empty(4 * H, device=dev)
        lib = _lib.load()
        M = T * mb
        # the projection and the scan forward as one kernel where the library
        # takes it for this micro-batch (HS_PROJ_SCAN=0 times the two calls),
        # or where the caller asks for it (fused=True)
        self.fused = bool(lib.hs_projection_scan_supported(T, mb, D, H)) if fused is None else fused
        self.ws = _lib.workspace(max(lib.hs_parallel_workspace_bytes(T, mb, D, H),
                                     lib.hs_scan_split_workspace_bytes(T, mb, H),
                                     lib.hs_linear_presplit_workspace_bytes(M, 4 * H, D),
                                     lib.hs_projection_scan_workspace_bytes(T, mb, D, H)), dev)
        self.status = _lib.status_word(dev)
        # dZ travels from the scan backward to the gradient GEMMs as its fp16
        # split (hi, lo) with one scale word; the forward's max c feeds the
        # split scale's bound
        self.dz_split = torch.empty(lib.hs_split_bytes(M, 4 * H), dtype=torch.uint8, device=dev)
        # x's split serves both the projection and the weight gradient
        self.x_split = torch.empty(lib.hs_split_bytes(M, D), dtype=torch.uint8, device=dev)
        self.words = torch.zeros(64, dtype=torch.int32, device=dev)  # [0] Kf, [16] dZ scale, [32] x scale
        self.names = (("proj_scan", "scan_bwd", "linear_bwd") if self.fused else
                      ("proj_gemm", "scan_fwd", "scan_bwd", "linear_bwd"))
        self.ms = {n: 0.0 for n in self.names}
        self.launches = 0

    @staticmethod
    def _part(t, m):
        """The first m sequences' worth of a [T, mb, ...] buffer, as a
        contiguous [T, m, ...] tensor (the same storage)."""
        n = t.numel() // t.shape[1] * m
        return t.view(-1)[:n].view(t.shape[0], m, *t.shape[2:])

    def run(self, x, G, record=False):
        L, P = self.L, self.L.ptr
        T, D, H = self.cfg["T"], self.cfg["D"], self.cfg["H"]
        st = L.stream_ptr(self.dev)
        evs = []
        for i, mb in enumerate(self.sizes):
            M = T * mb
            xs, Gs = x[i], G[i]
            z, out, c, dx = (self._part(t, mb) for t in (self.z, self.out, self.c, self.dx))
            c0, h_n, c_n = self.c0[:mb], self.h_n[:mb], self.c_n[:mb]
            e = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.names) + 1)] if record else None
            if record:
                e[0].record()
            x_scale = P(self.words[32:])
            cmax, dz_scale = P(self.words[0:]), P(self.words[16:])
            L.call("hs_split", P(xs), M, D, P(self.x_split), x_scale, st)
            if self.fused:
                # Z, out, c, h_n, c_n and the backward's bound in one kernel
                L.call("hs_projection_scan_forward", P(self.x_split), x_scale, P(self.W_ih), P(self.b_ih),
                       P(c0), P(z), P(out), P(c), P(h_n), P(c_n), T, mb, D, H,
                       1e-6, P(self.ws), self.ws.numel(), cmax, P(self.status), st)
            else:
                L.call("hs_linear_forward_presplit", P(self.x_split), x_scale, P(self.W_ih), P(self.b_ih),
                       P(z), M, 4 * H, D, P(self.ws), self.ws.numel(), P(self.status), st)
                if record:
                    e[1].record()
                L.call("hs_scan_forward_kf", P(z), P(c0), P(out), P(c), P(h_n),
                       P(c_n), T, mb, H, 1e-6, P(self.ws), self.ws.numel(), cmax, P(self.status), st)
            if record:
                e[len(self.names) - 2].record()
            # the scan backward writes dZ as the fp16 split the GEMMs read
            L.call("hs_scan_backward_split", P(z), P(c), P(c0), P(Gs), None, None, cmax,
                   P(self.dz_split), dz_scale, None, P(self.db_mb), T, mb, H, 1e-6, P(self.ws),
                   self.ws.numel(), P(self.status), st)
            if record:
                e[len(self.names) - 1].record()
            # dX and dW_ih (accumulated over micro-batches) in one call
            L.call("hs_linear_backward_presplit", P(self.dz_split), dz_scale, None, P(self.x_split), x_scale,
                   P(self.W_ih), P(dx), P(self.dW), M, 4 * H, D, 1 if i else 0, P(self.ws), self.ws.numel(),
                   P(self.status), st)
            if record:
                e[len(self.names)].record()
            self.db.add_(self.db_mb) if i else self.db.copy_(self.db_mb)
            # projection: absmax + split of x and of W_ih, GEMM; scan forward
            # 1 (fused: the same splits and one kernel for both); scan
            # backward: bound (3), scan, rowsum, check, conditional re-run and
            # split (2, return at once unless needed); backward GEMMs: absmax +
            # split of W_ih, 2 GEMMs, split-K reduce (x's split is the
            # projection's)
            self.launches += self.launches_per_mb()
            if record:
                evs.append(e)
        return evs

    def launches_per_mb(self):
        return (5 if self.fused else 5 + 1) + 8 + 5

    def per_step_launches(self):
        return self.launches_per_mb() * self.nmb

    def collect(self, evs):
        for e in evs:
            for k, n in enumerate(self.names):
                self.ms[n] += e[k].elapsed_time(e[k + 1])

    def units(self, kernel):
        """Work of one average call (launch counts are per micro-batch)."""
        T, D, H, mb = self.cfg["T"], self.cfg["D"], self.cfg["H"], self.mb_mean
        if kernel in ("scan_fwd", "scan_bwd"):
            return T * mb * H
        nprod = 2 if kernel == "linear_bwd" else 1  # dX and dW_ih; proj_scan: the projection's flops
        return nprod * 2.0 * T * mb * 4 * H * D  # flops of the call


class PrefetchedInputs:
    """The step's inputs for a graphed end-to-end leg: each step's
    host-to-device copies run on a copy stream into a device staging buffer,
    issued right after the previous step's replay was launched (so that they
    overlap it), and are moved into the graph's static input buffers (a
    device-to-device copy) before the step's own replay.  A step that finds
    no copy in flight (the first of the warm-up or of the timed region: the
    step before it does not prefetch across that boundary) issues its own, so
    that every timed step copies its inputs from pinned host memory inside
    the timed region."""

    def __init__(self, host, static, dev):
        self.host, self.static = host, static
        self.stage = [torch.empty_like(t) for t in static]
        self.cs = torch.cuda.Stream(dev)
        self.free = torch.cuda.Event()
        self.free.record()
        self.ready = None

    def issue(self):
        with torch.cuda.stream(self.cs):
            self.cs.wait_event(self.free)  # the staging buffer was read by the last move
            for st, h in zip(self.stage, self.host):
                st.copy_(h, non_blocking=True)
            self.ready = torch.cuda.Event()
            self.ready.record()

    def consume(self):
        if self.ready is None:
            self.issue()
        torch.cuda.current_stream().wait_event(self.ready)
        self.ready = None
        for t, st in zip(self.static, self.stage):
            t.copy_(st, non_blocking=True)
        self.free = torch.cuda.Event()
        self.free.record()


def use_graph(args, cfg, B_local, world):
    """Whether the parallel step is captured in a CUDA graph: on one GPU (no
    collective inside the step), for steps of at most 2^16 tokens per rank,
    whose kernels take a few tens of microseconds; --graph
    on/off overrides.  Returns True or None."""
    mode = getattr(args, "graph", "auto")
    if world > 1 or mode == "off":
        return None
    if mode == "on" or cfg["T"] * B_local <= (1 << 16):
        return True
    return None


def cublas_refs(cfg, mb, dev):
    """cuBLAS TF32 and FP32 throughput (TF/s) on one micro-batch's three GEMM
    shapes: projection [TB,D]x[D,4H], dgrad [TB,4H]x[4H,D], wgrad
    [4H,TB]x[TB,D]."""
    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    M, N, K = T * mb, 4 * H, D
    shapes = {"proj_gemm": (M, K, N), "dgrad": (M, N, K), "wgrad": (N, M, K)}
    out = {}
    old = torch.backends.cuda.matmul.allow_tf32
    try:
        for name, (m, k, n) in shapes.items():
            a = torch.randn(m, k, device=dev)
            b = torch.randn(k, n, device=dev)
            r = {}
            for tf32, key in ((True, "cublas_tf32_tflops"), (False, "cublas_fp32_tflops")):
                torch.backends.cuda.matmul.allow_tf32 = tf32
                c = a @ b
                torch.cuda.synchronize(dev)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(3):
                    c = a @ b
                e1.record()
                torch.cuda.synchronize(dev)
                r[key] = 2.0 * m * n * k * 3 / (e0.elapsed_time(e1) / 1e3) / 1e12
            out[name] = r
            del a, b, c
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
        torch.cuda.empty_cache()
    return out


def run_ours(args, cfg, rank, world, dev):
    import torch.distributed as dist

    import prlstm_b200
    from prlstm_b200 import _lib
    from prlstm_b200.data_parallel import GradAllReducer

    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    B_global = cfg["B"]
    if cfg["mode"] == "parallel":
        assert B_global % world == 0
        B_local = B_global // world
    else:
        B_local = B_global  # recurrent configs: every rank runs the full config (replicas)
    params = make_params(cfg)
    if cfg["mode"] == "parallel":
        x, G = make_data(cfg, B_local, rank, dev, mb=micro_batches(B_local, H))
    else:
        x, G = make_data(cfg, B_local, rank, dev)
    peak_hbm, peak_tf_burst, peak_tf, peak_kind = _peaks()

    # one SUM all-reduce of the packed gradients per step (batch sharding:
    # summed shard gradients equal the full-batch gradients)
    reducer = GradAllReducer()

    def allreduce(tensors):
        if world > 1:
            reducer(tensors)

    # launch without waiting (NCCL runs on its own stream): finish() later
    allreduce.start = lambda tensors: reducer.start(tensors) if world > 1 else None

    def sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    result = {}
    if cfg["mode"] == "parallel":
        step = ParallelStep(cfg, params, B_local, dev)
        for _ in range(args.warmup):
            step.run(x, G)
            allreduce([step.dW, step.db])
        sync()
        _lib.check_device_status(dev)
        step.ms = {n: 0.0 for n in step.names}
        step.launches = 0
        graph = use_graph(args, cfg, B_local, world)
        if graph is not None:
            # Launch-bound step (kernels of a few tens of us): the whole step
            # is captured once in a CUDA graph and replayed, so the timed
            # region holds every kernel of every step without the per-call
            # host work.  The per-kernel breakdown comes from an ungraphed
            # pass after it (device times do not depend on how the kernels
            # were launched).
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                step.run(x, G)
            torch.cuda.current_stream(dev).wait_stream(side)
            with torch.cuda.graph(graph):
                step.run(x, G)
            graph.replay()
            sync()
            _lib.check_device_status(dev)
            step.launches = 0
        clocks = ClockSampler(_gpu_id(dev))
        clocks.start()
        sync()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        allev = []
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
                step.launches += step.per_step_launches()
            else:
                allev.extend(step.run(x, G, record=True))
            allreduce([step.dW, step.db])
        t1.record()
        sync()
        ck = clocks.stop()
        ms = t0.elapsed_time(t1)
        if graph is not None:
            launches = step.launches
            for _ in range(args.steps):
                allev.extend(step.run(x, G, record=True))
            sync()
            step.launches = launches
            result["launch"] = "cuda_graph (one capture of the step, replayed every step)"
            del graph
            dev_ms = sum(e[0].elapsed_time(e[-1]) for e in allev) / args.steps
            if ms / args.steps < 0.5 * dev_ms:
                raise RuntimeError(f"graphed step {ms / args.steps:.4f} ms is shorter than half the ungraphed "
                                   f"device time {dev_ms:.4f} ms: the capture missed the step's kernels")
        step.collect(allev)
        _lib.check_device_status(dev)
        ms = max_over_ranks(ms)
        tokens = T * B_global * args.steps
        result["value"] = tokens / (ms / 1e3)
        result["ms_per_step"] = ms / args.steps
        result["gpu_launches"] = step.launches
        result["clocks"] = ck
        nl = args.steps * step.nmb
        kern = {}
        for n in step.names:
            avg_ms = step.ms[n] / nl
            if n.startswith("scan"):
                per_unit = 24.0 if n == "scan_fwd" else 40.0
                ach = per_unit * step.units(n) / (avg_ms / 1e3) / 1e9
                kern[n] = {"bound": "hbm", "avg_ms": avg_ms, "achieved": ach, "unit": "GB/s",
                           "frac": ach / peak_hbm, "share": step.ms[n] / max(1e-9, sum(step.ms.values()))}
            else:
                ach = step.units(n) / (avg_ms / 1e3) / 1e12
                kern[n] = {"bound": "tensor", "avg_ms": avg_ms, "achieved": ach, "unit": "TFLOP/s",
                           "frac": ach / peak_tf, "frac_of_burst_peak": ach / peak_tf_burst,
                           "share": step.ms[n] / max(1e-9, sum(step.ms.values()))}
        dom = max(kern, key=lambda n: kern[n]["share"])
        d = kern[dom]
        units = step.units(dom)
        per = {"scan_fwd": 24.0, "scan_bwd": 40.0}.get(dom)
        result["roofline"] = {
            "kernel": dom, "bound": d["bound"], "achieved": round(d["achieved"], 2),
            "peak": peak_hbm if d["bound"] == "hbm" else peak_tf, "unit": d["unit"],
            "frac": round(d["frac"], 4), "peak_kind": peak_kind,
            "peak_basis": ("hbm_gbs (copy)" if d["bound"] == "hbm" else
                           "bf16_tflops_sustained: the kernel is timed inside a multi-second step"),
            "traffic": _traffic(dom, units),
            "algorithmic_per_launch": (per * units) if per else units,
        }
        # Library references for the GEMMs, timed here on the same shapes:
        # cuBLAS TF32 (one tf32 product, ~1e-3 accurate; three of them bound
        # an fp32-accurate 3xTF32 GEMM) and cuBLAS FP32 (the same accuracy as
        # ours).  Measured after the timed region, outside it.
        if not args.no_cublas_ref:
            refs = cublas_refs(cfg, step.mb, dev)
            # the backward call holds both products: its references are their
            # time-weighted combination (equal FLOPs each)
            rb = {k: 2.0 / (1.0 / refs["dgrad"][k] + 1.0 / refs["wgrad"][k]) for k in refs["dgrad"]}
            refs = {("proj_scan" if step.fused else "proj_gemm"): refs["proj_gemm"], "linear_bwd": rb}
            for n, r in refs.items():
                kern[n].update(r)
                kern[n]["speedup_vs_cublas_fp32"] = kern[n]["achieved"] / r["cublas_fp32_tflops"]
        # The GEMMs are float32-accurate through three 16-bit tensor-core
        # products per fp32 product (fp16 hi/lo split), so their ceiling is a
        # third of the measured 16-bit dense peak.
        for n in kern:
            if kern[n]["bound"] == "tensor":
                kern[n]["f16x3_ceiling_tflops"] = peak_tf / 3.0
                kern[n]["frac_of_f16x3_ceiling"] = kern[n]["achieved"] / (peak_tf / 3.0)
        if dom in kern and kern[dom]["bound"] == "tensor":
            result["roofline"]["peak_burst"] = peak_tf_burst
            result["roofline"]["frac_of_burst_peak"] = round(kern[dom]["frac_of_burst_peak"], 4)
            result["roofline"]["f16x3_ceiling"] = round(peak_tf / 3.0, 1)
            result["roofline"]["frac_of_f16x3_ceiling"] = round(kern[dom]["frac_of_f16x3_ceiling"], 4)
        if step.fused:
            # the fused kernel's DRAM bytes per unit (t, b, h): x's split
            # (4 D / H B), Z written (16 B), out and c written (8 B)
            f = kern["proj_scan"]
            byt = (24.0 + 4.0 * D / H) * step.units("scan_bwd")
            f["hbm_bytes_per_launch"] = byt
            f["hbm_gbs"] = round(byt / (f["avg_ms"] / 1e3) / 1e9, 1)
        result["kernels"] = {n: {k: (round(v, 4) if isinstance(v, float) else v) for k, v in kern[n].items()}
                             for n in kern}
        # the scans of the step (with the projection fused, the forward's
        # scan has no kernel of its own: the backward's alone)
        scan = {n: kern[n] for n in ("scan_fwd", "scan_bwd") if n in kern}
        tot_ms = sum(v["avg_ms"] for v in scan.values())
        per_unit = (24.0 if "scan_fwd" in scan else 0.0) + 40.0
        ach = per_unit * step.units("scan_bwd") / (tot_ms / 1e3) / 1e9
        result["scan_roofline"] = {"kernels": sorted(scan), "bound": "hbm", "achieved": round(ach, 1),
                                   "peak": peak_hbm, "unit": "GB/s", "frac": round(ach / peak_hbm, 4),
                                   "peak_kind": peak_kind}
        # The scans on their own (plain float32 entry points, one micro-batch,
        # after the timed region): inside the step the GEMMs hold the SM clock
        # down under the power cap and the issue-bound scans slow with it.
        result["scan_alone"] = scan_alone(step, G[0], dev, peak_hbm)
        fused_here = step.fused
        del step
        torch.cuda.empty_cache()
        if not fused_here and H % 32 == 0:
            result["fused_projection_scan_step"] = fused_variant(args, cfg, params, x, G, B_local, dev, sync,
                                                                max_over_ranks, peak_hbm)
        # ---------------- e2e through the public module API, host buffers
        if not args.no_e2e:
            result["e2e"] = e2e_parallel(args, cfg, params, x, G, B_local, world, dev, sync,
                                         max_over_ranks, allreduce)
    else:
        result.update(run_recurrent(args, cfg, params, x, G, B_local, world, dev, sync,
                                    max_over_ranks, allreduce, peak_tf, peak_kind))
    if result.get("e2e") and not args.no_e2e:
        result["e2e"]["h2d_roofline"] = h2d_roofline(result["e2e"], cfg, world, dev, sync)
    return result


def fused_variant(args, cfg, params, x, G, B_local, dev, sync, max_over_ranks, peak_hbm, steps=3):
    """The same step with the projection and the scan forward as one kernel
    (hs_projection_scan_forward), where the library's default takes the two
    calls for this shape: timed the same way (CUDA events, max over ranks,
    no gradient all-reduce), with the forward's algorithmic DRAM bytes per
    micro-batch of both variants.  Reported beside the headline, which
    stays on the library's default path."""
    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    step = ParallelStep(cfg, params, B_local, dev, fused=True)
    for _ in range(2):
        step.run(x, G)
    sync()
    step.ms = {n: 0.0 for n in step.names}
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    allev = []
    for _ in range(steps):
        allev.extend(step.run(x, G, record=True))
    t1.record()
    sync()
    ms = max_over_ranks(t0.elapsed_time(t1))
    step.collect(allev)
    from prlstm_b200 import _lib
    _lib.check_device_status(dev)
    units = T * step.mb_mean * H  # (t, b, h) per micro-batch
    nl = steps * step.nmb
    res = {
        "what": "the same training step with hs_projection_scan_forward in place of the projection GEMM and "
                "the scan forward (not the library default for this shape)",
        "value": T * cfg["B"] * steps / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms / steps,
        "kernels_ms": {n: round(step.ms[n] / nl, 4) for n in step.names},
        # forward DRAM bytes per micro-batch (x's split read by both)
        "forward_hbm_bytes_per_microbatch": {"fused": (24.0 + 4.0 * D / H) * units,
                                             "two_calls": (40.0 + 4.0 * D / H) * units},
    }
    del step
    torch.cuda.empty_cache()
    return res


def h2d_roofline(e2e, cfg, world, dev, sync, nbytes=1 << 30, reps=4):
    """Ceiling of the end-to-end number set by the host->device copies: the
    pinned-memory H2D bandwidth measured here (every rank copying at once, so
    the aggregate includes contention on the host side), and the tokens/s the
    step's H2D bytes allow at that bandwidth."""
    import torch.distributed as dist

    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dst.copy_(src, non_blocking=True)
    sync()
    best = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sync()
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize(dev)
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    t = torch.tensor([best], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    agg = float(t.item())
    del src, dst
    # bytes per step over all ranks (each rank reports its own share)
    h2d_total = e2e["h2d_bytes_per_step"] * world
    tokens = cfg["T"] * cfg["B"] * (world if cfg["mode"] != "parallel" else 1)
    bound = tokens / (h2d_total / (agg * 1e9))
    return {"h2d_gbs_per_gpu": round(best, 2), "h2d_gbs_aggregate": round(agg, 2),
            "h2d_bytes_per_step_all_ranks": h2d_total, "bound_value": bound, "unit": "tokens/s",
            "frac": e2e["value"] / bound,
            "how": "1 GiB pinned->device copy, best of 4, all ranks at once"}


def scan_alone(step, G0, dev, peak_hbm, reps=5):
    """The scans timed alone with CUDA events on one micro-batch of the
    step's own inputs (every rank runs it; rank 0 reports).  "step_kernels"
    are the calls the training step makes: hs_scan_forward_kf and the
    split-writing hs_scan_backward_split (its bound pass over dout, the scan
    writing dZ as the fp16 split, the checks); "float32_dz" the plain entry
    points, hs_scan_forward and hs_scan_backward writing float32 dZ.  Both
    against the same algorithmic bytes: 24 B forward, 40 B backward per
    (t, b, h)."""
    L, P = step.L, step.L.ptr
    T, H, mb = step.cfg["T"], step.cfg["H"], step.mb
    st = L.stream_ptr(dev)
    dz = torch.empty_like(step.z)

    def fwd32():
        L.call("hs_scan_forward", P(step.z), P(step.c0), P(step.out), P(step.c), None, None, T, mb, H, 1e-6,
               P(step.ws), step.ws.numel(), P(step.status), st)

    def bwd32():
        L.call("hs_scan_backward", P(step.z), P(step.c), P(step.c0), P(G0), None, None, P(dz), None,
               P(step.db_mb), T, mb, H, 1e-6, P(step.ws), step.ws.numel(), P(step.status), st)

    kf, dz_scale = P(step.words[0:]), P(step.words[16:])

    def fwd_kf():
        L.call("hs_scan_forward_kf", P(step.z), P(step.c0), P(step.out), P(step.c), P(step.h_n), P(step.c_n),
               T, mb, H, 1e-6, P(step.ws), step.ws.numel(), kf, P(step.status), st)

    def bwd_split():
        L.call("hs_scan_backward_split", P(step.z), P(step.c), P(step.c0), P(G0), None, None, kf,
               P(step.dz_split), dz_scale, None, P(step.db_mb), T, mb, H, 1e-6, P(step.ws), step.ws.numel(),
               P(step.status), st)

    def timed(f):
        for _ in range(2):
            f()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            f()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    out = {"workload": f"one micro-batch, T={T}, B={mb}, H={H}", "reps": reps}
    for key, pair in (("step_kernels", (fwd_kf, bwd_split)), ("float32_dz", (fwd32, bwd32))):
        ent = {}
        for name, f, bpe in (("scan_fwd", pair[0], 24.0), ("scan_bwd", pair[1], 40.0)):
            ms = timed(f)
            gbs = bpe * T * mb * H / (ms / 1e3) / 1e9
            ent[name] = {"avg_ms": round(ms, 4), "achieved": round(gbs, 1), "unit": "GB/s",
                         "frac": round(gbs / peak_hbm, 4)}
        tot = ent["scan_fwd"]["avg_ms"] + ent["scan_bwd"]["avg_ms"]
        gbs = 64.0 * T * mb * H / (tot / 1e3) / 1e9
        ent["combined"] = {"achieved": round(gbs, 1), "frac": round(gbs / peak_hbm, 4)}
        out[key] = ent
    del dz
    return out


def e2e_parallel(args, cfg, params, x, G, B_local, world, dev, sync, max_over_ranks, allreduce):
    import prlstm_b200

    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    mb = x[0].shape[1]  # the micro-batches of make_data (micro_batches)
    nmb = len(x)
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=True).to(dev)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    # the step's inputs, in pinned host memory, one buffer per micro-batch
    hx = [t.cpu().pin_memory() for t in x]
    hG = [t.cpu().pin_memory() for t in G]
    x.clear()
    G.clear()
    torch.cuda.empty_cache()
    loss_host = torch.empty(1, pin_memory=True)
    copy_stream = torch.cuda.Stream(dev)
    ahead = []  # the next step's first micro-batch, when this step prefetched it

    def issue(i):
        with torch.cuda.stream(copy_stream):
            nxt = (hx[i].to(dev, non_blocking=True), hG[i].to(dev, non_blocking=True))
            ev = torch.cuda.Event()
            ev.record()
        return nxt, ev

    def one_step(prefetch=True):
        m.zero_grad(set_to_none=True)
        loss = torch.zeros((), device=dev)
        # double-buffered host->device copies on a side stream; during the
        # last micro-batch the next step's first one is copied (not across the
        # warm-up/timed boundary, so each timed step's copies are all inside
        # the timed region)
        nxt, ev = ahead.pop() if ahead else issue(0)
        for i in range(nmb):
            torch.cuda.current_stream(dev).wait_event(ev)
            xd, Gd = nxt
            xd.requires_grad_(True)
            xd.record_stream(torch.cuda.current_stream(dev))
            Gd.record_stream(torch.cuda.current_stream(dev))
            if i + 1 < nmb:
                nxt, ev = issue(i + 1)
            elif prefetch:
                ahead.append(issue(0))
            out, _ = m(xd)
            lo = (out * Gd).sum()
            lo.backward()
            loss += lo.detach()
        grads = [p.grad for p in m.parameters() if p.grad is not None]
        allreduce(grads)
        loss_host.copy_(loss.reshape(1), non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return float(loss_host.item())

    graphed = None
    if use_graph(args, cfg, B_local, world) is not None and nmb == 1:
        # A launch-bound step through the module as a user graphs it: the
        # forward and backward captured once (torch.cuda.graph), replayed
        # every step on static input buffers that the step's host->device
        # copies fill; the loss is read back after each replay.
        sx = torch.empty(T, mb, D, device=dev)
        sG = torch.empty(T, mb, H, device=dev)
        sx.copy_(hx[0])
        sG.copy_(hG[0])
        xleaf = sx.detach().requires_grad_(True)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                m.zero_grad(set_to_none=True)
                out, _ = m(xleaf)
                (out * sG).sum().backward()
        torch.cuda.current_stream(dev).wait_stream(side)
        m.zero_grad(set_to_none=True)
        xleaf.grad = None
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out, _ = m(xleaf)
            sloss = (out * sG).sum()
            sloss.backward()

        pf = PrefetchedInputs([hx[0], hG[0]], [sx, sG], dev)

        def graphed(prefetch=True):
            pf.consume()  # this step's inputs, copied while the previous step ran
            g.replay()
            if prefetch:
                pf.issue()  # the next step's inputs, overlapping this replay
            loss_host.copy_(sloss.detach().reshape(1), non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            return float(loss_host.item())

        one_step = graphed

    warm = max(1, min(args.warmup, 2))
    for w in range(warm):
        one_step(prefetch=w + 1 < warm)
    sync()
    steps = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        one_step(prefetch=s + 1 < steps)
    e1.record()
    sync()
    ms = max_over_ranks(e0.elapsed_time(e1))
    h2d = sum(t.numel() * 4 for t in hx) + sum(t.numel() * 4 for t in hG)
    res = {"value": T * cfg["B"] * steps / (ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "steps": steps}
    if graphed is not None:
        res["launch"] = ("module forward + backward captured in a CUDA graph (torch.cuda.graph), replayed per "
                         "step; each step's host-to-device copies overlap the previous step's replay")
    return res


def run_recurrent(args, cfg, params, x, G, B_local, world, dev, sync, max_over_ranks, allreduce,
                  peak_tf, peak_kind):
    import prlstm_b200
    from prlstm_b200 import _lib

    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    P = _lib.ptr
    lib = _lib.load()
    W_ih, W_hh, b_ih, b_hh, a = (t.to(dev).contiguous() for t in params)
    h_save = torch.empty(T + 1, B_local, H, device=dev)
    c_save = torch.empty(T + 1, B_local, H, device=dev)
    acts = torch.empty(T, B_local, 4 * H, device=dev)
    dx = torch.empty(T, B_local, D, device=dev)
    dW_ih, dW_hh = torch.empty_like(W_ih), torch.empty_like(W_hh)
    db_ih, db_hh, da = torch.empty(4 * H, device=dev), torch.empty(4 * H, device=dev), torch.empty(4, device=dev)
    ws = _lib.workspace(lib.hs_recurrent_workspace_bytes(T, B_local, D, H), dev)
    status = _lib.status_word(dev)

    def step(record=False):
        st = _lib.stream_ptr(dev)  # the current stream: the capture stream inside a graph capture
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
        if record:
            e[0].record()
        _lib.call("hs_recurrent_forward", P(x), None, None, P(W_ih), P(W_hh), P(b_ih), P(b_hh),
                  P(a), P(h_save), P(c_save), P(acts), T, B_local, D, H, P(ws), ws.numel(),
                  P(status), st)
        if record:
            e[1].record()
        if world == 1:
            _lib.call("hs_recurrent_backward", P(x), P(W_ih), P(W_hh), P(b_hh), P(a), P(h_save),
                      P(c_save), P(acts), P(G), None, None, P(dx), P(dW_ih), P(dW_hh), P(db_ih),
                      P(db_hh), P(da), T, B_local, D, H, P(ws), ws.numel(), P(status), st)
        else:
            # weight gradients first; their all-reduce (NCCL's stream) overlaps
            # the input-gradient GEMM dX = dgates . W_ih (acts holds dgates)
            _lib.call("hs_recurrent_backward", P(x), P(W_ih), P(W_hh), P(b_hh), P(a), P(h_save),
                      P(c_save), P(acts), P(G), None, None, None, P(dW_ih), P(dW_hh), P(db_ih),
                      P(db_hh), P(da), T, B_local, D, H, P(ws), ws.numel(), P(status), st)
            pending = allreduce.start([dW_ih, dW_hh, db_ih, db_hh, da])
            _lib.call("hs_linear_dgrad", P(acts), P(W_ih), P(dx), T * B_local, 4 * H, D, P(ws), ws.numel(),
                      P(status), st)
            pending.finish()
        if record:
            e[2].record()
        return e

    for _ in range(args.warmup):
        step()
    sync()
    _lib.check_device_status(dev)
    # Both directions on the cluster kernels (plain cluster launches, no
    # cooperative launch): the step is captured once in a CUDA graph and
    # replayed, as for the launch-bound parallel configs; the fwd/bwd
    # breakdown comes from an ungraphed pass after the timed region.
    paths = [lib.hs_recurrent_path(B_local, H, d) for d in (0, 1)]
    graph = None
    if world == 1 and getattr(args, "graph", "auto") != "off" and paths == [2, 2]:
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        sync()
        _lib.check_device_status(dev)
    clocks = ClockSampler(_gpu_id(dev))
    clocks.start()
    sync()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    if graph is not None:
        for _ in range(args.steps):
            graph.replay()
    else:
        evs = [step(record=True) for _ in range(args.steps)]
    t1.record()
    sync()
    ck = clocks.stop()
    if graph is not None:
        evs = [step(record=True) for _ in range(args.steps)]
        sync()
        del graph
    _lib.check_device_status(dev)
    ms = max_over_ranks(t0.elapsed_time(t1))
    fwd = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    bwd = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    if paths == [2, 2] and world == 1 and ms / args.steps < 0.5 * (fwd + bwd):
        raise RuntimeError(f"graphed recurrent step {ms / args.steps:.4f} ms is shorter than half the ungraphed "
                           f"device time {fwd + bwd:.4f} ms: the capture missed the step's kernels")
    flops = 24.0 * T * B_local * H * (D + H)
    tokens = T * B_local * world * args.steps
    ach = flops / ((fwd + bwd) / 1e3) / 1e12
    # Per-step latency bound of the recurrence: the larger of the step's
    # FLOPs at the tensor peak and the step's W_hh bytes at the aggregate
    # shared-memory bandwidth (128 B/clk/SM at the measured under-load clock).
    # The forward step is one [B,H]x[H,4H] product, the backward step two.
    pk = _peaks_raw()
    mhz = (pk.get("clocks_under_load") or {}).get("sm_mhz_median") or pk.get("sm_max_mhz") or 1965.0
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    smem_bw = 128.0 * nsm * mhz * 1e6  # bytes/s
    whh_bytes = 4.0 * H * H * 4
    step_flop = 8.0 * B_local * H * H
    bound_f = max(step_flop / (peak_tf * 1e12), whh_bytes / smem_bw) * 1e6
    bound_b = max(2 * step_flop / (peak_tf * 1e12), whh_bytes / smem_bw) * 1e6
    us_f, us_b = fwd * 1e3 / T, bwd * 1e3 / T
    kname = {0: "ffma", 1: "tcgen05", 2: "cluster (DSMEM exchange)"}
    res = {"value": tokens / (ms / 1e3), "ms_per_step": ms / args.steps, "clocks": ck,
           "gpu_launches": None,
           "recurrent": {"fwd_ms": fwd, "bwd_ms": bwd, "us_per_step_fwd": us_f,
                         "us_per_step_bwd": us_b,
                         "step_kernel": {"fwd": kname.get(paths[0], "?"), "bwd": kname.get(paths[1], "?")},
                         "step_bound_us": {"fwd": round(bound_f, 3), "bwd": round(bound_b, 3),
                                           "smem_gbs": round(smem_bw / 1e9, 1), "sm_mhz": mhz},
                         "frac_of_step_bound": {"fwd": round(bound_f / us_f, 4),
                                                "bwd": round(bound_b / us_b, 4)}},
           "roofline": {"kernel": "recurrent fwd+bwd", "bound": "tensor", "achieved": round(ach, 3),
                        "peak": peak_tf, "unit": "TFLOP/s", "frac": round(ach / peak_tf, 5),
                        "peak_kind": peak_kind, "traffic": None,
                        "note": "latency-bound recurrence: see recurrent.frac_of_step_bound"}}
    if paths == [2, 2] and world == 1 and getattr(args, "graph", "auto") != "off":
        res["launch"] = "cuda_graph (one capture of the step, replayed every step)"
    if args.no_e2e:
        return res
    # e2e through the module API with host buffers
    m = prlstm_b200.HeadStartLSTM(D, H).to(dev)
    with torch.no_grad():
        for p, v in zip(m.parameters(), params):
            p.copy_(v)
    hx_ = x.cpu().pin_memory()
    hG_ = G.cpu().pin_memory()
    loss_host = torch.empty(1, pin_memory=True)

    def e2e_step(prefetch=True):  # copies on the compute stream: nothing to prefetch
        m.zero_grad(set_to_none=True)
        xd = hx_.to(dev, non_blocking=True).requires_grad_(True)
        Gd = hG_.to(dev, non_blocking=True)
        out, _ = m(xd)
        lo = (out * Gd).sum()
        lo.backward()
        allreduce([p.grad for p in m.parameters()])
        loss_host.copy_(lo.detach().reshape(1), non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    graphed = "launch" in res
    if graphed:
        # the module's forward and backward captured once (torch.cuda.graph)
        # on static inputs that each step's host-to-device copies fill
        sx, sG = torch.empty_like(x), torch.empty_like(G)
        sx.copy_(hx_)
        sG.copy_(hG_)
        xleaf = sx.detach().requires_grad_(True)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                m.zero_grad(set_to_none=True)
                out, _ = m(xleaf)
                (out * sG).sum().backward()
        torch.cuda.current_stream(dev).wait_stream(side)
        m.zero_grad(set_to_none=True)
        xleaf.grad = None
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out, _ = m(xleaf)
            sloss = (out * sG).sum()
            sloss.backward()

        pf = PrefetchedInputs([hx_, hG_], [sx, sG], dev)

        def e2e_step(prefetch=True):
            pf.consume()
            g.replay()
            if prefetch:
                pf.issue()
            loss_host.copy_(sloss.detach().reshape(1), non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

    for w in range(args.warmup):
        e2e_step(prefetch=w + 1 < args.warmup)
    sync()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(args.steps):
        e2e_step(prefetch=s + 1 < args.steps)
    e1.record()
    sync()
    ms_e = max_over_ranks(e0.elapsed_time(e1))
    res["e2e"] = {"value": tokens / (ms_e / 1e3), "unit": "tokens/s",
                  "h2d_bytes_per_step": (x.numel() + G.numel()) * 4, "d2h_bytes_per_step": 4}
    if graphed:
        res["e2e"]["launch"] = ("module forward + backward captured in a CUDA graph (torch.cuda.graph), replayed "
                                "per step; each step's host-to-device copies overlap the previous step's replay")
    # launches per step (approximate): projection GEMM, weight staging (the
    # tensor-core path: max |a W_hh| then the split tiles), the recurrent
    # kernel per window of batch groups (one launch on the cluster path), the
    # gradient GEMMs, colsum, unscale, da
    nb = (B_local + 31) // 32
    nk = [1 if pth == 2 else nb for pth in paths]
    res["gpu_launches"] = args.steps * ((1 + (2 if paths[0] == 1 else 1) + nk[0]) +
                                        ((2 if paths[1] == 1 else 1) + nk[1] + 6))
    return res


# ------------------------------------------------------------------ reference arm
def _stock_reference():
    """The unmodified reference package (an offline pip install of the
    reference tree under baseline/_ref), or None when it is absent."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "headstartlstm")):
        return None
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    import headstartlstm

    return headstartlstm


def _host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, cfg, budget_s=None):
    """The reference's CPU path on all host cores: the stock package through
    its public API (HeadStartLSTM(D, H, backend="torch", parallel=...) ->
    forward -> sum(out*G).backward(), __init__.py:169-233) when it is
    installed under baseline/_ref, else the oracle port of the same
    algorithm.  Long-sequence parallel configs run a bounded sample of the
    batch per step: its size is chosen from one calibration step of one
    sequence so the warm-up and timed steps take about `budget_s` seconds.
    Returns (tokens/s, cores, sample, seconds per step, kind)."""
    ncores = _host_cores()
    torch.set_num_threads(ncores)
    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    parallel = cfg["mode"] == "parallel"
    params = make_params(cfg)
    ref = _stock_reference()
    if ref is not None:
        kind = "reference"
        m = ref.HeadStartLSTM(D, H, backend="torch", parallel=parallel)
        with torch.no_grad():
            for p, v in zip(m.parameters(), params):
                p.copy_(v)

        def fwd_bwd(x, G):
            m.zero_grad(set_to_none=True)
            xd = x.detach().requires_grad_(True)
            out, _ = m(xd)
            (out * G).sum().backward()
    else:
        from oracle import hs_oracle as O

        kind = "port"

        def fwd_bwd(x, G):
            O.module_forward_backward(params, x, G, parallel=parallel)

    gen = torch.Generator().manual_seed(1)
    Bs = cfg["B"]
    if parallel and T >= 4096:
        x1 = torch.randn(T, 1, D, generator=gen)
        G1 = torch.randn(T, 1, H, generator=gen)
        fwd_bwd(x1, G1)  # first call: allocator and thread-pool warm-up
        t0 = time.perf_counter()
        fwd_bwd(x1, G1)
        t1 = time.perf_counter() - t0
        nstep = args.warmup + args.steps
        Bs = int(max(1, min(8, (budget_s or 120.0) / max(1e-3, nstep * t1))))
        sample = (f"T={T}, B={Bs} of {cfg['B']} sequences per step (sequences are independent, "
                  "tokens/s scales with B)")
    else:
        sample = f"full config (T={T}, B={Bs})"
    x = torch.randn(T, Bs, D, generator=gen)
    G = torch.randn(T, Bs, H, generator=gen)
    for _ in range(args.warmup):
        fwd_bwd(x, G)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fwd_bwd(x, G)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = T * Bs * len(times) / total
    return value, ncores, sample, total / len(times), kind


def run_reference_gpu(args, cfg, dev):
    """The reference's own GPU paths on this GPU, for comparison (not the
    driver's reference arm): the Triton backend (CUDA graphs over per-step
    Triton cell kernels and cuBLAS, _triton.py:327-470) for recurrent
    configs, the parallel=True torch path (_parallel.py:38-74, ATen on CUDA)
    for parallel configs, each fwd + sum(out*G).backward() with x requiring
    grad.  Imports the reference package installed under baseline/_ref (an
    offline pip install of the reference tree; absent -> unavailable).
    Parallel configs run micro-batches of MICRO_BATCH sequences, as ours do;
    tokens/s counts the whole batch."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "headstartlstm")):
        return None, "reference package not installed under baseline/_ref"
    sys.path.insert(0, ref_root)
    import headstartlstm

    T, D, H = cfg["T"], cfg["D"], cfg["H"]
    params = make_params(cfg)
    parallel = cfg["mode"] == "parallel"
    mb = min(MICRO_BATCH, cfg["B"]) if parallel else cfg["B"]
    nmb = cfg["B"] // mb
    m = headstartlstm.HeadStartLSTM(D, H, backend="triton" if not parallel else "torch",
                                    parallel=parallel).to(dev)
    with torch.no_grad():
        for pp, v in zip(m.parameters(), params):
            pp.copy_(v)
    gen = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(T, mb, D, device=dev, generator=gen)
    G = torch.randn(T, mb, H, device=dev, generator=gen)

    def step():
        for _ in range(nmb):
            xd = x.detach().requires_grad_(True)
            out, _ = m(xd)
            (out * G).sum().backward()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    backend = "parallel torch path (ATen CUDA)" if parallel else "triton backend"
    return {"value": T * cfg["B"] / (ms / 1e3), "ms_per_step": ms, "backend": backend,
            "micro_batch": mb if parallel else None}, None


def reference_gpu_beside(args, cfg, line, dev):
    """The reference's stock GPU paths (run_reference_gpu: its Triton
    backend for the recurrent configs, its parallel=True torch path for the
    parallel ones) on the headline config and on each float32 config this
    run timed, with this build's device-timed value over the reference's.
    Not the driver's reference arm (the CPU path): a comparison on the same
    GPU, recorded in the same JSON line.  Each failure is recorded, never
    raised."""
    out = {}
    todo = [(args.config, cfg, line["value"])]
    todo += [(n, dict(CONFIGS[n]), e["value"]) for n, e in line.get("configs", {}).items()
             if n in CONFIGS and isinstance(e, dict) and "value" in e]
    for name, c, ours in todo:
        big = c["T"] * c["B"] >= (1 << 20)
        sub = argparse.Namespace(steps=1 if big else 5, warmup=1 if big else 2)
        torch.cuda.empty_cache()
        try:
            r, why = run_reference_gpu(sub, c, dev)
        except Exception as e:  # an out-of-memory or a compile failure of the reference
            r, why = None, f"{type(e).__name__}: {e}"[:300]
        if r is None:
            out[name] = {"unavailable": why}
        else:
            r["steps"] = sub.steps
            r["ours_over_reference"] = ours / r["value"]
            out[name] = r
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--config", default="cfg4", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) leg")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the global batch (small cases for profiling)")
    ap.add_argument("--no-cublas-ref", action="store_true",
                    help="skip timing cuBLAS TF32/FP32 on the GEMM shapes (GEMM ceilings)")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="override T (small cases for profiling)")
    ap.add_argument("--graph", default="auto", choices=["auto", "on", "off"],
                    help="capture the parallel step in a CUDA graph (auto: launch-bound steps on one GPU)")
    ap.add_argument("--no-configs", action="store_true",
                    help="time only the headline config (not configs[0-3] after it)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU paths beside each config")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["B"] = args.batch
    if args.seq_len:
        cfg["T"] = args.seq_len
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "train-step tokens/s (T*B fwd+bwd)"
    base = {"metric": metric, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded, config distributions)", "vs_baseline": None}
    workload = (f"{args.config}: {cfg['mode']} mode fwd+bwd of sum(out*G), T={cfg['T']}, "
                f"B={cfg['B']}, D={cfg['D']}, H={cfg['H']}")

    if args.impl == "reference":
        if rank != 0:
            return
        value, cores, sample, sec, kind = run_reference(args, cfg, budget_s=150.0)
        line = dict(base, impl="reference", value=value, ms_per_step=sec * 1e3,
                    scaling="strong" if cfg["mode"] == "parallel" else "weak",
                    config={"workload": workload, "T": cfg["T"], "B": cfg["B"], "D": cfg["D"],
                            "H": cfg["H"], "mode": cfg["mode"], "parallelism": "cpu"},
                    cpu_baseline={"value": value, "unit": "tokens/s", "cores": cores,
                                  "kind": kind, "sample": sample},
                    e2e={"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0},
                    gpu_launches=0)
        print(json.dumps(line), flush=True)
        return

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.impl == "reference-gpu":
        if rank != 0:
            return
        res, why = run_reference_gpu(args, cfg, dev)
        if res is None:
            print(json.dumps({"impl": "reference-gpu", "unavailable": why}), flush=True)
            return
        line = dict(base, impl="reference-gpu", value=res["value"], ms_per_step=res["ms_per_step"],
                    scaling="strong" if cfg["mode"] == "parallel" else "weak",
                    config={"workload": workload, "T": cfg["T"], "B": cfg["B"], "D": cfg["D"],
                            "H": cfg["H"], "mode": cfg["mode"], "micro_batch": res["micro_batch"],
                            "parallelism": "dp1", "backend": res["backend"]},
                    gpu_launches=None)
        print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    res = run_ours(args, cfg, rank, world, dev)
    line = dict(base)
    line.update(value=res["value"], ms_per_step=res["ms_per_step"],
                scaling="strong" if cfg["mode"] == "parallel" else "weak",
                config=_config_obj(args.config, cfg, world, workload),
                roofline=res.get("roofline"), e2e=res.get("e2e"), clocks=res.get("clocks"),
                gpu_launches=res.get("gpu_launches"))
    for k in ("kernels", "scan_roofline", "scan_alone", "fused_projection_scan_step", "recurrent", "launch"):
        if k in res:
            line[k] = res[k]
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref_args = argparse.Namespace(warmup=1, steps=2)
        value, cores, sample, _, kind = run_reference(ref_args, cfg, budget_s=25.0)
        line["cpu_baseline"] = {"value": value, "unit": "tokens/s", "cores": cores,
                                "kind": kind, "sample": sample}
    # The other configs of the benchmark, after the headline, in the same
    # run: each with its own device-timed value, e2e and (rank 0, N=1) the
    # reference's CPU path on the same host cores.
    if args.config == "cfg4" and not args.no_configs:
        line["configs"] = {}
        for name in ("cfg0", "cfg1", "cfg2", "cfg3"):
            c = dict(CONFIGS[name])
            sub = argparse.Namespace(**vars(args))
            sub.steps = max(args.steps, 10)
            sub.warmup = max(args.warmup, 3)
            sub.no_cublas_ref = True
            r = run_ours(sub, c, rank, world, dev)
            ent = {"value": r["value"], "unit": "tokens/s", "ms_per_step": r["ms_per_step"],
                   "steps": sub.steps, "mode": c["mode"],
                   "scaling": "strong" if c["mode"] == "parallel" else "weak (replicas)",
                   "config": _config_obj(name, c, world, None), "e2e": r.get("e2e"),
                   "roofline": r.get("roofline"), "gpu_launches": r.get("gpu_launches")}
            if "recurrent" in r:
                ent["recurrent"] = r["recurrent"]
            if "launch" in r:
                ent["launch"] = r["launch"]
            if "scan_roofline" in r:
                ent["scan_roofline"] = r["scan_roofline"]
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                ref_args = argparse.Namespace(warmup=1, steps=2)
                value, cores, sample, _, kind = run_reference(ref_args, c)
                ent["cpu_baseline"] = {"value": value, "unit": "tokens/s", "cores": cores,
                                       "kind": kind, "sample": sample}
                ent["vs_cpu_baseline"] = ent["value"] / value
                if ent.get("e2e"):
                    ent["e2e_vs_cpu_baseline"] = ent["e2e"]["value"] / value
            line["configs"][name] = ent
            torch.cuda.empty_cache()
        # configs[3]'s bf16-input variant, through the module API, and
        # configs[4] in bf16 (the bf16 tensor-core GEMMs and dZ writer)
        line["configs"]["cfg3_bf16"] = run_bf16_module(args, dict(CONFIGS["cfg3"]), world, dev, rank)
        torch.cuda.empty_cache()
        line["configs"]["cfg4_bf16"] = run_bf16_module(args, dict(CONFIGS["cfg4"]), world, dev, rank, steps=4)
        torch.cuda.empty_cache()
    # The reference's own GPU paths on this GPU, beside each float32 config
    # of this run: rank 0 at N=1, after everything else.
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        line["reference_gpu"] = reference_gpu_beside(args, cfg, line, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_bf16_module(args, cfg, world, dev, rank, steps=10, warmup=3):
    """A config with bfloat16 inputs and parameters (the reduced-precision
    variant): fwd + sum(out*G) backward through prlstm_b200.HeadStartLSTM,
    inputs resident on the device, CUDA events around the steps.  Recurrent
    configs: every rank runs the full config (replicas).  Parallel configs:
    the batch is split over ranks and run in the float32 headline's
    micro-batches (micro_batches; gradients accumulated, then all-reduced).
    tokens/s is the whole job's."""
    import torch.distributed as dist

    import prlstm_b200

    T, B, D, H = cfg["T"], cfg["B"], cfg["D"], cfg["H"]
    parallel = cfg["mode"] == "parallel"
    params = make_params(cfg)
    m = prlstm_b200.HeadStartLSTM(D, H, parallel=parallel).to(dev, torch.bfloat16)
    with torch.no_grad():
        for p_, v in zip(m.parameters(), params):
            p_.copy_(v)
    B_local = B // world if parallel else B
    if parallel:
        xs, Gs = make_data(cfg, B_local, rank, dev, mb=micro_batches(B_local, H))
        xs = [t.to(torch.bfloat16) for t in xs]
        Gs = [t.to(torch.bfloat16) for t in Gs]
    else:
        x, G = make_data(cfg, B, rank, dev)
        xs, Gs = [x.to(torch.bfloat16)], [G.to(torch.bfloat16)]
        del x, G
    torch.cuda.empty_cache()

    def step():
        m.zero_grad(set_to_none=True)
        for x, G in zip(xs, Gs):
            xd = x.detach().requires_grad_(True)
            out, _ = m(xd)
            (out * G).sum().backward()  # bf16 product, float32 accumulation in the sum
        if parallel and world > 1:
            for p_ in m.parameters():
                if p_.grad is not None:
                    dist.all_reduce(p_.grad)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    name = "cfg4" if parallel else "cfg3"
    if parallel:
        dtype = ("bf16 inputs and parameters: bf16 x bf16 tensor-core products (exact) with f32 accumulation, "
                 "f32 scan and state, dZ rounded to bf16 for the gradient products")
        tol = ("2e-2 normwise vs float64 fed the bf16-rounded inputs (tests/test_gpu_bf16.py, "
               "tests/test_gpu_bf16_path.py at this config's micro-batch)")
    else:
        dtype = "bf16 inputs and parameters, f32 arithmetic"
        tol = "2e-2 normwise vs float64 fed the bf16-rounded inputs (tests/test_gpu_bf16.py)"
    tokens = T * (B if parallel else B * world)
    return {"value": tokens * steps / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms / steps,
            "steps": steps, "dtype": dtype, "scaling": "strong" if parallel else "weak (replicas)",
            "config": _config_obj(name, cfg, world, None), "tolerance": tol}


def _config_obj(name, cfg, world, workload):
    o = {"workload": workload or (f"{name}: {cfg['mode']} mode fwd+bwd of sum(out*G), T={cfg['T']}, "
                                  f"B={cfg['B']}, D={cfg['D']}, H={cfg['H']}"),
         "T": cfg["T"], "B": cfg["B"], "D": cfg["D"], "H": cfg["H"], "mode": cfg["mode"],
         "micro_batch": micro_batches(cfg["B"] // world, cfg["H"]) if cfg["mode"] == "parallel" else None,
         "parallelism": f"dp{world}" if cfg["mode"] == "parallel" or world == 1 else f"{world} replicas",
         "l2": ("inputs larger than L2 (z of one micro-batch is 8.6-9.9 GB)" if name == "cfg4"
                else "no flush; the working set of one step is noted by T, B, D, H")}
    return o


if __name__ == "__main__":
    main()
