#!/usr/bin/env python
"""Decode-MLP benchmark: 28-layer Llama-3.2-3B MLP stack with E4M3 weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--m 8] [--impl ours|reference]

One step = one decode step of M tokens through all 28 layers
(RMSNorm -> fused gate||up + SiLU*up -> down + residual), weights resident in
HBM (2.12 GB of E4M3 per step, far above the 126 MB L2, so every step streams
from HBM without an explicit flush).  With N > 1 (torchrun), the stack is
tensor-parallel: gate/up column shards, down K shards, and one fp16 sum of
the 3072-wide partials per layer -- fused into the GEMVs over peer memory
(--tp-mode fused, the default) or an NCCL all-reduce between them
(--tp-mode nccl).

Prints one JSON line (rank 0): value = algorithmic HBM TB/s of the whole job
(bytes all ranks stream / max-over-ranks device time), plus us/layer, the
roofline of the dominant kernel, end-to-end time through the C ABI with host
buffers, the CPU baseline and the clocks seen.

``--impl reference`` times the reference's own CPU implementation of the path
(its fp64 host GEMV loop, compiled from its sources into oracle/_ref, run on
all host cores) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "llama-3.2-3b-instruct-gemm-optimization_b200"
METRIC = "MLP GEMV µs/layer & achieved HBM TB/s (% of ~8 TB/s) at M=1,8; 1/2/4/8 GPU"
HIDDEN, INTER, LAYERS = 3072, 8192, 28
FALLBACK_HBM_GBS = 6650.0


def load_module(name, path, package=False):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [str(path.parent)]} if package else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def layer_bytes(M: int, tp: int = 1):
    """Algorithmic bytes per layer per rank: W + scales + activations in/out."""
    inter = INTER // tp
    gu = 2 * HIDDEN * inter + 2 * inter * 4 + 2 * M * HIDDEN + 2 * M * inter
    dn = inter * HIDDEN + HIDDEN * 4 + 2 * M * inter + 2 * M * HIDDEN + 2 * M * HIDDEN
    return gu, dn


class ClockSampler:
    """nvidia-smi sampling while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        self.proc.wait()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = float(rows[0][2])
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        power = [float(r[3]) for r in rows if r[3].replace(".", "", 1).isdigit()]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------
# Weights
# ---------------------------------------------------------------------------
def make_layers(b2g, torch, device, tp: int, rank: int, ops, M: int, keep_raw: bool = False):
    """28 layers of N(0, 0.02) weights, E4M3 per-channel FP32 (quantised over
    the full matrix, then sharded), prepacked for this rank.  keep_raw keeps
    every layer's raw [K, N] E4M3 codes (the reference kernels' layout)."""
    gu_op, dn_op = ops
    inter = INTER // tp
    cs = slice(rank * inter, (rank + 1) * inter)
    layers = []
    for l in range(LAYERS):
        q = []
        for j, (K, N) in enumerate(((HIDDEN, INTER), (HIDDEN, INTER), (INTER, HIDDEN))):
            g = torch.Generator(device=device)
            g.manual_seed(1000 + 3 * l + j)
            W = (torch.randn(K, N, generator=g, device=device, dtype=torch.float32) * 0.02).half()
            qq, ss = b2g.quantize_e4m3(W, "channel_fp32")
            del W
            q.append((qq, ss))
        (qg, sg), (qu, su), (qd, sd) = q
        pgu = gu_op.prepack(qg[:, cs].contiguous(), qu[:, cs].contiguous())
        sgu = torch.cat([sg[cs], su[cs]]).contiguous()
        pd = dn_op.prepack(qd[cs, :].contiguous())
        layers.append({"pgu": pgu, "sgu": sgu, "pd": pd, "sd": sd,
                       "q0": (qg, qu, qd) if (l == 0 or keep_raw) else None})
    return layers


# ---------------------------------------------------------------------------
# The model's other decode projections on the same op
# ---------------------------------------------------------------------------
ADJACENT = (("qkv_proj", 3072, 5120), ("o_proj", 3072, 3072), ("lm_head", 3072, 128256))


def adjacent_shapes(b2g, torch, device, M: int, reps: int = 5) -> dict:
    """qkv_proj, o_proj and lm_head of Llama-3.2-3B (E4M3, per-channel FP32
    scales, M rows): per-launch time and algorithmic bandwidth, each launch
    on its own copy of the weights (copies > 256 MB in total, so HBM-fed),
    chained with PDL and the L2 prefetch of the next launch as in the step."""
    out = {}
    for name, K, N in ADJACENT:
        op = b2g.GemvOp(K, N, max_m=8)
        g = torch.Generator(device=device)
        g.manual_seed(77)
        W = (torch.randn(K, N, generator=g, device=device, dtype=torch.float32) * 0.02).half()
        q, s = b2g.quantize_e4m3(W, "channel_fp32")
        del W
        base = op.prepack(q)
        del q
        copies = max(2, -(-(256 << 20) // base.numel()))
        packs = [base] + [base.clone() for _ in range(copies - 1)]
        x = torch.randn(M, K, generator=g, device=device, dtype=torch.float32).half()
        y = torch.empty(M, N, dtype=torch.float16, device=device)
        ws = op.workspace(device)

        launches = [(lambda i=i, p=p: op.enqueue(x, p, s, y=y, workspace=ws, pdl=True,
                                                 prefetch=(op, packs[(i + 1) % len(packs)])))
                    for i, p in enumerate(packs)]
        passes = max(2, -(-56 // len(packs)))
        us = _chain_us(torch, launches, reps, passes)
        alg = op.packed_bytes() + 4 * N + 2 * M * K + 2 * M * N
        out[name] = {"K": K, "N": N, "m": M, "us_per_launch": round(us, 3), "alg_bytes": alg,
                     "achieved_gbs": round(alg / us / 1e3, 1), "grid": op.plan(M)["grid"],
                     "launches_timed": reps * passes * len(packs), "timing": "CUDA graph replay"}
        del packs, base
    return out


# ---------------------------------------------------------------------------
# Per-configuration figures: each GEMV of the decode MLP on its own, chained
# over 28 distinct weight sets (2.1 GB for FP8 U + D, 1.4 GB for FP16 U:
# every launch streams from HBM), with programmatic dependent launch and the
# L2 prefetch of the next launch's weights exactly as the stack chains them.
# ---------------------------------------------------------------------------
def _graph_of(torch, one_pass, passes: int = 1):
    """A CUDA graph of `passes` calls of one_pass (after one eager call, so
    plans and lazy state exist), replayed 3 times as warm-up.  Timing a graph
    measures the device: eager launches through the Python binding take
    longer to issue than a ~10 us GEMV takes to run."""
    one_pass()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(passes):
            one_pass()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    return g


def _chain_us(torch, launches, reps: int, passes: int = 2) -> float:
    """Device time per launch of a chain of launches, replayed as a CUDA
    graph of `passes` passes over the chain (CUDA events on the launching
    stream, after 3 warm-up replays)."""
    def one_pass():
        for f in launches:
            f()
    g = _graph_of(torch, one_pass, passes)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    g.reset()
    return e0.elapsed_time(e1) * 1e3 / (reps * passes * len(launches))


def gemv_bytes(K: int, N: int, M: int, wbytes: int, scale_bytes: int) -> int:
    """Algorithmic bytes of one GEMV: W + scales + x + y."""
    return K * N * wbytes + N * scale_bytes + 2 * M * K + 2 * M * N


def per_config(b2g, torch, device, layers, hbm: float, ms: tuple, reps: int = 5) -> dict:
    """FP16 U at M=1; FP8 U (3072->8192) and D (8192->3072) at M in ms; the
    CUDA-core FFMA variant against the tensor-core path at M=8.  Needs every
    layer's raw E4M3 codes (layers[l]["q0"])."""
    out = {}

    def rec(name, K, N, M, us, alg, **kw):
        out[name] = {"K": K, "N": N, "m": M, "us_per_launch": round(us, 3), "alg_bytes": alg,
                     "achieved_gbs": round(alg / us / 1e3, 1), "frac_of_measured_hbm": round(alg / us / 1e3 / hbm, 4),
                     **kw}

    g = torch.Generator(device=device)
    g.manual_seed(0)
    xs = {M: torch.randn(M, INTER, generator=g, device=device, dtype=torch.float32).half() for M in ms}
    y = torch.empty(max(ms), INTER, dtype=torch.float16, device=device)
    for name, (K, N, j) in {"fp8_U": (HIDDEN, INTER, 0), "fp8_D": (INTER, HIDDEN, 2)}.items():
        op = b2g.GemvOp(K, N, max_m=8)
        packs = [op.prepack(layers[l]["q0"][j]) for l in range(LAYERS)]
        scales = [layers[l]["sd"] if j == 2 else layers[l]["sgu"][:INTER] for l in range(LAYERS)]
        ws = op.workspace(device)
        for M in ms:
            x = xs[M][:, :K]
            x = x.contiguous()

            def mk(i, op=op, x=x, M=M):
                return lambda: op.enqueue(x, packs[i], scales[i], y=y[:M, :N], workspace=ws, pdl=True,
                                          prefetch=(op, packs[(i + 1) % LAYERS]))
            us = _chain_us(torch, [mk(i) for i in range(LAYERS)], reps)
            rec(f"{name}_m{M}", K, N, M, us, gemv_bytes(K, N, M, 1, 4), grid=op.plan(M)["grid"])
        if 8 in ms:
            # the CUDA-core FFMA variant against the tensor-core path at M = 8
            op.set_option(b2g.OPT_MATH, b2g.MATH_FFMA)
            x = xs[8][:, :K].contiguous()
            us = _chain_us(torch, [(lambda i=i: op.enqueue(x, packs[i], scales[i], y=y[:8, :N], workspace=ws, pdl=True,
                                                           prefetch=(op, packs[(i + 1) % LAYERS])))
                                   for i in range(LAYERS)], reps)
            rec(f"{name}_m8_ffma", K, N, 8, us, gemv_bytes(K, N, 8, 1, 4), grid=op.plan(8)["grid"])
        del packs
    # FP16 U, M = 1: W ~ N(0, 0.02) and x ~ N(0, 1), 28 distinct weight sets
    op = b2g.GemvOp(HIDDEN, INTER, weight_dtype="fp16", scale_mode="none", max_m=8)
    raw, packs = [], []
    for l in range(LAYERS):
        gl = torch.Generator(device=device)
        gl.manual_seed(l)
        w = (torch.randn(HIDDEN, INTER, generator=gl, device=device, dtype=torch.float32) * 0.02).half()
        packs.append(op.prepack(w))
        raw.append(w)
    x = torch.randn(1, HIDDEN, generator=g, device=device, dtype=torch.float32).half()
    ws = op.workspace(device)
    us = _chain_us(torch, [(lambda i=i: op.enqueue(x, packs[i], None, y=y[:1], workspace=ws, pdl=True,
                                                   prefetch=(op, packs[(i + 1) % LAYERS])))
                           for i in range(LAYERS)], reps)
    rec("fp16_U_m1", HIDDEN, INTER, 1, us, gemv_bytes(HIDDEN, INTER, 1, 2, 0), grid=op.plan(1)["grid"])
    del packs
    return out, raw


# ---------------------------------------------------------------------------
# The reference's own GPU kernels (kernels/gemv_fp8.cu run_gemv, compiled for
# sm_100a by baseline/Makefile) on the same weights
# ---------------------------------------------------------------------------
REF_GPU_LIB = ROOT / "baseline" / "_ref" / "libref_gpu.so"


def reference_kernels(torch, layers, h, M: int, our_ms_per_step: float, fp16_sets=None):
    """Times the reference GEMV path on the 28-layer stack: per layer and token
    its three M=1 GEMVs (gate, up, down; memset + gemv_chunk_kernel + cast
    each, kernels/gemv_fp8.cu:276-283), M tokens one after another (the
    reference has no M>1 path), weights rotating over the 28 distinct layers.
    RMSNorm, SiLU*up and the residual are not counted (the reference has no
    kernels for them).  Variant/grid/KU: the best of a sweep on this GPU over
    the reference's own knobs, and its shipped L4 setting for comparison."""
    import ctypes
    if not REF_GPU_LIB.exists():
        return {"unavailable": "baseline/_ref/libref_gpu.so not built (make -C baseline needs the reference sources)"}
    L = ctypes.CDLL(str(REF_GPU_LIB))
    L.ref_gpu_gemv_fp8.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5
    dev = h.device
    x = h[0].contiguous()
    a = torch.randn(INTER, device=dev).half()
    y_acc = torch.empty(INTER, dtype=torch.float32, device=dev)
    y = torch.empty(INTER, dtype=torch.float16, device=dev)

    def gemv(w, xv, K, N, cfg):
        st = L.ref_gpu_gemv_fp8(w.data_ptr(), xv.data_ptr(), y_acc.data_ptr(), y.data_ptr(), K, N, *cfg)
        if st != 0:
            raise RuntimeError(f"reference gemv failed: CUDA error {st}")

    def timed(fn, reps):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    L.ref_gpu_gemv_fp16.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4
    shapes = {"gate_up": (HIDDEN, INTER, 0, x), "down": (INTER, HIDDEN, 2, a)}
    best, shipped = {}, {}
    for name, (K, N, j, xv) in shapes.items():
        ws = [layers[l]["q0"][j] for l in range(LAYERS)]

        def sweep_one(cfg):
            return timed(lambda: [gemv(w, xv, K, N, cfg) for w in ws], 2) * 1e3 / LAYERS
        shipped_cfg = (L.ref_gpu_fp8_best_variant(), L.ref_gpu_fp8_best_grid(N), L.ref_gpu_fp8_best_ku(N))
        sweep_one(shipped_cfg)
        shipped[name] = {"cfg": shipped_cfg, "us": round(sweep_one(shipped_cfg), 2)}
        results = []
        for variant in range(4):
            for grid in (20, 48, 96, 148, 296, 592):
                for ku in (2, 4, 8):
                    results.append((sweep_one((variant, grid, ku)), (variant, grid, ku)))
        us, cfg = min(results)
        best[name] = {"cfg": cfg, "us": round(us, 2)}

    # The reference's FP16 GEMV (kernels/gemv_fp16.cu run_gemv) at 3072 -> 8192,
    # M = 1, over 28 distinct FP16 weight sets: best of its variant x grid sweep.
    fp16_best = None
    if fp16_sets is not None:
        def gemv16(w, cfg):
            st = L.ref_gpu_gemv_fp16(w.data_ptr(), x.data_ptr(), y_acc.data_ptr(), y.data_ptr(), HIDDEN, INTER, *cfg)
            if st != 0:
                raise RuntimeError(f"reference fp16 gemv failed: CUDA error {st}")
        res16 = []
        for variant in range(4):
            for grid in (14, 29, 48, 96, 148, 296, 592):
                cfg = (variant, grid)
                timed(lambda: [gemv16(w, cfg) for w in fp16_sets], 1)
                res16.append((timed(lambda: [gemv16(w, cfg) for w in fp16_sets], 2) * 1e3 / len(fp16_sets), cfg))
        us16, cfg16 = min(res16)
        fp16_best = {"us": round(us16, 2), "cfg_variant_grid": cfg16}

    def step():
        for l in range(LAYERS):
            qg, qu, qd = layers[l]["q0"]
            for _ in range(M):
                gemv(qg, x, HIDDEN, INTER, best["gate_up"]["cfg"])
                gemv(qu, x, HIDDEN, INTER, best["gate_up"]["cfg"])
                gemv(qd, a, INTER, HIDDEN, best["down"]["cfg"])
    step()
    ms = timed(step, 3)
    return {"what": "reference kernels/gemv_fp8.cu run_gemv (memset + gemv_chunk_kernel + cast), sm_100a build, "
                    f"3 GEMVs x {M} tokens x {LAYERS} layers per step, best sweep config",
            "ms_per_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / LAYERS, 2),
            "per_gemv_us_best": {k: v["us"] for k, v in best.items()},
            "best_cfg_variant_grid_ku": {k: v["cfg"] for k, v in best.items()},
            "per_gemv_us_shipped_l4_cfg": {k: v["us"] for k, v in shipped.items()},
            "fp16_gate_up_m1_best": fp16_best,
            "ours_speedup": round(ms / our_ms_per_step, 2)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's fp64 host loop on all cores
# ---------------------------------------------------------------------------
def cpu_reference_sample(q_host, M: int, min_seconds: float = 8.0):
    """Times the reference's cpu_reference_e4m3 (kernels/gemv_fp8.cu:313-323)
    over layer 0's three projections for M tokens, K-split over all cores.
    Falls back to the oracle's C port when oracle/_ref was not built."""
    orc = load_module("oracle", ROOT / "oracle" / "oracle.py")
    cores = orc.cpu_count()
    R = orc.ref()
    shapes = [(HIDDEN, INTER), (HIDDEN, INTER), (INTER, HIDDEN)]
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal((M, K), dtype=np.float32).astype(np.float16).view(np.uint16)
          for K, _ in shapes]
    nbytes = sum(K * N + N * 4 + 2 * M * K + 2 * M * N for K, N in shapes)
    if R is not None:
        kind = "reference"
        plans = [R.ref_cpu_plan_create(q.ctypes.data, 1, K, N, cores)
                 for q, (K, N) in zip(q_host, shapes)]

        def once():
            for pl, x, (K, N) in zip(plans, xs, shapes):
                y = np.empty((M, N), np.float64)
                R.ref_cpu_plan_run(pl, np.ascontiguousarray(x), M, y)
    else:
        kind = "port"
        os.environ.setdefault("OMP_NUM_THREADS", str(cores))

        def once():
            for q, x, (K, N) in zip(q_host, xs, shapes):
                orc.gemv_loop(q, orc.WTYPE_FP8, x.view(np.float16))
    t0 = time.perf_counter()
    reps = 0
    while True:
        once()
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = time.perf_counter() - t0
    if R is not None:
        for pl in plans:
            R.ref_cpu_plan_destroy(pl)
    return {
        "value": nbytes * reps / dt / 1e12, "unit": "TB/s", "cores": cores, "kind": kind,
        "sample": (f"{reps} x layer-0 gate, up and down E4M3 GEMVs (3072x8192, 3072x8192, "
                   f"8192x3072) for M={M} tokens through the reference's fp64 host loop, "
                   f"K split over {cores} threads; RMSNorm/SiLU not included"),
        "seconds": dt, "us_per_layer": dt / reps * 1e6,
    }


# ---------------------------------------------------------------------------
# The GPU arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist
    b2g = load_module("b2g", PKG_DIR / "__init__.py", package=True)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    tp = world
    M = args.m
    inter = INTER // tp
    if tp == 1:
        # One GPU: the library's stack (two launches per layer, chained).
        st = b2g.Stack(HIDDEN, INTER, LAYERS, max_m=M)
        gu_op, dn_op = st.gate_up, st.down
        tps = None
    else:
        # Tensor parallel: the package's TPStack (column/K shards, residual on
        # rank 0, the partials summed per layer: fused exchange or NCCL).
        import importlib
        st = None
        tps = importlib.import_module("b2g.tp").TPStack(HIDDEN, INTER, LAYERS, rank=rank, world=world, max_m=M,
                                                        fused=args.tp_mode == "fused")
        tps.exchange = args.tp_exchange
        gu_op, dn_op = tps.gate_up, tps.down
    pipe = {"auto": b2g.PIPE_AUTO, "registers": b2g.PIPE_REGISTERS, "tma": b2g.PIPE_TMA}[args.pipe]
    for op in (gu_op, dn_op):
        op.set_option(b2g.OPT_PIPE, pipe)
        if args.math == "ffma":
            op.set_option(b2g.OPT_MATH, b2g.MATH_FFMA)
    if st is not None and args.stack_mode != "per_layer":
        st.set_mode(args.stack_mode)
    want_ref = tp == 1 and not args.no_ref_kernels and REF_GPU_LIB.exists()
    layers = make_layers(b2g, torch, device, tp, rank, (gu_op, dn_op), M, keep_raw=want_ref)
    for i, L in enumerate(layers):
        (st or tps).set_layer(i, L["pgu"], L["sgu"], L["pd"], L["sd"])
    if tps is not None and tps.fused:
        tps.setup_comm(device)
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    g = torch.Generator(device=device)
    g.manual_seed(7)
    h0 = torch.randn(M, HIDDEN, generator=g, device=device, dtype=torch.float32).half()
    h = h0.clone()
    act = torch.empty(M, inter, dtype=torch.float16, device=device)
    ws = torch.empty(max(gu_op.workspace_bytes(), dn_op.workspace_bytes()), dtype=torch.uint8,
                     device=device)
    ws.zero_()

    def step_ops():
        tps.enqueue(h, act, ws)

    def step_stack():
        st.enqueue(h, act, ws)

    step = step_stack if st is not None else step_ops
    launches_per_step = 2 * LAYERS  # the stack's default per-layer mode and the TP path

    # CUDA graph of one step (the serving path); direct launches as a fallback
    graph = None
    try:
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()  # warm the side stream
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
    except Exception as e:  # pragma: no cover - reported in the JSON line
        graph = None
        graph_error = repr(e)
    run = graph.replay if graph is not None else step

    def timed(fn, k):
        if tp > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if tp > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for _ in range(args.warmup):
        run()
    h.copy_(h0)
    sampler = ClockSampler(local)
    if rank == 0:
        sampler.start()
    ms = timed(run, args.steps)
    ms_direct = timed(step, max(3, args.steps // 4)) / max(3, args.steps // 4) * args.steps
    clocks = sampler.stop() if rank == 0 else None

    gu_b, dn_b = layer_bytes(M, tp)
    bytes_rank = (gu_b + dn_b) * LAYERS
    ms_step = ms / args.steps
    value = bytes_rank * tp / (ms_step * 1e-3) / 1e12

    hbm, peak_kind = peaks()
    reps = max(5, args.steps // 20)
    detail_extra = {}
    if st is not None:
        # The stack's other execution modes (one persistent cooperative
        # launch per step, on the register or the TMA pipeline), for
        # comparison; recorded, not fatal.
        for mode in ("persistent", "persistent_tma", "per_layer"):
            if mode == args.stack_mode:
                continue
            try:
                st.set_mode(mode)
                for _ in range(3):
                    step_stack()
                ms_pl = timed(step_stack, reps) / reps
                detail_extra[f"{mode}_ms_per_step"] = round(ms_pl, 5)
                detail_extra[f"{mode}_us_per_layer"] = round(ms_pl * 1e3 / LAYERS, 3)
            except Exception as e:
                detail_extra[f"{mode}_error"] = f"{type(e).__name__}: {e}"
        st.set_mode(args.stack_mode)
        # The same stack at every M of the metric's configs (one decode MLP
        # layer = fused gate||up + down, 28 distinct layers per step), each
        # replayed as a CUDA graph of one step; recorded, not fatal.
        per_m = {}
        for Mi in (1, 2, 4, 8):
            try:
                hi, acti = h0[:Mi].clone(), act[:Mi].clone()

                def step_mi():
                    st.enqueue(hi, acti, ws)
                step_mi()
                gi = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gi):
                    step_mi()
                for _ in range(3):
                    gi.replay()
                msi = timed(gi.replay, reps) / reps
                gi.reset()
                bi = sum(layer_bytes(Mi, tp)) * LAYERS
                per_m[f"m{Mi}"] = {"us_per_layer": round(msi * 1e3 / LAYERS, 3),
                                   "tb_s": round(bi / (msi * 1e-3) / 1e12, 4),
                                   "frac_of_measured_hbm": round(bi / (msi * 1e-3) / 1e9 / peaks()[0], 4)}
            except Exception as e:
                per_m[f"m{Mi}"] = {"error": f"{type(e).__name__}: {e}"}
        detail_extra["stack_per_m"] = per_m

    # ---- dominant kernel: the fused RMSNorm + gate||up + SiLU*up GEMV (two
    # thirds of the bytes), its 28 layers back to back exactly as the step
    # chains them (PDL, L2 prefetch of the next launch); CUDA events on the
    # launching stream.
    def gu_sweep():
        for i, L in enumerate(layers):
            gu_op.enqueue(h, L["pgu"], L["sgu"], y=act, workspace=ws, pdl=True,
                          prefetch=(gu_op, layers[(i + 1) % LAYERS]["pgu"]))
    g_gu = _graph_of(torch, gu_sweep)
    ms_gu = timed(g_gu.replay, reps) / (reps * LAYERS)
    g_gu.reset()
    achieved = gu_b / (ms_gu * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"gate_up_m{M}_tp{tp}")
    gu_plan = gu_op.plan(M)
    # the gate||up launch carries the exchange only when it gathers the rows itself
    exch = 1 if tp > 1 and tps.fused and tps.exchange == "gather_launch" else 0
    gu_kernel = (f"gemv_tma_kernel<2,1,{exch}>" if gu_plan["pipe"] == b2g.PIPE_TMA
                 else f"gemv_streamk_kernel<2,1,{gu_plan['math']},{3 if exch else 0}>")
    roofline = {"kernel": f"{gu_kernel} (RMSNorm + gate||up + SiLU*up)",
                "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "traffic": traffic,
                "peak_source": f"{peak_kind} hbm_gbs (STREAM-style copy)",
                "alg_bytes_per_launch": gu_b, "us_per_launch": round(ms_gu * 1e3, 3)}

    def dn_sweep():
        for i, L in enumerate(layers):
            dn_op.enqueue(act, L["pd"], L["sd"], y=h, residual=h if rank == 0 else None,
                          workspace=ws, pdl=True, prefetch=(dn_op, layers[(i + 1) % LAYERS]["pd"]))
    g_dn = _graph_of(torch, dn_sweep)
    ms_dn = timed(g_dn.replay, reps) / (reps * LAYERS)
    g_dn.reset()

    # ---- end to end through the C ABI with host buffers
    h_host = h0.cpu().pin_memory()
    out_host = torch.empty_like(h_host).pin_memory()

    def e2e_step():
        h.copy_(h_host, non_blocking=True)
        step()
        out_host.copy_(h, non_blocking=True)
    for _ in range(3):
        e2e_step()
    k_e2e = max(5, args.steps // 4)
    ms_e2e = timed(e2e_step, k_e2e) / k_e2e
    e2e_value = bytes_rank * tp / (ms_e2e * 1e-3) / 1e12

    # ---- every GEMV configuration on its own (one GPU; recorded, not fatal)
    cfgs, fp16_raw = None, None
    if tp == 1 and want_ref:
        try:
            cfgs, fp16_raw = per_config(b2g, torch, device, layers, hbm, (1, 2, 4, 8))
        except Exception as e:
            cfgs = {"error": f"{type(e).__name__}: {e}"}

    # ---- the reference's own GPU kernels on the same weights (one GPU)
    ref_k = None
    if tp == 1 and not args.no_ref_kernels:
        ref_k = reference_kernels(torch, layers, h0, M, ms_step, fp16_sets=fp16_raw)
        if isinstance(cfgs, dict) and "error" not in cfgs and "unavailable" not in ref_k:
            # The reference has no M > 1 path: M tokens are M launches of its best config.
            pg = ref_k["per_gemv_us_best"]
            for name, c in cfgs.items():
                if name.startswith("fp8_U_m") and not name.endswith("ffma"):
                    c["reference_us"] = round(c["m"] * pg["gate_up"], 2)
                elif name.startswith("fp8_D_m") and not name.endswith("ffma"):
                    c["reference_us"] = round(c["m"] * pg["down"], 2)
                elif name == "fp16_U_m1" and ref_k.get("fp16_gate_up_m1_best"):
                    c["reference_us"] = ref_k["fp16_gate_up_m1_best"]["us"]
                if "reference_us" in c:
                    c["speedup_vs_reference"] = round(c["reference_us"] / c["us_per_launch"], 2)
    del fp16_raw

    # ---- the model's other decode projections (one GPU; recorded, not fatal:
    # the step's numbers above stand whatever happens here)
    adj = None
    if tp == 1 and not args.no_adjacent:
        try:
            adj = adjacent_shapes(b2g, torch, device, M)
        except Exception as e:
            adj = {"error": f"{type(e).__name__}: {e}"}

    # ---- CPU baseline (rank 0 at N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        qh = [t.cpu().numpy() for t in layers[0]["q0"]]
        cpu = cpu_reference_sample(qh, M, args.cpu_seconds)

    plan_gu, plan_dn = gu_op.plan(M), dn_op.plan(M)
    err = b2g.device_error()
    if world > 1:  # the worst device error over ranks (a peer wait that expired anywhere voids the run)
        e = torch.tensor([err], dtype=torch.int32, device=device)
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
        err = int(e.item())
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            # tensor parallel over one fixed workload at every N: strong scaling
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp8_e4m3", "data": "synthetic",
            "config": {
                "workload": (f"{LAYERS}-layer Llama-3.2-3B decode MLP stack, M={M}: RMSNorm(eps 1e-5) -> "
                             f"fused gate||up 3072->2x8192 + SiLU*up -> down 8192->3072 + residual; "
                             f"E4M3 weights, per-channel FP32 scales, fp16 activations, fp32 accumulate"),
                "hidden": HIDDEN, "intermediate": INTER, "layers": LAYERS, "m": M,
                "parallelism": f"tp{tp}" + (f" ({args.tp_mode} all-reduce"
                                            + (f", {args.tp_exchange} exchange" if args.tp_mode == "fused" else "")
                                            + ")" if tp > 1 else ""),
                "weights_per_step_bytes": bytes_rank * tp,
                "l2": (f"inputs larger than L2: {bytes_rank * tp / 1e9:.2f} GB of weights streamed per step "
                       "(L2 126 MB), no flush"),
                "timing": "CUDA graph replay of one step" if graph is not None else "direct launches",
                "data": "N(0,0.02) weights and N(0,1) hidden state from seeded device RNG",
            },
            "us_per_layer": round(ms_step * 1e3 / LAYERS, 3),
            "us_per_token_step": round(ms_step * 1e3, 2),
            "hbm_frac_of_measured": round(value * 1e3 / tp / hbm, 4),
            "roofline": roofline,
            "e2e": {"value": round(e2e_value, 4), "unit": "TB/s", "h2d_bytes_per_step": 2 * M * HIDDEN,
                    "d2h_bytes_per_step": 2 * M * HIDDEN, "ms_per_step": round(ms_e2e, 5),
                    "path": ("pinned host h -> b2g_stack_enqueue (C ABI) -> pinned host h" if st is not None
                             else f"pinned host h -> TPStack ({args.tp_mode} all-reduce) -> pinned host h")},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "detail": {
                **detail_extra,
                "reference_kernels_sm100": ref_k,
                "per_config": cfgs,
                "adjacent_decode_projections": adj,
                "direct_launch_ms_per_step": round(ms_direct / args.steps, 5),
                "gate_up_us_per_launch": round(ms_gu * 1e3, 3),
                "gate_up_alg_bytes": gu_b,
                "gate_up_achieved_gbs": round(gu_b / (ms_gu * 1e-3) / 1e9, 1),
                "down_us_per_launch": round(ms_dn * 1e3, 3),
                "down_alg_bytes": dn_b,
                "down_achieved_gbs": round(dn_b / (ms_dn * 1e-3) / 1e9, 1),
                "plan_gate_up": plan_gu, "plan_down": plan_dn, "device_error": err,
                "gpu": torch.cuda.get_device_name(device),
            },
        }
        if graph is None:
            line["detail"]["graph_error"] = graph_error
        print(json.dumps(line), flush=True)
    # Release the captured graph (it holds NCCL work when tp > 1) before the
    # process group goes: `run` is a bound method that keeps it alive.
    torch.cuda.synchronize()
    run = None
    if graph is not None:
        graph.reset()
        graph = None
    if tps is not None and tps.fused:
        dist.barrier()  # no rank unmaps a peer buffer another rank may still write
        tps.close_comm()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if err:
        sys.exit(f"device error {err} recorded during the run: the timing is void")


def run_reference(args):
    """The reference's CPU implementation of the path (its fp64 host loop,
    kernels/gemv_fp8.cu:313-323, compiled from its sources; the oracle's C
    port when oracle/_ref was not built) on all host cores.  One step = the
    three E4M3 GEMVs (gate, up, down) of `n` decode layers at M tokens, n
    chosen so that warm-up and timed steps together take about
    --ref-seconds; the layers cycle over two distinct weight sets (150 MB,
    beyond the host's caches).  RMSNorm, SiLU*up and the residual are not
    part of it: the reference has no CPU code for them."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    orc = load_module("oracle", ROOT / "oracle" / "oracle.py")
    syn = load_module("b2g_synthetic", PKG_DIR / "synthetic.py")
    M = args.m
    cores = orc.cpu_count()
    R = orc.ref()
    shapes = [(HIDDEN, INTER), (HIDDEN, INTER), (INTER, HIDDEN)]
    sets = []
    for l in range(2):
        qs = []
        for j, (K, N) in enumerate(shapes):
            q, _ = orc.quantize_e4m3(syn.weights(1000 + 3 * l + j, K, N), orc.SCALE_CHANNEL_FP32)
            qs.append(q)
        sets.append(qs)
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal((M, K), dtype=np.float32).astype(np.float16) for K, _ in shapes]
    if R is not None:
        kind = "reference"
        plans = [[R.ref_cpu_plan_create(q.ctypes.data, 1, K, N, cores) for q, (K, N) in zip(qs, shapes)]
                 for qs in sets]

        def layer(i):
            for pl, x, (K, N) in zip(plans[i % 2], xs, shapes):
                R.ref_cpu_plan_run(pl, np.ascontiguousarray(x.view(np.uint16)), M, np.empty((M, N), np.float64))
    else:
        kind = "port"
        os.environ.setdefault("OMP_NUM_THREADS", str(cores))

        def layer(i):
            for q, x in zip(sets[i % 2], xs):
                orc.gemv_loop(q, orc.WTYPE_FP8, x)
    t0 = time.perf_counter()
    layer(0)
    t_layer = time.perf_counter() - t0
    n = int(max(1, min(LAYERS, args.ref_seconds / (max(1, args.steps + args.warmup) * t_layer))))

    def step():
        for i in range(n):
            layer(i)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    if R is not None:
        for pls in plans:
            for pl in pls:
                R.ref_cpu_plan_destroy(pl)
    ms_step = sum(times) / len(times) * 1e3
    nbytes = n * sum(K * N + N * 4 + 2 * M * K + 2 * M * N for K, N in shapes)
    v = nbytes / (ms_step * 1e-3) / 1e12
    sample = (f"each step: {n} decode layer(s) x 3 E4M3 GEMVs (3072x8192, 3072x8192, 8192x3072) at M={M} "
              f"through the reference's fp64 host loop, K split over {cores} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "fp8_e4m3", "data": "synthetic",
        "config": {"workload": (f"{LAYERS}-layer Llama-3.2-3B decode MLP stack, M={M}: the reference's CPU "
                                f"loop over {n} of its layers per step (the GEMVs only: RMSNorm, SiLU*up and "
                                f"the residual have no CPU code in the reference)"),
                   "hidden": HIDDEN, "intermediate": INTER, "layers": LAYERS, "m": M,
                   "layers_per_step": n, "parallelism": "host cores"},
        "us_per_layer": round(ms_step * 1e3 / n, 1),
        "cpu_baseline": {"value": v, "unit": "TB/s", "cores": cores, "kind": kind, "sample": sample,
                         "seconds_timed": round(sum(times), 3)},
        "e2e": {"value": v, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# --timeline: where each launch of the decode step spends its time
# ---------------------------------------------------------------------------
TRACE_LIB = PKG_DIR / "libb200gemv_trace.so"
PHASES = ("start", "waited", "staged", "streamed", "end")


def run_timeline(args):
    """Per-CTA phase timestamps (%globaltimer) of every launch of one graph
    replay of the stack, from the trace build of the library (B2G_TRACE;
    built next to the library if missing).  Points: 0 start, 1 past the
    dependency wait, 2 inputs staged (after the CTA barrier), 3 this warp's
    weights streamed (thread 0), 4 end.  Prints one JSON line per M: per
    kernel, the means over the middle layers of each phase's median over
    CTAs, and of the critical-path marks measured from the launch's first
    release (its earliest CTA past the wait)."""
    import ctypes
    import torch
    build = load_module("b2g_build", PKG_DIR / "build.py")
    if not TRACE_LIB.exists():
        build.build(force=True, out=TRACE_LIB, defines=["B2G_TRACE"])
    b2g = load_module("b2g", PKG_DIR / "__init__.py", package=True)
    b2g.LIB_PATH = TRACE_LIB
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    st = b2g.Stack(HIDDEN, INTER, LAYERS, max_m=8)
    layers = make_layers(b2g, torch, device, 1, 0, (st.gate_up, st.down), 8)
    for i, L in enumerate(layers):
        st.set_layer(i, L["pgu"], L["sgu"], L["pd"], L["sd"])
    ws = torch.zeros(max(st.gate_up.workspace_bytes(), st.down.workspace_bytes()), dtype=torch.uint8, device=device)
    lib = ctypes.CDLL(str(TRACE_LIB))
    n_launch, n_cta = 64, 160
    grids = (st.gate_up.plan(8)["grid"], st.down.plan(8)["grid"])
    for M in sorted({args.m, 1}, reverse=True):
        h = torch.randn(M, HIDDEN, device=device).half()
        act = torch.empty(M, INTER, device=device, dtype=torch.float16)
        g = _graph_of(torch, lambda: st.enqueue(h, act, ws))
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        buf = np.zeros((n_launch, n_cta, 8), dtype=np.uint64)
        if lib.b2g_debug_trace(ctypes.c_void_p(buf.ctypes.data), ctypes.c_size_t(buf.nbytes)) != 0:
            raise RuntimeError("b2g_debug_trace failed")
        g.reset()
        nl = 2 * LAYERS
        order = np.argsort(buf[:, 0, 0].astype(np.int64))[-nl:]  # the last replay's launches, in time order
        rows = []
        for i, slot in enumerate(order):
            t = buf[slot, :grids[i % 2], :5].astype(np.int64)
            rows.append({k: (int(t[:, j].min()), int(np.median(t[:, j])), int(t[:, j].max()))
                         for j, k in enumerate(PHASES)})
        mid = range(4, nl - 4)

        def mean(kind, f):
            return round(float(np.mean([f(i) for i in mid if i % 2 == kind])) / 1e3, 3)
        out = {"timeline": "stack per-layer mode, one graph replay", "m": M, "layers": LAYERS,
               "us_per_layer": round((rows[nl - 4]["waited"][0] - rows[4]["waited"][0]) / ((nl - 8) / 2) / 1e3, 3)}
        for kind, name in ((0, "gate_up"), (1, "down")):
            out[name] = {
                "grid": grids[kind],
                "release_after_previous_last_end": mean(kind, lambda i: rows[i]["waited"][0] - rows[i - 1]["end"][2]),
                "wait_exit_spread": mean(kind, lambda i: rows[i]["waited"][2] - rows[i]["waited"][0]),
                "staging_median": mean(kind, lambda i: rows[i]["staged"][1] - rows[i]["waited"][1]),
                "stream_median": mean(kind, lambda i: rows[i]["streamed"][1] - rows[i]["staged"][1]),
                "epilogue_median": mean(kind, lambda i: rows[i]["end"][1] - rows[i]["streamed"][1]),
                "last_staged_after_release": mean(kind, lambda i: rows[i]["staged"][2] - rows[i]["waited"][0]),
                "last_streamed_after_release": mean(kind, lambda i: rows[i]["streamed"][2] - rows[i]["waited"][0]),
                "last_end_after_release": mean(kind, lambda i: rows[i]["end"][2] - rows[i]["waited"][0]),
            }
        print(json.dumps(out), flush=True)
    err = b2g.device_error()
    if err:
        raise RuntimeError(f"device error {err}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--m", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0,
                    help="--impl reference: host time budget of warm-up + timed steps")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ref-kernels", action="store_true", help="skip timing the reference's GPU kernels")
    ap.add_argument("--no-adjacent", action="store_true", help="skip timing qkv_proj / o_proj / lm_head")
    ap.add_argument("--tp-mode", choices=["fused", "nccl"], default="fused",
                    help="N > 1: all-reduce fused into the GEMVs over peer memory, or NCCL")
    ap.add_argument("--tp-exchange", choices=["reduce", "gather_kernel", "gather_launch"], default="reduce",
                    help="N > 1, fused: how the ranks' rows are summed (TPStack.exchange)")
    ap.add_argument("--pipe", choices=["auto", "registers", "tma"], default="auto",
                    help="how the GEMV launches feed their weights (B2G_OPT_PIPE)")
    ap.add_argument("--math", choices=["mma", "ffma"], default="mma",
                    help="the GEMV launches' math: tensor-core mma.sync, or the CUDA-core FFMA variant (B2G_OPT_MATH)")
    ap.add_argument("--stack-mode", choices=["per_layer", "persistent", "persistent_tma"], default="per_layer",
                    help="one GPU: the stack's execution mode for the timed step")
    ap.add_argument("--timeline", action="store_true",
                    help="one GPU: per-phase timestamps of the stack's launches (trace build), not the bench line")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decode-MLP layers (28 = Llama-3.2-3B; fewer only for small profiling captures)")
    args = ap.parse_args()
    globals()["LAYERS"] = args.layers
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.timeline:
        run_timeline(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
