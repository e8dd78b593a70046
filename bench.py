#!/usr/bin/env python
"""Decode-MLP benchmark: 28-layer Llama-3.2-3B MLP stack with E4M3 weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--m 8] [--impl ours|reference]

One step = one decode step of M tokens through all 28 layers
(RMSNorm -> fused gate||up + SiLU*up -> down + residual), weights resident in
HBM (2.12 GB of E4M3 per step, far above the 126 MB L2, so every step streams
from HBM without an explicit flush).  With N > 1 (torchrun), the stack is
tensor-parallel: gate/up column shards, down K shards, and an NCCL fp16
all-reduce of the 3072-wide partials per layer.

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
def make_layers(b2g, torch, device, tp: int, rank: int, ops, M: int):
    """28 layers of N(0, 0.02) weights, E4M3 per-channel FP32 (quantised over
    the full matrix, then sharded), prepacked for this rank."""
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
                       "q0": (qg, qu, qd) if l == 0 else None})
    return layers


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
        # One GPU: the library's stack (one cooperative launch for all layers).
        st = b2g.Stack(HIDDEN, INTER, LAYERS, max_m=M)
        gu_op, dn_op = st.gate_up, st.down
    else:
        st = None
        gu_op = b2g.GemvOp(HIDDEN, inter, max_m=M,
                           fuse=b2g.FUSE_GATE_UP_SILU | b2g.FUSE_RMSNORM_INPUT)
        dn_op = b2g.GemvOp(inter, HIDDEN, max_m=M,
                           fuse=b2g.FUSE_RESIDUAL_ADD if rank == 0 else b2g.FUSE_NONE)
    layers = make_layers(b2g, torch, device, tp, rank, (gu_op, dn_op), M)
    if st is not None:
        for i, L in enumerate(layers):
            st.set_layer(i, L["pgu"], L["sgu"], L["pd"], L["sd"])
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
        for i, L in enumerate(layers):
            nxt = layers[(i + 1) % LAYERS]
            gu_op.enqueue(h, L["pgu"], L["sgu"], y=act, workspace=ws, pdl=True,
                          prefetch=(dn_op, L["pd"]))
            dn_op.enqueue(act, L["pd"], L["sd"], y=h, residual=h if rank == 0 else None,
                          workspace=ws, pdl=True, prefetch=(gu_op, nxt["pgu"]))
            if tp > 1:
                dist.all_reduce(h)

    def step_stack():
        st.enqueue(h, act, ws)

    step = step_stack if st is not None else step_ops
    launches_per_step = (LAYERS + 31) // 32 if st is not None else 2 * LAYERS

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
        # The per-layer launch path of the same stack, for comparison.
        st.set_mode("per_layer")
        for _ in range(3):
            step_stack()
        ms_pl = timed(step_stack, reps) / reps
        st.set_mode("persistent")
        detail_extra["per_layer_launches_ms_per_step"] = round(ms_pl, 5)
        detail_extra["per_layer_launches_us_per_layer"] = round(ms_pl * 1e3 / LAYERS, 3)

    # ---- dominant kernel.  One GPU: the stack kernel is the step's only
    # launch, so its duration is the graph replay time per step.
    if st is not None:
        achieved = bytes_rank / (ms_step * 1e-3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get(f"stack_m{M}")
        roofline = {"kernel": "stack_kernel<1> (28 layers: RMSNorm + gate||up + SiLU*up, down + residual)",
                    "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(achieved / hbm, 4), "traffic": traffic,
                    "peak_source": f"{peak_kind} hbm_gbs (STREAM-style copy)",
                    "alg_bytes_per_launch": bytes_rank,
                    "us_per_launch": round(ms_step * 1e3, 3)}

    # ---- per-op kernels: fused RMSNorm + gate||up + SiLU*up, 28 layers back to back
    def gu_sweep():
        for i, L in enumerate(layers):
            gu_op.enqueue(h, L["pgu"], L["sgu"], y=act, workspace=ws, pdl=True,
                          prefetch=(gu_op, layers[(i + 1) % LAYERS]["pgu"]))
    for _ in range(3):
        gu_sweep()
    ms_gu = timed(gu_sweep, reps) / (reps * LAYERS)
    if st is None:
        achieved = gu_b / (ms_gu * 1e-3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get(f"gate_up_m{M}_tp{tp}")
        roofline = {"kernel": "gemv_streamk_kernel<2,1,0> (RMSNorm + gate||up + SiLU*up)",
                    "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(achieved / hbm, 4), "traffic": traffic,
                    "peak_source": f"{peak_kind} hbm_gbs (STREAM-style copy)",
                    "alg_bytes_per_launch": gu_b, "us_per_launch": round(ms_gu * 1e3, 3)}

    def dn_sweep():
        for i, L in enumerate(layers):
            dn_op.enqueue(act, L["pd"], L["sd"], y=h, residual=h if rank == 0 else None,
                          workspace=ws, pdl=True, prefetch=(dn_op, layers[(i + 1) % LAYERS]["pd"]))
    for _ in range(3):
        dn_sweep()
    ms_dn = timed(dn_sweep, reps) / (reps * LAYERS)

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

    # ---- CPU baseline (rank 0 at N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        qh = [t.cpu().numpy() for t in layers[0]["q0"]]
        cpu = cpu_reference_sample(qh, M, args.cpu_seconds)

    plan_gu, plan_dn = gu_op.plan(M), dn_op.plan(M)
    err = b2g.device_error()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "fp8_e4m3", "data": "synthetic",
            "config": {
                "workload": (f"28-layer Llama-3.2-3B decode MLP stack, M={M}: RMSNorm(eps 1e-5) -> "
                             f"fused gate||up 3072->2x8192 + SiLU*up -> down 8192->3072 + residual; "
                             f"E4M3 weights, per-channel FP32 scales, fp16 activations, fp32 accumulate"),
                "hidden": HIDDEN, "intermediate": INTER, "layers": LAYERS, "m": M,
                "parallelism": f"tp{tp}", "weights_per_step_bytes": bytes_rank * tp,
                "l2": "inputs larger than L2: 2.12 GB of weights streamed per step (L2 126 MB), no flush",
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
                             else "pinned host h -> b2g_enqueue_ex per layer + NCCL all-reduce -> pinned host h")},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "detail": {
                **detail_extra,
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
    if graph is not None:
        del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    orc = load_module("oracle", ROOT / "oracle" / "oracle.py")
    # E4M3 weights of layer 0 with the FP32 per-channel rule, generated on the host
    syn = load_module("b2g_synthetic", PKG_DIR / "synthetic.py")
    qs = []
    for j, (K, N) in enumerate(((HIDDEN, INTER), (HIDDEN, INTER), (INTER, HIDDEN))):
        q, _ = orc.quantize_e4m3(syn.weights(1000 + j, K, N), orc.SCALE_CHANNEL_FP32)
        qs.append(q)
    for _ in range(args.warmup and 1):
        pass
    per = []
    for _ in range(max(1, args.steps)):
        per.append(cpu_reference_sample(qs, args.m, min_seconds=args.cpu_seconds / max(1, args.steps)))
    v = statistics.median(p["value"] for p in per)
    cb = dict(per[0])
    cb["value"] = v
    us_layer = statistics.median(p["us_per_layer"] for p in per)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": us_layer * LAYERS / 1e3,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "fp8_e4m3", "data": "synthetic",
        "config": {"workload": (f"28-layer Llama-3.2-3B decode MLP stack, M={args.m} (CPU sample: "
                                f"layer 0's three E4M3 GEMVs, scaled to the stack)"),
                   "hidden": HIDDEN, "intermediate": INTER, "layers": LAYERS, "m": args.m,
                   "parallelism": "host cores"},
        "us_per_layer": us_layer,
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--m", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
