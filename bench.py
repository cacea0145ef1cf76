#!/usr/bin/env python
"""MoE verify-layer throughput on B200 (SpecMoE FusedMoE path), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2-256] [--impl reference]

A step is one pass of the MoE layer (route, expert FFN = gate/up GEMM + SiLU*mul + down
GEMM, combine) over one verify batch of T synthetic tokens, inputs resident in HBM.  The
timed region is K back-to-back replays of a CUDA graph holding one layer call, between
CUDA events on the launching stream, bracketed by a barrier and a device synchronise,
max over ranks, after a soak of the same replays (the eager, ctypes-per-call time is
reported beside it).  Expert weights (2.8 GB for Mixtral-8x7B) are far larger than the
126 MB L2, so consecutive steps do not reuse weights from L2.  The FFN kernel's duration
for the roofline comes from the library's device-side timers over exactly the K timed
launches; the timed output is checked against the fp32 CPU oracle (``parity``).

N > 1: expert parallelism (ae_b200/ep.py), strong scaling: the same verify batch of T
tokens per step, T/N on each rank; rank r holds experts [r*E/N, (r+1)*E/N); the kernels
move the rows over NVLink peer memory (``--ep-transport p2p``, the default; NCCL
all-to-alls are timed beside it), the whole batch's output is checked against the
oracle on rank 0, and Mixtral-8x22B (C5) runs the same way.

Extra keys: roofline (dominant kernel = the fused expert-FFN kernel, HBM bound), parity,
cpu_baseline (the CPU oracle port of the reference's arithmetic on this host), e2e
(FusedMoE.forward with host inputs copied in and the output copied out every step),
clocks, gpu_launches, kernels_us (per-kernel µs from a staged pass), sweep (other verify
batch sizes), c1_flushed (C1 with the L2 flushed), c5_single_gpu, prefill_t2048 (the
prefill-sized call on the CTA-pair path against the measured bf16 GEMM peaks), and further
blocks.

``--impl reference``: rank 0 times the reference's arithmetic on the host cores (the
reference has no CPU expert path of its own; its Triton GPU kernel is the GPU side), the
other ranks exit without work.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE verify-layer tokens/sec"
UNIT = "tokens/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while work runs."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 9:
                continue
            self.rows.append((time.time(), parts))

    def mark(self):
        return time.time()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [p for (t, p) in self.rows if t0 <= t <= t1]
        if self.uuid:
            mine = [p for p in rows if self.uuid in p[0] or p[0] in self.uuid]
            rows = mine or rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(p[1]) for p in rows if p[1].replace(".", "").isdigit()]
        smax = [float(p[2]) for p in rows if p[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for p in rows:
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max(float(p[3]) for p in rows if p[3].replace(".", "").isdigit())
                if any(p[3].replace(".", "").isdigit() for p in rows) else None}


def device_uuid(dev):
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


# ---------------------------------------------------------------------------- CPU arm

def cpu_port_time(cfg, seed: int, max_seconds: float = 20.0, max_reps: int = 5, pool_cpu=None, x=None,
                  logits=None):
    """Time the CPU oracle port of the layer (routing + bf16-storage expert FFN) on all host
    threads.  Returns (tokens_per_s, seconds_per_layer, threads, reps)."""
    from oracle import moe_oracle as mo  # the CPU baseline leg is the one bench leg allowed to use it
    from ae_b200 import configs

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if pool_cpu is None:
        pool_cpu = configs.make_pool(cfg, "cpu", seed=seed)
    if x is None:
        x, logits = configs.make_inputs(cfg, "cpu", seed=seed)
    pages = torch.arange(cfg.E)

    def one():
        w, ids = mo.select_experts(logits, cfg.k, cfg.renormalize)
        return mo.stack_fused_moe(x, pool_cpu, pages, w, ids, compute_dtype=torch.bfloat16)

    one()  # warm-up (thread pool, page faults)
    times = []
    t_start = time.perf_counter()
    while len(times) < max_reps and (time.perf_counter() - t_start) < max_seconds:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return cfg.T / med, med, threads, len(times)


def config_of(cfg, world: int) -> dict:
    """The ``config`` object of the JSON line, the same on both arms for a given N."""
    if world == 1:
        return {"workload": cfg.name, "T": cfg.T, "H": cfg.H, "I": cfg.I, "E": cfg.E, "k": cfg.k,
                "parallelism": "single",
                "l2": "inputs larger than L2 (expert weights %.2f GB per step)" % (cfg.weight_bytes() / 1e9)}
    E_loc, T_r = cfg.E // world, cfg.T // world
    return {"workload": cfg.name + f", expert-parallel over {world} GPUs ({T_r} tokens and {E_loc} experts per GPU)",
            "T": cfg.T, "T_per_gpu": T_r, "H": cfg.H, "I": cfg.I, "E": cfg.E, "k": cfg.k,
            "experts_per_gpu": E_loc, "parallelism": f"ep{world}",
            "l2": "inputs larger than L2 (expert weights %.2f GB per GPU per step)" % (cfg.weight_bytes(E_loc) / 1e9)}


def run_reference_arm(args, cfg, rank, world):
    if rank != 0:
        return
    from ae_b200 import configs
    torch.manual_seed(0)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    pool_cpu = configs.make_pool(cfg, "cpu", seed=0)
    x, logits = configs.make_inputs(cfg, "cpu", seed=0)
    from oracle import moe_oracle as mo
    pages = torch.arange(cfg.E)

    def step():
        w, ids = mo.select_experts(logits, cfg.k, cfg.renormalize)
        mo.stack_fused_moe(x, pool_cpu, pages, w, ids, compute_dtype=torch.bfloat16)

    t0 = time.perf_counter()
    step()
    one = time.perf_counter() - t0
    budget = 150.0
    steps, warm = args.steps, args.warmup
    if one * (steps + warm) > budget:
        steps = max(1, int(budget / one) - 1)
        warm = 1
    for _ in range(max(0, warm - 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    el = time.perf_counter() - t0
    value = cfg.T * steps / el
    sample = (f"{steps} full layer calls of {cfg.T} tokens (all {cfg.E} experts, bf16 storage, fp32 accumulate "
              f"in torch CPU GEMMs) on {threads} host threads")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": 1000 * el / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_of(cfg, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU expert path (FusedMoE.forward_cpu is unreachable); this arm runs the "
                "oracle's CPU restatement of stack_fused_moe + select_experts",
    }
    emit(line)


# ---------------------------------------------------------------------------- GPU arm

def algorithmic(cfg, touched: int, T: int | None = None):
    """Algorithmic bytes (the survey's measurement rules: touched experts' weights, tokens
    in and out, router logits; intermediate caches not counted) of the FFN kernel
    (touched weights + the token rows it reads) and of the whole layer, and the layer's
    flops."""
    H, I, E = cfg.H, cfg.I, cfg.E
    T = cfg.T if T is None else T
    ffn = touched * 3 * H * I * 2 + T * H * 2
    layer = touched * 3 * H * I * 2 + 2 * T * H * 2 + T * E * 2
    flops = 6 * H * I * T * cfg.k
    return ffn, layer, flops


def stage_means(tm: dict, busy: bool = False) -> dict:
    """Mean µs per call of each stage of the chain from the library's stage clock (a stage
    runs from its first kernel block passing its wait to the next stage's; with ``busy``,
    the part until the stage's kernel finished)."""
    out = {}
    key = "stage_busy_ns" if busy else "stage_ns"
    for name, ns in tm.get(key, {}).items():
        n = tm["stage_calls"][name]
        if n:
            out[name] = round(ns / n / 1e3, 2)
    return out


def touched_experts(logits, k: int, renormalize: bool = True) -> int:
    """Experts that at least one token picks, from the library's own routing of the logits."""
    from ae_b200 import ops
    _, ids = ops.topk(logits, k, renormalize)
    return int((torch.bincount(ids.flatten().long(), minlength=logits.shape[1]) > 0).sum())


def graph_of(fn, dev, with_stream: bool = False):
    """Capture one call of ``fn`` into a CUDA graph.  The warm call runs on the stream the
    capture then uses, so the library's per-stream workspace exists before the capture and
    the graph holds the kernels only (no allocation, no workspace initialisation)."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        fn()
    torch.cuda.synchronize(dev)
    return (g, side) if with_stream else g


def timed_steps(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / 1000.0


def load_traffic(cfg_key):
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(cfg_key)
    except Exception:
        return None


def parity_vs_oracle(out, x, logits, pool_cpu, pages, k, renormalize, ids=None, ref=None):
    """Parity of a layer output against the fp32 CPU oracle on the same inputs: routing ids
    bit-exact, max-abs and relative-L2 error, and the bar (max-abs <= 2e-2, or the
    reference arithmetic's own error where that is larger; relative-L2 <= 1e-2)."""
    from oracle import moe_oracle as mo  # the checker only
    xc, lc = x.cpu(), logits.cpu()
    rw, rids = mo.select_experts(lc, k, renormalize)
    pc = pages.cpu()
    ref = mo.stack_fused_moe(xc, pool_cpu, pc, rw, rids, rounding="fp32")
    ref_r = mo.stack_fused_moe(xc, pool_cpu, pc, rw, rids, rounding="reference").float()
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    ref_err = float((ref_r - ref).abs().max())
    bar = max(2e-2, ref_err)
    res = {"max_abs": max_abs, "rel_l2": rel, "reference_rounding_max_abs": ref_err,
           "bar": {"max_abs": bar, "rel_l2": 1e-2}, "within_bar": bool(max_abs <= bar and rel <= 1e-2),
           "against": "fp32 CPU oracle (oracle/moe_oracle.py) on the timed inputs"}
    if ids is not None:
        res["ids_exact"] = bool((ids.cpu().numpy() == rids).all())
    return res


def run_ours(args, cfg, rank, world, dev):
    from ae_b200 import configs, ops
    from ae_b200.layers.FusedMoE import FusedMoE

    hbm_peak, tc_peak, peak_kind = peaks()
    stream = torch.cuda.current_stream(dev)
    pool = configs.make_pool(cfg, dev, seed=rank)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=rank)
    out = torch.empty_like(x)
    Tk = cfg.T * cfg.k

    def step():
        ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, out=out)

    sampler = ClockSampler(device_uuid(dev))
    sampler.start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    # eager launches (a host-side ctypes call per layer), for reference
    eager = timed_steps(step, args.steps, stream)
    # the timed region replays a CUDA graph of one layer call per step (the reference
    # engine captures its verify step as well); launches are the same three kernels
    graph, cap_stream = graph_of(step, dev, with_stream=True)
    ws = ops.Workspace.lookup(dev, cap_stream)
    # soak with the replays that are then timed, so the timed region starts in the power
    # and clock state it runs in
    t_soak = time.time()
    soak_end = t_soak + args.soak
    while True:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize(dev)
        if time.time() >= soak_end:
            break
    ops.read_timers(ws, reset=True)
    torch.cuda.synchronize(dev)
    elapsed = timed_steps(graph.replay, args.steps, stream)
    torch.cuda.synchronize(dev)
    t_timed_end = time.time()
    # device-side timer of the FFN kernel over exactly the timed launches
    tm = ops.read_timers(ws)
    clocks = sampler.summary(t_soak, t_timed_end)
    sampler.stop()
    if tm["ffn_launches"] != args.steps:
        raise RuntimeError(f"FFN timer saw {tm['ffn_launches']} launches in {args.steps} timed steps")
    ffn_s = tm["ffn_ns"] / tm["ffn_launches"] * 1e-9
    stages = {"stage_us": stage_means(tm), "kernel_busy_us": stage_means(tm, busy=True)}
    if not torch.isfinite(out.float()).all():
        raise RuntimeError("non-finite layer output")
    timed_out = out.clone()

    # staged pass: per-kernel durations from CUDA events between the three launches of a
    # layer call (eager; a cross-check of the in-graph FFN timer)
    L = ops.StagedLayer(cfg.T, cfg.E, cfg.k, cfg.H, cfg.I, x.dtype, dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.staged_steps)]
    for i in range(3):
        L.route(logits, x, cfg.renormalize)
        L.ffn(pool, pages, x)
        L.combine(out)
    for e in evs:
        e[0].record(stream)
        L.route(logits, x, cfg.renormalize)
        e[1].record(stream)
        L.ffn(pool, pages, x)
        e[2].record(stream)
        L.combine(out)
        e[3].record(stream)
    torch.cuda.synchronize(dev)
    names = ["route", "ffn", "combine"]
    kern_us = {n: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs) * 1000.0 for i, n in enumerate(names)}
    v = L.views()
    off = v["expert_off"].cpu()
    touched = int(((off[1:] - off[:-1]) > 0).sum())
    splits = ops.splits(cfg.E, cfg.H, cfg.I, Tk)
    ffn_bytes, layer_bytes, flops = algorithmic(cfg, touched)
    del L

    # end to end through the drop-in module: host inputs in, host output out, every step
    moe = FusedMoE(cfg.E, cfg.k, cfg.H, cfg.I, params_dtype=x.dtype, renormalize=cfg.renormalize, tp_size=1)
    moe.ws.gpu_cache = pool
    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    dx = torch.empty_like(x)
    dl = torch.empty_like(logits)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        r = moe(dx, dl, pages)
        hout.copy_(r, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    e2e_el = timed_steps(e2e_step, args.steps, stream)

    # parity of the timed output against the fp32 oracle (rank 0, N = 1), and the routing
    # ids of one more call on the same inputs (whose output must equal the timed one)
    parity = None
    pool_cpu = None
    if rank == 0 and not args.no_parity:
        pool_cpu = pool.cpu()
        w_chk = torch.empty(cfg.T, cfg.k, dtype=torch.float32, device=dev)
        ids_chk = torch.empty(cfg.T, cfg.k, dtype=torch.int32, device=dev)
        again = ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, topk_weights=w_chk, topk_ids=ids_chk)
        torch.cuda.synchronize(dev)
        parity = parity_vs_oracle(timed_out, x, logits, pool_cpu, pages, cfg.k, cfg.renormalize, ids=ids_chk)
        parity["repeat_bitwise_equal"] = bool(torch.equal(again, timed_out))

    # other verify batch sizes of the same layer (N = 1)
    sweep = {}
    if not args.no_sweep:
        for Ts in args.sweep:
            if Ts == cfg.T:
                continue
            xs, ls = configs.make_inputs(cfg, dev, seed=1, T=Ts)
            os_ = torch.empty_like(xs)

            def s():
                ops.moe_forward(xs, ls, pool, pages, cfg.k, cfg.renormalize, out=os_)

            for _ in range(5):
                s()
            gs = graph_of(s, dev)
            for _ in range(3):
                gs.replay()
            torch.cuda.synchronize(dev)
            n = max(10, args.steps // 2)
            el_s = timed_steps(gs.replay, n, stream)
            us = el_s / n * 1e6
            t_s = touched_experts(ls, cfg.k, cfg.renormalize)
            sweep[f"T{Ts}"] = {"us_per_layer": round(us, 2), "tokens_per_s": round(Ts / (el_s / n), 1),
                               "experts_touched": t_s,
                               "layer_hbm_frac": round(algorithmic(cfg, t_s, Ts)[1] / (el_s / n) / 1e9 / hbm_peak, 4)}
            del gs

    # the whole MixtralMoE block (gate + experts): gate fused into the routing launch vs.
    # the reference's arrangement of a separate half-precision gate GEMM (cuBLAS, like
    # ReplicatedLinear) followed by the layer
    gated = None
    if not args.no_sweep:
        xg, wg = configs.make_gate_inputs(cfg, dev, seed=2)
        og = torch.empty_like(xg)

        def fused():
            ops.moe_forward_gated(xg, wg, pool, pages, cfg.k, cfg.renormalize, out=og)

        def unfused():
            lg = torch.matmul(xg, wg.t())
            ops.moe_forward(xg, lg, pool, pages, cfg.k, cfg.renormalize, out=og)

        gated = {"api": "ae_b200.layers.mixtral_moe.MixtralMoE.forward (smb_moe_forward_gated)",
                 "timing": "graph replays, the two arrangements alternated 4 times, median"}
        graphs = {}
        for name, fn in (("fused_gate", fused), ("separate_gate_gemm", unfused)):
            for _ in range(5):
                fn()
            graphs[name] = graph_of(fn, dev)
        samples = {name: [] for name in graphs}
        n = max(10, args.steps // 4)
        for _ in range(4):
            for name, gg in graphs.items():
                for _ in range(3):
                    gg.replay()
                samples[name].append(timed_steps(gg.replay, n, stream) / n * 1e6)
        for name, sv in samples.items():
            gated[f"{name}_us_per_layer"] = round(statistics.median(sv), 2)
        del graphs

    # the small configuration of the reference's CPU path (C1), L2 flushed between replays
    c1 = None
    if not args.no_sweep:
        c1 = bench_flushed_config(configs.BY_KEY["c1"], dev, stream, max(20, args.steps), hbm_peak)

    # Mixtral-8x22B (C5, T = 512) on this GPU: the expert-parallel configuration's N = 1 point
    c5 = None
    if not args.no_sweep:
        c5 = bench_single_config(configs.BY_KEY["c5"], dev, stream, max(10, args.steps // 2), hbm_peak)

    # prefill-sized call (survey row f4): C2 at T = 2048 on the CTA-pair path
    prefill = None
    if not args.no_sweep:
        prefill = bench_prefill_config(configs.BY_KEY["c2-2048"], dev, stream, max(40, args.steps), args.no_parity)

    # the fine-grained configuration with a shared expert (60 routed experts of I 1408,
    # top-4, shared expert I 5632 as 4 pseudo-experts in the same launch, Zipf routing)
    fine = None
    if not args.no_sweep:
        fine = bench_shared_config(configs.BY_KEY["c3"], dev, stream, max(10, args.steps // 2), hbm_peak)

    # the 32-layer verify step (Mixtral-8x7B architecture, batch 4 x 32-token draft tree on
    # a 2048-token KV cache), MoE layers isolated by CUDA events around each MoE call
    verify = None
    if not args.no_sweep and not args.no_verify:
        verify = bench_verify_step(dev, stream, hbm_peak)

    # expert pages streamed from page-locked host memory while the layer runs (all 8
    # experts cross PCIe, as with the reference's decode_weight_cache_ratio = 0)
    streamed = None
    if not args.no_sweep:
        streamed = bench_streaming(cfg, pool, pages, x, logits, dev, stream)

    # CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        if pool_cpu is None:
            pool_cpu = pool.cpu()
        tps, sec, threads, reps = cpu_port_time(cfg, 0, pool_cpu=pool_cpu, x=x.cpu(), logits=logits.cpu())
        cpu = {"value": round(tps, 2), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{reps} full layer calls of {cfg.T} tokens ({cfg.name}), median {sec * 1000:.1f} ms, "
                         f"oracle CPU restatement, bf16 storage / fp32 accumulate, {threads} threads"}
    del pool_cpu

    if rank != 0:
        return
    step_s = elapsed / args.steps
    achieved = ffn_bytes / ffn_s / 1e9
    traffic = load_traffic(args.config)
    line = {
        "metric": METRIC,
        "value": round(world * cfg.T * args.steps / elapsed, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_s * 1000, 5),
        "us_per_layer": round(step_s * 1e6, 2),
        "launch_mode": "cuda_graph (one layer call per replay)",
        "eager_us_per_layer": round(eager / args.steps * 1e6, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: expert weights N(0,0.02) bf16, tokens N(0,1), router logits x@Wr^T "
                f"(Wr std {cfg.router_std:.4g})",
        "config": config_of(cfg, world),
        "layout": {"experts_touched": touched, "splits": splits},
        "roofline": {"bound": "hbm", "kernel": "ffn_gemm_kernel (gate/up + down, one launch)",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                     "alg_bytes_per_launch": ffn_bytes,
                     "duration_us": round(ffn_s * 1e6, 2),
                     "timing": f"device timer of every FFN launch in the timed region ({tm['ffn_launches']} "
                               "launches: first CTA past its wait on the router to the last CTA done, "
                               "%globaltimer), averaged",
                     "traffic": traffic},
        "layer_roofline": {"alg_bytes": layer_bytes, "achieved_gbs": round(layer_bytes / step_s / 1e9, 1),
                           "frac_hbm": round(layer_bytes / step_s / 1e9 / hbm_peak, 4),
                           "tflops": round(flops / step_s / 1e12, 2),
                           "frac_tensor": round(flops / step_s / 1e12 / tc_peak, 4)},
        "stages_us": stages,
        "kernels_us": {n: round(u, 2) for n, u in kern_us.items()},
        "kernels_timing": "CUDA events between eager launches of the three kernels (staged pass after the timed "
                          "region)",
        "parity": parity,
        "cpu_baseline": cpu,
        "e2e": {"value": round(world * cfg.T * args.steps / e2e_el, 2), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * x.element_size() + logits.numel() * logits.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "api": "ae_b200.layers.FusedMoE.FusedMoE.forward"},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
        "sweep": sweep,
        "c1_flushed": c1,
        "c5_single_gpu": c5,
        "prefill_t2048": prefill,
        "gated_block": gated,
        "shared_expert_config": fine,
        "verify_32_layers": verify,
        "streamed_pages": streamed,
    }
    emit(line)


def bench_single_config(cfg, dev, stream, n, hbm_peak):
    """Graph-replay time of one layer call of another routed configuration on this GPU
    (inputs larger than L2), with its HBM roofline fraction and the FFN kernel's device timer."""
    from ae_b200 import configs, ops
    pool = configs.make_pool(cfg, dev, seed=0)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=0)
    out = torch.empty_like(x)

    def step():
        ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, out=out)

    for _ in range(3):
        step()
    gr, cs = graph_of(step, dev, with_stream=True)
    ws = ops.Workspace.lookup(dev, cs)
    for _ in range(3):
        gr.replay()
    ops.read_timers(ws, reset=True)
    el = timed_steps(gr.replay, n, stream)
    tm = ops.read_timers(ws)
    touched = touched_experts(logits, cfg.k, cfg.renormalize)
    ffn_b, layer_b, flops = algorithmic(cfg, touched)
    t = el / n
    ffn_s = tm["ffn_ns"] / max(1, tm["ffn_launches"]) * 1e-9
    del gr, pool
    torch.cuda.empty_cache()
    return {"workload": cfg.name, "T": cfg.T, "us_per_layer": round(t * 1e6, 2),
            "tokens_per_s": round(cfg.T / t, 1), "experts_touched": touched, "alg_bytes": layer_b,
            "layer_hbm_frac": round(layer_b / t / 1e9 / hbm_peak, 4),
            "ffn_us": round(ffn_s * 1e6, 2), "ffn_hbm_frac": round(ffn_b / ffn_s / 1e9 / hbm_peak, 4),
            "splits": ops.splits(cfg.E, cfg.H, cfg.I, cfg.T * cfg.k),
            "api": "ae_b200.ops.moe_forward (smb_moe_forward)", "timing": f"{n} graph replays"}


def bench_prefill_config(cfg, dev, stream, n, no_parity=False):
    """Prefill-sized layer call (C2 at T = 2048: 256 routed slots per expert on average, the
    CTA-pair path with the 2-SM MMA): graph replays after a soak of the same replays, TFLOP/s
    of the layer and of the FFN kernel's device timer against the measured bf16 GEMM peaks
    (sustained: a kernel timed inside a long, power-capped loop, like this one), and the
    output checked against the fp32 CPU oracle."""
    from ae_b200 import configs, ops
    pool = configs.make_pool(cfg, dev, seed=0)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=0)
    out = torch.empty_like(x)
    ids = torch.empty(cfg.T, cfg.k, dtype=torch.int32, device=dev)

    def step():
        ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, out=out, topk_ids=ids)

    for _ in range(3):
        step()
    gr, cs = graph_of(step, dev, with_stream=True)
    ws = ops.Workspace.lookup(dev, cs)
    sampler = ClockSampler(device_uuid(dev))
    sampler.start()
    t_soak = time.time()
    while time.time() < t_soak + 1.5:
        timed_steps(gr.replay, 10, stream)
    ops.read_timers(ws, reset=True)
    el = timed_steps(gr.replay, n, stream)
    t1w = time.time()
    tm = ops.read_timers(ws)
    time.sleep(0.15)
    clocks = sampler.summary(t_soak + 0.5, t1w + 0.1)  # the settled part of the soak and the timed replays
    sampler.stop()
    _, _, flops = algorithmic(cfg, cfg.E)
    t = el / n
    ffn_s = tm["ffn_ns"] / max(1, tm["ffn_launches"]) * 1e-9
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        sus, burst, kind = float(pk["bf16_tflops_sustained"]), float(pk["bf16_tflops"]), "measured"
    except Exception:
        sus, burst, kind = 1400.0, 1590.0, "fallback"
    res = {"workload": cfg.name, "T": cfg.T, "path": "CTA pairs (tcgen05.mma.cta_group::2), two launches",
           "us_per_layer": round(t * 1e6, 2), "tokens_per_s": round(cfg.T / t, 1),
           "layer_tflops": round(flops / t / 1e12, 1), "ffn_us": round(ffn_s * 1e6, 2),
           "ffn_tflops": round(flops / ffn_s / 1e12, 1),
           "frac_of_sustained_bf16_peak": {"layer": round(flops / t / 1e12 / sus, 4),
                                           "ffn": round(flops / ffn_s / 1e12 / sus, 4)},
           "frac_of_burst_bf16_peak": {"layer": round(flops / t / 1e12 / burst, 4),
                                       "ffn": round(flops / ffn_s / 1e12 / burst, 4)},
           "peaks_tflops": {"sustained": sus, "burst": burst, "kind": kind},
           "stages_us": stage_means(tm), "kernel_busy_us": stage_means(tm, busy=True),
           "clocks": clocks, "timing": f"{n} graph replays after a 1.5 s soak of the same replays (clocks: soak and timed replays)",
           "api": "ae_b200.ops.moe_forward (smb_moe_forward)"}
    if not no_parity:
        res["parity"] = parity_vs_oracle(out, x, logits, pool.cpu(), pages, cfg.k, cfg.renormalize, ids=ids)
    del gr, pool
    torch.cuda.empty_cache()
    return res


def bench_flushed_config(cfg, dev, stream, n, hbm_peak, flush_bytes: int = 256 << 20):
    """Layer time of a configuration whose weights are only ~1.4x the L2 (C1: 176 MB): each
    replay is timed alone between CUDA events, with a 256 MB buffer written before it
    (outside the events) so that no weights are served from L2, and then a second 256 MB
    buffer read, so that the L2 holds clean lines: otherwise writing back the first
    buffer's dirty lines (about the L2's size) would fall inside the timed call."""
    from ae_b200 import configs, ops
    pool = configs.make_pool(cfg, dev, seed=0)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=0)
    out = torch.empty_like(x)
    scratch = torch.empty(flush_bytes, dtype=torch.uint8, device=dev)
    clean = torch.ones(flush_bytes // 4, dtype=torch.int32, device=dev)

    def step():
        ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, out=out)

    for _ in range(3):
        step()
    gr, cs = graph_of(step, dev, with_stream=True)
    ws = ops.Workspace.lookup(dev, cs)
    times = []
    for i in range(n + 3):
        if i == 3:
            ops.read_timers(ws, reset=True)
        scratch.fill_(i & 0xFF)
        clean.max()  # reads 256 MB: the written lines are evicted (and written back) here
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        gr.replay()
        b.record(stream)
        b.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b) * 1e-3)
    tm = ops.read_timers(ws)
    touched = touched_experts(logits, cfg.k, cfg.renormalize)
    ffn_b, layer_b, _ = algorithmic(cfg, touched)
    t = statistics.median(times)
    ffn_s = tm["ffn_ns"] / max(1, tm["ffn_launches"]) * 1e-9
    stages = stage_means(tm, busy=True)
    del gr, pool, scratch, clean
    return {"workload": cfg.name, "T": cfg.T, "us_per_layer": round(t * 1e6, 2),
            "tokens_per_s": round(cfg.T / t, 1), "experts_touched": touched, "alg_bytes": layer_b,
            "layer_hbm_frac": round(layer_b / t / 1e9 / hbm_peak, 4),
            "ffn_us": round(ffn_s * 1e6, 2), "ffn_hbm_frac": round(ffn_b / ffn_s / 1e9 / hbm_peak, 4),
            "kernel_busy_us": stages, "splits": ops.splits(cfg.E, cfg.H, cfg.I, cfg.T * cfg.k),
            "l2": f"{flush_bytes >> 20} MB buffer written, then another {flush_bytes >> 20} MB read, before every "
                  "timed replay (outside the events)",
            "timing": f"median of {n} single graph replays"}


def bench_shared_config(cfg, dev, stream, n, hbm_peak):
    """Graph-replay time of one layer call of a shared-expert configuration (routed top-k
    plus a sigmoid-gated shared expert), with its HBM roofline fraction."""
    from ae_b200 import configs, ops
    x, logits = configs.make_inputs(cfg, dev, seed=0)
    routed = configs.make_pool(cfg, dev, seed=0)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    H, Is = cfg.H, cfg.shared_I
    w1 = (torch.randn(Is, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn(Is, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(H, Is, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wsg = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    shared = ops.shared_expert_pages(w1, w3, w2, cfg.I)
    ns = shared.shape[0]
    pool = torch.cat([routed, shared])
    del routed, w1, w3, w2
    pages = torch.arange(cfg.E + ns, device=dev, dtype=torch.int64)
    out = torch.empty_like(x)
    sw = torch.empty(cfg.T, dtype=torch.float32, device=dev)

    def step():
        torch.sigmoid(torch.matmul(x, wsg.unsqueeze(1)).squeeze(1).float(), out=sw)
        ops.moe_forward_shared(x, logits, pool, pages, cfg.k, ns, sw, cfg.renormalize, out=out)

    for _ in range(5):
        step()
    gr = graph_of(step, dev)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize(dev)
    el = timed_steps(gr.replay, n, stream)
    touched = touched_experts(logits, cfg.k, cfg.renormalize)
    alg = (touched * 3 * cfg.I * H + 3 * Is * H) * 2 + 2 * cfg.T * H * 2 + cfg.T * cfg.E * 2
    us = el / n * 1e6
    del gr
    return {"workload": cfg.name + f" + shared expert I{Is} ({ns} pseudo-experts)", "T": cfg.T,
            "us_per_layer": round(us, 2), "tokens_per_s": round(cfg.T / (el / n), 1),
            "experts_touched": touched, "alg_bytes": alg,
            "layer_hbm_frac": round(alg / (el / n) / 1e9 / hbm_peak, 4),
            "api": "ae_b200.ops.moe_forward_shared (smb_moe_forward_shared)",
            "note": "sigmoid shared gate (torch GEMV) + one library call per replay"}


def bench_streaming(cfg, pool, pages, x, logits, dev, stream, reps: int = 3):
    """Layer time with every expert page copied from page-locked host memory in the same
    step: streamed (per-page copies + ready flags, the FFN starts at once) against copying
    all pages first and then running the resident layer, and the copies alone."""
    from ae_b200 import ops
    from ae_b200.streaming import ExpertPageStreamer
    host = pool.cpu().pin_memory()
    st = ExpertPageStreamer(host, num_pages=cfg.E, device=dev)
    out = torch.empty_like(x)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    res = {"streamed": [], "copy_then_compute": [], "copy_only": []}
    for _ in range(reps + 1):
        torch.cuda.synchronize(dev)
        a, b = ev(), ev()
        a.record(stream)
        st.load(range(cfg.E))
        st.forward(x, logits, cfg.k, pages, out=out)
        b.record(stream)
        torch.cuda.synchronize(dev)
        res["streamed"].append(a.elapsed_time(b))
        if st.status(x, cfg.E, cfg.k) != 0:
            raise RuntimeError("streamed layer reported a device error")
        a, b, c = ev(), ev(), ev()
        a.record(stream)
        for p in range(cfg.E):
            st.pool[p].copy_(host[p], non_blocking=True)
        c.record(stream)
        ops.moe_forward(x, logits, st.pool, pages, cfg.k, cfg.renormalize, out=out)
        b.record(stream)
        torch.cuda.synchronize(dev)
        res["copy_then_compute"].append(a.elapsed_time(b))
        res["copy_only"].append(a.elapsed_time(c))
    med = {k: statistics.median(v[1:]) for k, v in res.items()}
    nbytes = cfg.E * pool.shape[1] * pool.element_size()
    del st, host
    return {"workload": cfg.name + ", all expert pages copied host -> device in the step",
            "streamed_ms": round(med["streamed"], 3), "copy_then_compute_ms": round(med["copy_then_compute"], 3),
            "copy_only_ms": round(med["copy_only"], 3),
            "h2d_gbs": round(nbytes / (med["copy_only"] * 1e-3) / 1e9, 1), "bytes": nbytes,
            "api": "ae_b200.streaming.ExpertPageStreamer (smb_moe_page_copy + smb_moe_forward_streamed)",
            "note": "median of %d; one cudaMemcpyAsync per page" % reps}


def bench_verify_step(dev, stream, hbm_peak, steps: int = 5):
    """Verify step of a random-init 32-layer Mixtral-8x7B decoder (ae_b200/verify.py):
    batch 4 x 32 draft tokens (a seeded tree) over a 2048-token bf16 KV cache, 128 tokens
    per MoE layer.  Returns the MoE layers' device time (events around each call), the
    whole step and the MoE share."""
    from ae_b200.verify import MIXTRAL_8X7B, VerifyDecoder, accept_greedy, random_tree
    cfg = MIXTRAL_8X7B
    B, n, cache = 4, 32, 2048
    dec = VerifyDecoder(cfg, batch=B, cache_len=cache, max_draft=n, device=dev, seed=0)
    parents = random_tree(n, seed=0)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    tokens = torch.randint(0, cfg.vocab, (B, n), generator=g, device=dev)
    for _ in range(3):
        dec.forward(tokens, parents)
    torch.cuda.synchronize(dev)
    moe_us, step_us = [], []
    for _ in range(steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(cfg.layers)]
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        logits = dec.forward(tokens, parents, moe_events=ev)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        moe_us.append(statistics.mean(a.elapsed_time(b) for a, b in ev) * 1000.0)
        step_us.append(s0.elapsed_time(s1) * 1000.0)
    acc, n_acc = accept_greedy(logits, tokens, parents, logits[:, 0])
    T = B * n
    layer_bytes = cfg.E * 3 * cfg.H * cfg.I * 2 + 2 * T * cfg.H * 2
    m = statistics.median(moe_us)
    out = {"workload": "C4 Mixtral-8x7B 32-layer verify step: batch 4 x 32-token draft tree, 2048-token bf16 KV "
                       "cache, random-init weights",
           "tokens_per_moe_layer": T, "moe_us_per_layer": round(m, 2),
           "moe_layer_hbm_frac": round(layer_bytes / (m * 1e-6) / 1e9 / hbm_peak, 4),
           "step_ms": round(statistics.median(step_us) / 1000.0, 3),
           "moe_share_of_step": round(m * cfg.layers / statistics.median(step_us), 4),
           "api": "ae_b200.verify.VerifyDecoder (MoE: smb_moe_forward_gated per layer)",
           "accepted_tokens_per_seq": n_acc.tolist(),
           "note": "eager launches; attention is torch SDPA with a tree mask; MoE time from CUDA events around "
                   "each MoE call, median over %d steps" % steps}
    del dec
    torch.cuda.empty_cache()
    return out


EP_STAGES = ("route", "ffn", "final_combine")


def ep_time(moe, x, logits, dev, stream, steps, soak=0.0):
    """Graph-replay time of ``steps`` expert-parallel layer calls (max over ranks) with the
    ranks' device timers over exactly those calls.  Returns (seconds, timers per rank as a
    [world, 6] tensor on every rank, launch mode)."""
    import torch.distributed as dist

    def step():
        return moe(x, logits)

    graph = None
    mode = "cuda_graph (one expert-parallel layer call per replay)"
    try:
        graph = graph_of(step, dev)
        run = graph.replay
        for _ in range(3):
            run()
    except Exception as exc:  # capture unsupported here: time the eager calls instead
        mode = f"eager (graph capture failed: {type(exc).__name__})"
        run = step
    torch.cuda.synchronize(dev)
    end = time.time() + soak
    while True:
        for _ in range(20):
            run()
        torch.cuda.synchronize(dev)
        if time.time() >= end:
            break
    moe.timers(reset=True)
    dist.barrier()
    torch.cuda.synchronize(dev)
    elapsed = timed_steps(run, steps, stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    tm = moe.timers()
    st = stage_means(tm)
    sb = stage_means(tm, busy=True)
    mine = torch.tensor([elapsed, tm.get("ffn_ns", 0) / max(1, tm.get("ffn_launches", 0)) * 1e-3,
                         tm.get("recv_wait_ns", 0) / max(1, tm.get("recv_waits", 0)) * 1e-3,
                         tm.get("combine_wait_ns", 0) / max(1, tm.get("combine_waits", 0)) * 1e-3,
                         tm.get("ffn_launches", 0), tm.get("recv_waits", 0)] +
                        [st.get(n, 0.0) for n in EP_STAGES] + [sb.get(n, 0.0) for n in EP_STAGES],
                        device=dev, dtype=torch.float64)
    every = [torch.empty_like(mine) for _ in range(dist.get_world_size())]
    dist.all_gather(every, mine)
    every = torch.stack(every)
    del graph
    torch.cuda.synchronize(dev)
    return float(every[:, 0].max()), every.cpu(), mode


def ep_parity(cfg, moe, x, logits, rank, world, dev):
    """Every rank's output and routing ids of one more call on its timed inputs, gathered
    on rank 0 and checked over the whole batch against the fp32 CPU oracle (all experts,
    the same seeded pages) and against the single-GPU library layer.  Collective."""
    import torch.distributed as dist
    from ae_b200 import configs, ops
    T_r = x.shape[0]
    w = torch.empty(T_r, cfg.k, dtype=torch.float32, device=dev)
    ids = torch.empty(T_r, cfg.k, dtype=torch.int32, device=dev)
    out = moe(x, logits, topk_weights=w, topk_ids=ids).clone()
    torch.cuda.synchronize(dev)
    outs = [torch.empty_like(out) for _ in range(world)]
    idss = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(outs, out)
    dist.all_gather(idss, ids)
    res = None
    if rank == 0:
        from oracle import moe_oracle as mo  # the checker only
        xs, ls = zip(*[configs.make_inputs(cfg, dev, seed=r, T=T_r) for r in range(world)])
        xs, ls = torch.cat(xs), torch.cat(ls)
        full = configs.make_pool(cfg, dev, seed=0)
        pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
        single = ops.moe_forward(xs, ls, full, pages, cfg.k, cfg.renormalize)
        torch.cuda.synchronize(dev)
        got = torch.cat(outs)
        res = parity_vs_oracle(got, xs, ls, full.cpu(), pages, cfg.k, cfg.renormalize, ids=torch.cat(idss))
        sm, sr = mo.error_metrics(got.float().cpu(), single.float().cpu())
        res["vs_single_gpu_layer"] = {"max_abs": sm, "rel_l2": sr}
        res["against"] += f"; whole batch of {cfg.T} tokens gathered from {world} ranks"
        del full, single
        torch.cuda.empty_cache()
    dist.barrier()
    return res


def run_ep(args, cfg, rank, world, dev):
    """N > 1: expert parallelism, strong scaling.  One verify batch of T tokens per step is
    spread over the N ranks (T/N each); rank r holds experts [r*E/N, (r+1)*E/N); rows are
    dispatched and returned by the kernels over peer memory (the default, ``--ep-transport
    p2p``) or with fixed-capacity NCCL all-to-alls (``nccl``), with no host synchronisation
    either way, so the step is replayed from a CUDA graph (ae_b200/ep.py).  The other
    transport is timed on the same ranks for comparison, the output is checked against the
    oracle, and Mixtral-8x22B (C5) is timed the same way."""
    import torch.distributed as dist
    from ae_b200 import configs
    from ae_b200.ep import ExpertParallelMoE

    hbm_peak, tc_peak, peak_kind = peaks()
    stream = torch.cuda.current_stream(dev)
    if cfg.T % world or cfg.E % world:
        raise SystemExit(f"{cfg.name}: T={cfg.T} and E={cfg.E} must divide by {world} GPUs")
    E_loc = cfg.E // world
    T_r = cfg.T // world
    pool = configs.make_pool(cfg, dev, seed=0, experts=range(rank * E_loc, (rank + 1) * E_loc))
    x, logits = configs.make_inputs(cfg, dev, seed=rank, T=T_r)
    moe = ExpertParallelMoE(cfg.E, cfg.k, cfg.H, cfg.I, pool, max_tokens=T_r, transport=args.ep_transport)

    def step():
        return moe(x, logits)

    sampler = ClockSampler(device_uuid(dev))
    sampler.start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    eager = timed_steps(step, args.steps, stream)
    el = torch.tensor([eager], device=dev, dtype=torch.float64)
    dist.all_reduce(el, op=dist.ReduceOp.MAX)
    eager = float(el.item())
    t_soak = time.time()
    elapsed, per_rank, mode = ep_time(moe, x, logits, dev, stream, args.steps, soak=args.soak)
    t_end = time.time()
    clocks = sampler.summary(t_soak, t_end)
    sampler.stop()
    if args.ep_transport == "p2p":
        mode = mode.replace("per replay)", "per replay: rows moved by the kernels over peer memory, no collective)")

    parity = None if args.no_parity else ep_parity(cfg, moe, x, logits, rank, world, dev)

    # the same layer with the other transport, graph replays, max over ranks
    other = "nccl" if args.ep_transport == "p2p" else "p2p"
    moe2 = ExpertParallelMoE(cfg.E, cfg.k, cfg.H, cfg.I, pool, max_tokens=T_r, transport=other)
    for _ in range(3):
        moe2(x, logits)
    t2, _, _ = ep_time(moe2, x, logits, dev, stream, args.steps)
    moe2.close()

    # the local expert FFN of a step on the rows this rank received, replayed from a
    # graph and timed alone (the dominant work of a rank)
    send, state = moe.backend.dispatch(x, logits, world, moe.C)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    torch.cuda.synchronize(dev)
    hdr = recv.view(world, moe.C + 1, cfg.H)[:, 0].contiguous().view(torch.int32)[:, :E_loc].cpu()
    n_recv = int(hdr.sum())
    touched = int((hdr.sum(0) > 0).sum())

    def experts():
        moe.backend.experts(recv, world, moe.C, pool, moe.pages, E_loc)

    g_exp = graph_of(experts, dev)
    for _ in range(3):
        g_exp.replay()
    t_exp = timed_steps(g_exp.replay, 20, stream) / 20
    ffn_bytes = touched * 3 * cfg.H * cfg.I * 2 + n_recv * cfg.H * 2 * 2
    ach = torch.tensor([ffn_bytes / t_exp / 1e9], device=dev, dtype=torch.float64)
    dist.all_reduce(ach, op=dist.ReduceOp.MIN)
    del g_exp

    # e2e through the public EP layer with host inputs and outputs, every step
    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    dx = torch.empty_like(x)
    dl = torch.empty_like(logits)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        hout.copy_(moe(dx, dl), non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e2e_el = timed_steps(e2e_step, args.steps, stream)
    t = torch.tensor([e2e_el], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_el = float(t.item())
    torch.cuda.synchronize(dev)
    moe.close()
    del pool

    # Mixtral-8x22B (C5): T = 512 per step, T/N tokens and E/N experts per rank
    c5 = None
    if not args.no_sweep:
        c5 = ep_config_block(configs.BY_KEY["c5"], rank, world, dev, stream, max(10, args.steps // 2),
                             hbm_peak, args.ep_transport, args.no_parity)

    if rank != 0:
        return
    step_s = elapsed / args.steps
    achieved = float(ach.item())
    pr = per_rank.numpy()
    line = {
        "metric": METRIC,
        "value": round(cfg.T * args.steps / elapsed, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_s * 1000, 5),
        "us_per_layer": round(step_s * 1e6, 2),
        "launch_mode": mode,
        "eager_us_per_layer": round(eager / args.steps * 1e6, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: expert weights N(0,0.02) bf16, tokens N(0,1), router logits x@Wr^T "
                f"(Wr std {cfg.router_std:.4g})",
        "config": config_of(cfg, world),
        "roofline": {"bound": "hbm", "kernel": "local experts on the received rows (smb_moe_ep_experts: "
                                                "route_kernel + ffn_gemm_kernel), slowest rank",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind, "traffic": None},
        "per_rank_device_timers_us": {
            "ffn": [round(float(v), 2) for v in pr[:, 1]],
            "recv_flag_wait": [round(float(v), 2) for v in pr[:, 2]],
            "return_flag_wait": [round(float(v), 2) for v in pr[:, 3]],
            "stages": {n: [round(float(v), 2) for v in pr[:, 6 + i]] for i, n in enumerate(EP_STAGES)},
            "stage_kernel_busy": {n: [round(float(v), 2) for v in pr[:, 6 + len(EP_STAGES) + i]]
                                  for i, n in enumerate(EP_STAGES)},
            "timing": "device timers over the timed replays (means per call): FFN kernel (first CTA past its "
                      "wait to last CTA done), expert-side wait for the sources' rows, source-side wait for "
                      "the returned rows; stages of the chain from the arena's stage clock (dispatch, receive "
                      "routing, FFN with the returned rows written, final combine up to the next call's dispatch)"},
        "parity": parity,
        "cpu_baseline": None,
        "e2e": {"value": round(cfg.T * args.steps / e2e_el, 2), "unit": UNIT,
                "h2d_bytes_per_step": world * (x.numel() * x.element_size() + logits.numel() * logits.element_size()),
                "d2h_bytes_per_step": world * x.numel() * x.element_size(),
                "api": f"ae_b200.ep.ExpertParallelMoE.forward (transport={args.ep_transport})"},
        f"{other}_transport_us_per_layer": round(t2 / args.steps * 1e6, 2),
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
        "c5_expert_parallel": c5,
    }
    emit(line)


def ep_config_block(cfg, rank, world, dev, stream, n, hbm_peak, transport, no_parity):
    """Another configuration through the expert-parallel layer on the same ranks: graph
    replays, max over ranks, per-GPU HBM fraction, parity over the whole batch."""
    from ae_b200 import configs
    from ae_b200.ep import ExpertParallelMoE
    E_loc, T_r = cfg.E // world, cfg.T // world
    pool = configs.make_pool(cfg, dev, seed=0, experts=range(rank * E_loc, (rank + 1) * E_loc))
    x, logits = configs.make_inputs(cfg, dev, seed=rank, T=T_r)
    moe = ExpertParallelMoE(cfg.E, cfg.k, cfg.H, cfg.I, pool, max_tokens=T_r, transport=transport)
    for _ in range(3):
        moe(x, logits)
    el, per_rank, _ = ep_time(moe, x, logits, dev, stream, n)
    parity = None if no_parity else ep_parity(cfg, moe, x, logits, rank, world, dev)
    moe.close()
    del moe, pool
    torch.cuda.empty_cache()
    t = el / n
    per_gpu_bytes = cfg.weight_bytes(E_loc)
    pr = per_rank.numpy()
    return {"workload": cfg.name + f", expert-parallel over {world} GPUs ({T_r} tokens and {E_loc} experts per GPU)",
            "T": cfg.T, "us_per_layer": round(t * 1e6, 2), "tokens_per_s": round(cfg.T / t, 1),
            "per_gpu_weight_bytes": per_gpu_bytes,
            "per_gpu_hbm_frac": round(per_gpu_bytes / t / 1e9 / hbm_peak, 4),
            "ffn_us_per_rank": [round(float(v), 2) for v in pr[:, 1]],
            "parity": parity, "transport": transport, "timing": f"{n} graph replays, max over ranks"}


def run_ep_rank(args, cfg, dev):
    """Diagnostic (``--ep-rank G``): one rank's share of a G-rank expert-parallel layer call
    on this GPU, with local buffers instead of peers (for profiling; no metric line): the
    dispatch of T/G tokens, the local experts on a receive buffer built from G sources'
    chunks for this rank, and the final combine, each timed from graph replays."""
    from ae_b200 import configs, ops
    from ae_b200.ep import CudaBackend
    G = args.ep_rank
    E_loc, T_r = cfg.E // G, cfg.T // G
    C = T_r * cfg.k
    pool = configs.make_pool(cfg, dev, seed=0, experts=range(0, E_loc))
    pages = torch.arange(E_loc, device=dev, dtype=torch.int64)
    b = CudaBackend(cfg.E, cfg.k, cfg.H, cfg.I, torch.bfloat16, dev)
    recv = torch.zeros(G * (C + 1), cfg.H, dtype=torch.bfloat16, device=dev)
    for src in range(G):
        xs, ls = configs.make_inputs(cfg, dev, seed=src, T=T_r)
        send, _ = b.dispatch(xs, ls, G, C)
        recv[src * (C + 1):(src + 1) * (C + 1)] = send[0:C + 1]
    x, lg = configs.make_inputs(cfg, dev, seed=0, T=T_r)
    send, state = b.dispatch(x, lg, G, C)
    back = torch.zeros(G * C, cfg.H, dtype=torch.bfloat16, device=dev)
    steps = {"dispatch": lambda: b.dispatch(x, lg, G, C),
             "experts": lambda: b.experts(recv, G, C, pool, pages, E_loc),
             "combine": lambda: b.combine(back, state, T_r, G, C)}
    stream = torch.cuda.current_stream(dev)
    res = {}
    for name, fn in steps.items():
        for _ in range(3):
            fn()
        gr = graph_of(fn, dev)
        for _ in range(3):
            gr.replay()
        if name == "experts":
            ws = b._bufs[("ws_exp", G, C)]
            ops.read_timers_at(ws.data_ptr(), ws.numel(), dev, reset=True)
        res[name + "_us"] = round(timed_steps(gr.replay, args.steps, stream) / args.steps * 1e6, 2)
        if name == "experts":
            tm = ops.read_timers_at(ws.data_ptr(), ws.numel(), dev)
            res["ffn_us"] = round(tm["ffn_ns"] / max(1, tm["ffn_launches"]) / 1e3, 2)
            wbytes = E_loc * 3 * cfg.H * cfg.I * 2
            res["ffn_hbm_frac"] = round(wbytes / (res["ffn_us"] * 1e-6) / 1e9 / peaks()[0], 4)
    if os.environ.get("SMB_SPLIT_K"):
        res["split_k"] = int(os.environ["SMB_SPLIT_K"])
    hdr = recv.view(G, C + 1, cfg.H)[:, 0].contiguous().view(torch.int32)[:, :E_loc]
    res["rows_received"] = int(hdr.sum())
    emit({"ep_rank_emulation": {"workload": cfg.name, "ranks": G, "experts_per_rank": E_loc, **res}})


def run_power_probe(args, cfg, dev):
    """Diagnostic (``--power-probe``, no metric line): layer time against the SM clock.  One
    graph of a layer call is replayed in blocks of 40: once after a 2 s idle gap, then back
    to back for ``--probe-seconds``, then once more after a 3 s idle gap; each block reports
    its µs per layer, the FFN kernel's device timer and the SM clock / throttle reasons
    sampled during it."""
    from ae_b200 import configs, ops
    pool = configs.make_pool(cfg, dev, seed=0)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=0)
    out = torch.empty_like(x)

    def step():
        ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, out=out)

    for _ in range(5):
        step()
    g, cs = graph_of(step, dev, with_stream=True)
    ws = ops.Workspace.lookup(dev, cs)
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(device_uuid(dev))
    sampler.start()
    blocks = []

    def block(tag, n=40):
        ops.read_timers(ws, reset=True)
        t0 = time.time()
        el = timed_steps(g.replay, n, stream)
        tm = ops.read_timers(ws)
        t1 = time.time()
        c = sampler.summary(t0 - 0.15, t1 + 0.15)
        blocks.append({"tag": tag, "us_per_layer": round(el / n * 1e6, 2),
                       "ffn_us": round(tm["ffn_ns"] / max(1, tm["ffn_launches"]) / 1e3, 2),
                       "sm_mhz": c["sm_mhz"], "reasons": c["reasons"]})

    time.sleep(2.0)
    block("after_idle_2s")
    end = time.time() + args.probe_seconds
    while time.time() < end:
        block("sustained")
    time.sleep(3.0)
    block("after_idle_3s")
    sampler.stop()
    hot = [b for b in blocks if b["tag"] == "sustained"]
    hot = hot[len(hot) // 2:]  # the settled half
    emit({"power_probe": {"workload": cfg.name, "blocks_first_last": blocks[:2] + blocks[-2:],
                          "sustained_median_us": statistics.median(b["us_per_layer"] for b in hot),
                          "sustained_median_ffn_us": statistics.median(b["ffn_us"] for b in hot),
                          "sustained_median_sm_mhz": statistics.median(b["sm_mhz"] or 0 for b in hot),
                          "blocks": len(blocks)}})


_JSON_OUT = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's real stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def _stdout_to_stderr() -> None:
    """Keep a private handle on stdout for the JSON line and send everything else that
    writes to file descriptor 1 (library banners such as NCCL's version line, C-level
    prints, stray Python prints) to stderr."""
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def main():
    _stdout_to_stderr()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c2-256")
    ap.add_argument("--soak", type=float, default=1.5, help="seconds of untimed load before timing")
    ap.add_argument("--staged-steps", type=int, default=20)
    ap.add_argument("--sweep", type=int, nargs="*", default=[16, 64])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-verify", action="store_true", help="skip the 32-layer verify-step block")
    ap.add_argument("--ep-rank", type=int, default=0,
                    help="diagnostic: time one rank's kernels of a G-rank expert-parallel call on this GPU")
    ap.add_argument("--ep-transport", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: rows over peer memory by the kernels, or NCCL all-to-alls")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed output")
    ap.add_argument("--power-probe", action="store_true",
                    help="diagnostic: layer time against the SM clock over a sustained run (no metric line)")
    ap.add_argument("--probe-seconds", type=float, default=8.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    from ae_b200 import configs
    cfg = configs.BY_KEY[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, cfg, rank, world)
        return

    from ae_b200 import build
    if rank == 0:
        build.build()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.ep_rank > 0:
        run_ep_rank(args, cfg, dev)
        return
    if args.power_probe:
        run_power_probe(args, cfg, dev)
        return
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        dist.barrier()
    try:
        if world > 1:
            run_ep(args, cfg, rank, world, dev)
        else:
            run_ours(args, cfg, rank, world, dev)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
