#!/usr/bin/env python
"""MoE verify-layer throughput on B200 (SpecMoE FusedMoE path), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2-256] [--impl reference]

A step is one pass of the MoE layer (route, expert FFN = gate/up GEMM + SiLU*mul + down
GEMM, combine) over one verify batch of T synthetic tokens, inputs resident in HBM.  The
timed region is K back-to-back replays of a CUDA graph holding one layer call, between
CUDA events on the launching stream, bracketed by a barrier and a device synchronise,
max over ranks (the eager, ctypes-per-call time is reported beside it).  Expert weights (2.8 GB for
Mixtral-8x7B) are far larger than the 126 MB L2, so consecutive steps do not reuse
weights from L2.

N > 1: expert parallelism (ae_b200/ep.py), strong scaling: the same verify batch of T
tokens per step, T/N on each rank; rank r holds experts [r*E/N, (r+1)*E/N); rows are
dispatched and returned with NCCL all-to-all.

Extra keys: roofline (dominant kernel = the fused expert-FFN kernel, HBM bound), cpu_baseline (the CPU
oracle port of the reference's arithmetic on this host), e2e (FusedMoE.forward with host
inputs copied in and the output copied out every step), clocks, gpu_launches, kernels
(per-kernel µs from a staged pass), sweep (other verify batch sizes).

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


def run_reference_arm(args, cfg, rank):
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
        "config": {"workload": cfg.name, "T": cfg.T, "H": cfg.H, "I": cfg.I, "E": cfg.E, "k": cfg.k},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU expert path (FusedMoE.forward_cpu is unreachable); this arm runs the "
                "oracle's CPU restatement of stack_fused_moe + select_experts",
    }
    emit(line)


# ---------------------------------------------------------------------------- GPU arm

def algorithmic(cfg, touched: int, Tk: int, splits: int):
    """Algorithmic bytes of the FFN kernel (touched experts' weights + its token rows in +
    fp32 partials out) and of the whole layer (weights + tokens in and out + logits), and
    the layer's flops."""
    H, I, T, E = cfg.H, cfg.I, cfg.T, cfg.E
    ffn = touched * 3 * H * I * 2 + Tk * H * 2 + splits * Tk * H * 4
    layer = touched * 3 * H * I * 2 + 2 * T * H * 2 + T * E * 2
    flops = 6 * H * I * Tk
    return ffn, layer, flops


def graph_of(fn, dev):
    """Capture one call of ``fn`` into a CUDA graph (after a warm call on the capture
    stream, so its workspace exists before capture)."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize(dev)
    return g


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


def run_ours(args, cfg, rank, world, dev):
    import torch.distributed as dist
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

    # warm-up and clock soak
    sampler = ClockSampler(device_uuid(dev))
    sampler.start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    t_soak = time.time()
    soak_end = t_soak + args.soak
    while time.time() < soak_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize(dev)

    # eager launches (host-side ctypes call per layer), for reference
    torch.cuda.synchronize(dev)
    eager = timed_steps(step, args.steps, stream)
    # the timed region replays a CUDA graph of one layer call per step (the verify step
    # of the reference engine is graph-captured as well); launches are the same kernels
    graph = graph_of(step, dev)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    elapsed = timed_steps(graph.replay, args.steps, stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t_timed_end = time.time()
    el = torch.tensor([elapsed], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
    elapsed = float(el.item())
    clocks = sampler.summary(t_soak, t_timed_end)
    sampler.stop()
    if not torch.isfinite(out.float()).all():
        raise RuntimeError("non-finite layer output")

    # staged pass: per-kernel durations (events between the three launches of a layer call)
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
    ffn_bytes, layer_bytes, flops = algorithmic(cfg, touched, Tk, splits)

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
    if world > 1:
        dist.barrier()
    e2e_el = timed_steps(e2e_step, args.steps, stream)
    t = torch.tensor([e2e_el], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_el = float(t.item())

    # other verify batch sizes of the same layer (rank 0 view, N=1 only)
    sweep = {}
    if world == 1 and not args.no_sweep:
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
            sweep[f"T{Ts}"] = {"us_per_layer": round(us, 2), "tokens_per_s": round(Ts / (el_s / n), 1),
                               "layer_hbm_frac": round(algorithmic(
                                   configs.MoEConfig(cfg.name, cfg.H, cfg.I, cfg.E, cfg.k, Ts, cfg.router_std),
                                   cfg.E, Ts * cfg.k, splits)[1] / (el_s / n) / 1e9 / hbm_peak, 4)}

    # the whole MixtralMoE block (gate + experts): gate fused into the routing launch vs.
    # the reference's arrangement of a separate half-precision gate GEMM (cuBLAS, like
    # ReplicatedLinear) followed by the layer
    gated = None
    if world == 1 and not args.no_sweep:
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
        for name, v in samples.items():
            gated[f"{name}_us_per_layer"] = round(statistics.median(v), 2)
        del graphs

    # the fine-grained configuration with a shared expert (60 routed experts of I 1408,
    # top-4, shared expert I 5632 as 4 pseudo-experts in the same launch, Zipf routing)
    fine = None
    if world == 1 and not args.no_sweep:
        fine = bench_shared_config(configs.BY_KEY["c3"], dev, stream, max(10, args.steps // 2), hbm_peak)

    # the 32-layer verify step (Mixtral-8x7B architecture, batch 4 x 32-token draft tree on
    # a 2048-token KV cache), MoE layers isolated by CUDA events around each MoE call
    verify = None
    if world == 1 and not args.no_sweep and not args.no_verify:
        verify = bench_verify_step(dev, stream, hbm_peak)

    # expert pages streamed from page-locked host memory while the layer runs (all 8
    # experts cross PCIe, as with the reference's decode_weight_cache_ratio = 0)
    streamed = None
    if world == 1 and not args.no_sweep:
        streamed = bench_streaming(cfg, pool, pages, x, logits, dev, stream)

    # CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        pool_cpu = pool.cpu()
        tps, sec, threads, reps = cpu_port_time(cfg, 0, pool_cpu=pool_cpu, x=x.cpu(), logits=logits.cpu())
        cpu = {"value": round(tps, 2), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{reps} full layer calls of {cfg.T} tokens ({cfg.name}), median {sec * 1000:.1f} ms, "
                         f"oracle CPU restatement, bf16 storage / fp32 accumulate, {threads} threads"}
        del pool_cpu

    if rank != 0:
        return
    step_s = elapsed / args.steps
    ffn_s = kern_us["ffn"] * 1e-6
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
        "config": {"workload": cfg.name, "T": cfg.T, "H": cfg.H, "I": cfg.I, "E": cfg.E, "k": cfg.k,
                   "experts_touched": touched, "splits": splits,
                   "parallelism": "replicas" if world > 1 else "single",
                   "l2": "inputs larger than L2 (expert weights %.2f GB per step)" % (cfg.weight_bytes() / 1e9)},
        "roofline": {"bound": "hbm", "kernel": "ffn_gemm_kernel (gate/up + down, one launch)",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                     "alg_bytes_per_launch": ffn_bytes, "traffic": traffic},
        "layer_roofline": {"alg_bytes": layer_bytes, "achieved_gbs": round(layer_bytes / step_s / 1e9, 1),
                           "frac_hbm": round(layer_bytes / step_s / 1e9 / hbm_peak, 4),
                           "tflops": round(flops / step_s / 1e12, 2),
                           "frac_tensor": round(flops / step_s / 1e12 / tc_peak, 4)},
        "kernels_us": {n: round(u, 2) for n, u in kern_us.items()},
        "cpu_baseline": cpu,
        "e2e": {"value": round(world * cfg.T * args.steps / e2e_el, 2), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * x.element_size() + logits.numel() * logits.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "api": "ae_b200.layers.FusedMoE.FusedMoE.forward"},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
        "sweep": sweep,
        "gated_block": gated,
        "shared_expert_config": fine,
        "verify_32_layers": verify,
        "streamed_pages": streamed,
    }
    emit(line)


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
    ids = torch.topk(logits.float(), cfg.k, dim=1).indices
    touched = int((torch.bincount(ids.flatten(), minlength=cfg.E) > 0).sum())
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


def run_ep(args, cfg, rank, world, dev):
    """N > 1: expert parallelism, strong scaling.  One verify batch of T tokens per step is
    spread over the N ranks (T/N each); rank r holds experts [r*E/N, (r+1)*E/N); rows are
    dispatched and returned by the kernels over peer memory (the default, ``--ep-transport
    p2p``) or with fixed-capacity NCCL all-to-alls (``nccl``), with no host synchronisation
    either way, so the step is replayed from a CUDA graph (ae_b200/ep.py).  The other
    transport is timed on the same ranks for comparison."""
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
    mode = ("cuda_graph (one expert-parallel layer call per replay: rows moved by the kernels over peer "
            "memory, no collective)" if args.ep_transport == "p2p" else
            "cuda_graph (one expert-parallel layer call per replay, NCCL inside the graph)")
    graph = None
    try:
        graph = graph_of(step, dev)
        run = graph.replay
        for _ in range(3):
            run()
    except Exception as exc:  # capture unsupported here: time the eager calls instead
        mode = f"eager (graph capture failed: {type(exc).__name__})"
        run = step
    torch.cuda.synchronize(dev)
    t_soak = time.time()
    soak_end = t_soak + args.soak
    while time.time() < soak_end:
        for _ in range(20):
            run()
        torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    elapsed = timed_steps(run, args.steps, stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    t_end = time.time()
    el = torch.tensor([elapsed, eager], device=dev, dtype=torch.float64)
    dist.all_reduce(el, op=dist.ReduceOp.MAX)
    elapsed, eager = float(el[0].item()), float(el[1].item())
    clocks = sampler.summary(t_soak, t_end)
    sampler.stop()

    # the same layer with the other transport, graph replays, max over ranks
    other = "nccl" if args.ep_transport == "p2p" else "p2p"
    moe2 = ExpertParallelMoE(cfg.E, cfg.k, cfg.H, cfg.I, pool, max_tokens=T_r, transport=other)

    def step2():
        return moe2(x, logits)

    for _ in range(3):
        step2()
    g2 = graph_of(step2, dev)
    for _ in range(3):
        g2.replay()
    dist.barrier()
    torch.cuda.synchronize(dev)
    t2 = torch.tensor([timed_steps(g2.replay, args.steps, stream) / args.steps], device=dev, dtype=torch.float64)
    dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    del g2
    torch.cuda.synchronize(dev)
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
    del graph
    torch.cuda.synchronize(dev)
    moe.close()
    if rank != 0:
        return
    step_s = elapsed / args.steps
    achieved = float(ach.item())
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
        "config": {"workload": cfg.name + f", expert-parallel over {world} GPUs ({T_r} tokens and {E_loc} "
                                          "experts per GPU)",
                   "T": cfg.T, "T_per_gpu": T_r, "H": cfg.H, "I": cfg.I, "E": cfg.E, "k": cfg.k,
                   "experts_per_gpu": E_loc, "parallelism": f"ep{world}",
                   "l2": "inputs larger than L2 (expert weights %.2f GB per GPU per step)"
                         % (cfg.weight_bytes(E_loc) / 1e9)},
        "roofline": {"bound": "hbm", "kernel": "local experts on the received rows (smb_moe_ep_experts: "
                                                "route_kernel + ffn_gemm_kernel + combine_kernel), slowest rank",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind, "traffic": None},
        "cpu_baseline": None,
        "e2e": {"value": round(cfg.T * args.steps / e2e_el, 2), "unit": UNIT,
                "h2d_bytes_per_step": world * (x.numel() * x.element_size() + logits.numel() * logits.element_size()),
                "d2h_bytes_per_step": world * x.numel() * x.element_size(),
                "api": f"ae_b200.ep.ExpertParallelMoE.forward (transport={args.ep_transport})"},
        f"{other}_transport_us_per_layer": round(float(t2.item()) * 1e6, 2),
        "gpu_launches": 5 * args.steps,
        "clocks": clocks,
    }
    emit(line)


def run_ep_rank(args, cfg, dev):
    """Diagnostic (``--ep-rank G``): one rank's share of a G-rank expert-parallel layer call
    on this GPU, with local buffers instead of peers (for profiling; no metric line): the
    dispatch of T/G tokens, the local experts on a receive buffer built from G sources'
    chunks for this rank, and the final combine, each timed from graph replays."""
    from ae_b200 import configs
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
        res[name + "_us"] = round(timed_steps(gr.replay, args.steps, stream) / args.steps * 1e6, 2)
    hdr = recv.view(G, C + 1, cfg.H)[:, 0].contiguous().view(torch.int32)[:, :E_loc]
    res["rows_received"] = int(hdr.sum())
    emit({"ep_rank_emulation": {"workload": cfg.name, "ranks": G, "experts_per_rank": E_loc, **res}})


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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    from ae_b200 import configs
    cfg = configs.BY_KEY[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, cfg, rank)
        return

    from ae_b200 import build
    if rank == 0:
        build.build()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.ep_rank > 0:
        run_ep_rank(args, cfg, dev)
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
