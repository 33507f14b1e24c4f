#!/usr/bin/env python3
"""Benchmark of the B200 expert hot path (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|layer]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1: one replica per GPU)

Workload `decode` (default; BASELINE config 4, the configuration the headline metric is quoted on):
greedy batch-1 decode of a Qwen3-30B-A3B-shape model -- 48 layers, hidden 2048, 32 q / 4 kv heads of
128, 128 experts top-8, intermediate 768, vocab 151936; Q4_K attention/gate/up/embedding, Q6_K
down/output, F32 router/norms; seeded random weights written as a GGUF (synth.config4_30b) and loaded
through eahmmf_engine_load. A 512-token random-id prompt is prefilled (untimed), then W decode steps
warm up and K decode steps are timed. One step = one token = one forward pass (48 layers + output GEMV
+ argmax), replayed as the captured CUDA graph.

  value     decode tokens/s over all ranks: K * ranks / (device time of the K steps, CUDA events on the
            engine's stream, max over ranks). Each step streams ~2 GB of weights (far above the 126 MB
            L2), so no flush is needed between steps.
  e2e       eahmmf_engine_greedy through the C ABI with host buffers: the 512-token prompt copied in,
            prefill, K generated tokens copied out; K / wall time of the call.
  roofline  k_moe_gateup (the Q4_K MoE decode kernel the target names) at T = 1: algorithmic bytes
            (the 8 routed experts' gate and up matrices + staged activations + h outputs) / its mean
            duration over every layer of a few eager decode steps (CUDA events around the kernel on
            its stream), against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the reference engine itself (oracle/_ref, compiled from the reference sources) on the
            same GGUF, all host threads: decode tokens/s after a short prompt (rank 0 at N = 1).

Workload `layer`: one MoE layer of the same shape on decode batches T = 1..8 (one
step = eight layer calls, 36 tokens), L2 flushed before every call; value = tokens/s of the layer.

--impl reference times the reference CPU implementation alone on the same workload (all host threads).
Multi-GPU: the path has no exchange step at these configurations; N ranks run N replicas ("replicas
only", weak scaling); the step time is the maximum over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "eahmmf_inference_prototype_v-0.1.0_b200")
ORACLE = os.path.join(ROOT, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "Qwen3-30B-A3B-shape Q4_K decode tok/s; MoE-layer achieved HBM GB/s vs ~8 TB/s"
T_LIST = (1, 2, 3, 4, 5, 6, 7, 8)
D, FF, E, K = 2048, 768, 128, 8
TOKENS_PER_STEP = sum(T_LIST)
LAUNCHES_PER_CALL = 3  # routing + prep, gate/up (+ h prep), down + combine
GATEUP_STAGE = 2       # index of the gate/up kernel in eahmmf_cuda_moe_profile_read's stages
LAYER_CONFIG = {"workload": "config2: Qwen3-30B-A3B-shape MoE layer decode, T=1..8 tokens per step",
          "hidden": D, "experts": E, "top_k": K, "moe_intermediate": FF, "gate_up": "Q4_K", "down": "Q6_K",
          "tokens_per_step": TOKENS_PER_STEP, "l2": "flushed (256 MiB memset) before every layer call, untimed"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ---- clocks sampled during the timed region -----------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.proc:
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---- inputs ---------------------------------------------------------------------------------------
def step_inputs(step: int, T: int, rank: int):
    import synth
    seed = 1000 * step + T + 7919 * rank
    return (synth.activations(T, D, seed=seed), synth.activations(T, D, seed=seed + 500),
            synth.router_logits(T, E, seed=seed + 900))


# ---- reference CPU arm ------------------------------------------------------------------------------
def reference_step(ref, ex, step: int) -> int:
    for T in T_LIST:
        x, xn, lg = step_inputs(step, T, 0)
        ref.moe_layer(x, xn, lg, list(ex.gate), list(ex.up), list(ex.down), ex.types, ex.row_bytes, K)
    return TOKENS_PER_STEP


def cpu_reference(ex, steps: int, warmup: int, budget_s: float | None = None):
    """Reference CPU tokens/s: `steps` steps, or as many as fit in budget_s seconds when given."""
    import oracle
    ref = oracle.Reference(threads=os.cpu_count() or 1)
    for s in range(warmup):
        reference_step(ref, ex, s)
    t0 = time.perf_counter()
    done = 0
    while True:
        reference_step(ref, ex, warmup + done)
        done += 1
        el = time.perf_counter() - t0
        if budget_s is None and done >= steps:
            break
        if budget_s is not None and (el >= budget_s or done >= 1000):
            break
    return TOKENS_PER_STEP * done / el, ref.threads, done


# ---- our arm --------------------------------------------------------------------------------------
def layer_ours(args, rank: int, world: int, local: int):
    import torch
    import eahmmf_b200 as eb
    import synth

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ex = synth.expert_set()
    layer = eb.MoeLayer.from_expert_set(ex, n_used=K)
    ws = torch.zeros(layer.workspace_bytes(max(T_LIST)), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    nsteps = args.warmup + args.steps
    host = {(s, T): step_inputs(s, T, rank) for s in range(nsteps) for T in T_LIST}
    devin = {k: tuple(torch.from_numpy(a).to(dev) for a in v) for k, v in host.items()}
    pinned = {k: tuple(torch.from_numpy(a).pin_memory() for a in v) for k, v in host.items()}
    bytes_g, bytes_u = ex.gate.shape[1], ex.up.shape[1]

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(dev)

    # device-timed layer calls (no instrumentation between the kernels of a call)
    step_us, launches = [], 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with Clocks(local) as clk:
        for s in range(nsteps):
            t_step = 0.0
            for T in T_LIST:
                x, xn, lg = devin[(s, T)]
                xo = x.clone()
                flush.zero_()
                ev0.record(stream)
                rc = layer(T, xn, lg, xo, ws, stream=stream, d_status=status)
                ev1.record(stream)
                if rc:
                    raise RuntimeError(f"eahmmf_cuda_moe_layer failed: {rc}")
                ev1.synchronize()
                if s >= args.warmup:
                    t_step += ev0.elapsed_time(ev1) * 1e3
                    launches += LAUNCHES_PER_CALL
            if s >= args.warmup:
                step_us.append(t_step)
        barrier()
    if int(status.item()):
        raise RuntimeError(f"kernel status {int(status.item())}")

    # roofline pass: the same steps again with the library's stage events on the call's stream, which
    # time each kernel on its own (the events stop the next kernel from starting early)
    eb.MoeLayer.profile(True)
    gu_us, gu_bytes, gu_n = 0.0, 0, 0
    for s in range(args.warmup, nsteps):
        for T in T_LIST:
            x, xn, lg = devin[(s, T)]
            xo = x.clone()
            flush.zero_()
            if layer(T, xn, lg, xo, ws, stream=stream, d_status=status):
                raise RuntimeError("eahmmf_cuda_moe_layer failed")
            stages = eb.MoeLayer.profile_read()
            ids, _ = layer.routing(ws, T)
            gu_us += float(stages[GATEUP_STAGE])
            gu_bytes += len(np.unique(ids)) * (bytes_g + bytes_u) + T * D * 3 + T * K * FF * 4
            gu_n += 1
    eb.MoeLayer.profile(False)
    barrier()

    # end-to-end through the C ABI with host buffers
    e2e_us = []
    h2d = d2h = 0
    for s in range(args.warmup, nsteps):
        t_step = 0.0
        for T in T_LIST:
            hx, hxn, hlg = pinned[(s, T)]
            out = torch.empty_like(hx).pin_memory()
            dx, dxn, dlg = (torch.empty(a.shape, dtype=a.dtype, device=dev) for a in (hx, hxn, hlg))
            flush.zero_()
            ev0.record(stream)
            dx.copy_(hx, non_blocking=True)
            dxn.copy_(hxn, non_blocking=True)
            dlg.copy_(hlg, non_blocking=True)
            layer(T, dxn, dlg, dx, ws, stream=stream)
            out.copy_(dx, non_blocking=True)
            ev1.record(stream)
            ev1.synchronize()
            t_step += ev0.elapsed_time(ev1) * 1e3
            if s == args.warmup:
                h2d += (hx.numel() + hxn.numel() + hlg.numel()) * 4
                d2h += out.numel() * 4
        e2e_us.append(t_step)

    t_total = float(np.sum(step_us))
    if world > 1:
        import torch.distributed as dist
        v = torch.tensor([t_total, float(np.sum(e2e_us))], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t_total, e2e_total = float(v[0]), float(v[1])
    else:
        e2e_total = float(np.sum(e2e_us))
    ms_step = t_total / args.steps / 1e3
    value = TOKENS_PER_STEP * args.steps * world / (t_total * 1e-6)
    e2e_value = TOKENS_PER_STEP * args.steps * world / (e2e_total * 1e-6)
    peak, peak_kind = peaks()
    achieved = gu_bytes / (gu_us * 1e-6) / 1e9 if gu_us > 0 else 0.0
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get("k_moe_gateup", {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        pass
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8/s8 tensor-core MMA, s32 -> fp32 accumulate (fp32 activations)",
        "data": "synthetic (seeded)", "config": dict(LAYER_CONFIG, parallelism=f"replicas x{world}"),
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if peak else None, "traffic": traffic,
                     "kernel": "k_moe_gateup", "peak_source": peak_kind,
                     "timing": f"CUDA events around the kernel on its stream, {gu_n} launches over the timed steps"},
        "clocks": clk.summary(),
        "layer_us_per_step": {"mean": float(np.mean(step_us)), "min": float(np.min(step_us))},
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, n = cpu_reference(ex, steps=1, warmup=1, budget_s=args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                "sample": f"{n} steps of T=1..8 ({TOKENS_PER_STEP} tokens each) through the "
                                          "reference CPU MoE block (oracle/_ref)"}
    return line


# ---- decode workload (config 4) ----------------------------------------------------------------------
N_PROMPT = 512
DECODE_CONFIG = {"workload": "config4: Qwen3-30B-A3B-shape greedy batch-1 decode, 48 layers, 512-token prompt",
                 "model": "qwen3moe 30B-A3B shape (synthetic weights)", "layers": 48, "hidden": 2048,
                 "heads": "32q/4kv x 128", "experts": 128, "top_k": 8, "moe_intermediate": 768, "vocab": 151936,
                 "types": "Q4_K attn/gate/up/embd, Q6_K down/output, F32 router/norms", "global_batch": 1,
                 "prompt": N_PROMPT, "l2": "not flushed: each step streams ~2 GB of weights (> 126 MB L2)"}
GATEUP_BYTES_T1 = 8 * 2 * 768 * 1152 + 2048 * 3 + 8 * 768 * 4  # routed experts' gate+up, XF digits, h


def decode_model(rank: int):
    """Path of the config-4 GGUF (generated once per machine; rank 0 writes, the others wait)."""
    import synth
    cfg = synth.config4_30b()
    d = os.environ.get("EAHMMF_MODEL_DIR", "/tmp/eahmmf_models")
    path = os.path.join(d, f"{cfg.name}-L{cfg.n_layer}-{synth.config_digest(cfg)}.gguf")
    if rank == 0:
        return synth.cached_gguf(cfg, d, workers=max(1, min(48, (os.cpu_count() or 2) - 1)))
    t0 = time.time()
    while not os.path.exists(path):
        if time.time() - t0 > 1800:
            raise RuntimeError("timed out waiting for rank 0 to write the model")
        time.sleep(2)
    return path


def decode_prompt(rank: int, n: int = N_PROMPT):
    import synth
    return synth._rng(4, 0x50, rank).integers(0, 151936, n).astype(np.int32)


def cpu_decode(path: str, steps: int, warmup: int, budget_s: float | None):
    """Reference engine decode tokens/s on the host: a short prompt, then single-token forward passes
    (Engine::forward through eref_engine_eval), `steps` of them or as many as fit in budget_s."""
    import oracle
    ref = oracle.Reference(threads=os.cpu_count() or 1)
    n_prompt = 8
    eng = ref.engine(path, n_prompt + warmup + max(steps, 4096 if budget_s else steps) + 8)
    prompt = decode_prompt(0, n_prompt)
    lg = eng.eval(prompt, 0, 32)
    pos = n_prompt
    for _ in range(warmup):
        lg = eng.eval([int(lg.argmax())], pos, 1)
        pos += 1
    t0, done = time.perf_counter(), 0
    while True:
        lg = eng.eval([int(lg.argmax())], pos, 1)
        pos += 1
        done += 1
        el = time.perf_counter() - t0
        if (budget_s is None and done >= steps) or (budget_s is not None and el >= budget_s):
            break
        if pos >= eng.dims["n_ctx"] - 1:
            break
    eng.close()
    return done / el, ref.threads, done, n_prompt


def decode_ours(args, rank: int, world: int, local: int, path: str):
    import torch
    import eahmmf_b200 as eb

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n_ctx = N_PROMPT + args.warmup + args.steps + 16
    eng = eb.Engine(path, n_ctx)
    prompt = decode_prompt(rank)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(dev)

    # prefill + first token (untimed), warm-up steps (captures the step graph), then the timed steps
    rc, first, _ = eng.greedy(prompt, 1, 64)
    if rc:
        raise RuntimeError(f"eahmmf_engine_greedy failed: {rc}")
    rc, warm, _ = eng.decode(args.warmup)
    if rc:
        raise RuntimeError(f"eahmmf_engine_decode failed: {rc}")
    barrier()
    with Clocks(local) as clk:
        rc, toks, ms = eng.decode(args.steps)
        barrier()
    if rc:
        raise RuntimeError(f"eahmmf_engine_decode failed: {rc}")
    nodes = eng.graph_nodes()

    # per-operation profile of a few eager steps, and the MoE stages inside them
    eng.profile(True)
    eb.MoeLayer.profile(True)
    eng.decode(4)
    ops = eng.profile_read()
    moe_stages = eb.MoeLayer.profile_read()
    eb.MoeLayer.profile(False)
    eng.profile(False)
    barrier()

    # end to end through the C ABI: host prompt in, K host tokens out
    t0 = time.perf_counter()
    rc, gen, _ = eng.greedy(prompt, args.steps, 64)
    e2e_s = time.perf_counter() - t0
    if rc:
        raise RuntimeError(f"eahmmf_engine_greedy failed: {rc}")
    # the captured-graph steps and the greedy call generate the same sequence
    seq = np.concatenate([first, warm, toks])[:args.steps]
    consistent = bool(np.array_equal(gen, seq))
    eng.close()

    t_ms = ms
    if world > 1:
        import torch.distributed as dist
        v = torch.tensor([t_ms, e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t_ms, e2e_s = float(v[0]), float(v[1])
    value = args.steps * world / (t_ms * 1e-3)
    peak, peak_kind = peaks()
    gu_us = float(moe_stages[GATEUP_STAGE]) if len(moe_stages) else 0.0
    achieved = GATEUP_BYTES_T1 / (gu_us * 1e-6) / 1e9 if gu_us > 0 else 0.0
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get("k_moe_gateup_decode_T1", {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        pass
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8/s8 tensor-core MMA, s32 -> fp32 accumulate (fp32 activations)",
        "data": "synthetic (seeded random weights, random-id prompt)",
        "config": dict(DECODE_CONFIG, parallelism=f"replicas x{world}"),
        "e2e": {"value": args.steps * world / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": N_PROMPT * 4,
                "d2h_bytes_per_step": args.steps * 4,
                "step": "one eahmmf_engine_greedy call: 512-token prompt in, prefill in 64-token passes, K tokens out"},
        "gpu_launches": nodes * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if peak else None, "traffic": traffic, "kernel": "k_moe_gateup (T=1)",
                     "peak_source": peak_kind,
                     "timing": "CUDA events around the gate/up kernel on its stream, mean over 4 eager steps x 48 layers"},
        "clocks": clk.summary(),
        "decode_ops_us_per_step": ops,
        "tokens_consistent": consistent,
        "moe_stages_us_per_layer": {"router": float(moe_stages[0]), "route": float(moe_stages[1]),
                                    "gateup": float(moe_stages[2]), "down_combine": float(moe_stages[3])}
        if len(moe_stages) else None,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, n, npr = cpu_decode(path, steps=1, warmup=1, budget_s=args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                "sample": f"{n} decode steps of the reference engine (oracle/_ref) on the same GGUF "
                                          f"after a {npr}-token prompt"}
    return line


# ---- ragged workload (config 3) ---------------------------------------------------------------------
RAGGED_CONFIG = {"workload": "config3: ragged continuous batch through one Qwen3-30B-A3B-shape MoE layer",
                 "sequences": 64, "tokens_per_sequence": "uniform 1..512", "hidden": D, "experts": E, "top_k": K,
                 "moe_intermediate": FF, "gate_up": "Q4_K", "down": "Q6_K",
                 "router_logits": "N(0,1) + log-Zipf(1.1) expert bias",
                 "l2": "not flushed: each call streams the 391 MB expert set and >1 GB of activations"}


def ragged_inputs(step: int, rank: int):
    import synth
    counts = synth.ragged_batch(64, 1, 512, seed=3 + 100 * step + rank)
    T = int(counts.sum())
    seed = 77 + 1000 * step + 7919 * rank
    return (T, synth.activations(T, D, seed=seed), synth.activations(T, D, seed=seed + 1),
            synth.router_logits(T, E, seed=seed + 2, zipf_bias=1.1))


def ragged_ours(args, rank: int, world: int, local: int):
    import torch
    import eahmmf_b200 as eb
    import synth

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ex = synth.expert_set()
    layer = eb.MoeLayer.from_expert_set(ex, n_used=K)
    nsteps = args.warmup + args.steps
    inputs = [ragged_inputs(s % 2, rank) for s in range(nsteps)]  # two distinct batches, alternating
    tmax = max(v[0] for v in inputs)
    ws = torch.zeros(layer.workspace_bytes(tmax), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    dev_in = [(T, torch.from_numpy(x).to(dev), torch.from_numpy(xn).to(dev), torch.from_numpy(lg).to(dev))
              for T, x, xn, lg in inputs[:2]]

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(dev)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    us, toks = [], 0
    barrier()
    with Clocks(local) as clk:
        for s in range(nsteps):
            T, x, xn, lg = dev_in[s % 2]
            xo = x.clone()
            ev0.record(stream)
            if layer(T, xn, lg, xo, ws, stream=stream, d_status=status):
                raise RuntimeError("eahmmf_cuda_moe_layer failed")
            ev1.record(stream)
            ev1.synchronize()
            if s >= args.warmup:
                us.append(ev0.elapsed_time(ev1) * 1e3)
                toks += T
        barrier()
    if int(status.item()):
        raise RuntimeError(f"kernel status {int(status.item())}")
    # stage pass: the tensor-core GEMM stages timed on their own (profiler events between the kernels)
    eb.MoeLayer.profile(True)
    T, x, xn, lg = dev_in[0]
    for _ in range(3):
        layer(T, xn, lg, x.clone(), ws, stream=stream)
    stages = eb.MoeLayer.profile_read()
    eb.MoeLayer.profile(False)
    # end to end: pinned host activations and logits in, the updated residual out
    T, hx, hxn, hlg = inputs[0]
    px, pxn, plg = (torch.from_numpy(a).pin_memory() for a in (hx, hxn, hlg))
    out = torch.empty_like(px).pin_memory()
    dx, dxn, dlg = (torch.empty(a.shape, dtype=a.dtype, device=dev) for a in (px, pxn, plg))
    e2e = []
    for _ in range(3):
        ev0.record(stream)
        dx.copy_(px, non_blocking=True)
        dxn.copy_(pxn, non_blocking=True)
        dlg.copy_(plg, non_blocking=True)
        layer(T, dxn, dlg, dx, ws, stream=stream)
        out.copy_(dx, non_blocking=True)
        ev1.record(stream)
        ev1.synchronize()
        e2e.append(ev0.elapsed_time(ev1) * 1e-3)
    t_total = float(np.sum(us)) * 1e-6
    if world > 1:
        import torch.distributed as dist
        v = torch.tensor([t_total], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t_total = float(v[0])
    flops = 2.0 * T * K * 3 * D * FF  # the three projections of every routed slot
    gemm_us = float(stages[2] + stages[3])
    achieved = flops / (gemm_us * 1e-6) / 1e12 if gemm_us > 0 else 0.0
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        peak = float(json.load(f).get("bf16_tflops", 1590.0))
    line = {
        "metric": "ragged MoE-layer tokens/s (config 3)", "value": toks * world / t_total, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 tcgen05 MMA (weights f16 per-row scaled, activations f16 hi/lo), fp32 accumulate",
        "data": "synthetic (seeded)", "config": dict(RAGGED_CONFIG, tokens_per_step=toks // args.steps,
                                                     parallelism=f"replicas x{world}"),
        "e2e": {"value": T / min(e2e), "unit": "tok/s", "h2d_bytes_per_step": int(T * (2 * D + E) * 4),
                "d2h_bytes_per_step": int(T * D * 4)},
        "gpu_launches": 11 * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "kernel": "k_gemm_tc<gate/up> + k_gemm_tc<down>",
                     "peak_source": "measured (cuBLAS bf16 burst)",
                     "timing": "CUDA events around the two GEMM stages (with the h repack between them)"},
        "stages_us": {"router": float(stages[0]), "route_dequant_pack": float(stages[1]),
                      "gateup": float(stages[2]), "down_pack_combine": float(stages[3])},
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        ref = oracle.Reference(threads=os.cpu_count() or 1)
        n = 256
        x, xn, lg = inputs[0][1][:n], inputs[0][2][:n], inputs[0][3][:n]
        ref.moe_layer(x, xn, lg, list(ex.gate), list(ex.up), list(ex.down), ex.types, ex.row_bytes, K)
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 20.0) or reps == 0:
            ref.moe_layer(x, xn, lg, list(ex.gate), list(ex.up), list(ex.down), ex.types, ex.row_bytes, K)
            reps += 1
        v = n * reps / (time.perf_counter() - t0)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": ref.threads, "kind": "reference",
                                "sample": f"{reps} x {n} tokens of the batch through the reference CPU MoE block "
                                          "(oracle/_ref, 64-token passes)"}
    return line


def profile_ragged(T: int) -> int:
    """No timing: three grouped-path calls of the config-2 layer on T ragged tokens (the small case for
    ncu captures of the tcgen05 GEMMs)."""
    import torch
    import eahmmf_b200 as eb
    import synth
    ex = synth.expert_set()
    layer = eb.MoeLayer.from_expert_set(ex, n_used=8)
    xt = torch.from_numpy(synth.activations(T, ex.D, 5)).cuda()
    lg = torch.from_numpy(synth.router_logits(T, ex.n_expert, 6, zipf_bias=1.1)).cuda()
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    for _ in range(3):
        if layer(T, xt, lg, xt.clone(), ws):
            raise RuntimeError("eahmmf_cuda_moe_layer failed")
    torch.cuda.synchronize()
    print(json.dumps({"profile_ragged": T, "ok": True}))
    return 0


# ---- expert-parallel workload (config 5) ---------------------------------------------------------------
EP_SEQS = 32
EP_CONFIG = {"workload": "config5: Qwen3-235B-A22B-shape MoE layer, expert-parallel decode step",
             "hidden": 4096, "experts": 128, "top_k": 8, "moe_intermediate": 1536, "gate_up": "Q4_K", "down": "Q6_K",
             "sequences": EP_SEQS, "tokens_per_step": EP_SEQS,
             "l2": "not flushed: the routed experts of a step are ~100 MB per rank and change every step"}


def ep_ours(args, rank: int, world: int, local: int):
    import torch
    import torch.distributed as dist
    import ep
    import synth

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world == 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", rank=0, world_size=1, init_method="tcp://127.0.0.1:" + str(29600 + local),
                                timeout=timedelta(seconds=120), device_id=dev)
    ex = synth.expert_set(D=4096, FF=1536, n_expert=128, seed=5, d_sigma=0.002)
    layer = ep.EpMoeLayer(ex, n_used=8, device=dev)
    del ex
    T = EP_SEQS // world + (1 if rank < EP_SEQS % world else 0)
    nsteps = args.warmup + args.steps
    xs = [(torch.from_numpy(synth.activations(T, 4096, seed=1000 * s + rank)).to(dev),
           torch.from_numpy(synth.activations(T, 4096, seed=1000 * s + 500 + rank)).to(dev),
           torch.from_numpy(synth.router_logits(T, 128, seed=1000 * s + 900 + rank)).to(dev)) for s in range(nsteps)]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    dist.barrier()
    torch.cuda.synchronize(dev)
    with Clocks(local) as clk:
        for s in range(nsteps):
            x, xn, lg = xs[s]
            xo = x.clone()
            dist.barrier()
            ev0.record()
            layer(xn, lg, xo)
            ev1.record()
            ev1.synchronize()
            if s >= args.warmup:
                times.append(ev0.elapsed_time(ev1))
        dist.barrier()
        torch.cuda.synchronize(dev)
    t = torch.tensor([float(np.sum(times))], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_ms = float(t[0])
    value = EP_SEQS * args.steps / (t_ms * 1e-3)
    line = {"metric": "EP MoE-layer decode tokens/s (config 5, 32 sequences)", "value": value, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "u8/s8 tensor-core MMA, fp32 activations; fp32 rows over NCCL all-to-all",
            "data": "synthetic (seeded)", "config": dict(EP_CONFIG, parallelism=f"ep{world}"),
            "clocks": clk.summary(), "gpu_launches": None}
    if world == 1 and dist.is_initialized():
        dist.destroy_process_group()
    return line


def profile_decode(n_layer: int) -> int:
    """No timing: a config-4-shape model with n_layer layers (generated if absent), an 8-token prompt
    in one pass and 4 greedy tokens (3 captured-graph steps). The case ncu captures of the decode
    kernels are taken on: 48 layers for the launch list, 2 layers (1.2 GB) for full captures."""
    import synth
    cfg = synth.config4_30b(n_layer=n_layer)
    path = synth.cached_gguf(cfg, workers=max(1, min(48, (os.cpu_count() or 2) - 1)))
    import eahmmf_b200 as eb
    eng = eb.Engine(path, 64)
    rc, out, _ = eng.greedy(decode_prompt(0, 8), 4, 8)
    eng.close()
    if rc:
        raise RuntimeError(f"eahmmf_engine_greedy returned {rc}")
    print(json.dumps({"profile_decode": n_layer, "tokens": [int(v) for v in out], "ok": True}))
    return 0


def profile_prefill(n_layer: int) -> int:
    """No timing: a config-4-shape model with n_layer layers, one 512-token prompt through eval in
    passes of 64 (the prompt half of the e2e step). The case the prefill launch list is taken on."""
    import synth
    cfg = synth.config4_30b(n_layer=n_layer)
    path = synth.cached_gguf(cfg, workers=max(1, min(48, (os.cpu_count() or 2) - 1)))
    import eahmmf_b200 as eb
    eng = eb.Engine(path, 1024)
    rc, lg = eng.eval(decode_prompt(0, 512), 0, 64)
    eng.close()
    if rc:
        raise RuntimeError(f"eahmmf_engine_eval returned {rc}")
    print(json.dumps({"profile_prefill": n_layer, "argmax": int(np.argmax(lg)), "ok": True}))
    return 0


def profile_case(T: int) -> int:
    """Three calls of the config-2 MoE layer at T tokens on fixed seeded inputs, nothing timed: the
    small case ncu captures are taken on (a few hundred MB on the device)."""
    import torch
    import eahmmf_b200 as eb
    import synth
    ex = synth.expert_set()
    layer = eb.MoeLayer.from_expert_set(ex, n_used=8)
    xt = torch.from_numpy(synth.activations(T, ex.D, 5)).cuda()
    lg = torch.from_numpy(synth.router_logits(T, ex.n_expert, 6)).cuda()
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    for _ in range(3):
        st = layer(T, xt, lg, xt.clone(), ws)
        if st:
            raise RuntimeError(f"eahmmf_cuda_moe_layer returned {st}")
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": T, "ok": True}))
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (decode: 128, layer: 20)")
    ap.add_argument("--warmup", type=int, default=None, help="warm-up steps (decode: 8, layer: 3)")
    ap.add_argument("--workload", choices=("decode", "layer", "ragged", "ep"), default="decode")
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--profile-case", type=int, metavar="T", default=0,
                    help="no timing: run the config-2 layer three times at T tokens (a small case for ncu)")
    ap.add_argument("--profile-ragged", type=int, metavar="T", default=0,
                    help="no timing: three grouped-path layer calls on T ragged tokens (a small case for ncu)")
    ap.add_argument("--profile-decode", type=int, metavar="LAYERS", default=0,
                    help="no timing: 8-token prompt + 4 greedy tokens on a config-4-shape model of LAYERS layers")
    ap.add_argument("--profile-prefill", type=int, metavar="LAYERS", default=0,
                    help="no timing: one 512-token prompt in passes of 64 on a config-4-shape model of LAYERS layers")
    args = ap.parse_args()
    if args.profile_prefill:
        return profile_prefill(args.profile_prefill)
    if args.profile_case:
        return profile_case(args.profile_case)
    if args.profile_decode:
        return profile_decode(args.profile_decode)
    if args.profile_ragged:
        return profile_ragged(args.profile_ragged)
    decode = args.workload == "decode"
    if args.steps is None:
        args.steps = 256 if decode else 5 if args.workload == "ragged" else 20
    if args.warmup is None:
        args.warmup = 8 if decode else 3
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference" and decode:
        if rank != 0:
            return 0
        path = decode_model(0)
        v, cores, n, npr = cpu_decode(path, steps=min(args.steps, 24), warmup=1, budget_s=None)
        line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": n, "warmup": 1,
                "ms_per_step": 1e3 / v, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "fp32 (reference CPU)", "data": "synthetic (seeded random weights, random-id prompt)",
                "config": dict(DECODE_CONFIG, parallelism="reference CPU", prompt=npr), "impl": "reference",
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                 "sample": f"{n} decode steps of the reference engine (oracle/_ref) on the same GGUF "
                                           f"after a {npr}-token prompt (bounded: the reference takes ~0.2 s/token)"},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    if args.impl == "reference":
        if rank != 0:
            return 0
        import synth
        ex = synth.expert_set()
        v, cores, n = cpu_reference(ex, steps=args.steps, warmup=args.warmup)
        line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
                "ms_per_step": TOKENS_PER_STEP / v * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp32 (reference CPU)", "data": "synthetic (seeded)",
                "config": dict(LAYER_CONFIG, parallelism="reference CPU"), "impl": "reference",
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                 "sample": f"{n} steps of T=1..8 through the reference CPU MoE block (oracle/_ref)"},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    path = decode_model(rank) if decode else None  # before any CUDA work (spawned writer processes)
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    try:
        if decode:
            line = decode_ours(args, rank, world, local, path)
        elif args.workload == "ragged":
            line = ragged_ours(args, rank, world, local)
        elif args.workload == "ep":
            line = ep_ours(args, rank, world, local)
        else:
            line = layer_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
