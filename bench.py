#!/usr/bin/env python3
"""Benchmark of the B200 expert hot path (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|layer|ragged|ep]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1: one process per GPU)

Workload `decode` (default; BASELINE config 4, the configuration the headline metric is quoted on):
greedy batch-1 decode of a Qwen3-30B-A3B-shape model -- 48 layers, hidden 2048, 32 q / 4 kv heads of
128, 128 experts top-8, intermediate 768, vocab 151936; Q4_K attention/gate/up/embedding, Q6_K
down/output, F32 router/norms; seeded random weights written as a GGUF (synth.config4_30b) and loaded
through eahmmf_engine_load. A 512-token random-id prompt is prefilled (timed apart: `prefill`), then W
decode steps warm up and K decode steps are timed. One step = one token = one forward pass (48 layers +
output GEMV + argmax), replayed as the captured CUDA graph.

  value     decode tokens/s over all ranks: K * ranks / (device time of the K steps, CUDA events on the
            engine's stream, max over ranks). Each step streams ~2 GB of weights (far above the 126 MB
            L2), so no flush is needed between steps.
  e2e       the same decode driven from the host through the C ABI (eahmmf_engine_step: token in from
            pinned memory, one forward pass, next token out, synchronised), after an untimed prefill of
            the same prompt -- the reference arm's decode follows its prefill the same way.
            e2e_with_prompt: one eahmmf_engine_greedy call with the prompt inside the timed region.
  roofline  k_moe_gateup (the Q4_K MoE decode kernel the target names) at T = 1: algorithmic bytes
            (the 8 routed experts' gate and up matrices + staged activations + h outputs) / its mean
            duration over every layer of a few eager decode steps (CUDA events around the kernel on
            its stream), against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the reference engine itself (oracle/_ref, compiled from the reference sources) on the
            same GGUF and prompt, all host threads (rank 0 at N = 1); its greedy tokens are compared with
            ours over the steps both produce (tokens_match_reference; exit 1 on a mismatch).
  ep        the config-5 expert-parallel MoE layer (Qwen3-235B-A22B shape, 32 sequences per step) over
            the job's N ranks (ep.py: NCCL all-to-all of fixed-capacity blocks), with its stage times.

Workload `layer`: one MoE layer of the same shape on decode batches T = 1..8 (one
step = eight layer calls, 36 tokens), L2 flushed before every call; value = tokens/s of the layer.
Workload `ragged` (config 3) and `ep` (config 5 alone) as described at their functions.

--impl reference times the reference CPU implementation alone on the same workload (all host threads).
Multi-GPU: the decode path has no exchange step, so N ranks run N replicas (weak scaling, step time the
maximum over ranks); the `ep` object measures the path that does exchange, over the same N ranks.
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
            traffic = json.load(f).get("k_moe_gateup_T8", {}).get("dram_bytes_per_launch")
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
                     "traffic_case": "dram bytes of one launch at T = 8 (profiles/traffic.json); achieved is the mean "
                                     "over T = 1..8",
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
EXTRA_STEPS = 600  # untimed steps after the timed ones: the clock sampler (100 ms period) sees >= 1 s of decode
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


def cpu_decode(path: str, prompt, steps: int, warmup: int, budget_s: float | None):
    """The reference engine on the host (oracle/_ref, all host threads): the prompt through Engine::eval
    in 64-token passes (timed apart), its argmax, `warmup` untimed single-token forward passes, then
    `steps` timed ones -- or, with budget_s, as many more as fit in that many seconds. The reference's
    own generate loop (qwen3moe.cpp:1294-1310) with greedy selection (first maximum, :1103).
    Returns a dict: tok_s, cores, steps, prefill_s, ids (the first token, then every step's)."""
    import oracle
    ref = oracle.Reference(threads=os.cpu_count() or 1)
    n_ctx = len(prompt) + warmup + max(steps, 512 if budget_s else steps) + 8
    eng = ref.engine(path, n_ctx)
    t0 = time.perf_counter()
    lg = eng.eval(prompt, 0, 64)
    prefill_s = time.perf_counter() - t0
    ids = [int(np.argmax(lg))]
    pos = len(prompt)
    for _ in range(warmup):
        lg = eng.eval([ids[-1]], pos, 1)
        pos += 1
        ids.append(int(np.argmax(lg)))
    t0, done = time.perf_counter(), 0
    while True:
        lg = eng.eval([ids[-1]], pos, 1)
        pos += 1
        done += 1
        ids.append(int(np.argmax(lg)))
        el = time.perf_counter() - t0
        if done >= steps and (budget_s is None or el >= budget_s):
            break
        if pos >= eng.dims["n_ctx"] - 1:
            break
    eng.close()
    return {"tok_s": done / el, "cores": ref.threads, "steps": done, "prefill_s": prefill_s, "ids": ids}


BATCH_SEQS, BATCH_PROMPT, BATCH_STEPS = 32, 128, 32


def batched_decode(eng, rank: int):
    """Several sequences decoded together on the same model (eahmmf_engine_set_slots / prefill_slot /
    step_slots): 32 sequences with their own 128-token random prompts, then 32 greedy steps that each run
    one token of every sequence as a single forward pass. Tokens/s = sequence-tokens of the timed steps
    / wall time of those steps through the C ABI (each step copies its rows in and its tokens out).
    The engine returns to one slot afterwards."""
    import synth
    if eng.set_slots(BATCH_SEQS):
        return {"unavailable": "eahmmf_engine_set_slots failed"}
    rng = synth._rng(9, 0xB5, rank)
    toks, pos = [], []
    for s in range(BATCH_SEQS):
        p = rng.integers(0, 151936, BATCH_PROMPT).astype(np.int32)
        rc, first = eng.prefill_slot(s, p, 64)
        if rc:
            raise RuntimeError(f"eahmmf_engine_prefill_slot failed: {rc}")
        toks.append(first)
        pos.append(BATCH_PROMPT)
    slots = list(range(BATCH_SEQS))
    for _ in range(3):  # warm-up steps
        rc, toks = eng.step_slots(slots, pos, toks)
        pos = [p + 1 for p in pos]
    t0 = time.perf_counter()
    for _ in range(BATCH_STEPS):
        rc, toks = eng.step_slots(slots, pos, toks)
        if rc:
            raise RuntimeError(f"eahmmf_engine_step_slots failed: {rc}")
        pos = [p + 1 for p in pos]
    el = time.perf_counter() - t0
    eng.set_slots(1)
    return {"sequences": BATCH_SEQS, "prompt": BATCH_PROMPT, "steps": BATCH_STEPS,
            "tok_s": BATCH_SEQS * BATCH_STEPS / el, "ms_per_step": el / BATCH_STEPS * 1e3,
            "timing": "wall clock of the timed steps (host-driven, synchronous per step)"}


OVERSUB_LAYERS, OVERSUB_STEPS = 1, 24  # cache of one layer's experts: 1/48 of the model's


def oversubscribed_decode(path: str, rank: int, want):
    """The same model with a device cache of one layer's experts (1/48 of the experts' bytes) in HBM
    (eahmmf_engine_load_budget): the rest stay in host memory and reach the cache on demand, with the next layer's last routed
    experts prefetched while the current layer computes. The same 512-token prompt and greedy steps as
    the resident measurement (the prompt untimed); tokens/s of the timed steps (host-driven: the host
    makes each layer's routed experts resident), the cache counters, and whether the tokens equal the
    resident engine's."""
    import eahmmf_b200 as eb
    import synth
    cfg = synth.config4_30b()
    tg, tu, td = cfg.expert_types
    a256 = lambda v: (v + 255) // 256 * 256  # noqa: E731
    foot = a256(a256(a256(cfg.FF * synth.row_bytes(tg, cfg.D)) + cfg.FF * synth.row_bytes(tu, cfg.D)) +
                cfg.D * synth.row_bytes(td, cfg.FF))
    total = cfg.n_layer * cfg.n_expert * foot
    budget = OVERSUB_LAYERS * cfg.n_expert * foot
    t0 = time.perf_counter()
    e = eb.Engine(path, N_PROMPT + OVERSUB_STEPS + 16, expert_vram_bytes=budget)
    load_s = time.perf_counter() - t0
    try:
        rc, first, _ = e.greedy(decode_prompt(rank), 1, 64)
        if rc:
            raise RuntimeError(f"eahmmf_engine_greedy failed: {rc}")
        s0 = e.cache_stats()
        t0 = time.perf_counter()
        rc, toks, _ = e.decode(OVERSUB_STEPS)
        el = time.perf_counter() - t0
        if rc:
            raise RuntimeError(f"eahmmf_engine_decode failed: {rc}")
        s1 = e.cache_stats()
    finally:
        e.close()
    d = {k: s1[k] - s0[k] for k in ("hits", "misses", "prefetched", "prefetch_hits", "evictions", "bytes_h2d")}
    ids = [int(first[0])] + [int(v) for v in toks]
    return {"expert_vram_bytes": budget, "expert_bytes_total": total, "cache_experts": s1["slots"],
            "dma_from_mapping": bool(s1["dma"]), "load_s": load_s, "steps": OVERSUB_STEPS,
            "tok_s": OVERSUB_STEPS / el, "ms_per_step": el / OVERSUB_STEPS * 1e3,
            "hit_rate": d["hits"] / max(1, d["hits"] + d["misses"]), "h2d_gb_per_step": d["bytes_h2d"] / OVERSUB_STEPS / 1e9,
            "counters_timed_steps": d, "tokens_match_resident": ids == list(want[:len(ids)])}


def first_mismatch(a, b):
    m = min(len(a), len(b))
    d = np.nonzero(np.asarray(a[:m]) != np.asarray(b[:m]))[0]
    return (int(d[0]) if len(d) else None), m


def decode_ours(args, rank: int, world: int, local: int, path: str):
    import torch
    import eahmmf_b200 as eb

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n_ctx = N_PROMPT + args.warmup + args.steps + EXTRA_STEPS + 16
    t0 = time.perf_counter()
    eng = eb.Engine(path, n_ctx)
    load_s = time.perf_counter() - t0
    # the staged copy checked against the file: hash64 of every expert component, on the device
    t0 = time.perf_counter()
    vrc, n_checked, n_bad = eng.verify()
    verify_s = time.perf_counter() - t0
    if vrc or n_bad:
        raise RuntimeError(f"eahmmf_engine_verify: rc {vrc}, {n_bad} of {n_checked} expert components differ")
    prompt = decode_prompt(rank)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(dev)

    # prefill + first token (timed apart, wall clock of the call), warm-up steps (the first captures the
    # step graph), the timed steps (device events on the engine's stream), then untimed steps so that the
    # clock sampler covers more than a second of the same decode
    barrier()
    t0 = time.perf_counter()
    rc, first, _ = eng.greedy(prompt, 1, 64)
    prefill_s = time.perf_counter() - t0
    if rc:
        raise RuntimeError(f"eahmmf_engine_greedy failed: {rc}")
    with Clocks(local) as clk:
        rc, warm, _ = eng.decode(args.warmup)
        if rc:
            raise RuntimeError(f"eahmmf_engine_decode failed: {rc}")
        barrier()
        rc, toks, ms = eng.decode(args.steps)
        barrier()
        if rc:
            raise RuntimeError(f"eahmmf_engine_decode failed: {rc}")
        rc, _, _ = eng.decode(EXTRA_STEPS)
        if rc:
            raise RuntimeError(f"eahmmf_engine_decode failed: {rc}")
    nodes = eng.graph_nodes()
    seq = [int(v) for v in np.concatenate([first, warm, toks])]

    # per-operation profile of a few eager steps, and the MoE stages inside them
    eng.profile(True)
    eb.MoeLayer.profile(True)
    eng.decode(4)
    ops = eng.profile_read()
    moe_stages = eb.MoeLayer.profile_read()
    eb.MoeLayer.profile(False)
    eng.profile(False)
    barrier()

    # end to end through the C ABI, host-driven as the reference's generate loop: the same prompt
    # prefilled again (untimed), then per step eahmmf_engine_step -- the input token copied in from
    # pinned host memory, one forward pass, the next token and the status word copied back
    rc, lg = eng.eval(prompt, 0, 64)
    if rc:
        raise RuntimeError(f"eahmmf_engine_eval failed: {rc}")
    tok = int(np.argmax(lg))
    e2e_ids = [tok]
    for _ in range(args.warmup):
        rc, tok = eng.step(tok)
        if rc:
            raise RuntimeError(f"eahmmf_engine_step failed: {rc}")
        e2e_ids.append(tok)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rc, tok = eng.step(tok)
        if rc:
            raise RuntimeError(f"eahmmf_engine_step failed: {rc}")
        e2e_ids.append(tok)
    e2e_s = time.perf_counter() - t0
    # and one greedy call with the prompt inside the timed region
    barrier()
    t0 = time.perf_counter()
    rc, gen, _ = eng.greedy(prompt, args.steps, 64)
    e2e_prompt_s = time.perf_counter() - t0
    if rc:
        raise RuntimeError(f"eahmmf_engine_greedy failed: {rc}")
    consistent = bool(e2e_ids == seq and [int(v) for v in gen] == seq[:args.steps])
    batched = None if args.no_configs else batched_decode(eng, rank)
    eng.close()
    # one process (each rank would hold its own pinned copy of the model's 19 GB of experts)
    oversub = None if args.no_configs or world > 1 else oversubscribed_decode(path, rank, e2e_ids)

    t_ms = ms
    if world > 1:
        import torch.distributed as dist
        v = torch.tensor([t_ms, e2e_s, e2e_prompt_s, prefill_s], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t_ms, e2e_s, e2e_prompt_s, prefill_s = (float(u) for u in v)
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
        "e2e": {"value": args.steps * world / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 8,
                "step": "eahmmf_engine_step through the C ABI: the input token copied in from pinned host memory, one "
                        "forward pass, the next token and the status word copied back, synchronised; after an untimed "
                        "prefill of the same 512-token prompt (the reference arm's timed steps follow its prefill the "
                        "same way)"},
        "e2e_with_prompt": {"value": args.steps * world / e2e_prompt_s, "unit": "tok/s",
                            "h2d_bytes_per_step": N_PROMPT * 4 // args.steps, "d2h_bytes_per_step": 4,
                            "step": "one eahmmf_engine_greedy call: the 512-token prompt in, prefill in 64-token passes, "
                                    "K tokens out"},
        "prefill": {"tok_s": N_PROMPT / prefill_s, "ms": prefill_s * 1e3, "passes": "64-token eval passes + argmax"},
        "staging": {"load_s": load_s, "verify_s": verify_s, "components_verified": n_checked, "mismatches": n_bad,
                    "how": "GGUF mmap -> pinned double buffer -> HBM; hash64 of every expert component on the "
                           "device against the file's on the host"},
        "gpu_launches": nodes * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if peak else None, "traffic": traffic, "kernel": "k_moe_gateup (T=1)",
                     "peak_source": peak_kind,
                     "timing": "CUDA events around the gate/up kernel on its stream, mean over 4 eager steps x 48 layers"},
        "clocks": clk.summary(),
        "clocks_window": f"warm-up, the {args.steps} timed steps and {EXTRA_STEPS} more steps of the same decode "
                         "(the timed steps alone are shorter than the 100 ms sampling period)",
        "decode_ops_us_per_step": ops,
        "tokens_consistent": consistent,
        "moe_stages_us_per_layer": {"router": float(moe_stages[0]), "route": float(moe_stages[1]),
                                    "gateup": float(moe_stages[2]), "down_combine": float(moe_stages[3])}
        if len(moe_stages) else None,
        "tokens_match_reference": None,
        "batched_decode": batched,
        "oversubscribed_decode": oversub,
    }
    if not args.no_ep:
        line["ep"] = ep_measure(rank, world, local, dev, steps=20, warmup=3, cpu=(rank == 0 and world == 1 and
                                                                                  not args.no_cpu))
    if not args.no_configs:  # BASELINE configs 2 and 3 on the same ranks (short runs; their own CPU legs)
        sub = argparse.Namespace(steps=5, warmup=3, no_cpu=args.no_cpu, cpu_seconds=5.0)
        keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "config", "e2e", "roofline",
                "cpu_baseline", "stages_us", "layer_us_per_step", "dtype")
        c2 = layer_ours(sub, rank, world, local)
        line["config2_layer"] = {k: c2[k] for k in keep if k in c2}
        sub.steps = 3
        c3 = ragged_ours(sub, rank, world, local)
        line["config3_ragged"] = {k: c3[k] for k in keep if k in c3}
    if rank == 0 and world == 1 and not args.no_cpu:
        c = cpu_decode(path, prompt, steps=args.steps, warmup=args.warmup, budget_s=args.cpu_seconds)
        bad, m = first_mismatch(c["ids"], seq)
        line["tokens_match_reference"] = bad is None
        line["reference_tokens_compared"] = m
        line["first_mismatch"] = bad
        line["cpu_baseline"] = {"value": c["tok_s"], "unit": "tok/s", "cores": c["cores"], "kind": "reference",
                                "sample": f"{c['steps']} decode steps of the reference engine (oracle/_ref) on the same "
                                          f"GGUF after the same {N_PROMPT}-token prompt (prefill {c['prefill_s']:.1f} s, "
                                          f"untimed) and {args.warmup} warm-up steps",
                                "prefill_tok_s": N_PROMPT / c["prefill_s"]}
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
    gemm_us = float(stages[2])  # gate/up GEMM, h repack, down GEMM
    achieved = flops / (gemm_us * 1e-6) / 1e12 if gemm_us > 0 else 0.0
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        peak = float(json.load(f).get("bf16_tflops", 1590.0))
    line = {
        "metric": "ragged MoE-layer tokens/s (config 3)", "value": toks * world / t_total, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 tcgen05 MMA (weights and activations f16 with power-of-two row scales), fp32 accumulate",
        "data": "synthetic (seeded)", "config": dict(RAGGED_CONFIG, tokens_per_step=toks // args.steps,
                                                     parallelism=f"replicas x{world}"),
        "e2e": {"value": T / min(e2e), "unit": "tok/s", "h2d_bytes_per_step": int(T * (2 * D + E) * 4),
                "d2h_bytes_per_step": int(T * D * 4)},
        "gpu_launches": 10 * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "kernel": "k_gemm_tc<gate/up> + k_gemm_tc<down>",
                     "peak_source": "measured (cuBLAS bf16 burst)",
                     "timing": "CUDA events around the two GEMM kernels and the h repack between them"},
        "stages_us": {"router": float(stages[0]), "route_dequant_pack": float(stages[1]),
                      "gemms_and_h_repack": float(stages[2]), "combine": float(stages[3])},
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
EP_CONFIG = {"workload": "config5: Qwen3-235B-A22B-shape MoE layer, expert-parallel decode step of 32 sequences",
             "hidden": 4096, "experts": 128, "top_k": 8, "moe_intermediate": 1536, "gate_up": "Q4_K", "down": "Q6_K",
             "sequences": EP_SEQS, "tokens_per_step": EP_SEQS, "layers_of_model": 94,
             "l2": "not flushed: the routed experts of a step are ~1.3 GB over the ranks and alternate between two "
                   "token sets"}
EP_EXPERT_BYTES = 2 * 1536 * 2304 + 4096 * 1260  # one 235B-shape expert: Q4_K gate + up, Q6_K down


def ep_measure(rank: int, world: int, local: int, dev, steps: int = 20, warmup: int = 3, cpu: bool = False):
    """The config-5 expert-parallel MoE layer over the ranks of the job (ep.py: pack, one NCCL all-to-all of
    fixed-capacity blocks each way, assigned-expert application, expert-ordered combine; no host
    synchronisation). 32 decode tokens per step split over the ranks; each rank generates only its own
    128/world experts. Step time = CUDA events around the call on each rank, max over ranks. With `cpu`,
    the reference CPU MoE block (oracle/_ref) on the same 32 tokens (all experts: world 1 only)."""
    import torch
    import torch.distributed as dist
    import ep
    import synth

    own = not dist.is_initialized()
    if own:
        from datetime import timedelta
        port = 29600 + (os.getpid() % 1000)
        dist.init_process_group("nccl", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{port}",
                                timeout=timedelta(seconds=120), device_id=dev)
    try:
        E, K, D = 128, 8, 4096
        if E % world:
            return {"unavailable": f"{E} experts do not split over {world} ranks"}
        E_loc = E // world
        ex = synth.expert_set(D=D, FF=1536, n_expert=E, seed=5, d_sigma=0.002,
                              experts=range(rank * E_loc, (rank + 1) * E_loc))
        t_max = -(-EP_SEQS // world)
        T = EP_SEQS // world + (1 if rank < EP_SEQS % world else 0)
        layer = ep.EpMoeLayer(ex, E, K, t_max, device=dev)
        sets = []
        for s in range(2):  # two token sets, alternating
            seed = 1000 * s + 31 * rank
            sets.append(tuple(torch.from_numpy(a).to(dev) for a in (
                synth.activations(T, D, seed=seed), synth.activations(T, D, seed=seed + 500),
                synth.router_logits(T, E, seed=seed + 900))))
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for i in range(warmup + steps):
            x, xn, lg = sets[i % 2]
            xo = x.clone()
            dist.barrier()
            torch.cuda.synchronize(dev)
            ev0.record()
            layer(xn, lg, xo)
            ev1.record()
            ev1.synchronize()
            if i >= warmup:
                times.append(ev0.elapsed_time(ev1))
        if layer.be.check():
            raise RuntimeError(f"EP kernels raised status {layer.be.check()}")
        # one call with events between the stages
        stg = ep.stage_events()
        x, xn, lg = sets[0]
        dist.barrier()
        torch.cuda.synchronize(dev)
        layer(xn, lg, x.clone(), stages=stg)
        st_ms = ep.stage_ms(stg)
        n_uniq = int(torch.unique(layer.eid[layer.eid >= 0]).numel())
        v = torch.tensor([float(np.sum(times))] + [st_ms[k] for k in ep.STAGE_NAMES], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t_ms = float(v[0])
        stages = {k: float(v[1 + i]) for i, k in enumerate(ep.STAGE_NAMES)}
        peak, peak_kind = peaks()
        exp_bytes = n_uniq * EP_EXPERT_BYTES
        achieved = exp_bytes / (st_ms["experts"] * 1e-3) / 1e9 if st_ms["experts"] > 0 else 0.0
        out = {"metric": "EP MoE-layer decode tokens/s (config 5, 32 sequences per step)",
               "value": EP_SEQS * steps / (t_ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": steps,
               "warmup": warmup, "ms_per_step": t_ms / steps, "scaling": "strong",
               "config": dict(EP_CONFIG, parallelism=f"ep{world}", experts_per_rank=E_loc),
               "stages_ms_max_over_ranks": stages,
               "roofline_experts_rank0": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                          "frac": achieved / peak if peak else None, "peak_source": peak_kind,
                                          "bytes": exp_bytes,
                                          "what": f"{n_uniq} distinct routed experts' weights on rank 0 / its "
                                                  "assigned-expert stage (unpack + experts + return)"},
               "dispatch": "fixed-capacity blocks, one equal-split NCCL all-to-all each way, no host sync"}
        if cpu and world == 1:
            import oracle
            ref = oracle.Reference(threads=os.cpu_count() or 1)
            x, xn, lg = (a.cpu().numpy() for a in sets[0])
            args_ = (list(ex.gate), list(ex.up), list(ex.down), ex.types, ex.row_bytes, K)
            ref.moe_layer(x, xn, lg, *args_)
            t0, reps = time.perf_counter(), 0
            while reps < 3 or time.perf_counter() - t0 < 5.0:
                ref.moe_layer(x, xn, lg, *args_)
                reps += 1
            layer_s = (time.perf_counter() - t0) / reps
            out["cpu_baseline"] = {"value": EP_SEQS / layer_s, "unit": "tok/s", "cores": ref.threads,
                                   "kind": "reference", "layer_ms": layer_s * 1e3,
                                   "model_step_ms_extrapolated": 94 * layer_s * 1e3,
                                   "sample": f"{reps} calls of the reference CPU MoE block (oracle/_ref) on the same "
                                             "32 tokens; x 94 layers gives the reduced-layer extrapolation of a "
                                             "235B-shape decode step's MoE time"}
        return out
    finally:
        if own:
            dist.destroy_process_group()


def ep_ours(args, rank: int, world: int, local: int):
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    with Clocks(local) as clk:
        out = ep_measure(rank, world, local, dev, steps=args.steps, warmup=args.warmup,
                         cpu=(rank == 0 and world == 1 and not args.no_cpu))
    out.update({"higher_is_better": True, "vs_baseline": None,
                "dtype": "u8/s8 tensor-core MMA, fp32 activations; fp32 rows over NCCL all-to-all",
                "data": "synthetic (seeded)", "clocks": clk.summary(), "gpu_launches": None})
    return out


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
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg (and the reference token check)")
    ap.add_argument("--no-ep", action="store_true", help="decode: skip the config-5 expert-parallel measurement")
    ap.add_argument("--no-configs", action="store_true", help="decode: skip the short config-2 and config-3 runs")
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
        c = cpu_decode(path, decode_prompt(0), steps=args.steps, warmup=args.warmup, budget_s=None)
        v = c["tok_s"]
        line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": c["steps"],
                "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp32 (reference CPU)",
                "data": "synthetic (seeded random weights, random-id prompt)",
                "config": dict(DECODE_CONFIG, parallelism="reference CPU"), "impl": "reference",
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": c["cores"], "kind": "reference",
                                 "sample": f"{c['steps']} decode steps of the reference engine (oracle/_ref) on the "
                                           f"same GGUF after the same {N_PROMPT}-token prompt (prefill "
                                           f"{c['prefill_s']:.1f} s, untimed) and {args.warmup} warm-up steps"},
                "prefill": {"tok_s": N_PROMPT / c["prefill_s"], "ms": c["prefill_s"] * 1e3},
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
    if line.get("tokens_match_reference") is False:
        print(f"greedy tokens differ from the reference engine's at step {line.get('first_mismatch')}",
              file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
