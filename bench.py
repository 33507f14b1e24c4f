#!/usr/bin/env python3
"""Benchmark of the B200 expert hot path (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1: one replica per GPU)

Workload (the configuration the headline metric is quoted on): one Qwen3-30B-A3B-shape
MoE layer -- hidden 2048, 128 experts top-8, intermediate 768, Q4_K gate/up and Q6_K down, router
logits ~N(0,1), activations ~N(0,1), all seeded -- run on decode batches of T = 1..8 tokens. One step
is eight layer calls, T = 1, 2, ..., 8 (36 tokens); routing inputs change every step.

  value     tokens/s of the layer over all ranks: 36 * ranks / (device time of a step). Each layer
            call is timed with CUDA events on its stream; the L2 is flushed (256 MiB memset) before
            every call, outside the timed events.
  e2e       the same through the C ABI with host buffers: pinned host->device copies of the step's
            activations and logits, the call, and the device->host copy of the updated residual,
            all inside the timed events.
  roofline  the gate/up kernel (the step's largest weight stream): algorithmic bytes (weights of the
            routed experts + staged activations + outputs) / its duration, timed by CUDA events on the
            call's stream in a second pass over the same steps (stage events between the kernels would
            serialise them, so they are kept out of the pass that gives `value`), against the measured
            HBM copy bandwidth of this pool (MEASURED_PEAKS.json).
  cpu_baseline  the reference's own CPU code (oracle/_ref, compiled from the reference sources) on a
            bounded sample of the same workload, rank 0 at N = 1.

--impl reference times the reference CPU implementation alone on the same workload (all host threads).
Multi-GPU: the path has no exchange step at this configuration; N ranks run N replicas ("replicas only",
weak scaling); the step time is the maximum over ranks.
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
CONFIG = {"workload": "config2: Qwen3-30B-A3B-shape MoE layer decode, T=1..8 tokens per step",
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
def run_ours(args, rank: int, world: int, local: int):
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
        "data": "synthetic (seeded)", "config": dict(CONFIG, parallelism=f"replicas x{world}"),
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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--profile-case", type=int, metavar="T", default=0,
                    help="no timing: run the config-2 layer three times at T tokens (a small case for ncu)")
    args = ap.parse_args()
    if args.profile_case:
        return profile_case(args.profile_case)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank != 0:
            return 0
        import synth
        ex = synth.expert_set()
        v, cores, n = cpu_reference(ex, steps=args.steps, warmup=args.warmup)
        line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
                "ms_per_step": TOKENS_PER_STEP / v * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp32 (reference CPU)", "data": "synthetic (seeded)",
                "config": dict(CONFIG, parallelism="reference CPU"), "impl": "reference",
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                 "sample": f"{n} steps of T=1..8 through the reference CPU MoE block (oracle/_ref)"},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        line = run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
