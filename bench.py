#!/usr/bin/env python3
"""Benchmark: the routed FP8 MoE layer of MiMo-V2.5 on B200.

One step = one whole routed MoE layer at decode/verifier width 8: 8 tokens of
hidden 4096, sigmoid no-aux top-8 router over 256 experts (bf16 weight + f32
bias), dynamic FP8 activations, per selected expert fused gate/up + staged
SwiGLU + down over e4m3 weights with 128x128 f32 block scales, weighted
combine.  Weights, router and tokens are seeded synthetic tensors with the
checkpoint's shapes and distributions (no network for the checkpoint).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value      mean device time per layer (us), inputs resident in HBM, K layers
           enqueued back to back on one stream, CUDA events around them; each
           step routes a different token batch, so every step streams its own
           ~57 experts (~1.4 GB) from HBM -- far more than L2, no flush needed.
e2e        the same layer through the C ABI with HOST buffers (pinned), the
           H2D copy of the tokens and the D2H copy of the output inside the
           timed region, one synchronous call per step.
roofline   the fused gate/up GEMV (the dominant kernel): algorithmic bytes per
           launch / its CUDA-event duration, against MEASURED_PEAKS.json's HBM.
cpu_baseline  the CPU restatement of the reference's routed layer (oracle/,
           f32 reference order, all host threads) on the same routed layer.

With --gpus N > 1 (torchrun, one rank per GPU) each rank runs its own replica
of the layer; the line reports the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, EXPERTS, WIDTH = 4096, 2048, 256, 8
# DRAM traffic / algorithmic bytes of the fused gate/up GEMV, from one ncu
# capture of a 32-expert layer (profiles/k_gemv_mma_c2_small.md): 507.55 MB
# read+written for 503.84 MB of algorithmic bytes.  Traffic grows in
# proportion to the experts streamed, so the full-size launch's traffic is
# this ratio times its algorithmic bytes.
GATE_UP_TRAFFIC_RATIO = 507.55 / 503.84
METRIC = "routed FP8 MoE layer us @width 8"
CONFIG = {
    "workload": "C2: full routed MoE layer, decode/verifier width 8 (BASELINE.json configs[2])",
    "hidden": HIDDEN, "intermediate": INTER, "experts": EXPERTS, "top_k": 8, "tokens": WIDTH,
    "weights": "e4m3 + 128x128 f32 block scales, N(0,0.02) quantized per block (amax/448, RNE)",
    "router": "bf16 [256,4096] N(0,0.02) + f32 bias N(0,0.01)",
    "l2": "no flush: each step routes a fresh token batch and streams ~1.4 GB of experts (>> 126 MB L2)",
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML while running."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    handle = h
            if handle is None and pynvml.nvmlDeviceGetCount() == 1:
                handle = pynvml.nvmlDeviceGetHandleByIndex(0)
            self._nv, self._h = pynvml, handle
            if handle is not None:
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv, self._h = None, None

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self._h is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------- CPU baseline
def cpu_layer_baseline(x_np, sel, wts, bank_np, budget_s=12.0):
    """The reference's routed layer (src/text_endpoint.rs:5290) restated on the
    CPU (oracle/, f32 reference order, libm exp), all host threads."""
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    times = []
    t_end = time.perf_counter() + budget_s
    while not times or (time.perf_counter() < t_end and len(times) < 20):
        t0 = time.perf_counter()
        O.routed_layer(x_np, sel, wts, bank_np, O.ACC_F32, O.EXP_LIBM)
        times.append(time.perf_counter() - t0)
    return statistics.mean(times) * 1e6, threads, len(times)


def bank_to_host(bank, experts):
    out = []
    for e in range(len(bank)):
        if e in experts:
            g, u, d = bank[e]
            out.append(tuple(t.cpu().numpy() for p in (g, u, d) for t in (p.weight, p.scale)))
        else:
            out.append(None)
    # the oracle only touches selected experts; fill the rest with a tiny stand-in
    filler = next(o for o in out if o is not None)
    return [o if o is not None else filler for o in out]


# -------------------------------------------------------------- reference
def run_reference(args, rank):
    """--impl reference: the reference's CPU path (restated, oracle/) on this
    arm's config; rank 0 only."""
    if rank != 0:
        return
    import numpy as np
    import torch
    from mimo_prismwing_b200 import synth
    from oracle import oracle as O
    # same seeded layer as our arm, generated on the CPU
    experts_needed = None
    w, bias = synth.router(EXPERTS, HIDDEN, 7, "cpu")
    x = synth.activations(WIDTH, HIDDEN, 1000, "cpu")
    logits = O.router_logits(x.numpy(), w.view(torch.int16).numpy().view(np.uint16))
    sel, wts, _, _, _ = O.noaux_topk(logits, bias.numpy())
    experts_needed = sorted(set(sel.ravel().tolist()))
    bank_np = []
    filler = None
    for e in range(EXPERTS):
        if e in experts_needed:
            g, u, d = synth.expert(HIDDEN, INTER, 1000 + e, "cpu")
            t = tuple(a.numpy() for p in (g, u, d) for a in (p.weight, p.scale))
            bank_np.append(t)
            filler = filler or t
        else:
            bank_np.append(None)
    bank_np = [b if b is not None else filler for b in bank_np]
    times = []
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    for _ in range(max(1, args.warmup // 3)):
        O.routed_layer(x.numpy(), sel, wts, bank_np, O.ACC_F32, O.EXP_LIBM)
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.routed_layer(x.numpy(), sel, wts, bank_np, O.ACC_F32, O.EXP_LIBM)
        times.append(time.perf_counter() - t0)
    us = statistics.mean(times) * 1e6
    line = {
        "metric": METRIC, "value": round(us, 3), "unit": "us", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": dict(CONFIG, unique_experts=len(experts_needed)),
        "cpu_baseline": {"value": round(us, 3), "unit": "us", "cores": threads, "kind": "port",
                         "sample": f"one routed layer (8 tokens, {len(experts_needed)} experts) x {len(times)} steps; "
                                   "oracle/pw_oracle.c routed layer, f32 reference order, libm exp"},
        "e2e": {"value": round(us, 3), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import WideMoeRuntime

    torch.cuda.set_device(local_rank)
    dev = f"cuda:{local_rank}"
    rt = WideMoeRuntime.compile_with_fused_gate_up(local_rank)
    bank = [synth.expert(HIDDEN, INTER, 1000 + e, dev) for e in range(EXPERTS)]
    handle = rt.create_bank(bank)
    w, bias = synth.router(EXPERTS, HIDDEN, 7, dev)
    n_batches = args.steps + args.warmup
    xs = [synth.activations(WIDTH, HIDDEN, 1000 + i + 7919 * rank, dev) for i in range(n_batches)]
    y = torch.empty((WIDTH, HIDDEN), device=dev)
    stream = torch.cuda.Stream(device=dev)
    rt.set_stream(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timing (the `value`)
    for i in range(args.warmup):
        rt.moe_layer(xs[args.steps + i], w, bias, handle, asynchronous=True, out=y)
    stream.synchronize()
    assert rt.error_flags() == 0, rt.last_error()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for i in range(args.steps):
                rt.moe_layer(xs[i], w, bias, handle, asynchronous=True, out=y)
            ev1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    barrier()
    flags = rt.error_flags()
    if flags:
        raise RuntimeError(f"device error flags {flags}")
    ms = ev0.elapsed_time(ev1)
    us_per_layer = ms * 1e3 / args.steps

    # ---- per-kernel profile + bytes (separate pass, synchronous calls)
    rt.set_profiling(True)
    prof_keys = ["quantize_ms", "router_ms", "schedule_ms", "gate_up_ms", "down_ms", "combine_ms"]
    prof = {k: 0.0 for k in prof_keys}
    gu_bytes = dn_bytes = 0
    uniq = []
    per_expert_gu = 2 * INTER * HIDDEN + 2 * (INTER // 128) * (HIDDEN // 128) * 4
    per_expert_dn = INTER * HIDDEN + (HIDDEN // 128) * (INTER // 128) * 4
    P = WIDTH * 8
    for i in range(args.steps):
        ex = rt.moe_layer(xs[i], w, bias, handle, stats=True, out=y)
        p = rt.last_profile()
        launches_per_layer = p["launches"]
        for k in prof_keys:
            prof[k] += p[k]
        U = ex.unique_experts
        uniq.append(U)
        # weights + scales + activation codes/scales read + outputs written
        gu_bytes += U * per_expert_gu + P * (HIDDEN + HIDDEN // 128 * 4) + P * (INTER + INTER // 128 * 4)
        dn_bytes += U * per_expert_dn + P * (INTER + INTER // 128 * 4) + P * HIDDEN * 4
    rt.set_profiling(False)
    gu_ms = prof["gate_up_ms"] / args.steps
    dn_ms = prof["down_ms"] / args.steps
    hbm, peak_kind = peaks()
    gu_gbs = gu_bytes / args.steps / (gu_ms * 1e-3) / 1e9
    dn_gbs = dn_bytes / args.steps / (dn_ms * 1e-3) / 1e9
    layer_bytes = (gu_bytes + dn_bytes) / args.steps + EXPERTS * HIDDEN * 2
    layer_gbs = layer_bytes / (us_per_layer * 1e-6) / 1e9

    # ---- end to end through the C ABI with pinned host buffers
    xh = [x.cpu().pin_memory() for x in xs[: args.steps]]
    rt.set_stream(None)
    for i in range(min(3, args.warmup)):
        rt.moe_layer(xh[i], w, bias, handle, stats=False)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        rt.moe_layer(xh[i], w, bias, handle, stats=False)
    e2e_us = (time.perf_counter() - t0) * 1e6 / args.steps
    barrier()

    # ---- max over ranks
    vals = torch.tensor([us_per_layer, e2e_us, gu_gbs], device=dev, dtype=torch.float64)
    if world > 1:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        mn = vals.clone()
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        us_per_layer, e2e_us = float(mx[0]), float(mx[1])
        gu_gbs = float(mn[2])

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sel_ex = rt.moe_layer(xs[0], w, bias, handle, want_routes=True, out=y)
        sel = sel_ex.selected.cpu().numpy().astype(np.uint32)
        wts = sel_ex.weights.cpu().numpy()
        bank_np = bank_to_host(bank, set(sel.ravel().tolist()))
        cpu_us, threads, reps = cpu_layer_baseline(xs[0].cpu().numpy(), sel, wts, bank_np)
        cpu = {"value": round(cpu_us, 1), "unit": "us", "cores": threads, "kind": "port",
               "sample": f"step 0's routed layer (8 tokens, {len(set(sel.ravel().tolist()))} experts) x {reps}; "
                         "oracle/pw_oracle.c routed layer, f32 reference order, libm exp"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(us_per_layer, 3), "unit": "us", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us_per_layer / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3xe4m3->f32",
            "data": "synthetic (seeded, checkpoint shapes)",
            "config": dict(CONFIG, parallelism=f"replicas x{world}" if world > 1 else "single GPU",
                           unique_experts_mean=round(statistics.mean(uniq), 2)),
            "e2e": {"value": round(e2e_us, 3), "unit": "us", "h2d_bytes_per_step": WIDTH * HIDDEN * 4,
                    "d2h_bytes_per_step": WIDTH * HIDDEN * 4 + 4},
            "gpu_launches": launches_per_layer * args.steps,
            "roofline": {"bound": "hbm", "kernel": "k_gemv fused gate/up + SwiGLU",
                         "achieved": round(gu_gbs, 1), "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(gu_gbs / hbm, 4),
                         "traffic": int(gu_bytes / args.steps * GATE_UP_TRAFFIC_RATIO),
                         "bytes_per_launch": int(gu_bytes / args.steps), "us_per_launch": round(gu_ms * 1e3, 2)},
            "layer_roofline": {"achieved": round(layer_gbs, 1), "unit": "GB/s", "frac": round(layer_gbs / hbm, 4),
                               "bytes_per_layer": int(layer_bytes)},
            "kernels_us": {k.replace("_ms", ""): round(v / args.steps * 1e3, 2) for k, v in prof.items()},
            "down_gemv_gbs": round(dn_gbs, 1),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    rt.close()


def main():
    global EXPERTS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=EXPERTS,
                    help="smaller banks only for profiling captures (the metric is quoted at 256)")
    args = ap.parse_args()
    EXPERTS = args.experts
    CONFIG["experts"] = EXPERTS
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        if args.impl == "ours":
            torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl" if args.impl == "ours" else "gloo",
                                timeout=datetime.timedelta(seconds=300))
    try:
        if args.impl == "reference":
            run_reference(args, rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
