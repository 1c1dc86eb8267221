#!/usr/bin/env python
"""MoE-layer throughput on B200: the GLM-5.2 MoE layer (router -> top-8 ->
permutation -> routed + shared SwiGLU experts -> combine) through the C ABI of
hummingflight_b200/libhf_moe.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One JSON line on rank 0. `value` is MoE-layer tokens/s over the whole job
(tokens x layers / device time, max over ranks) with inputs resident in HBM;
`e2e` is the same metric through hf_moe_forward_host (pinned host buffers,
H2D of x and D2H of the output inside the timed region). Workload: config 1
by default (decode, 64 tokens, one layer); weights and activations are the
seeded synthetic tensors of hummingflight_b200/configs.py, generated in HBM.

`--impl reference` times the reference's own CPU MoE path (compute/cpu_kernels.cpp
+ compute/moe_router.h built unmodified into oracle/_ref, AVX2 build, all host
threads) on a bounded token sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from hummingflight_b200.configs import GLM, WORKLOADS, layer_flops, zipf_bias  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
REASON_BITS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, device: int, period_ms: int = 50):
        self.rows = []
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-i", str(device), "-lms", str(period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.p.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 3:
                self.rows.append(parts)

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        for a, b, r in self.rows:
            try:
                sm.append(float(a))
                mx.append(float(b))
                bits = int(r, 16)
                for bit, name in REASON_BITS.items():
                    if bits & bit and name != "gpu_idle":
                        reasons.add(name)
            except ValueError:
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "samples": len(sm),
                "reasons": sorted(reasons)}


def phase_bytes(shape, counts, T, k, path, gemv_max):
    """Algorithmic HBM bytes (and useful flops) of each phase from the routing
    of one forward: every active expert's weights once, activations and
    intermediates once, split by the path each expert segment takes."""
    H, I, Is, E = shape.hidden, shape.inter, shape.shared_inter, shape.num_experts
    inter = np.array([I] * E + [Is], np.int64)
    c = counts.astype(np.int64).copy()
    if Is == 0:
        c[E] = 0
    live = (c > 0) & (inter > 0)
    if path == "gemv":
        on_gemv = live
    elif path == "gemm":
        on_gemv = np.zeros_like(live)
    else:
        on_gemv = live & (c <= gemv_max)
    out = {"active": int((c[:E] > 0).sum())}
    for name, sel in (("gemv", on_gemv), ("gemm", live & ~on_gemv)):
        w_gu = int((2 * inter[sel] * H * 2).sum())
        w_d = int((H * inter[sel] * 2).sum())
        slots = int(c[sel].sum())
        mid_b = int((c[sel] * inter[sel]).sum()) * 4  # fp32 (GEMV) or BF16 hi + lo (GEMM)
        out[f"{name}_gate_up"] = w_gu + slots * H * 2 + mid_b
        out[f"{name}_down"] = w_d + mid_b + slots * H * 4
        out[f"{name}_gate_up_flops"] = int((2 * 2 * c[sel] * inter[sel] * H).sum())
        out[f"{name}_down_flops"] = int((2 * c[sel] * inter[sel] * H).sum())
    n_slots = int(c.sum())
    out["router"] = E * H * 2 + T * H * 2 + T * E * 4
    out["combine"] = n_slots * H * 4 + T * H * 4 + T * k * 8
    out["total_weights"] = E * H * 2 + int((3 * inter[live] * H * 2).sum())
    return out


# ---------------------------------------------------------------- reference arm (CPU)
def reference_sample(wl, max_tokens=8):
    from oracle import oracle as O
    s = wl.shape
    d = O.Dims(s.hidden, s.num_experts, s.top_k, s.inter, s.shared_inter, s.scale, s.norm_topk)
    flavour = "avx2" if O.ref_available("avx2") else "port"
    ntok = min(max_tokens, wl.tokens)
    x = O.bf16_to_f32(O.gen_x_bf16(wl.x_seed, wl.tokens, s.hidden))[:ntok]
    bias = zipf_bias(s.num_experts, wl.weight_seeds[0]) if wl.bias == "zipf" else None
    if flavour == "avx2":
        R = O.RefLayer(d, wl.weight_seeds[0], 0, bias=bias, flavour="avx2")
        R.prepare(x)
        return R, x, "reference", O.ref_lib("avx2").hfr_threads()
    raise RuntimeError("oracle/_ref was not built (the reference's CPU kernels)")


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        R, x, kind, cores = reference_sample(wl, args.ref_tokens)
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": "reference", "unavailable": str(e)}))
        return
    for _ in range(args.warmup):
        R.forward(x)
    t = 0.0
    for _ in range(args.steps):
        t += R.forward(x)["seconds"]
    ntok = x.shape[0]
    value = ntok * args.steps / t
    sample = (f"first {ntok} tokens of {wl.name} (layer 0), {args.steps} passes; weights "
              f"generated before timing, resident in host RAM")
    line = {"metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 weights, fp32 math", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": wl.name, "tokens_per_step": ntok, "layers": 1},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "cpu": cpu_model(), "nproc": os.cpu_count(), "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(wl, budget_s):
    try:
        R, x, kind, cores = reference_sample(wl, 8)
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "tokens/s", "cores": None, "kind": "reference",
                "sample": f"unavailable: {e}"}
    t, n, passes = 0.0, 0, 0
    while (t < budget_s and passes < 50) or passes < 1:
        t += R.forward(x)["seconds"]
        n += x.shape[0]
        passes += 1
    R.close()
    return {"value": n / t, "unit": "tokens/s", "cores": cores, "kind": kind,
            "cpu": cpu_model(), "nproc": os.cpu_count(),
            "sample": f"{passes} passes over the first {x.shape[0]} tokens of {wl.name} "
                      f"({t:.1f} s of CPU time), reference AVX2 build, per-token moeLayer"}


# ---------------------------------------------------------------- our arm (GPU)
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "gemm"])
    ap.add_argument("--cpu-budget-s", type=float, default=10.0)
    ap.add_argument("--ref-tokens", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=0,
                    help="profiling case: fewer routed experts (same per-expert shape)")
    ap.add_argument("--tokens", type=int, default=0, help="profiling case: override T")
    ap.add_argument("--inter", type=int, default=0,
                    help="profiling case: override the (routed and shared) intermediate size")
    ap.add_argument("--gemv-max", type=int, default=0,
                    help="AUTO path: segments up to this many tokens use the GEMV (0 = default)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    wl = WORKLOADS[args.config]
    if args.experts or args.tokens or args.inter:
        from dataclasses import replace
        shape = replace(wl.shape, num_experts=args.experts or wl.shape.num_experts,
                        inter=args.inter or wl.shape.inter,
                        shared_inter=args.inter or wl.shape.shared_inter)
        wl = replace(wl, shape=shape, tokens=args.tokens or wl.tokens,
                     name=f"{wl.name}_E{shape.num_experts}_T{args.tokens or wl.tokens}"
                          f"_I{shape.inter}")
    if args.impl == "reference":
        run_reference(args, wl)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from hummingflight_b200.moe import MoELayer

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    shape = wl.shape
    # strong scaling: the workload's global batch is split across the ranks and
    # the experts are sharded (expert parallelism, E/world per GPU)
    T_glob, H = wl.tokens, shape.hidden
    if T_glob % world or shape.num_experts % world:
        raise SystemExit(f"{wl.name}: tokens and experts must divide by {world} ranks")
    T = T_glob // world
    uid = None
    if world > 1:
        from hummingflight_b200.ep import broadcast_unique_id
        uid = broadcast_unique_id(dist, rank, torch.device("cuda", local))
    L = MoELayer(shape, wl.layers, T, local, args.path, args.gemv_max, rank, world, uid)
    bias = zipf_bias(shape.num_experts, wl.weight_seeds[0]) if wl.bias == "zipf" else None
    for l, seed in enumerate(wl.weight_seeds):
        L.synth_layer(l, seed, 0, bias)
    stream = torch.cuda.current_stream()
    x_all = torch.empty((T_glob, H), dtype=torch.int16, device="cuda")
    from hummingflight_b200.moe import synth_bf16_normal
    synth_bf16_normal(x_all, wl.x_seed, 0, 0, 0, 1.0)
    x = x_all[rank * T:(rank + 1) * T].contiguous().view(torch.bfloat16)
    del x_all
    outs = [torch.empty((T, H), dtype=torch.float32, device="cuda") for _ in range(wl.layers)]

    def step():
        for l in range(wl.layers):
            L.forward(l, x, out=outs[l])

    _, r = L.forward(0, x, out=outs[0], routing=True)
    ids = r["topk_ids"]
    if world > 1:
        got = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(got, ids)
        ids = torch.cat(got)
    # rank 0's expert work: its local experts over the whole batch + shared on its tokens
    glob = np.bincount(ids.cpu().numpy().ravel(), minlength=shape.num_experts)
    el = shape.num_experts // world
    counts = np.zeros(shape.num_experts + 1, np.int64)
    counts[:el] = glob[:el]
    counts[shape.num_experts] = T
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    L.profile_read()  # drop warm-up launch counts

    def timed_pass():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        m = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([m], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            m = float(t.item())
        return m

    # pass 1 (the value): K steps as a user runs them. Pass 2: the same K steps
    # with a CUDA event pair around every phase, for the per-kernel durations of
    # the roofline; those events cost a few us per phase boundary, so they stay
    # out of the first pass.
    clk = ClockSampler(local)
    ms = timed_pass()
    launches = int(sum(v[1] for v in L.profile_read().values()))
    L.profile(True)
    ms_profiled = timed_pass()
    clocks = clk.stop()
    L.profile(False)
    prof = L.profile_read()
    tokens_per_step = T_glob * wl.layers
    value = tokens_per_step / (ms / 1e3)

    # end to end through hf_moe_forward_host: pinned host x in, pinned host out back
    xh = torch.empty((T, H), dtype=torch.int16, pin_memory=True)
    xh.copy_(x.view(torch.int16).cpu())
    oh = torch.empty((T, H), dtype=torch.float32, pin_memory=True)
    xh_np, oh_np = xh.numpy().view(np.uint16), oh.numpy()
    for _ in range(3):
        for l in range(wl.layers):
            L.forward_host(l, xh_np, oh_np, stream=stream)
    e_steps = max(3, args.steps // 4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(e_steps):
        for l in range(wl.layers):
            L.forward_host(l, xh_np, oh_np, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    if rank == 0:
        hbm, tflops_peak, peak_kind = peaks()
        # the library's AUTO rule: the GEMV only for a single token
        gemv_max = args.gemv_max or (1 if T <= 1 else 0)
        pb = phase_bytes(shape, counts, T, L.k, args.path, gemv_max)
        dom = max(("gemv_gate_up", "gemv_down", "router", "route", "combine",
                   "gemm_gate_up", "gemm_down"), key=lambda p: prof[p][0])
        dom_ms, dom_n = prof[dom]
        per_launch_ms = dom_ms / max(1, dom_n)
        alg = pb.get(dom)
        flops = pb.get(dom + "_flops")
        # prefill-sized segments are tensor-bound; decode streams weights (HBM-bound)
        tensor_bound = bool(flops) and flops / max(1, alg) > 0.5 * 1e3 * tflops_peak / hbm
        if tensor_bound:
            achieved = flops / (per_launch_ms / 1e3) / 1e12
        else:
            achieved = alg / (per_launch_ms / 1e3) / 1e9 if alg else None
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get(f"{wl.name}:{dom}")
        layer_bytes = pb["total_weights"] + T * H * 2 + T * H * 4
        line = {
            "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded, generated in HBM)",
            "config": {"workload": wl.name, "tokens": T_glob, "tokens_per_rank": T,
                       "layers": wl.layers,
                       "hidden": H, "experts": shape.num_experts, "top_k": shape.top_k,
                       "inter": shape.inter, "shared_inter": shape.shared_inter,
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "path": args.path, "active_experts": pb["active"],
                       "l2": "no flush: weights streamed per step (%.1f GB) exceed the 126 MB L2"
                             % (pb["total_weights"] / 1e9)},
            "e2e": {"value": tokens_per_step / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T_glob * H * 2 * wl.layers,
                    "d2h_bytes_per_step": T_glob * H * 4 * wl.layers},
            "gpu_launches": launches,
            "phase_timing": {"pass": "second timed pass of the same K steps with per-phase "
                                     "CUDA events on the forward's stream",
                             "ms_per_step_with_events": ms_profiled},
            # rank 0's weight stream per second, and useful flops of the whole job
            "layer_hbm_gbs": layer_bytes * wl.layers / (ms / 1e3) / 1e9,
            "layer_tflops": layer_flops(shape, T_glob) * wl.layers / (ms / 1e3) / 1e12,
            "phases_ms_per_step": {p: v[0] / args.steps for p, v in prof.items() if v[1] or v[0] > 0},
            "roofline": {"bound": "tensor" if tensor_bound else "hbm", "kernel": dom,
                         "achieved": achieved,
                         "peak": tflops_peak if tensor_bound else hbm,
                         "unit": "TFLOP/s" if tensor_bound else "GB/s",
                         "frac": (achieved / (tflops_peak if tensor_bound else hbm))
                         if achieved else None,
                         "peak_kind": peak_kind, "traffic": traffic,
                         # against the nominal 8 TB/s HBM3e and 2.25 PFLOP/s dense BF16
                         "frac_nominal": (achieved / (2250.0 if tensor_bound else 8000.0))
                         if achieved else None,
                         "algorithmic_bytes_per_launch": alg,
                         "algorithmic_flops_per_launch": flops,
                         "launch_ms": per_launch_ms},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_budget_s)
        print(json.dumps(line))
    L.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
