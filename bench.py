#!/usr/bin/env python
"""MoE-layer throughput on B200: the GLM-5.2 MoE layer (router -> top-8 ->
permutation -> routed + shared SwiGLU experts -> combine) through the C ABI of
hummingflight_b200/libhf_moe.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One JSON line on rank 0. The workload is config 3 by default: a stack of 8
GLM MoE layers (seeds 10-17, 155 GB of BF16 weights resident in HBM), 16384
tokens a step, expert-parallel over the ranks (E/N experts per GPU, the
global batch split evenly: strong scaling). `value` is MoE-layer tokens/s of
the whole job (tokens x layers / device time, max over ranks) with inputs
resident in HBM; `e2e` is the same metric through hf_moe_forward_host
(pinned host buffers, H2D of x and D2H of the output inside the timed
region). On one GPU the same run then measures configs 2 (prefill, 4096
tokens) and 0 (batch-1 decode) on one layer and reports them under
`sub_results`, each with its own roofline.

Inputs: seeded synthetic tensors (hummingflight_b200/configs.py) generated in
HBM. The generator is an Irwin-Hall(4) normal, so weights and activations are
bounded at +-3.46 sigma of the N(0, sigma) the configs name.

`--probe gemv` / `--probe ingest` run the GEMV-twin and checkpoint-ingest
measurements instead (see probe_gemv / probe_ingest).

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

from hummingflight_b200.configs import (GLM, WORKLOADS, ZIPF_BETA, layer_flops,  # noqa: E402
                                        zipf_bias, zipf_stats)

FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NOMINAL_HBM_GBS, NOMINAL_TFLOPS = 8000.0, 2250.0
REASON_BITS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}
SUB_CONFIGS = (2, 0)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained",
                                                     d["bf16_tflops"])),
                "kind": "measured"}
    return dict(FALLBACK, kind="fallback")


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a timed region."""

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

    def ready(self, timeout_s: float = 10.0):
        """Wait (bounded) until nvidia-smi delivers samples, then drop them:
        it takes longer to start than a short timed region lasts."""
        if self.p is None:
            return
        t0 = time.time()
        while not self.rows and time.time() - t0 < timeout_s and self.p.poll() is None:
            time.sleep(0.02)
        self.rows.clear()

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
    # expert outputs: one FP16 plane when no segment can take the GEMV (the
    # library's rule; HF_Y_F16=0 keeps fp32), else fp32
    no_gemv = path == "gemm" or (path == "auto" and gemv_max == 0)
    y_e = 2 if no_gemv and os.environ.get("HF_Y_F16") != "0" else 4
    for name, sel in (("gemv", on_gemv), ("gemm", live & ~on_gemv)):
        w_gu = int((2 * inter[sel] * H * 2).sum())
        w_d = int((H * inter[sel] * 2).sum())
        slots = int(c[sel].sum())
        # mid per element: fp32 on the GEMV, one FP16 plane on the GEMM's FP16
        # down pass (a BF16 hi + lo pair with HF_DOWN_F16=0)
        mid_e = 4 if name == "gemv" or os.environ.get("HF_DOWN_F16") == "0" else 2
        mid_b = int((c[sel] * inter[sel]).sum()) * mid_e
        out[f"{name}_gate_up"] = w_gu + slots * H * 2 + mid_b
        out[f"{name}_down"] = w_d + mid_b + slots * H * y_e
        out[f"{name}_gate_up_flops"] = int((2 * 2 * c[sel] * inter[sel] * H).sum())
        out[f"{name}_down_flops"] = int((2 * c[sel] * inter[sel] * H).sum())
    n_slots = int(c.sum())
    out["router"] = E * H * 2 + T * H * 2 + T * E * 4
    out["router_flops"] = 2 * T * E * H
    out["combine"] = n_slots * H * y_e + T * H * 4 + T * k * 8
    out["total_weights"] = E * H * 2 + int((3 * inter[live] * H * 2).sum())
    return out


def sum_dicts(ds):
    out = {}
    for d in ds:
        for k, v in d.items():
            out[k] = out.get(k, 0) + v
    return out


# ---------------------------------------------------------------- reference arm (CPU)
def reference_sample(wl, max_tokens):
    from oracle import oracle as O
    s = wl.shape
    d = O.Dims(s.hidden, s.num_experts, s.top_k, s.inter, s.shared_inter, s.scale, s.norm_topk)
    ntok = min(max_tokens, wl.tokens)
    x = O.bf16_to_f32(O.gen_x_rows_bf16(wl.x_seed, range(ntok), s.hidden)).reshape(ntok, -1)
    bias = zipf_bias(s.num_experts, wl.weight_seeds[0]) if wl.bias == "zipf" else None
    if not O.ref_available("avx2"):
        raise RuntimeError("oracle/_ref was not built (the reference's CPU kernels)")
    R = O.RefLayer(d, wl.weight_seeds[0], 0, bias=bias, flavour="avx2")
    R.prepare(x)
    return R, x, "reference", O.ref_lib("avx2").hfr_threads()


def sample_text(wl, ntok):
    return (f"first {ntok} of the {wl.tokens} tokens of {wl.name}, layer 0 of {wl.layers} "
            f"(every layer has the same shape and per-token cost); weights generated before "
            f"timing, resident in host RAM; per-token moeLayer")


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
    sample = sample_text(wl, ntok) + f", {args.steps} passes"
    line = {"metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 weights, fp32 math", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": wl.name, "tokens_per_step": ntok, "layers": 1,
                       "same_config": ntok == wl.tokens and wl.layers == 1},
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


def cpu_baseline(wl, budget_s, ntok):
    try:
        R, x, kind, cores = reference_sample(wl, ntok)
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
            "sample": sample_text(wl, x.shape[0]) + f", {passes} passes ({t:.1f} s of CPU "
                      f"time), reference AVX2 build"}


# ---------------------------------------------------------------- probes
# `--probe gemv`: device time of the gemv_bf16_f32 twin (hf_gemv_bf16_f32) on
# the matrix shapes of its call sites -- the attention projections of
# glm_forward.cpp:314-408 (q_a, q_b, kv_a, kv_b, o_proj), the DSA indexer, the
# router and an LM head. Each shape runs 60 times back to back from a CUDA
# graph (no host launch cost in the time), cycling through enough copies of
# the weight to pass 512 MB per cycle, so every launch streams its matrix from
# HBM rather than L2. Prints the mean time per launch, matrix bytes / time and
# the error against a torch fp32 product (relative to the largest output).
GEMV_SHAPES = {"q_a": (2048, 6144), "q_b": (16384, 2048), "kv_a": (576, 6144),
               "kv_b": (28672, 512), "o_proj": (6144, 16384), "idx_wq_b": (4096, 2048),
               "idx_wk": (128, 6144), "router": (256, 6144), "lm_head": (151552, 6144)}


def probe_gemv(launches=60):
    import torch

    from hummingflight_b200 import moe as M
    for name, (m, k) in GEMV_SHAPES.items():
        nb = m * k * 2
        ncopy = max(1, min(64, (512 << 20) // nb + 1))
        As = [(torch.randn(m, k, device="cuda") * 0.05).to(torch.bfloat16).view(torch.int16)
              for _ in range(ncopy)]
        x = torch.randn(k, device="cuda")
        y = torch.zeros(m, device="cuda")
        M.gemv_bf16_f32(As[0], x, y, m, k)
        ref = As[0].view(torch.bfloat16).float() @ x
        err = ((y - ref).abs().max() / ref.abs().max()).item()
        for i in range(5):
            M.gemv_bf16_f32(As[i % ncopy], x, y, m, k)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=torch.cuda.Stream()):
            for i in range(launches):
                M.gemv_bf16_f32(As[i % ncopy], x, y, m, k)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        t_ms = a.elapsed_time(b) / launches
        print(f"{name:9s} {m:6d} x {k:5d}: {t_ms * 1000:7.1f} us  {nb / t_ms / 1e6:6.0f} GB/s  "
              f"rel err {err:.1e}  ({ncopy} copies)", flush=True)
        del g, As


# `--probe ingest`: checkpoint ingest throughput, safetensors shards (in the
# page cache) -> resident HBM weights through hf_moe_load_safetensors. Writes
# one GLM-shaped MoE layer (`--probe-experts` routed experts of 75.5 MB, the
# router and the bias) as shards in the checkpoint's tensor names, loads it
# `--probe-repeat` times and prints one JSON line: the load rate beside the
# two ceilings of the path -- a pinned host-to-device copy of 1 GiB (the DMA
# bound) and a pread of the shards with the loader's thread count (the
# page-cache bound). Every expert holds the same random bytes.
def _write_shards(d, E, H, I, Is, nshards, layer=0):
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from safetensors_writer import write_file
    rng = np.random.default_rng(0)
    blk = {k: rng.integers(0, 1 << 16, (I, H) if k != "down" else (H, I), dtype=np.uint16)
           for k in ("gate", "up", "down")}
    pre = f"model.layers.{layer}.mlp."
    tensors = [(pre + "gate.weight", "BF16", (E, H),
                rng.integers(0, 1 << 16, (E, H), dtype=np.uint16)),
               (pre + "gate.e_score_correction_bias", "F32", (E,),
                rng.uniform(-0.1, 0.1, E).astype(np.float32))]
    for e in range(E):
        for k in ("gate", "up", "down"):
            tensors.append((pre + f"experts.{e}.{k}_proj.weight", "BF16", blk[k].shape, blk[k]))
    sh = {k: blk[k][:Is] if k != "down" else blk[k][:, :Is] for k in blk}
    for k in ("gate", "up", "down"):
        tensors.append((pre + f"shared_experts.{k}_proj.weight", "BF16", sh[k].shape,
                        np.ascontiguousarray(sh[k])))
    per = (len(tensors) + nshards - 1) // nshards
    paths = []
    for s in range(nshards):
        p = os.path.join(d, f"model-{s + 1:05d}-of-{nshards:05d}.safetensors")
        write_file(p, tensors[s * per:(s + 1) * per])
        paths.append(p)
    return paths


def _pread_rate(paths, threads):
    import concurrent.futures as cf
    import time
    chunk = 16 << 20
    jobs = []
    for p in paths:
        n = os.path.getsize(p)
        jobs += [(p, o, min(chunk, n - o)) for o in range(0, n, chunk)]
    bufs = [np.empty(chunk, np.uint8) for _ in range(threads)]
    fds = {p: os.open(p, os.O_RDONLY) for p in paths}

    def run(tid):
        for i in range(tid, len(jobs), threads):
            p, o, n = jobs[i]
            os.preadv(fds[p], [memoryview(bufs[tid])[:n]], o)

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(run, range(threads)))
    dt = time.perf_counter() - t0
    for fd in fds.values():
        os.close(fd)
    return sum(j[2] for j in jobs) / dt / 1e9


def _h2d_rate(torch, nbytes=1 << 30, reps=5):
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        dst.copy_(src, non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    return nbytes * reps / (a.elapsed_time(b) / 1e3) / 1e9


def probe_a2a(sizes_mb):
    """NCCL all-to-all bandwidth for comparison with the expert-parallel
    dispatch (run under torchrun, one rank per GPU): per rank `mb` MB of bf16
    split evenly over the ranks, 10 timed calls after 3, CUDA events, max over
    ranks. Without a GPU it runs on gloo and the CPU (a check of the plumbing
    only; its numbers mean nothing)."""
    import torch
    import torch.distributed as dist
    cuda = torch.cuda.is_available()
    dist.init_process_group("nccl" if cuda else "gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = "cpu"
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dev = "cuda"
    for mb in sizes_mb:
        n = (int(mb * (1 << 20)) // 2) // world * world
        a = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        b = torch.empty_like(a)
        for _ in range(3):
            dist.all_to_all_single(b, a)
        if cuda:
            torch.cuda.synchronize()
        dist.barrier()
        t0 = time.time()
        if cuda:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        for _ in range(10):
            dist.all_to_all_single(b, a)
        if cuda:
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 10
        else:
            ms = (time.time() - t0) * 1e3 / 10
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out = n * 2 * (world - 1) / world
            print(json.dumps({"probe": "a2a", "mb_per_rank": mb, "world": world,
                              "ms": round(float(t.item()), 4),
                              "gbs_out_per_rank": round(out / float(t.item()) / 1e6, 1),
                              "device": dev}), flush=True)
    dist.destroy_process_group()


def probe_ingest(E, nshards, repeat):
    import shutil
    import tempfile

    import torch

    from hummingflight_b200 import _lib
    from hummingflight_b200.configs import LayerShape
    from hummingflight_b200.moe import MoELayer
    H, I, Is = 6144, 2048, 2048
    d = tempfile.mkdtemp(prefix="hf_ingest_")
    try:
        paths = _write_shards(d, E, H, I, Is, nshards)
        L = MoELayer(LayerShape(H, E, min(8, E), I, Is, 2.5, True), 1, 8, 0, "auto")
        runs = [L.load_safetensors(0, paths, 0) for _ in range(repeat)]
        best = min(r["seconds"] for r in runs)
        nbytes = runs[0]["bytes"]
        threads = max(1, min(8, (os.cpu_count() or 2) // 2))
        line = {"metric": "checkpoint ingest GB/s (safetensors page cache -> HBM)",
                "value": nbytes / best / 1e9, "unit": "GB/s", "bytes": nbytes, "experts": E,
                "tensors": runs[0]["tensors"], "shards": nshards,
                "seconds": [round(r["seconds"], 4) for r in runs],
                "ceilings": {"h2d_pinned_gbs": _h2d_rate(torch),
                             "pread_gbs": _pread_rate(paths, threads),
                             "reader_threads": threads}}
        L.close()
        _lib.lib().hf_ingest_release_staging()
        print(json.dumps(line))
    finally:
        shutil.rmtree(d, ignore_errors=True)


# ---------------------------------------------------------------- our arm (GPU)
class Job:
    """One workload resident on this rank: the layers, x and outputs."""

    def __init__(self, wl, args, rank, world, local, dist=None, uid=None):
        import torch

        from hummingflight_b200.moe import MoELayer, synth_bf16_normal
        self.wl, self.rank, self.world = wl, rank, world
        shape = wl.shape
        T_glob, H = wl.tokens, shape.hidden
        if T_glob % world or shape.num_experts % world:
            raise SystemExit(f"{wl.name}: tokens and experts must divide by {world} ranks")
        self.T = T = T_glob // world
        E = shape.num_experts
        self.L = MoELayer(shape, wl.layers, T, local, args.path, args.gemv_max, rank, world, uid)
        self.bias = zipf_bias(E, wl.weight_seeds[0]) if wl.bias == "zipf" else None
        for l, seed in enumerate(wl.weight_seeds):
            self.L.synth_layer(l, seed, 0, self.bias)
        x_all = torch.empty((T_glob, H), dtype=torch.int16, device="cuda")
        self.orders = [np.arange(E)] * wl.layers
        self.placement = "contiguous"
        if world > 1 and args.placement == "balanced":
            # Expert placement by load: route a calibration batch (the same
            # size, other tokens: x seed + 1000) through every layer, sum the
            # per-expert token counts over the ranks, and give each rank E/W
            # experts of about equal work (tokens + 128 token-equivalents for
            # an active expert's weight stream), then load the layer again.
            from hummingflight_b200.moe import balanced_placement
            synth_bf16_normal(x_all, wl.x_seed + 1000, 0, 0, 0, 1.0)
            xc = x_all[rank * T:(rank + 1) * T].contiguous().view(torch.bfloat16)
            self.orders = []
            for l, seed in enumerate(wl.weight_seeds):
                ids = self.L.route(l, xc)["topk_ids"]
                cnt = torch.bincount(ids.reshape(-1).long(), minlength=E)
                dist.all_reduce(cnt)
                c = cnt.cpu().numpy().astype(np.int64)
                order = balanced_placement(c + 128 * (c > 0), world)
                self.orders.append(order)
                self.L.set_placement(l, order)
                self.L.synth_layer(l, seed, 0, self.bias)
            del xc
            self.placement = "balanced (calibration batch: x seed + 1000)"
        synth_bf16_normal(x_all, wl.x_seed, 0, 0, 0, 1.0)
        self.x = x_all[rank * T:(rank + 1) * T].contiguous().view(torch.bfloat16)
        del x_all
        self.outs = [torch.empty((T, H), dtype=torch.float32, device="cuda")
                     for _ in range(wl.layers)]
        # the routing of every layer (global counts: all ranks' tokens)
        self.counts_glob, self.counts_rank0 = [], []
        el = E // world
        for l in range(wl.layers):
            _, r = self.L.forward(l, self.x, out=self.outs[l], routing=True)
            ids = r["topk_ids"]
            if world > 1:
                got = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(got, ids)
                ids = torch.cat(got)
            glob = np.bincount(ids.cpu().numpy().ravel(), minlength=E)
            self.counts_glob.append(glob)
            # rank 0's expert work: its local experts over the whole batch + shared on its tokens
            c0 = np.zeros(E + 1, np.int64)
            c0[:el] = glob[self.orders[l][:el]]
            c0[E] = T
            self.counts_rank0.append(c0)
        torch.cuda.synchronize()

    def step(self):
        for l in range(self.wl.layers):
            self.L.forward(l, self.x, out=self.outs[l])

    def close(self):
        self.L.close()
        self.outs = None
        self.x = None


def timed(job, steps, world, dist, stream):
    """K steps bracketed by a barrier and a device synchronize; CUDA events on
    the launching stream; the max over ranks."""
    import torch
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        job.step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    m = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([m], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        m = float(t.item())
    return m


def measure(job, args, world, dist, stream, local, steps):
    """Pass 1 (the value): K steps as a user runs them. Pass 2: the same K
    steps with a CUDA event pair around every phase, for the per-kernel
    durations of the roofline (those events cost a few us per phase boundary,
    so they stay out of the first pass)."""
    import torch
    L = job.L
    for _ in range(args.warmup):
        job.step()
    torch.cuda.synchronize()
    L.profile_read()  # drop warm-up launch counts
    clk = ClockSampler(local)
    clk.ready()
    if world > 1:
        dist.barrier()
    ms = timed(job, steps, world, dist, stream)
    launches = int(sum(v[1] for v in L.profile_read().values()))
    L.profile(True)
    ms_profiled = timed(job, steps, world, dist, stream)
    clocks = clk.stop()
    L.profile(False)
    prof = L.profile_read()
    return {"ms": ms, "ms_profiled": ms_profiled, "launches": launches, "prof": prof,
            "clocks": clocks, "steps": steps}


def e2e_ms(job, world, dist, stream, steps):
    """Same steps through hf_moe_forward_host: pinned host x in, pinned fp32
    out back, inside the timed region, every layer."""
    import torch
    T, H = job.T, job.wl.shape.hidden
    xh = torch.empty((T, H), dtype=torch.int16, pin_memory=True)
    xh.copy_(job.x.view(torch.int16).cpu())
    oh = torch.empty((T, H), dtype=torch.float32, pin_memory=True)
    xh_np, oh_np = xh.numpy().view(np.uint16), oh.numpy()

    def one():
        for l in range(job.wl.layers):
            job.L.forward_host(l, xh_np, oh_np, stream=stream)

    one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize()
    m = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([m], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        m = float(t.item())
    return m


def roofline(job, meas, args, pk, steps):
    """The dominant kernel's algorithmic bytes or flops per launch (summed
    over the layers of a step from each layer's realised routing) over its
    average CUDA-event duration."""
    wl, shape = job.wl, job.wl.shape
    T = job.T
    gemv_max = args.gemv_max or (1 if T <= 1 else 0)  # the library's AUTO rule
    pb = sum_dicts(phase_bytes(shape, c, T, job.L.k, args.path, gemv_max)
                   for c in job.counts_rank0)
    prof = meas["prof"]
    dom = max(("gemv_gate_up", "gemv_down", "router", "route", "combine",
               "gemm_gate_up", "gemm_down"), key=lambda p: prof[p][0])
    dom_ms, dom_n = prof[dom]
    per_step_launches = max(1, dom_n // steps)
    per_launch_ms = dom_ms / max(1, dom_n)
    alg = pb.get(dom, 0) / per_step_launches
    flops = pb.get(dom + "_flops", 0) / per_step_launches
    hbm, tfl = pk["hbm_gbs"], pk["bf16_tflops"]
    # flops/byte above half the machine balance: report against the tensor peak
    tensor_bound = bool(flops) and flops / max(1, alg) > 0.5 * 1e3 * tfl / hbm
    if tensor_bound:
        achieved = flops / (per_launch_ms / 1e3) / 1e12
    else:
        achieved = alg / (per_launch_ms / 1e3) / 1e9 if alg else None
    # DRAM bytes per launch from ncu: measured on this workload, or -- where the
    # full workload is too large to capture -- the ratio of DRAM traffic to
    # algorithmic bytes measured on a small case of the same kernel, scaled to
    # this launch's algorithmic bytes
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            t = json.load(f).get(f"{wl.name}:{dom}")
        if isinstance(t, dict) and alg:
            traffic = t["traffic_over_algorithmic"] * alg
        elif isinstance(t, (int, float)):
            traffic = t
    peak = tfl if tensor_bound else hbm
    return pb, {"bound": "tensor" if tensor_bound else "hbm", "kernel": dom,
                "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s" if tensor_bound else "GB/s",
                "frac": achieved / peak if achieved else None,
                "peak_kind": pk["kind"], "traffic": traffic,
                "frac_nominal": (achieved / (NOMINAL_TFLOPS if tensor_bound else NOMINAL_HBM_GBS))
                if achieved else None,
                "algorithmic_bytes_per_launch": alg, "algorithmic_flops_per_launch": flops,
                "launch_ms": per_launch_ms, "launches_per_step": per_step_launches}


def layer_summary(job, meas, pb, pk):
    """Whole-layer figures: weights + activations streamed, useful flops."""
    wl, shape = job.wl, job.wl.shape
    T, H = job.T, shape.hidden
    ms = meas["ms"]
    layer_bytes = pb["total_weights"] + wl.layers * (T * H * 2 + T * H * 4)
    flops = layer_flops(shape, wl.tokens) * wl.layers
    s = {"hbm_gbs": layer_bytes / (ms / 1e3) / 1e9, "tflops": flops / (ms / 1e3) / 1e12}
    s["hbm_frac"] = s["hbm_gbs"] / pk["hbm_gbs"]
    s["tflops_frac_burst"] = s["tflops"] / pk["bf16_tflops"]
    s["tflops_frac_sustained"] = s["tflops"] / pk["bf16_tflops_sustained"]
    t_bytes = layer_bytes / (pk["hbm_gbs"] * 1e9) * 1e3
    t_flops = flops / (pk["bf16_tflops"] * 1e12) * 1e3
    s["roofline_ms"] = max(t_bytes, t_flops)
    s["roofline_bound"] = "hbm" if t_bytes >= t_flops else "tensor"
    s["roofline_frac"] = s["roofline_ms"] / ms
    s["bytes_per_step"] = layer_bytes
    s["flops_per_step"] = flops
    return s


def sub_result(wl, args, local, stream, pk):
    """Config 0 or 2 on one GPU: one layer, its own timing, roofline and clocks."""
    import torch
    job = Job(wl, args, 0, 1, local)
    steps = 1000 if wl.tokens <= 64 else max(args.steps, 30)  # >= ~0.1 s timed
    meas = measure(job, args, 1, None, stream, local, steps)
    pb, rl = roofline(job, meas, args, pk, steps)
    lay = layer_summary(job, meas, pb, pk)
    out = {"workload": wl.name, "tokens": wl.tokens, "layers": wl.layers,
           "ms_per_step": meas["ms"], "value": wl.tokens * wl.layers / (meas["ms"] / 1e3),
           "unit": "tokens/s", "steps": steps, "active_experts": pb["active"],
           "layer": lay, "roofline": rl, "gpu_launches": meas["launches"],
           "phases_ms_per_step": {p: v[0] / steps for p, v in meas["prof"].items()
                                  if v[1] or v[0] > 0},
           "clocks": meas["clocks"]}
    job.close()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "gemm"])
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--ref-tokens", type=int, default=24,
                    help="tokens of the workload the reference arm runs per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="skip the config 2 / 0 sub-results")
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="expert placement over the ranks (N > 1)")
    ap.add_argument("--experts", type=int, default=0,
                    help="profiling case: fewer routed experts (same per-expert shape)")
    ap.add_argument("--tokens", type=int, default=0, help="profiling case: override T")
    ap.add_argument("--layers", type=int, default=0, help="profiling case: first N layers")
    ap.add_argument("--inter", type=int, default=0,
                    help="profiling case: override the (routed and shared) intermediate size")
    ap.add_argument("--gemv-max", type=int, default=0,
                    help="AUTO path: segments up to this many tokens use the GEMV (0 = default)")
    ap.add_argument("--probe", default="", choices=["", "gemv", "ingest", "a2a"],
                    help="instead of the layer benchmark: the GEMV twin on the attention "
                         "shapes, checkpoint ingest throughput, or (under torchrun) NCCL "
                         "all-to-all bandwidth")
    ap.add_argument("--probe-mb", type=float, nargs="+", default=[32, 116, 512],
                    help="a2a probe: MB per rank")
    ap.add_argument("--probe-experts", type=int, default=32)
    ap.add_argument("--probe-shards", type=int, default=4)
    ap.add_argument("--probe-repeat", type=int, default=3)
    args = ap.parse_args()
    if args.probe == "gemv":
        probe_gemv()
        return
    if args.probe == "ingest":
        probe_ingest(args.probe_experts, args.probe_shards, args.probe_repeat)
        return
    if args.probe == "a2a":
        probe_a2a(args.probe_mb)
        return
    args.warmup = max(3, args.warmup)
    wl = WORKLOADS[args.config]
    profiling_case = bool(args.experts or args.tokens or args.inter or args.layers)
    if profiling_case:
        from dataclasses import replace
        shape = replace(wl.shape, num_experts=args.experts or wl.shape.num_experts,
                        inter=args.inter or wl.shape.inter,
                        shared_inter=args.inter or wl.shape.shared_inter)
        seeds = wl.weight_seeds[:args.layers] if args.layers else wl.weight_seeds
        wl = replace(wl, shape=shape, tokens=args.tokens or wl.tokens, weight_seeds=seeds,
                     name=f"{wl.name}_E{shape.num_experts}_T{args.tokens or wl.tokens}"
                          f"_I{shape.inter}_L{len(seeds)}")
    if args.impl == "reference":
        run_reference(args, wl)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    uid = None
    if world > 1:
        from hummingflight_b200.ep import broadcast_unique_id
        uid = broadcast_unique_id(dist, rank, torch.device("cuda", local))
    stream = torch.cuda.current_stream()
    pk = peaks()

    job = Job(wl, args, rank, world, local, dist, uid)
    meas = measure(job, args, world, dist, stream, local, args.steps)
    ranks_phases = None
    if world > 1:  # every rank's phase times (second pass) and routed rows
        el = wl.shape.num_experts // world
        mine = {"phases": {p: v[0] / args.steps for p, v in meas["prof"].items() if v[0] > 0},
                "ms_profiled": meas["ms_profiled"],
                "routed_rows": int(sum(int(c[o[rank * el:(rank + 1) * el]].sum())
                                       for c, o in zip(job.counts_glob, job.orders)))}
        ranks_phases = [None] * world
        dist.all_gather_object(ranks_phases, mine)
    e_steps = max(3, args.steps // 4)
    e2e = e2e_ms(job, world, dist, stream, e_steps)
    shape, T_glob, T = wl.shape, wl.tokens, job.T
    tokens_per_step = T_glob * wl.layers
    line = None
    if rank == 0:
        pb, rl = roofline(job, meas, args, pk, args.steps)
        lay = layer_summary(job, meas, pb, pk)
        H = shape.hidden
        line = {
            "metric": "MoE-layer tokens/s", "value": tokens_per_step / (meas["ms"] / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": meas["ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, generated in HBM; Irwin-Hall(4) normals, "
                    "bounded at +-3.46 sigma)",
            "config": {"workload": wl.name, "tokens": T_glob, "tokens_per_rank": T,
                       "layers": wl.layers, "hidden": H, "experts": shape.num_experts,
                       "top_k": shape.top_k, "inter": shape.inter,
                       "shared_inter": shape.shared_inter,
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "expert_placement": job.placement,
                       "path": args.path,
                       "active_experts_layer0": int((job.counts_glob[0] > 0).sum()),
                       "profiling_case": profiling_case,
                       "l2": "no flush: weights streamed per step (%.1f GB on rank 0) exceed "
                             "the 126 MB L2" % (pb["total_weights"] / 1e9)},
            "e2e": {"value": tokens_per_step / (e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T_glob * H * 2 * wl.layers,
                    "d2h_bytes_per_step": T_glob * H * 4 * wl.layers, "ms_per_step": e2e},
            "gpu_launches": meas["launches"],
            "phase_timing": {"pass": "second timed pass of the same K steps with per-phase "
                                     "CUDA events on the forward's stream (rank 0)",
                             "ms_per_step_with_events": meas["ms_profiled"]},
            "layer": lay,
            "phases_ms_per_step": {p: v[0] / args.steps for p, v in meas["prof"].items()
                                   if v[1] or v[0] > 0},
            "roofline": rl,
            "clocks": meas["clocks"],
        }
        if ranks_phases:
            gemm = [sum(v for p, v in r["phases"].items() if p.startswith("gemm"))
                    for r in ranks_phases]
            rows = [r["routed_rows"] for r in ranks_phases]
            line["ranks"] = {
                "phases_ms_per_step": [r["phases"] for r in ranks_phases],
                "routed_rows_per_step": rows,
                "rows_max_over_mean": max(rows) / (sum(rows) / len(rows)),
                "gemm_ms_max_over_mean": max(gemm) / (sum(gemm) / len(gemm)),
                "slowest_rank_by_gemm": int(np.argmax(gemm))}
        if wl.bias == "zipf":
            z = zipf_stats(job.counts_glob[0], wl.weight_seeds[0], shape.top_k)
            z["beta"] = ZIPF_BETA
            z["hottest_share_per_layer"] = [float(c.max() / c.sum()) for c in job.counts_glob]
            z["zero_experts_per_layer"] = [int((c == 0).sum()) for c in job.counts_glob]
            line["zipf"] = z
    job.close()
    del job
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if world == 1 and not args.no_sub and not profiling_case and args.config not in SUB_CONFIGS:
        line["sub_results"] = {WORKLOADS[c].name: sub_result(WORKLOADS[c], args, local, stream, pk)
                               for c in SUB_CONFIGS}
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_budget_s, args.ref_tokens)
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
