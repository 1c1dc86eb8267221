"""Checkpoint ingest throughput: safetensors shards (in the page cache) ->
resident HBM weights through hf_moe_load_safetensors.

    python -m hummingflight_b200.ingest_bench [--experts 32] [--shards 4] [--dir DIR]

Writes one GLM-shaped MoE layer (H = 6144, I = I_s = 2048, `--experts`
routed experts of 75.5 MB, the router and the bias) as safetensors shards in
the checkpoint's tensor names, loads it into a context `--repeat` times and
prints one JSON line: the load rate (tensor bytes / wall time) beside the two
ceilings of the path -- a pinned host-to-device copy of 1 GiB (the DMA bound)
and a pread of the shards into host memory with the loader's thread count
(the page-cache bound). The weights' values do not matter here: every expert
holds the same random bytes.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import shutil
import tempfile
import time

import numpy as np


def write_shards(d, E, H, I, Is, nshards, layer=0):
    from .safetensors_writer import write_file
    rng = np.random.default_rng(0)
    blk = {k: rng.integers(0, 1 << 16, (I, H) if k != "down" else (H, I), dtype=np.uint16)
           for k in ("gate", "up", "down")}
    pre = f"model.layers.{layer}.mlp."
    tensors = [(pre + "gate.weight", "BF16", (E, H), rng.integers(0, 1 << 16, (E, H),
                                                                   dtype=np.uint16)),
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


def pread_rate(paths, threads):
    """Host read bandwidth of the shards from the page cache, `threads` readers."""
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


def h2d_rate(torch, nbytes=1 << 30, reps=5):
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=32)
    ap.add_argument("--shards", type=int, default=4)
    ap.add_argument("--repeat", type=int, default=3)
    ap.add_argument("--dir", default="")
    a = ap.parse_args()
    import torch
    from .configs import LayerShape
    from .moe import MoELayer
    from . import _lib

    H, I, Is, E = 6144, 2048, 2048, a.experts
    d = a.dir or tempfile.mkdtemp(prefix="hf_ingest_")
    try:
        paths = write_shards(d, E, H, I, Is, a.shards)
        L = MoELayer(LayerShape(H, E, min(8, E), I, Is, 2.5, True), 1, 8, 0, "auto")
        runs = [L.load_safetensors(0, paths, 0) for _ in range(a.repeat)]
        best = min(r["seconds"] for r in runs)
        nbytes = runs[0]["bytes"]
        threads = max(1, min(8, (os.cpu_count() or 2) // 2))
        line = {
            "metric": "checkpoint ingest GB/s (safetensors page cache -> HBM)",
            "value": nbytes / best / 1e9, "unit": "GB/s", "bytes": nbytes,
            "experts": E, "tensors": runs[0]["tensors"], "shards": a.shards,
            "seconds": [round(r["seconds"], 4) for r in runs],
            "ceilings": {"h2d_pinned_gbs": h2d_rate(torch),
                         "pread_gbs": pread_rate(paths, threads), "reader_threads": threads},
        }
        L.close()
        _lib.lib().hf_ingest_release_staging()
        print(json.dumps(line))
    finally:
        if not a.dir:
            shutil.rmtree(d, ignore_errors=True)


if __name__ == "__main__":
    main()
