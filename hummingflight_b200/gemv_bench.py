"""Device time of the gemv_bf16_f32 twin (hf_gemv_bf16_f32) on the matrix
shapes of its call sites: the attention projections of glm_forward.cpp:314-408
(q_a, q_b, kv_a, kv_b, o_proj), the DSA indexer, the router and an LM head.

    python -m hummingflight_b200.gemv_bench

Each shape runs 60 times back to back from a CUDA graph (no host launch cost
in the time), cycling through enough copies of the weight to pass 512 MB per
cycle, so every launch streams its matrix from HBM rather than L2. Prints the
mean time per launch, matrix bytes / time, and the error against a torch fp32
product (relative to the largest output).
"""
from __future__ import annotations

import torch

from . import moe as M

SHAPES = {"q_a": (2048, 6144), "q_b": (16384, 2048), "kv_a": (576, 6144),
          "kv_b": (28672, 512), "o_proj": (6144, 16384), "idx_wq_b": (4096, 2048),
          "idx_wk": (128, 6144), "router": (256, 6144), "lm_head": (151552, 6144)}


def time_shape(m: int, k: int, launches: int = 60):
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
    return t_ms, nb / t_ms / 1e6, err, ncopy


def main():
    for name, (m, k) in SHAPES.items():
        t, gbs, err, ncopy = time_shape(m, k)
        print(f"{name:9s} {m:6d} x {k:5d}: {t * 1000:7.1f} us  {gbs:6.0f} GB/s  "
              f"rel err {err:.1e}  ({ncopy} copies)", flush=True)


if __name__ == "__main__":
    main()
