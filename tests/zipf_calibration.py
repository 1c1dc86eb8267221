"""Calibration of config 4's Zipf correction bias (test infrastructure).

Config 4 asks for expert popularity that follows Zipf(1.1) over the 256
experts. The bias is bias_e = beta * ln(p_e / p_max) over a seeded
popularity ranking (hummingflight_b200.configs.zipf_bias); beta sets how hard
the bias pulls against the router's own scores. This script bisects beta so
that the realised share of token-slots held by the top tenth of experts (by
Zipf rank) equals the target shape's (Zipf(1.1) capped at 1/8 per expert, the
most a top-8 router can give one expert: configs.zipf_target_shares), on
config 4's first layer and batch, and prints the realised statistics.

Routing here is the reference's rule (compute/moe_router.h:36-43: rank by
sigmoid score + bias, top 8) on router logits computed by numpy in fp32 from
the same BF16 weights and activations the device generates; its sums differ
from the device's only in order, which moves only near-tie tokens.

    python tests/zipf_calibration.py      # prints beta and the statistics
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from hummingflight_b200.configs import WORKLOADS, ZIPF_S, zipf_bias, zipf_stats  # noqa: E402
from oracle import oracle as O  # noqa: E402


def routing_scores(wseed: int, xseed: int, T: int, H: int, E: int) -> np.ndarray:
    """sigmoid(router . x) for T tokens (glm_forward.cpp:519-524), fp32."""
    x = O.bf16_to_f32(O.gen_x_bf16_c(xseed, T, H)).reshape(T, H)
    W = O.bf16_to_f32(O.gen_bf16_normal(wseed, 0, O.KIND_ROUTER, 0, 0.02, E * H)).reshape(E, H)
    logits = x @ W.T
    return (1.0 / (1.0 + np.exp(-logits))).astype(np.float32)


def routed_counts(scores: np.ndarray, bias: np.ndarray, k: int) -> np.ndarray:
    """Per-expert slot counts of top-k on scores + bias."""
    top = np.argpartition(-(scores + bias[None, :]), k - 1, axis=1)[:, :k]
    return np.bincount(top.ravel(), minlength=scores.shape[1])


def calibrate(wl=WORKLOADS[4], lo: float = 0.0, hi: float = 1.0, iters: int = 30):
    s = wl.shape
    seed = wl.weight_seeds[0]
    sc = routing_scores(seed, wl.x_seed, wl.tokens, s.hidden, s.num_experts)
    k = min(s.top_k, s.num_experts)

    def stats(beta):
        return zipf_stats(routed_counts(sc, zipf_bias(s.num_experts, seed, ZIPF_S, beta), k),
                          seed, k)

    target = stats(0.0)["target_top_decile_share"]
    for _ in range(iters):  # the top-decile share grows with beta
        mid = 0.5 * (lo + hi)
        if stats(mid)["top_decile_share"] < target:
            lo = mid
        else:
            hi = mid
    beta = 0.5 * (lo + hi)
    return beta, stats(beta)


if __name__ == "__main__":
    b, st = calibrate()
    print(f"ZIPF_BETA = {b:.4f}")
    for key, v in st.items():
        print(f"  {key}: {v}")
