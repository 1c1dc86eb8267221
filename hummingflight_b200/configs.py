"""Layer shapes and the seeded synthetic workloads.

GLM-5.2 MoE layer shape (model/config.h; MoE keys parsed at
model/config.cpp:108-117): hidden 6144, 256 routed experts, top-8,
moe_intermediate 2048, one shared expert (n_shared_experts * moe_intermediate =
2048), routed_scaling_factor 2.5, norm_topk_prob true, sigmoid scoring with
e_score_correction_bias (noaux_tc).

The five workloads are the benchmark configurations of this path. No dataset is
involved: every tensor is a pure function of (seed, layer, kind, expert, index)
(see hummingflight_b200/csrc/hf_synth.cu), BF16 weights ~N(0, 0.02),
BF16 activations ~N(0, 1), fp32 bias ~U(-0.1, 0.1).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class LayerShape:
    hidden: int = 6144
    num_experts: int = 256
    top_k: int = 8
    inter: int = 2048
    shared_inter: int = 2048
    scale: float = 2.5
    norm_topk: bool = True

    @property
    def expert_bytes(self) -> int:
        return 3 * self.hidden * self.inter * 2

    @property
    def shared_bytes(self) -> int:
        return 3 * self.hidden * self.shared_inter * 2

    @property
    def router_bytes(self) -> int:
        return self.num_experts * self.hidden * 2

    @property
    def layer_bytes(self) -> int:
        return (self.num_experts * self.expert_bytes + self.shared_bytes + self.router_bytes
                + 4 * self.num_experts)


GLM = LayerShape()


@dataclass(frozen=True)
class Workload:
    name: str
    tokens: int
    x_seed: int
    weight_seeds: tuple
    bias: str = "uniform"          # "uniform" or "zipf"
    shape: LayerShape = field(default=GLM)

    @property
    def layers(self) -> int:
        return len(self.weight_seeds)


WORKLOADS = {
    0: Workload("cfg0_decode_t1", 1, 0, (0,)),
    1: Workload("cfg1_decode_t64", 64, 1, (0,)),
    2: Workload("cfg2_prefill_t4096", 4096, 2, (0,)),
    3: Workload("cfg3_ep_t16384_x8", 16384, 10, tuple(range(10, 18))),
    4: Workload("cfg4_zipf_t8192_x8", 8192, 20, tuple(range(20, 28)), bias="zipf"),
}

ZIPF_S = 1.1
ZIPF_BETA = 0.12


def zipf_bias(num_experts: int, seed: int, s: float = ZIPF_S, beta: float = ZIPF_BETA):
    """Correction bias that makes expert popularity follow Zipf(s).

    Expert popularity p_r ~ r^-s over a seeded permutation of expert ids;
    bias_e = beta * ln(p_e / p_max). Because top-8 picks 8 distinct experts a
    token, an expert can hold at most 1/8 of the token-slots; the realised
    hottest share is measured and reported, not assumed.
    """
    rng = np.random.default_rng(seed)
    order = rng.permutation(num_experts)
    ranks = np.empty(num_experts, np.int64)
    ranks[order] = np.arange(1, num_experts + 1)
    lnp = -s * np.log(ranks.astype(np.float64))
    return (beta * (lnp - lnp.max())).astype(np.float32)


def decode_bytes(shape: LayerShape, tokens: int, active_experts: int) -> int:
    """Algorithmic HBM bytes of one decode layer: router + bias + every active
    expert once + shared once + x (bf16) + out (fp32)."""
    return (shape.router_bytes + 4 * shape.num_experts
            + active_experts * shape.expert_bytes
            + (shape.shared_bytes if shape.shared_inter else 0)
            + tokens * shape.hidden * 2 + tokens * shape.hidden * 4)


def layer_flops(shape: LayerShape, tokens: int) -> int:
    """Useful flops of one layer: router GEMM + k routed + 1 shared SwiGLU."""
    k = min(shape.top_k, shape.num_experts)
    routed = tokens * k * 2 * 3 * shape.hidden * shape.inter
    shared = tokens * 2 * 3 * shape.hidden * shape.shared_inter if shape.shared_inter else 0
    return 2 * tokens * shape.num_experts * shape.hidden + routed + shared


def expected_active(shape: LayerShape, tokens: int) -> float:
    k, E = shape.top_k, shape.num_experts
    return E * (1.0 - (1.0 - k / E) ** tokens)


__all__ = ["LayerShape", "GLM", "Workload", "WORKLOADS", "zipf_bias", "decode_bytes",
           "layer_flops", "expected_active"]
