"""The oracle (oracle/hf_oracle.c) against the reference's own outputs.

tests/golden/ holds vectors produced by the reference's unmodified
compute/cpu_kernels.cpp and compute/moe_router.h (tests/golden/make_golden.py):
its self-test inputs (src/self_test.cpp:53-70, :73-103, :125-138, :180-200), its expert-FFN
parity case (compute/cuda_backend.cpp:497-520) and GLMForward::moeLayer
(model/glm_forward.cpp:509-661) on seeded layers. The oracle restates the
scalar Linux build, so it must match that build bit for bit.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from hummingflight_b200.configs import GLM

G = os.path.join(os.path.dirname(__file__), "golden")


def kat(flavour="scalar"):
    with open(os.path.join(G, f"ref_kat_{flavour}.json")) as f:
        d = json.load(f)
    out = {}
    for k, v in d.items():
        a = np.array(v, dtype=np.int64)
        if k.endswith("_idx"):
            out[k] = a.astype(np.int32)
        elif k in ("gemv_A", "expert_w", "bf16_out"):
            out[k] = a.astype(np.uint16)
        else:
            out[k] = a.astype(np.uint32).view(np.float32)
    return out


def test_gemv_selftest_vectors_bit_exact():
    k = kat("scalar")
    A = k["gemv_A"].reshape(8, 33)
    y = O.gemv_bf16_f32(A, k["gemv_x"])
    assert np.array_equal(y.view(np.uint32), k["gemv_y"].view(np.uint32))
    # the reference self-test's own tolerance against its naive loop
    assert np.abs(y - k["gemv_y_naive"]).max() < 1e-3
    y2 = O.gemv_bf16_f32(A, k["gemv_x"], y=np.full(8, 7.0, np.float32), alpha=2.0, beta=0.5)
    assert np.array_equal(y2.view(np.uint32), k["gemv_y_alpha2_beta05_y7"].view(np.uint32))


def test_gemv_avx2_build_within_selftest_tolerance():
    k = kat("avx2")
    y = O.gemv_bf16_f32(k["gemv_A"].reshape(8, 33), k["gemv_x"])
    assert np.abs(y - k["gemv_y"]).max() < 1e-3


def test_bf16_rounding_known_answers():
    """BFloat16::fromF32 (dtype_bf16.h:27-33) on self_test.cpp:53-70's values and
    the rounding edges: ties to even both ways, exponent carries, subnormals,
    the largest finite value, infinities."""
    k = kat("scalar")
    assert np.array_equal(O.f32_to_bf16(k["bf16_in"]), k["bf16_out"])
    # and the widening back is exact
    back = O.bf16_to_f32(k["bf16_out"])
    assert np.array_equal(O.f32_to_bf16(back), k["bf16_out"])


def test_rmsnorm_selftest_vector_bit_exact():
    """self_test.cpp:125-138 (the math GLMForward::rmsNorm runs), no weight."""
    k = kat("scalar")
    y = O.rmsnorm(k["rmsnorm_x"], None, 1e-5)[0]
    assert np.array_equal(y.view(np.uint32), k["rmsnorm_y"].view(np.uint32))


def test_rmsnorm_weight_and_residual_follow_reference_order():
    """glm_forward.cpp:193 multiplies (x * rms) * w left to right; :795-796
    adds the MLP output to the residual. A weight of ones is the identity."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 96)).astype(np.float32)
    w = O.f32_to_bf16(rng.uniform(0.5, 1.5, 96).astype(np.float32))
    got = O.rmsnorm(x, w, 1e-5)
    plain = O.rmsnorm(x, None, 1e-5)
    wf = O.bf16_to_f32(w)
    assert np.array_equal(got, (plain * wf).astype(np.float32))
    ones = O.f32_to_bf16(np.ones(96, np.float32))
    assert np.array_equal(O.rmsnorm(x, ones, 1e-5), plain)
    m = rng.standard_normal((3, 96)).astype(np.float32)
    assert np.array_equal(O.residual_add(x, m), x + m)


def test_topk_known_answers():
    k = kat("scalar")
    s, b = k["topk_scores"], k["topk_bias_vec"]
    cases = {"topk_plain": (None, 3, 1.0, False), "topk_norm": (None, 3, 1.0, True),
             "topk_scaled": (None, 3, 2.5, False), "topk_bias": (b, 3, 1.0, False),
             "topk_k8_norm_scaled": (None, 8, 2.5, True)}
    for name, (bias, kk, sc, norm) in cases.items():
        idx, w, _ = O.topk_scores(s, bias, kk, sc, norm)
        assert np.array_equal(idx, k[name + "_idx"]), name
        assert np.array_equal(w.view(np.uint32), k[name + "_w"].view(np.uint32)), name
    # the literal expectations of src/self_test.cpp:180-200
    assert list(k["topk_plain_idx"]) == [2, 6, 4]
    assert k["topk_bias_idx"][0] == 6
    assert abs(float(np.sum(k["topk_norm_w"])) - 1.0) < 1e-5


def test_topk_edge_cases():
    s = np.array([0.5, 0.5, 0.2, 0.9], np.float32)
    idx, w, m = O.topk_scores(s, None, 2, 1.0, False)
    assert list(idx) == [3, 0]          # tie 0/1 -> lower id first
    assert m == 0.0
    idx, w, _ = O.topk_scores(s, None, 8, 1.0, True)   # k > E -> k = E
    assert len(idx) == 4
    idx, w, _ = O.topk_scores(s, None, 0, 1.0, True)
    assert len(idx) == 0
    z = np.zeros(4, np.float32)                         # sum == 0: no normalisation
    idx, w, _ = O.topk_scores(z, None, 2, 2.5, True)
    assert np.all(w == 0.0)


def test_expert_ffn_selftest_case():
    k = kat("scalar")
    h, i = 64, 32
    w = k["expert_w"]
    half = h * i
    y = np.zeros(h, np.float32)
    x = k["expert_x"]
    L = O.lib()
    L.hfo_expert_ffn(w[:half].ctypes.data_as(O._c_u16p), w[half:2 * half].ctypes.data_as(O._c_u16p),
                     w[2 * half:].ctypes.data_as(O._c_u16p), x.ctypes.data_as(O._c_f32p),
                     y.ctypes.data_as(O._c_f32p), h, i)
    assert np.array_equal(y.view(np.uint32), k["expert_y"].view(np.uint32))


@pytest.mark.parametrize("name", ["moe_small", "moe_mid", "moe_noshared", "moe_k_gt_e", "moe_zipf"])
def test_moe_layer_matches_reference(name):
    z = np.load(os.path.join(G, name + ".npz"))
    H, E, K, I, Is = (int(v) for v in z["dims"])
    d = O.Dims(H, E, K, I, Is, float(z["scale"]))
    T = z["out"].shape[0]
    x = O.bf16_to_f32(O.gen_x_bf16(int(z["xseed"]), T, H))
    bias = z["bias"] if z["bias"].size else None
    r = O.moe_layer_synth(d, int(z["wseed"]), 0, x, bias=bias, want_slots=True)
    k = min(K, E)
    assert np.array_equal(r["ids"], z["ids"][:, :k])
    assert np.array_equal(r["w"].view(np.uint32), z["w"][:, :k].view(np.uint32))
    assert np.array_equal(r["out"].view(np.uint32), z["out"].view(np.uint32))
    # per-slot expert outputs: harness layout [T, K+1, H] (shared last)
    ref_slots = z["slots"]
    for t in range(T):
        for i in range(k):
            assert np.array_equal(r["slots"][t * k + i], ref_slots[t, i])
        if Is:
            assert np.array_equal(r["slots"][T * k + t], ref_slots[t, K])
    # the AVX2 build differs only by summation order
    assert np.abs(r["out"] - z["out_avx2"]).max() < 1e-4


def test_moe_cfg0_full_size_matches_reference():
    z = np.load(os.path.join(G, "moe_cfg0.npz"))
    s = GLM
    d = O.Dims(s.hidden, s.num_experts, s.top_k, s.inter, s.shared_inter, s.scale)
    x = O.bf16_to_f32(O.gen_x_bf16(0, 1, s.hidden))
    r = O.moe_layer_synth(d, 0, 0, x)
    assert np.array_equal(r["ids"], z["ids"])
    assert np.array_equal(r["out"].view(np.uint32), z["out"].view(np.uint32))
    assert float(r["margins"][0]) > 1e-4


def test_permute_canonical_order():
    ids = np.array([[3, 1], [1, 0], [3, 2]], np.int32)
    counts, offsets, perm = O.permute(ids, 4, has_shared=True)
    assert list(counts) == [1, 2, 1, 2, 3]
    assert list(offsets) == [0, 1, 3, 4, 6, 9]
    # expert 0: (t1,s1)=3; expert 1: (t0,s1)=1,(t1,s0)=2; expert 2: (t2,s1)=5;
    # expert 3: (t0,s0)=0,(t2,s0)=4; shared: 6,7,8
    assert list(perm) == [3, 1, 2, 5, 0, 4, 6, 7, 8]


def test_generator_numpy_matches_c():
    n = 4099
    a = O.gen_bf16_normal(3, 2, O.KIND_UP, 9, 0.02, n)
    b = np.zeros(n, np.uint16)
    O.lib().hfo_gen_bf16_normal(3, 2, O.KIND_UP, 9, 0.02, n, b.ctypes.data_as(O._c_u16p))
    assert np.array_equal(a, b)
    v = O.bf16_to_f32(O.gen_bf16_normal(1, 0, O.KIND_GATE, 0, 0.02, 1 << 18))
    assert abs(v.std() - 0.02) < 5e-4 and abs(v.mean()) < 2e-4
