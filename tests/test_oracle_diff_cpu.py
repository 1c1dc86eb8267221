"""The oracle against the reference's own compiled CPU code on random inputs.

oracle/_ref/libhfref_scalar.so is the reference's compute/cpu_kernels.cpp (the
Linux build's sequential GEMV) and compute/moe_router.h, compiled unmodified,
with oracle/ref_harness.cpp restating moeLayer's glue. The golden fixtures
pin the oracle (oracle/hf_oracle.c) on fixed vectors; this test draws fresh
seeded inputs and requires the same bits from both:

* gemv_bf16_f32 (cpu_kernels.cpp:43-94): random M, K (not multiples of the
  vector width), alpha and beta, y read when beta == 0 too;
* topKScores (moe_router.h:29-57): random E up to 300, k 1..8 (k > E too),
  with and without bias, normalised or not, two scales. Continuous scores
  have no ties, and there the indices, their order and the weights must be
  bit-identical. Scores quantised to eighths tie often: std::partial_sort's
  order among equal keys is unspecified by the C++ standard, and the oracle
  (like the device kernels) takes the lower expert id first, so there only
  the selected keys -- the sorted biased scores -- must agree;
* the MoE layer (glm_forward.cpp:509-661) on small random shapes and
  generated weights: every output bit, every index and weight.

Skipped where the reference build is absent. No GPU.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.skipif(not O.ref_available("scalar"),
                                reason="the reference's CPU kernels are not built (oracle/_ref)")


def ref_topk(s, b, k, scale, norm):
    R = O.ref_lib("scalar")
    idx = np.zeros(8, np.int32)
    w = np.zeros(8, np.float32)
    n = R.hfr_topk_scores(O._p(s, O._c_f32p), len(s), O._p(b, O._c_f32p), k, scale, int(norm),
                          O._p(idx, O._c_i32p), O._p(w, O._c_f32p))
    return idx[:n], w[:n]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_gemv_bit_exact_on_random_shapes():
    R = O.ref_lib("scalar")
    rng = np.random.default_rng(21)
    for _ in range(300):
        M, K = int(rng.integers(1, 200)), int(rng.integers(1, 400))
        A = np.ascontiguousarray(O.f32_to_bf16(rng.standard_normal(M * K).astype(np.float32))
                                 .reshape(M, K))
        x = rng.standard_normal(K).astype(np.float32)
        y0 = rng.standard_normal(M).astype(np.float32)
        alpha, beta = float(rng.choice([1.0, 0.5, -2.0])), float(rng.choice([0.0, 1.0, 0.25]))
        got = O.gemv_bf16_f32(A, x, y0.copy(), alpha, beta)
        want = y0.copy()
        R.hfr_gemv_bf16_f32(O._p(A, O._c_u16p), O._p(x, O._c_f32p), O._p(want, O._c_f32p), M, K,
                            alpha, beta)
        assert np.array_equal(bits(got), bits(want)), (M, K, alpha, beta)


def test_topk_bit_exact_without_ties_and_same_keys_with_ties():
    rng = np.random.default_rng(22)
    for it in range(4000):
        E, k = int(rng.integers(1, 300)), int(rng.integers(1, 9))
        tie = it % 2 == 1
        s = rng.random(E, dtype=np.float32)
        b = None if rng.random() < 0.3 else (rng.random(E, dtype=np.float32) * 0.2 - 0.1)
        if tie:
            s = (np.floor(s * 8) / 8).astype(np.float32)
            if b is not None:
                b = (np.floor(b * 16) / 16).astype(np.float32)
        b = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
        scale, norm = float(rng.choice([1.0, 2.5])), bool(rng.integers(0, 2))
        i1, w1, _ = O.topk_scores(s, b, k, scale, norm)
        i2, w2 = ref_topk(s, b, k, scale, norm)
        assert len(i1) == len(i2) == min(k, E)
        if not tie:
            assert np.array_equal(i1, i2) and np.array_equal(bits(w1), bits(w2)), (E, k)
        else:
            key = s + (b if b is not None else np.float32(0))
            assert np.array_equal(np.sort(key[i1]), np.sort(key[i2])), (E, k)


@pytest.mark.parametrize("case", range(6))
def test_moe_layer_bit_exact_on_random_small_shapes(case):
    rng = np.random.default_rng(100 + case)
    H = 8 * int(rng.integers(4, 33))
    E = int(rng.choice([4, 8, 16, 32, 64]))
    K = int(rng.integers(1, 9))
    I = 8 * int(rng.integers(2, 17))
    Is = int(rng.choice([0, 8 * int(rng.integers(2, 17))]))
    norm = bool(rng.integers(0, 2))
    d = O.Dims(H, E, K, I, Is, float(rng.choice([1.0, 2.5])), norm)
    wseed, T = int(rng.integers(0, 1 << 30)), 5
    x = O.bf16_to_f32(O.gen_x_bf16(int(rng.integers(0, 1 << 30)), T, H)).reshape(T, H)
    ref = O.RefLayer(d, wseed, 0, flavour="scalar")
    ref.prepare(x)
    want = ref.forward(x)
    ref.close()
    got = O.moe_layer_synth(d, wseed, 0, x)
    k = min(K, E)
    assert np.array_equal(got["ids"], want["ids"][:, :k])
    assert np.array_equal(bits(got["w"]), bits(want["w"][:, :k]))
    assert np.array_equal(bits(got["out"]), bits(want["out"])), (H, E, K, I, Is)
