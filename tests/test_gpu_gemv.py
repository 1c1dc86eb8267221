"""The gemv_bf16_f32 device twin (hf_gemv_bf16_f32; compute/cpu_kernels.cpp:43-94)
on the shapes of its call sites in the attention block (glm_forward.cpp:314-408:
q_a, q_b, kv_a, kv_b, o_proj) and the indexer, against the oracle's sequential
restatement. The twin sums in a different order, so the bar is relative to the
row's magnitude: |y - y_ref| <= 1e-5 * sum_j |A_ij x_j| + 1e-6, far inside the
reference self-test's own 1e-3 (self_test.cpp:98-100). Also: alpha / beta,
y read at beta = 0 (NaN propagates as in the reference), K not a multiple of 8
and a misaligned x (scalar path), K = 0.
"""
import numpy as np
import pytest

from oracle import oracle as O

from test_gpu_moe import need_gpu

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def moe():
    from hummingflight_b200 import moe as M
    return M


def case(M_, K, seed):
    rng = np.random.default_rng(seed)
    A = O.f32_to_bf16((rng.standard_normal((M_, K)) * 0.05).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    return A, x


def check(A, x, y0, alpha, beta, got):
    ref = O.gemv_bf16_f32(A, x, y=y0, alpha=alpha, beta=beta)
    scale = np.abs(O.bf16_to_f32(A)).astype(np.float64) @ np.abs(x).astype(np.float64)
    bound = 1e-5 * (abs(alpha) * scale + abs(beta) * np.abs(y0)) + 1e-6
    assert np.all(np.abs(got.astype(np.float64) - ref) <= bound), \
        float(np.max(np.abs(got - ref) - bound))


@pytest.mark.parametrize("name,M_,K", [("q_a", 2048, 6144), ("q_b", 16384, 2048),
                                       ("kv_a", 576, 6144), ("kv_b", 28672, 512),
                                       ("o_proj", 6144, 16384), ("idx_wk", 128, 6144),
                                       ("odd_rows", 1000, 264), ("tiny", 3, 8)])
def test_gemv_twin_attention_shapes(name, M_, K):
    need_gpu()
    A, x = case(M_, K, M_ + K)
    y0 = np.random.default_rng(1).standard_normal(M_).astype(np.float32)
    for alpha, beta in ((1.0, 0.0), (0.5, 2.0)):
        y = torch.from_numpy(y0.copy()).cuda()
        moe().gemv_bf16_f32(torch.from_numpy(A.view(np.int16)).cuda(), torch.from_numpy(x).cuda(),
                            y, M_, K, alpha, beta)
        check(A, x, y0, alpha, beta, y.cpu().numpy())


def test_gemv_twin_scalar_paths_and_edges():
    need_gpu()
    M = moe()
    A, x = case(37, 33, 5)                       # K % 8 != 0
    y = torch.zeros(37, device="cuda")
    M.gemv_bf16_f32(torch.from_numpy(A.view(np.int16)).cuda(), torch.from_numpy(x).cuda(), y,
                    37, 33)
    check(A, x, np.zeros(37, np.float32), 1.0, 0.0, y.cpu().numpy())
    A, x = case(64, 256, 6)                      # x not 16-byte aligned
    xs = torch.zeros(257, device="cuda")
    xs[1:] = torch.from_numpy(x).cuda()
    y = torch.zeros(64, device="cuda")
    M.gemv_bf16_f32(torch.from_numpy(A.view(np.int16)).cuda(), xs[1:], y, 64, 256)
    check(A, x, np.zeros(64, np.float32), 1.0, 0.0, y.cpu().numpy())
    y = torch.full((4,), 3.0, device="cuda")     # K = 0: y = beta * y
    M.gemv_bf16_f32(torch.zeros(1, dtype=torch.int16, device="cuda"),
                    torch.zeros(1, device="cuda"), y, 4, 0, 1.0, 0.5)
    assert torch.equal(y.cpu(), torch.full((4,), 1.5))
    A, x = case(8, 64, 7)                        # beta = 0 still reads y: NaN stays NaN
    y = torch.full((8,), float("nan"), device="cuda")
    M.gemv_bf16_f32(torch.from_numpy(A.view(np.int16)).cuda(), torch.from_numpy(x).cuda(), y, 8, 64)
    assert torch.isnan(y).all()
