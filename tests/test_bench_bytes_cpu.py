"""bench.py's algorithmic bytes (the roofline numerators) follow the library's
formats: mid is one FP16 plane on the GEMM's FP16 down pass and fp32 on the
GEMV; expert outputs are one FP16 plane when no segment can take the GEMV
(GEMM path, or AUTO with no GEMV threshold) and fp32 otherwise; HF_DOWN_F16=0
and HF_Y_F16=0 restore the wider formats."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import bench  # noqa: E402
from hummingflight_b200.configs import LayerShape  # noqa: E402

S = LayerShape(256, 8, 2, 128, 64, 2.5, True)
T, K = 40, 2


def counts():
    c = np.zeros(S.num_experts + 1, np.int64)
    c[:S.num_experts] = T * K // S.num_experts
    c[S.num_experts] = T
    return c


def expect(y_e, mid_e):
    H, I, Is, E = S.hidden, S.inter, S.shared_inter, S.num_experts
    c = counts()
    slots = int(c.sum())
    mid = int((c[:E] * I).sum() + c[E] * Is) * mid_e
    w_d = E * H * I * 2 + H * Is * 2
    return w_d + mid + slots * H * y_e, slots * H * y_e + T * H * 4 + T * K * 8


@pytest.mark.parametrize("path,gemv_max,env,y_e,mid_e", [
    ("gemm", 0, {}, 2, 2),
    ("auto", 0, {}, 2, 2),
    ("gemm", 0, {"HF_Y_F16": "0"}, 4, 2),
    ("gemm", 0, {"HF_DOWN_F16": "0"}, 2, 4),
])
def test_gemm_bytes_follow_the_formats(monkeypatch, path, gemv_max, env, y_e, mid_e):
    for k in ("HF_Y_F16", "HF_DOWN_F16"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    pb = bench.phase_bytes(S, counts(), T, K, path, gemv_max)
    down, combine = expect(y_e, mid_e)
    assert pb["gemm_down"] == down
    assert pb["combine"] == combine


def test_gemv_possible_keeps_fp32_outputs(monkeypatch):
    monkeypatch.delenv("HF_Y_F16", raising=False)
    pb = bench.phase_bytes(S, counts(), T, K, "auto", 1)
    _, combine = expect(4, 2)
    assert pb["combine"] == combine
