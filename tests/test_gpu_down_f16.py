"""The FP16 down pass (csrc/hf_weights.cu): the resident down blocks are FP16
(w * 2^S per block) and the SwiGLU intermediate one FP16 plane (mid * 2^-6),
so the down GEMM runs one MMA pass instead of the BF16 hi + lo pair.

* The conversion keeps every BF16 weight: a block handed out through
  hf_moe_expert_device_ptr after forwards reads back bit for bit.
* Outputs stay within the north-star bars against the oracle on both passes
  (FP16, and HF_DOWN_F16=0: the BF16 hi + lo pass); the decode GEMV reads
  the FP16 block and gives the same bits as it does from the BF16 block.
* An intermediate beyond the FP16 range (|mid| > 4.2e6) is reported as
  HF_ERR_RANGE, never returned silently, and the context stays usable.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from hummingflight_b200.configs import LayerShape

from test_gpu_ingest import _wrap
from test_gpu_moe import close, need_gpu, x_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SHAPE = LayerShape(256, 16, 4, 128, 192, 2.5, True)
HERE = os.path.dirname(os.path.abspath(__file__))


def moe():
    from hummingflight_b200 import moe as M
    return M


@pytest.mark.parametrize("path", ["gemm", "auto"])
def test_down_blocks_read_back_exactly_after_forwards(path):
    need_gpu()
    M = moe()
    T = 300 if path == "gemm" else 1
    L = M.MoELayer(SHAPE, 1, T, 0, path)
    L.synth_layer(0, 91, 0)
    x, xb = x_dev(92, T, SHAPE.hidden, "bf16")
    out1 = L.forward(0, x)
    L.synchronize()
    n = 3 * SHAPE.hidden * SHAPE.inter
    for eid in (0, 7, SHAPE.num_experts - 1):
        got = _wrap(L.expert_device_ptr(0, eid), n).clone().cpu().numpy().view(np.uint16)
        assert np.array_equal(got, O.gen_expert(91, 0, eid, SHAPE.hidden, SHAPE.inter)), eid
    ns = 3 * SHAPE.hidden * SHAPE.shared_inter
    got = _wrap(L.expert_device_ptr(0, SHAPE.num_experts), ns).clone().cpu().numpy().view(np.uint16)
    assert np.array_equal(got, O.gen_expert(91, 0, SHAPE.num_experts, SHAPE.hidden,
                                            SHAPE.shared_inter))
    # after the read-back (blocks in BF16 again) the next forward converts and
    # gives the same bits as the first
    out2 = L.forward(0, x)
    L.synchronize()
    assert torch.equal(out1, out2)
    orc = O.moe_layer_synth(O.Dims(*[getattr(SHAPE, f) for f in
                                     ("hidden", "num_experts", "top_k", "inter",
                                      "shared_inter")]), 91, 0,
                            O.bf16_to_f32(xb).reshape(T, -1))
    close(out1.cpu().numpy(), orc["out"], f"fp16 down pass, {path}")
    L.close()


def test_intermediate_beyond_fp16_range_is_an_error():
    """Gate and up rows of 16.0 on activations of ones (H = 256): g = u = 4096
    and mid = silu(4096) * 4096 ~ 1.7e7, beyond the 4.2e6 the FP16 plane
    holds: the forward reports HF_ERR_RANGE, and a normal forward on the same
    context is correct again."""
    need_gpu()
    M = moe()
    H, E, K, I, Is = 256, 4, 2, 64, 64
    shape = LayerShape(H, E, K, I, Is, 2.5, True)
    T = 300
    L = M.MoELayer(shape, 1, T, 0, "gemm")
    router = np.zeros((E, H), np.uint16)
    big = O.f32_to_bf16(np.full(I * H, 16.0, np.float32))
    down = O.f32_to_bf16(np.full(H * I, 1e-3, np.float32))
    L.set_router(0, router, np.zeros(E, np.float32))
    for e in range(E):
        L.set_expert(0, e, np.concatenate([big, big, down]))
    L.set_shared(0, big, big, down)
    x = torch.ones((T, H), dtype=torch.bfloat16, device="cuda")
    L.forward(0, x)
    with pytest.raises(M.HfError) as e:
        L.synchronize()
    assert e.value.status == 8  # HF_ERR_RANGE
    L.synth_layer(0, 93, 0)
    xs, xb = x_dev(94, T, H, "bf16")
    out = L.forward(0, xs)
    L.synchronize()
    orc = O.moe_layer_synth(O.Dims(H, E, K, I, Is), 93, 0, O.bf16_to_f32(xb).reshape(T, H))
    close(out.cpu().numpy(), orc["out"], "after the range error")
    L.close()


def test_bf16_hi_lo_pass_still_available(tmp_path):
    """HF_DOWN_F16=0 (a fresh process) keeps the BF16 hi + lo down pass. On
    the GEMM (1500 tokens) both passes meet the bars against the oracle and
    agree to 5e-4 relative (the FP16 plane's rounding of mid, 2^-11); on the
    decode GEMV (one token) the FP16 block gives the same bits as the BF16."""
    need_gpu()
    code = r'''
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from oracle import oracle as O
from hummingflight_b200.moe import MoELayer
from hummingflight_b200.configs import LayerShape
s = LayerShape(256, 16, 4, 128, 192, 2.5, True)
for T, path, f in ((1500, "gemm", sys.argv[2]), (1, "auto", sys.argv[3])):
    L = MoELayer(s, 1, T, 0, path); L.synth_layer(0, 95, 0)
    xb = O.gen_x_bf16(96, T, 256)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    out = L.forward(0, x); L.synchronize()
    np.save(f, out.cpu().numpy())
    L.close()
'''
    outs = {}
    for flag in ("1", "0"):
        fa, fb = str(tmp_path / f"gemm_{flag}.npy"), str(tmp_path / f"gemv_{flag}.npy")
        env = dict(os.environ, HF_DOWN_F16=flag)
        p = subprocess.run([sys.executable, "-c", code, os.path.dirname(HERE), fa, fb], env=env,
                           capture_output=True, text=True, timeout=300)
        assert p.returncode == 0, p.stderr[-2000:]
        outs[flag] = (np.load(fa), np.load(fb))
    orc = O.moe_layer_synth(O.Dims(256, 16, 4, 128, 192), 95, 0,
                            O.bf16_to_f32(O.gen_x_bf16(96, 1500, 256)).reshape(1500, 256))
    for flag, (o, _) in outs.items():
        close(o, orc["out"], f"HF_DOWN_F16={flag}")
    a, b = outs["1"][0].astype(np.float64), outs["0"][0].astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 5e-4
    assert np.array_equal(outs["1"][1].view(np.uint32), outs["0"][1].view(np.uint32))
