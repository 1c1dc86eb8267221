"""Expert outputs as one FP16 plane (y * 2^-4) on forwards whose every segment
takes the tensor-core GEMM: the down GEMM's epilogue stores half the bytes, the
combine (and, across GPUs, the return) moves half.

* Outputs stay within the north-star bars against the oracle, and agree with
  the fp32 outputs (HF_Y_F16=0, a fresh process) to 5e-4 relative: the plane
  rounds each expert output to 11 bits.
* A finite output beyond the plane's range (|y| > 1.05e6) is reported as
  HF_ERR_RANGE, never returned silently, and the context stays usable.
* Single-token decode (the GEMV) keeps fp32 outputs: bit-identical with and
  without the plane.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from hummingflight_b200.configs import LayerShape

from test_gpu_moe import close, need_gpu, x_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
SHAPE = LayerShape(256, 16, 4, 128, 192, 2.5, True)


def moe():
    from hummingflight_b200 import moe as M
    return M


def _dims(s):
    return O.Dims(s.hidden, s.num_experts, s.top_k, s.inter, s.shared_inter)


def test_outputs_beyond_the_plane_are_an_error():
    """Gate and up rows of 0.25 on activations of ones (H = 256): g = u = 64,
    mid = silu(64) * 64 ~ 4096 (inside the mid plane); down rows of 8.0 over
    I = 64 give y = 64 * 8 * 4096 ~ 2.1e6, beyond the 1.05e6 the output plane
    holds: the forward reports HF_ERR_RANGE, and a normal forward on the same
    context is correct again."""
    need_gpu()
    M = moe()
    H, E, K, I, Is = 256, 4, 2, 64, 64
    shape = LayerShape(H, E, K, I, Is, 2.5, True)
    T = 300
    L = M.MoELayer(shape, 1, T, 0, "gemm")
    gu = O.f32_to_bf16(np.full(I * H, 0.25, np.float32))
    down = O.f32_to_bf16(np.full(H * I, 8.0, np.float32))
    L.set_router(0, np.zeros((E, H), np.uint16), np.zeros(E, np.float32))
    for e in range(E):
        L.set_expert(0, e, np.concatenate([gu, gu, down]))
    L.set_shared(0, gu, gu, down)
    x = torch.ones((T, H), dtype=torch.bfloat16, device="cuda")
    L.forward(0, x)
    with pytest.raises(M.HfError) as e:
        L.synchronize()
    assert e.value.status == 8  # HF_ERR_RANGE
    L.synth_layer(0, 97, 0)
    xs, xb = x_dev(98, T, H, "bf16")
    out = L.forward(0, xs)
    L.synchronize()
    orc = O.moe_layer_synth(_dims(shape), 97, 0, O.bf16_to_f32(xb).reshape(T, H))
    close(out.cpu().numpy(), orc["out"], "after the range error")
    L.close()


def test_plane_against_fp32_outputs(tmp_path):
    """HF_Y_F16=1 (default) and 0 in fresh processes: on the GEMM (1500
    tokens) both meet the bars against the oracle, and the outputs and
    per-slot outputs agree to 5e-4 relative; on the decode GEMV (one token)
    they give the same bits."""
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
    out, r = L.forward(0, x, routing=True, slot_out=True); L.synchronize()
    np.save(f, out.cpu().numpy())
    np.save(f + ".slots.npy", r["slot_out"].cpu().numpy())
    L.close()
'''
    outs = {}
    for flag in ("1", "0"):
        fa, fb = str(tmp_path / f"gemm_{flag}.npy"), str(tmp_path / f"gemv_{flag}.npy")
        env = dict(os.environ, HF_Y_F16=flag)
        p = subprocess.run([sys.executable, "-c", code, os.path.dirname(HERE), fa, fb], env=env,
                           capture_output=True, text=True, timeout=300)
        assert p.returncode == 0, p.stderr[-2000:]
        outs[flag] = (np.load(fa), np.load(fb), np.load(fa + ".slots.npy"))
    T = 1500
    orc = O.moe_layer_synth(_dims(SHAPE), 95, 0,
                            O.bf16_to_f32(O.gen_x_bf16(96, T, 256)).reshape(T, 256))
    for flag, (o, _, _) in outs.items():
        close(o, orc["out"], f"HF_Y_F16={flag}")
    a, b = outs["1"][0].astype(np.float64), outs["0"][0].astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 5e-4
    # per-slot outputs (the same routing: it does not depend on the outputs)
    sa, sb = outs["1"][2].astype(np.float64), outs["0"][2].astype(np.float64)
    assert np.linalg.norm(sa - sb) / np.linalg.norm(sb) < 5e-4
    assert np.array_equal(outs["1"][1].view(np.uint32), outs["0"][1].view(np.uint32))
