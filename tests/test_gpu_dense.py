"""GPU parity of the dense SwiGLU MLP entry (hf_dense_mlp_forward, the
reference's GLMForward::denseMlp, glm_forward.cpp:411-432) against the oracle's
expertFFNRaw restatement (the same three GEMVs and fp32 SwiGLU).

One token runs the GEMV pair, two or more the tcgen05 GEMM (bf16 activations
read in place, fp32 activations split into hi + lo planes). The weights are
three separate device allocations, as the reference's getWeightPtr hands them
out. Bars: max-abs 2e-2 and rel-L2 1e-3 per token, as for the MoE outputs.
"""
import numpy as np
import pytest

from oracle import oracle as O

from test_gpu_moe import close, need_gpu, x_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dense_weights(seed, H, I):
    from hummingflight_b200 import moe as M
    ws = []
    for kind, shape in ((O.KIND_GATE, (I, H)), (O.KIND_UP, (I, H)), (O.KIND_DOWN, (H, I))):
        t = torch.empty(shape, dtype=torch.int16, device="cuda")
        M.synth_bf16_normal(t, seed, 0, kind, 0, 0.02)
        ws.append(t)
    torch.cuda.synchronize()
    return ws


def oracle_rows(ws, xf, rows):
    g, u, d = (np.ascontiguousarray(w.cpu().numpy().view(np.uint16)) for w in ws)
    I, H = g.shape
    out = np.zeros((len(rows), H), np.float32)
    for j, t in enumerate(rows):
        xr = np.ascontiguousarray(xf[t], np.float32)
        O.lib().hfo_expert_ffn(g.ctypes.data_as(O._c_u16p), u.ctypes.data_as(O._c_u16p),
                               d.ctypes.data_as(O._c_u16p), xr.ctypes.data_as(O._c_f32p),
                               out[j].ctypes.data_as(O._c_f32p), H, I)
    return out


def run_dense(ws, x):
    from hummingflight_b200 import moe as M
    out, wsp = M.dense_mlp_forward(ws[0], ws[1], ws[2], x)
    M.dense_mlp_status(wsp)
    return out.cpu().numpy()


@pytest.mark.parametrize("T", [1, 2, 17, 100, 300, 1100])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_dense_small_matches_oracle(T, xdt):
    need_gpu()
    H, I = 256, 384
    ws = dense_weights(51, H, I)
    x, xb = x_dev(52 + T, T, H, xdt)
    got = run_dense(ws, x)
    ref = oracle_rows(ws, O.bf16_to_f32(xb).reshape(T, H), range(T))
    close(got, ref, f"dense T={T} {xdt}")


def test_dense_odd_inter_runs_gemv_path():
    """I = 200 is not 64-aligned: every token count takes the GEMV pair."""
    need_gpu()
    H, I, T = 256, 200, 5
    ws = dense_weights(53, H, I)
    x, xb = x_dev(54, T, H, "f32")
    close(run_dense(ws, x), oracle_rows(ws, O.bf16_to_f32(xb).reshape(T, H), range(T)),
          "dense I=200")


@pytest.mark.parametrize("T,xdt,rows", [(1, "f32", [0]), (64, "bf16", [0, 31, 63])])
def test_dense_glm_shape(T, xdt, rows):
    """GLM dense layers (0-2): H = 6144, I = 12288; sampled tokens."""
    need_gpu()
    H, I = 6144, 12288
    ws = dense_weights(55, H, I)
    x, xb = x_dev(56, T, H, xdt)
    got = run_dense(ws, x)
    ref = oracle_rows(ws, O.bf16_to_f32(xb).reshape(T, H), rows)
    close(got[rows], ref, f"dense GLM T={T}")


def test_dense_workspace_reuse_across_shapes():
    """One workspace sized for the largest call serves smaller calls in order."""
    need_gpu()
    from hummingflight_b200 import moe as M
    H, I = 256, 384
    ws = dense_weights(57, H, I)
    big = torch.empty(M.dense_mlp_workspace_size(300, H, I), dtype=torch.uint8, device="cuda")
    for T in (300, 1, 40):
        x, xb = x_dev(58 + T, T, H, "bf16")
        out, _ = M.dense_mlp_forward(ws[0], ws[1], ws[2], x, workspace=big)
        M.dense_mlp_status(big)
        close(out.cpu().numpy(), oracle_rows(ws, O.bf16_to_f32(xb).reshape(T, H), range(T)),
              f"reuse T={T}")
