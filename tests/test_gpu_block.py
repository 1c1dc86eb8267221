"""GPU parity of the MLP residual block around the layer (glm_forward.cpp:785-796):
hidden = hidden + mlp(rmsNorm(post_attention_layernorm, hidden)), with mlp the
MoE layer (hf_moe_block_forward) or the dense MLP (hf_dense_block_forward), and
of the RMSNorm twin (hf_rmsnorm, GLMForward::rmsNorm, glm_forward.cpp:185-197).

The oracle side is oracle/hf_oracle.c: hfo_rmsnorm (pinned bit-exact on the
reference's self-test vector), the MoE / expert-FFN restatements, then
hfo_residual_add. Hidden states are fp32 values that are not bf16-exact, so the
fp32 hand-off (the reference's) and the bf16 hand-off (rounded once) differ.
Bars: RMSNorm fp32 output within rel 1e-5 (only the squares' summation order
differs; the reference's sequential fp32 sum alone carries a relative error of
up to ~n * 2^-24, a few 1e-6 at n = 6144, half of it in rms), bf16 output within
one bf16 rounding step; block outputs
max-abs 2e-2 and rel-L2 1e-3 on both the block output and its MLP part;
indices bit-exact where the oracle's 8th/9th margin exceeds 1e-4.
"""
import numpy as np
import pytest

from oracle import oracle as O
from hummingflight_b200.configs import GLM, LayerShape

from test_gpu_moe import agreeing, check_routing, close, need_gpu
from test_gpu_dense import dense_weights, oracle_rows

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SMALL = LayerShape(256, 64, 8, 64, 128, 2.5, True)


def moe():
    from hummingflight_b200 import moe as M
    return M


def hidden_states(seed, T, H, scale=3.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((T, H)) * scale).astype(np.float32)


def norm_weight(seed, H):
    rng = np.random.default_rng(seed)
    return O.f32_to_bf16(rng.uniform(0.5, 1.5, H).astype(np.float32))


def dev_u16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def oracle_norm(h, w, act):
    xn = O.rmsnorm(h, w, 1e-5)
    if act == "bf16":
        xn = O.bf16_to_f32(O.f32_to_bf16(xn)).reshape(xn.shape)
    return xn


# ---------------------------------------------------------------- RMSNorm twin
@pytest.mark.parametrize("T,H", [(1, 6144), (7, 256), (300, 1024)])
@pytest.mark.parametrize("weighted", [True, False])
def test_rmsnorm_matches_oracle(T, H, weighted):
    need_gpu()
    M = moe()
    h = hidden_states(60 + T, T, H)
    w = norm_weight(61, H) if weighted else None
    ref = O.rmsnorm(h, w, 1e-5)
    hd = torch.from_numpy(h).cuda()
    wd = dev_u16(w) if weighted else None
    got = M.rmsnorm(hd, wd, 1e-5, "f32").cpu().numpy()
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)
    assert rel.max() < 1e-5, f"rmsnorm f32 rel {rel.max():.3e}"
    gb = M.rmsnorm(hd, wd, 1e-5, "bf16").cpu().view(torch.int16).numpy().view(np.uint16)
    rb = O.f32_to_bf16(ref)
    step = np.abs(gb.astype(np.int32) - rb.reshape(gb.shape).astype(np.int32))
    assert step.max() <= 1, "rmsnorm bf16 more than one rounding step away"
    assert (step > 0).mean() < 1e-2


def test_rmsnorm_on_reference_selftest_vector():
    """self_test.cpp:125-138 (n = 128, no weight) through the device twin."""
    need_gpu()
    from test_oracle_golden import kat
    k = kat("scalar")
    x = torch.from_numpy(k["rmsnorm_x"].reshape(1, 128).copy()).cuda()
    got = moe().rmsnorm(x, None, 1e-5).cpu().numpy()[0]
    assert np.abs(got - k["rmsnorm_y"]).max() <= 1e-6   # the self-test's own bar


# ---------------------------------------------------------------- MoE block
@pytest.mark.parametrize("T", [1, 5, 300])
@pytest.mark.parametrize("act", ["f32", "bf16"])
@pytest.mark.parametrize("inplace", [False, True])
def test_moe_block_matches_oracle(T, act, inplace):
    need_gpu()
    M = moe()
    H = SMALL.hidden
    L = M.MoELayer(SMALL, 1, max(T, 8), 0, "auto")
    L.synth_layer(0, 62, 0)
    h = hidden_states(63 + T, T, H)
    w = norm_weight(64, H)
    hd = torch.from_numpy(h).cuda()
    out, r = L.block_forward(0, hd, dev_u16(w), 1e-5, act, out=hd if inplace else None,
                             routing=True)
    L.synchronize()
    got = out.cpu().numpy()
    xn = oracle_norm(h, w, act)
    d = O.Dims(H, SMALL.num_experts, SMALL.top_k, SMALL.inter, SMALL.shared_inter, SMALL.scale)
    orc = O.moe_layer_synth(d, 62, 0, xn)
    ids = check_routing(r, orc["ids"], orc["margins"], SMALL.num_experts)
    ref = O.residual_add(h, orc["out"])
    a = agreeing(ids, orc["ids"])
    close(got[a], ref[a], f"moe block T={T} {act}")
    close((got - h)[a], orc["out"][a], f"moe block mlp part T={T} {act}")
    if inplace:
        assert out.data_ptr() == hd.data_ptr()
    L.close()


def test_moe_block_without_weight_and_zero_tokens():
    need_gpu()
    M = moe()
    H = SMALL.hidden
    L = M.MoELayer(SMALL, 1, 8, 0, "auto")
    L.synth_layer(0, 65, 0)
    h = hidden_states(66, 3, H)
    out = L.block_forward(0, torch.from_numpy(h).cuda(), None, 1e-6, "f32")
    L.synchronize()
    d = O.Dims(H, SMALL.num_experts, SMALL.top_k, SMALL.inter, SMALL.shared_inter, SMALL.scale)
    orc = O.moe_layer_synth(d, 65, 0, O.rmsnorm(h, None, 1e-6))
    close(out.cpu().numpy(), O.residual_add(h, orc["out"]), "moe block, no norm weight")
    empty = torch.empty((0, H), dtype=torch.float32, device="cuda")
    assert L.block_forward(0, empty, None).shape == (0, H)
    L.close()


def test_moe_block_glm_shape():
    """Full GLM layer (H = 6144, 256 experts, top-8, shared expert), 2 tokens."""
    need_gpu()
    M = moe()
    T, H = 2, GLM.hidden
    L = M.MoELayer(GLM, 1, 8, 0, "auto")
    L.synth_layer(0, 0, 0)
    h = hidden_states(67, T, H)
    w = norm_weight(68, H)
    out, r = L.block_forward(0, torch.from_numpy(h).cuda(), dev_u16(w), 1e-5, "f32",
                             routing=True)
    L.synchronize()
    d = O.Dims(H, GLM.num_experts, GLM.top_k, GLM.inter, GLM.shared_inter, GLM.scale)
    orc = O.moe_layer_synth(d, 0, 0, O.rmsnorm(h, w, 1e-5))
    ids = check_routing(r, orc["ids"], orc["margins"], GLM.num_experts)
    a = agreeing(ids, orc["ids"])
    got = out.cpu().numpy()
    close((got - h)[a], orc["out"][a], "glm moe block mlp part")
    close(got[a], O.residual_add(h, orc["out"])[a], "glm moe block")
    L.close()


# ---------------------------------------------------------------- dense block
@pytest.mark.parametrize("T", [1, 2, 64, 300])
@pytest.mark.parametrize("act", ["f32", "bf16"])
def test_dense_block_matches_oracle(T, act):
    need_gpu()
    M = moe()
    H, I = 256, 384
    ws = dense_weights(69, H, I)
    h = hidden_states(70 + T, T, H)
    w = norm_weight(71, H)
    hd = torch.from_numpy(h).cuda()
    out, wsp = M.dense_block_forward(ws[0], ws[1], ws[2], hd, dev_u16(w), 1e-5, act)
    M.dense_mlp_status(wsp)
    mlp = oracle_rows(ws, oracle_norm(h, w, act), range(T))
    got = out.cpu().numpy()
    close(got, O.residual_add(h, mlp), f"dense block T={T} {act}")
    close(got - h, mlp, f"dense block mlp part T={T} {act}")


@pytest.mark.parametrize("T", [1, 64])
def test_dense_block_in_place_glm_shape(T):
    """Dense layers 0-2 (H = 6144, I = 12288), in place like hiddenStates."""
    need_gpu()
    M = moe()
    H, I = 6144, 12288
    ws = dense_weights(72, H, I)
    h = hidden_states(73, T, H)
    w = norm_weight(74, H)
    hd = torch.from_numpy(h).cuda()
    out, wsp = M.dense_block_forward(ws[0], ws[1], ws[2], hd, dev_u16(w), 1e-5, "f32", out=hd)
    M.dense_mlp_status(wsp)
    assert out.data_ptr() == hd.data_ptr()
    rows = [0] if T == 1 else [0, 37, 63]
    mlp = oracle_rows(ws, O.rmsnorm(h, w, 1e-5), rows)
    got = hd.cpu().numpy()[rows]
    close(got, O.residual_add(h[rows], mlp), f"dense block glm T={T}")
    close(got - h[rows], mlp, f"dense block glm mlp part T={T}")
