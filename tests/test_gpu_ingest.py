"""GPU checks of checkpoint ingest (include/hf_ingest.h): a layer written as
safetensors shards, in the checkpoint's tensor names and per-projection layout
(weight_index.cpp:219-244), made resident by hf_moe_load_safetensors.

The shard contents are the seeded generator's weights (the same bytes that
hf_moe_synth_layer writes on the device), so the loaded layer must hold
exactly the synthesized layer's bytes and give bit-identical outputs; the
outputs are also checked against the oracle at the usual bars. Missing or
mis-shaped tensors must be refused.
"""
import numpy as np
import pytest

from oracle import oracle as O
from hummingflight_b200.configs import LayerShape

from st_cases import tensors_file
from test_gpu_moe import close, need_gpu, x_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SMALL = LayerShape(256, 64, 8, 64, 128, 2.5, True)
WSEED, MODEL_LAYER = 81, 5


def moe():
    from hummingflight_b200 import moe as M
    return M


def layer_tensors(shape, wseed):
    H, E, I, Is = shape.hidden, shape.num_experts, shape.inter, shape.shared_inter
    pre = f"model.layers.{MODEL_LAYER}.mlp."
    router = O.gen_bf16_normal(wseed, 0, O.KIND_ROUTER, 0, 0.02, E * H).reshape(E, H)
    bias = O.gen_f32_uniform(wseed, 0, O.KIND_BIAS, 0, -0.1, 0.1, E)
    t = [(pre + "gate.weight", "BF16", (E, H), router.tobytes()),
         (pre + "gate.e_score_correction_bias", "F32", (E,), bias.tobytes())]
    experts = []
    for e in range(E):
        g = O.gen_expert(wseed, 0, e, H, I)
        n = I * H
        x = f"experts.{e}."
        experts += [(pre + x + "gate_proj.weight", "BF16", (I, H), g[:n].tobytes()),
                    (pre + x + "up_proj.weight", "BF16", (I, H), g[n:2 * n].tobytes()),
                    (pre + x + "down_proj.weight", "BF16", (H, I), g[2 * n:].tobytes())]
    s = O.gen_expert(wseed, 0, E, H, Is)
    n = Is * H
    shared = [(pre + "shared_experts.gate_proj.weight", "BF16", (Is, H), s[:n].tobytes()),
              (pre + "shared_experts.up_proj.weight", "BF16", (Is, H), s[n:2 * n].tobytes()),
              (pre + "shared_experts.down_proj.weight", "BF16", (H, Is), s[2 * n:].tobytes())]
    return t, experts, shared


@pytest.fixture(scope="module")
def shards(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    t, experts, shared = layer_tensors(SMALL, WSEED)
    half = len(experts) // 2
    other = [(f"model.layers.{MODEL_LAYER}.self_attn.o_proj.weight", "BF16", (4, 4), bytes(32)),
             (f"model.layers.{MODEL_LAYER + 1}.mlp.gate.weight", "BF16", (4, 4), bytes(32))]
    p1, p2 = d / "model-00001-of-00002.safetensors", d / "model-00002-of-00002.safetensors"
    p1.write_bytes(tensors_file(t + experts[:half], metadata={"format": "pt"}))
    p2.write_bytes(tensors_file(other + experts[half:] + shared))
    return [str(p1), str(p2)], d


def test_loaded_layer_is_the_synthesized_layer(shards):
    need_gpu()
    M = moe()
    paths, _ = shards
    A = M.MoELayer(SMALL, 1, 300, 0, "auto")
    A.synth_layer(0, WSEED, 0)
    B = M.MoELayer(SMALL, 1, 300, 0, "auto")
    st = B.load_safetensors(0, paths, MODEL_LAYER)
    E = SMALL.num_experts
    assert st["experts"] == E and st["tensors"] == 2 + 3 * E + 3 and st["has_bias"] == 1
    blk = 3 * SMALL.hidden * SMALL.inter
    assert st["bytes"] == 2 * (E * SMALL.hidden + E * blk + 3 * SMALL.hidden * SMALL.shared_inter) \
        + 4 * E
    # the resident bytes of every expert, the shared expert and the router
    for eid in (0, 17, E - 1, E):
        n = blk if eid < E else 3 * SMALL.hidden * SMALL.shared_inter
        a = _wrap(A.expert_device_ptr(0, eid), n).clone()
        b = _wrap(B.expert_device_ptr(0, eid), n).clone()
        assert torch.equal(a, b), f"expert {eid}"
    (ra, ba), (rb, bb) = A.router_device_ptrs(0), B.router_device_ptrs(0)
    assert torch.equal(_wrap(ra, E * SMALL.hidden).clone(), _wrap(rb, E * SMALL.hidden).clone())
    assert torch.equal(_wrap(ba, 2 * E).clone(), _wrap(bb, 2 * E).clone())
    for T, xdt in ((1, "f32"), (16, "bf16"), (300, "bf16")):
        x, xb = x_dev(82 + T, T, SMALL.hidden, xdt)
        oa, ob = A.forward(0, x), B.forward(0, x)
        torch.cuda.synchronize()
        assert torch.equal(oa, ob), f"T={T}: outputs differ"
        if T <= 16:
            d = O.Dims(SMALL.hidden, E, SMALL.top_k, SMALL.inter, SMALL.shared_inter, SMALL.scale)
            orc = O.moe_layer_synth(d, WSEED, 0, O.bf16_to_f32(xb).reshape(T, SMALL.hidden))
            close(ob.cpu().numpy(), orc["out"], f"loaded layer T={T}")
    A.close()
    B.close()


def _wrap(ptr, n):
    """A torch view of n int16 at a device address owned by the library."""
    class _Cai:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(_Cai(), device="cuda")


def test_missing_or_misshapen_tensors_are_refused(shards, tmp_path):
    need_gpu()
    M = moe()
    from hummingflight_b200._lib import HfError
    paths, _ = shards
    L = M.MoELayer(SMALL, 1, 8, 0, "auto")
    with pytest.raises(HfError, match="missing"):
        L.load_safetensors(0, paths[:1], MODEL_LAYER)       # experts 32.. are in shard 2
    with pytest.raises(HfError, match="missing"):
        L.load_safetensors(0, paths, MODEL_LAYER + 2)       # no such layer
    with pytest.raises(HfError, match="shape"):
        L.load_safetensors(0, paths, MODEL_LAYER + 1)       # a 4 x 4 decoy router only
    t, experts, shared = layer_tensors(SMALL, WSEED)
    bad = list(t)
    bad[0] = (bad[0][0], "BF16", (SMALL.num_experts // 2, SMALL.hidden * 2), bad[0][3])
    p = tmp_path / "bad.safetensors"
    p.write_bytes(tensors_file(bad + experts + shared))
    with pytest.raises(HfError, match="shape"):
        L.load_safetensors(0, [str(p)], MODEL_LAYER)
    with pytest.raises(HfError, match="two shards"):
        L.load_safetensors(0, paths + [paths[0]], MODEL_LAYER)
    L.close()


def test_upload_one_tensor(shards):
    need_gpu()
    from hummingflight_b200.safetensors import SafeTensors
    paths, _ = shards
    name = f"model.layers.{MODEL_LAYER}.mlp.gate.weight"
    with SafeTensors(paths[0]) as f:
        host = f.read(name)
        dev = torch.empty(host.shape, dtype=torch.int16, device="cuda")
        f.upload(name, dev)
        torch.cuda.synchronize()
        assert np.array_equal(dev.cpu().numpy().view(np.uint16), host)


def test_set_expert_parts_matches_set_expert():
    need_gpu()
    M = moe()
    H, I = SMALL.hidden, SMALL.inter
    g = O.gen_expert(WSEED, 0, 3, H, I)
    n = I * H
    A = M.MoELayer(SMALL, 1, 8, 0, "gemv")
    A.synth_layer(0, WSEED, 0)
    A.set_expert_parts(0, 3, g[:n], g[n:2 * n], g[2 * n:])
    a = _wrap(A.expert_device_ptr(0, 3), 3 * n).clone()
    assert np.array_equal(a.cpu().numpy().view(np.uint16), g)
    A.close()


def test_load_checkpoint_layer_from_directory(shards):
    """The shards of the checkpoint directory (no index there: both files) hold
    the whole layer; the result is the synthesized layer's bytes."""
    need_gpu()
    M = moe()
    paths, d = shards
    from hummingflight_b200.safetensors import layer_shards
    assert layer_shards(str(d), MODEL_LAYER) == sorted(paths)
    L = M.MoELayer(SMALL, 1, 8, 0, "auto")
    st = L.load_checkpoint_layer(0, str(d), MODEL_LAYER)
    assert st["experts"] == SMALL.num_experts and st["has_bias"] == 1
    g = O.gen_expert(WSEED, 0, 5, SMALL.hidden, SMALL.inter)
    got = _wrap(L.expert_device_ptr(0, 5), g.size).clone().cpu().numpy().view(np.uint16)
    assert np.array_equal(got, g)
    L.close()
