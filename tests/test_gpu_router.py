"""The tcgen05 router (bf16 batches from 16 tokens: router rows x token rows on
the tensor cores, K split into runs whose partial logit planes the top-k sums
in order) against the SIMT router kernels and the oracle.

Both routers must pick the oracle's experts wherever the 8th/9th biased-score
margin exceeds 1e-4; between themselves the selections agree off such
near-ties and the routing weights within 1e-5.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from hummingflight_b200.configs import GLM, LayerShape

from test_gpu_moe import need_gpu, x_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def route_with(mode, shape, wseed, x, T):
    from hummingflight_b200 import moe as M
    old = os.environ.get("HF_ROUTER")
    os.environ["HF_ROUTER"] = mode
    try:
        L = M.MoELayer(shape, 1, T, 0, "auto")
    finally:
        if old is None:
            del os.environ["HF_ROUTER"]
        else:
            os.environ["HF_ROUTER"] = old
    L.synth_layer(0, wseed, 0)
    r = L.route(0, x)
    L.synchronize()
    out = {k: v.cpu().numpy() for k, v in r.items()}
    L.close()
    return out


@pytest.mark.parametrize("T", [16, 64, 300, 4096])
def test_tc_router_agrees_with_simt_on_glm(T):
    need_gpu()
    x, _ = x_dev(70 + T, T, GLM.hidden, "bf16")
    a = route_with("simt", GLM, 0, x, T)
    b = route_with("tc", GLM, 0, x, T)
    ok = a["margins"] > 1e-4
    assert ok.mean() > 0.9
    assert np.array_equal(a["topk_ids"][ok], b["topk_ids"][ok])
    same = (a["topk_ids"] == b["topk_ids"]).all(axis=1)
    assert np.abs(a["topk_weights"][same] - b["topk_weights"][same]).max() <= 1e-5
    if same.all():
        assert np.array_equal(a["counts"], b["counts"])
        assert np.array_equal(a["perm"], b["perm"])


@pytest.mark.parametrize("E,T", [(128, 40), (200, 70), (64, 16)])
def test_tc_router_small_shapes_match_oracle(E, T):
    """E = 128: one 128-row tile; E = 200: a second 128-row block that is
    partly past the last router row; E = 64: one partial tile."""
    need_gpu()
    H, k, I, Is = 512, 8, 128, 128
    shape = LayerShape(H, E, k, I, Is, 2.5, True)
    x, xb = x_dev(80 + E, T, H, "bf16")
    r = route_with("tc", shape, 81, x, T)
    d = O.Dims(H, E, k, I, Is, 2.5)
    ids_o, w_o, mg = O.route_synth(d, 81, 0, O.bf16_to_f32(xb).reshape(T, H))
    ok = mg > 1e-4
    assert np.array_equal(r["topk_ids"][ok], ids_o[ok])
    assert np.abs(r["topk_weights"][ok] - w_o[ok]).max() <= 1e-5
