"""hf_moe_route_noalloc: routing for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: an engine that gave every byte of device
memory to its resident expert weights, or a decode loop that must not take the
device-wide synchronization an allocation can bring. This entry point keeps
its scratch in a fixed array inside the library. The test calls it through the
C ABI several times in a row -- different token counts, activation types and
inputs, so leftovers of one call must not leak into the next -- and checks
every output against the context-based hf_moe_route, with the tolerance the
other GPU tests use (the kernels are the same, so the results are in fact
identical), and against the oracle's router + topKScores: indices equal off
near-ties, weights within 1e-5, counts / offsets / permutation bit-exact
against a CPU counting sort of the returned indices. The calls cover both
routing paths: up to 64 tokens one fused launch, 65..128 tokens (128 fills
the static scratch) the tiled router plus separate top-k and permutation
launches. The file name makes pytest collect it last.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _routing_outputs(T, k, E):
    dev = "cuda"
    return dict(topk_ids=torch.full((T, k), -1, dtype=torch.int32, device=dev),
                topk_weights=torch.full((T, k), -1.0, dtype=torch.float32, device=dev),
                counts=torch.full((E + 1,), -1, dtype=torch.int32, device=dev),
                offsets=torch.full((E + 2,), -1, dtype=torch.int32, device=dev),
                perm=torch.full((max(1, T * k + T),), -1, dtype=torch.int32, device=dev))


def _call(lib, router, bias, x, xdt, T, shape, out, stream):
    return lib.hf_moe_route_noalloc(
        router, bias, x.data_ptr() if x is not None else None, xdt, T, shape.hidden,
        shape.num_experts, shape.top_k, shape.scale, int(shape.norm_topk), 1,
        out["topk_ids"].data_ptr(), out["topk_weights"].data_ptr(), out["counts"].data_ptr(),
        out["offsets"].data_ptr(), out["perm"].data_ptr(), stream)


@pytest.mark.gpu
def test_route_noalloc_matches_route_and_oracle():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oracle import oracle as O
    from hummingflight_b200 import _lib
    from hummingflight_b200.configs import GLM, LayerShape
    from hummingflight_b200.moe import MoELayer

    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    small = LayerShape(256, 64, 8, 64, 128, 2.5, True)
    layers = {}
    for shape, wseed in ((GLM, 0), (small, 7)):
        L = MoELayer(shape, 1, 128, 0, "gemv")
        L.synth_layer(0, wseed, 0)
        layers[shape] = (L, wseed)
    # (shape, T, x seed, activation dtype): ordered so that every call differs
    # from the one before it in size or type; T = 128 fills the array
    calls = [(GLM, 64, 1, "bf16"), (GLM, 5, 3, "bf16"), (GLM, 128, 4, "bf16"),
             (GLM, 33, 5, "f32"), (small, 100, 6, "bf16"), (GLM, 0, 0, "bf16"),
             (GLM, 7, 8, "bf16")]
    for i, (shape, T, xseed, xdt) in enumerate(calls):
        L, wseed = layers[shape]
        router, bias = L.router_device_ptrs(0)
        H, E, k = shape.hidden, shape.num_experts, shape.top_k
        xb = O.gen_x_bf16(xseed, T, H)
        if xdt == "bf16":
            x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
            code = _lib.HF_BF16
        else:
            x = torch.from_numpy(O.bf16_to_f32(xb).reshape(T, H)).cuda()
            code = _lib.HF_F32
        ref = L.route(0, x)
        out = _routing_outputs(T, k, E)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = _call(lib, router, bias, x, code, T, shape, out, stream)
        torch.cuda.synchronize()
        assert st == _lib.HF_OK, lib.hf_last_error()
        if i > 0:  # after the first call's one-time set-up, nothing is allocated
            assert torch.cuda.mem_get_info()[0] == free_before
        if T == 0:  # an empty batch: zero counts and offsets, like hf_moe_route
            assert not out["counts"].any() and not out["offsets"].any()
            assert not ref["counts"].any() and not ref["offsets"].any()
            continue
        d = O.Dims(H, E, k, shape.inter, shape.shared_inter, shape.scale)
        ids_o, w_o, mg = O.route_synth(d, wseed, 0, O.bf16_to_f32(xb).reshape(T, H))
        firm = mg > 1e-4
        # the same as the context-based route (whose router may sum the logits
        # in another order: tokens closer to a tie than that may swap)
        ids, ids_r = out["topk_ids"].cpu().numpy(), ref["topk_ids"].cpu().numpy()
        assert np.array_equal(ids[firm], ids_r[firm])
        same_r = np.all(ids == ids_r, axis=1)
        assert same_r.mean() >= 0.9
        w, wr = out["topk_weights"].cpu().numpy(), ref["topk_weights"].cpu().numpy()
        assert np.abs(w[same_r] - wr[same_r]).max() <= 1e-6
        if same_r.all():
            assert torch.equal(out["counts"], ref["counts"])
            assert torch.equal(out["offsets"], ref["offsets"])
            assert torch.equal(out["perm"][:T * k + T], ref["perm"])
        # and to the oracle: router GEMV + sigmoid + topKScores, then the
        # canonical counting sort of the returned indices
        assert np.array_equal(ids[firm], ids_o[firm]), f"call {i}: indices"
        same = np.all(ids == ids_o, axis=1)
        assert same.mean() >= 0.9
        assert np.abs(w[same] - w_o[same]).max() <= 1e-5, f"call {i}: weights"
        c, off, perm = O.permute(ids, E, True)
        assert np.array_equal(out["counts"].cpu().numpy(), c)
        assert np.array_equal(out["offsets"].cpu().numpy(), off)
        assert np.array_equal(out["perm"].cpu().numpy()[:T * k + T], perm)
    # sizes beyond the static scratch are rejected with a clear error
    L, _ = layers[GLM]
    router, bias = L.router_device_ptrs(0)
    big = _routing_outputs(1, GLM.top_k, GLM.num_experts)
    x = torch.zeros((1, GLM.hidden), dtype=torch.bfloat16, device="cuda")
    st = _call(lib, router, bias, x, _lib.HF_BF16, 129, GLM, big, stream)
    assert st == _lib.HF_ERR_ARG
    assert b"static scratch" in lib.hf_last_error()
    for L, _ in layers.values():
        L.close()
