"""hf_moe_route_noalloc: routing for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: an engine that gave every byte of device
memory to its resident expert weights, or a decode loop that must not take the
device-wide synchronization an allocation can bring. This entry point keeps
its scratch in a fixed array inside the library. The test calls it through the
C ABI twice in a row (different token counts and inputs, so leftovers of the
first call must not leak into the second) and checks every output against the
context-based hf_moe_route, with the tolerance the other GPU tests use (the
kernels are the same, so the results are in fact identical). The file name
makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _routing_outputs(T, k, E):
    dev = "cuda"
    return dict(topk_ids=torch.full((T, k), -1, dtype=torch.int32, device=dev),
                topk_weights=torch.full((T, k), -1.0, dtype=torch.float32, device=dev),
                counts=torch.full((E + 1,), -1, dtype=torch.int32, device=dev),
                offsets=torch.full((E + 2,), -1, dtype=torch.int32, device=dev),
                perm=torch.full((T * k + T,), -1, dtype=torch.int32, device=dev))


@pytest.mark.gpu
def test_route_noalloc_matches_route_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oracle import oracle as O
    from hummingflight_b200 import _lib
    from hummingflight_b200.configs import GLM
    from hummingflight_b200.moe import MoELayer

    L = MoELayer(GLM, 1, 128, 0, "gemv")
    L.synth_layer(0, 0, 0)
    router, bias = L.router_device_ptrs(0)
    H, E, k = GLM.hidden, GLM.num_experts, GLM.top_k
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (T, xseed) in enumerate([(64, 1), (5, 3)]):
        xb = O.gen_x_bf16(xseed, T, H)
        x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
        ref = L.route(0, x)
        out = _routing_outputs(T, k, E)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = lib.hf_moe_route_noalloc(
            router, bias, x.data_ptr(), _lib.HF_BF16, T, H, E, k, GLM.scale,
            int(GLM.norm_topk), 1, out["topk_ids"].data_ptr(), out["topk_weights"].data_ptr(),
            out["counts"].data_ptr(), out["offsets"].data_ptr(), out["perm"].data_ptr(), stream)
        torch.cuda.synchronize()
        assert st == _lib.HF_OK, lib.hf_last_error()
        if call > 0:  # after the first call's one-time set-up, nothing is allocated
            assert torch.cuda.mem_get_info()[0] == free_before
        assert torch.equal(out["topk_ids"], ref["topk_ids"])
        w, wr = out["topk_weights"].cpu().numpy(), ref["topk_weights"].cpu().numpy()
        assert np.abs(w - wr).max() <= 1e-6
        assert torch.equal(out["counts"], ref["counts"])
        assert torch.equal(out["offsets"][:E + 2], ref["offsets"])
        assert torch.equal(out["perm"], ref["perm"])
    # sizes beyond the static scratch are rejected with a clear error
    big = _routing_outputs(1, k, E)
    st = lib.hf_moe_route_noalloc(router, bias, x.data_ptr(), _lib.HF_BF16, 129, H, E, k, 2.5, 1,
                                  1, big["topk_ids"].data_ptr(), big["topk_weights"].data_ptr(),
                                  big["counts"].data_ptr(), big["offsets"].data_ptr(),
                                  big["perm"].data_ptr(), stream)
    assert st == _lib.HF_ERR_ARG
    assert b"static scratch" in lib.hf_last_error()
    L.close()
