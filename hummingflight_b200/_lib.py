"""ctypes binding of libhf_moe.so (the C ABI declared in include/hf_moe.h and
include/hf_synth.h).

The library is built in-tree by hummingflight_b200/build.py. Loading fails
loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhf_moe.so")

c_int, c_float, c_size, c_u64, c_u32, c_vp = (ctypes.c_int, ctypes.c_float, ctypes.c_size_t,
                                              ctypes.c_uint64, ctypes.c_uint32, ctypes.c_void_p)

HF_OK, HF_ERR_ARG, HF_ERR_CUDA, HF_ERR_NCCL, HF_ERR_TIMEOUT, HF_ERR_OOM, HF_ERR_STATE, \
    HF_ERR_UNSUPPORTED = range(8)
HF_MEM_HOST, HF_MEM_DEVICE = 0, 1
HF_BF16, HF_F32 = 0, 1
HF_PATH_AUTO, HF_PATH_GEMV, HF_PATH_GEMM = 0, 1, 2


class HfMoeConfig(ctypes.Structure):
    _fields_ = [("hidden_size", c_int), ("num_experts", c_int), ("num_experts_per_tok", c_int),
                ("moe_intermediate_size", c_int), ("shared_intermediate_size", c_int),
                ("routed_scaling_factor", c_float), ("norm_topk_prob", c_int),
                ("num_layers", c_int), ("max_tokens", c_int), ("device", c_int),
                ("path", c_int), ("gemv_max_tokens", c_int), ("ep_rank", c_int),
                ("ep_world", c_int), ("ep_unique_id", c_vp)]


class HfMoeRouting(ctypes.Structure):
    _fields_ = [("topk_ids", c_vp), ("topk_weights", c_vp), ("margins", c_vp), ("counts", c_vp),
                ("offsets", c_vp), ("perm", c_vp), ("slot_out", c_vp)]


class HfError(RuntimeError):
    def __init__(self, status: int, fn: str, msg: str):
        super().__init__(f"{fn} -> {status_name(status)}: {msg}")
        self.status = status


# name -> (restype, argtypes); every entry point declared in include/*.h
SIGNATURES = {
    "hf_abi_version": (c_int, []),
    "hf_status_string": (ctypes.c_char_p, [c_int]),
    "hf_last_error": (ctypes.c_char_p, []),
    "hf_moe_create": (c_int, [ctypes.POINTER(c_vp), ctypes.POINTER(HfMoeConfig)]),
    "hf_moe_destroy": (c_int, [c_vp]),
    "hf_moe_set_router": (c_int, [c_vp, c_int, c_vp, c_vp, c_int]),
    "hf_moe_set_expert": (c_int, [c_vp, c_int, c_int, c_vp, c_int]),
    "hf_moe_set_shared": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_int]),
    "hf_moe_expert_device_ptr": (c_int, [c_vp, c_int, c_int, ctypes.POINTER(c_vp)]),
    "hf_moe_router_device_ptr": (c_int, [c_vp, c_int, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp)]),
    "hf_moe_mark_loaded": (c_int, [c_vp, c_int]),
    "hf_moe_forward": (c_int, [c_vp, c_int, c_vp, c_int, c_int, c_vp, ctypes.POINTER(HfMoeRouting), c_vp]),
    "hf_moe_forward_host": (c_int, [c_vp, c_int, c_vp, c_int, c_int, c_vp, c_vp]),
    "hf_moe_layer": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "hf_moe_block_forward": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_float, c_int, c_int,
                                     ctypes.POINTER(HfMoeRouting), c_vp]),
    "hf_moe_route": (c_int, [c_vp, c_int, c_vp, c_int, c_int, ctypes.POINTER(HfMoeRouting), c_vp]),
    "hf_ep_unique_id": (c_int, [c_vp]),
    "hf_ep_plan": (c_int, [c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hf_moe_route_noalloc": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_float,
                                     c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hf_moe_last_stats": (c_int, [c_vp, ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "hf_moe_synchronize": (c_int, [c_vp]),
    "hf_moe_set_wait_timeout": (c_int, [c_vp, c_u64]),
    "hf_moe_debug_stall": (c_int, [c_vp, c_int]),
    "hf_moe_profile": (c_int, [c_vp, c_int]),
    "hf_moe_profile_read": (c_int, [c_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)]),
    "hf_gemv_bf16_f32": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_float, c_float, c_vp]),
    "hf_topk_scores": (c_int, [c_vp, c_int, c_int, c_vp, c_int, c_float, c_int, c_vp, c_vp, c_vp]),
    "hf_dense_mlp_workspace_size": (c_size, [c_int, c_int, c_int]),
    "hf_dense_mlp_forward": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_size, c_vp]),
    "hf_dense_mlp_status": (c_int, [c_vp, c_vp]),
    "hf_dense_block_forward": (c_int, [c_vp, c_vp, c_vp, c_vp, c_float, c_int, c_vp, c_vp, c_int,
                                       c_int, c_int, c_vp, c_size, c_vp]),
    "hf_rmsnorm": (c_int, [c_vp, c_vp, c_float, c_int, c_int, c_vp, c_int, c_vp]),
    "hf_synth_bf16_normal": (c_int, [c_vp, c_u64, c_u64, c_u32, c_u32, c_u32, ctypes.c_double, c_vp]),
    "hf_synth_f32_uniform": (c_int, [c_vp, c_u64, c_u64, c_u32, c_u32, c_u32, c_float, c_float, c_vp]),
    "hf_moe_synth_layer": (c_int, [c_vp, c_int, c_u64, c_u32, c_vp, c_vp]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m hummingflight_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_name(s: int) -> str:
    try:
        return lib().hf_status_string(s).decode()
    except Exception:
        return str(s)


def check(status: int, fn: str) -> None:
    if status != HF_OK:
        msg = lib().hf_last_error().decode(errors="replace")
        raise HfError(status, fn, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
