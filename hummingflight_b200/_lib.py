"""ctypes binding of libhf_moe.so (the C ABI declared in include/hf_moe.h,
include/hf_synth.h and include/hf_ingest.h).

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
    HF_ERR_UNSUPPORTED, HF_ERR_RANGE = range(9)
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


class HfStOptions(ctypes.Structure):
    _fields_ = [("require_bf16", c_int), ("allow_f32", ctypes.POINTER(ctypes.c_char_p)),
                ("num_allow_f32", c_int), ("require_aligned_header", c_int),
                ("require_aligned_data", c_int)]


class HfStStats(ctypes.Structure):
    _fields_ = [(n, c_u64) for n in ("total", "accepted", "rejected", "duplicate_rejected",
                                     "dtype_rejected", "f32_allowed_accepted", "shape_rejected",
                                     "bounds_rejected", "byte_mismatch_rejected",
                                     "alignment_rejected")]


class HfIngestStats(ctypes.Structure):
    _fields_ = [("bytes", c_u64), ("tensors", c_int), ("experts", c_int),
                ("skipped_experts", c_int), ("has_bias", c_int), ("seconds", ctypes.c_double)]


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
    "hf_moe_ep_transport": (c_int, [c_vp, c_vp]),
    "hf_moe_ep_resync": (c_int, [c_vp]),
    "hf_moe_set_placement": (c_int, [c_vp, c_int, c_vp]),
    "hf_ep_balanced_placement": (c_int, [c_int, c_int, c_vp, c_vp]),
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
    "hf_moe_set_expert_parts": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_int]),
    "hf_st_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(HfStOptions), ctypes.POINTER(c_vp),
                           ctypes.POINTER(HfStStats)]),
    "hf_st_close": (c_int, [c_vp]),
    "hf_st_count": (c_int, [c_vp]),
    "hf_st_tensor": (c_int, [c_vp, c_int, ctypes.POINTER(ctypes.c_char_p),
                             ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(c_int),
                             ctypes.POINTER(ctypes.c_int64), c_int, ctypes.POINTER(c_u64),
                             ctypes.POINTER(c_u64)]),
    "hf_st_find": (c_int, [c_vp, ctypes.c_char_p]),
    "hf_st_read": (c_int, [c_vp, c_int, c_vp, c_u64]),
    "hf_st_upload": (c_int, [c_vp, c_int, c_vp, c_u64, c_int]),
    "hf_moe_load_safetensors": (c_int, [c_vp, c_int, c_int, ctypes.POINTER(ctypes.c_char_p), c_int,
                                        ctypes.POINTER(HfIngestStats)]),
    "hf_ingest_release_staging": (c_int, []),
    "hf_st_layer_shards": (c_int, [ctypes.c_char_p, c_int, c_vp, c_size, ctypes.POINTER(c_int)]),
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
