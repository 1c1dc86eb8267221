"""B200-native (sm_100a) MoE layer for HummingFlight.

The product is the C ABI in include/hf_moe.h, implemented by
hummingflight_b200/libhf_moe.so (hand-written CUDA in csrc/). This package
builds it (build.py), binds it with ctypes (_lib.py) and mirrors the
reference's MoE-layer interface for Python callers (moe.py).
"""
from .configs import GLM, WORKLOADS, LayerShape, Workload  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # moe.py imports torch lazily; keep `import hummingflight_b200` light.
    if name in ("MoELayer", "gemv_bf16_f32", "top_k_scores", "HfError"):
        from . import moe
        return getattr(moe, name)
    raise AttributeError(name)
