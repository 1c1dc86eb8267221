"""ctypes view of the parity oracle (TEST INFRASTRUCTURE, never the product).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs import this module. It loads

* ``oracle/liboracle.so`` -- the C restatement of the reference's MoE layer
  (oracle/hf_oracle.c), and
* ``oracle/_ref/libhfref_{avx2,scalar}.so`` -- the reference's own
  ``compute/cpu_kernels.cpp`` + ``compute/moe_router.h`` with the
  ``GLMForward::moeLayer`` glue restated (oracle/ref_harness.cpp), when they
  were built (they need the reference source tree at build time).

The numpy generator below mirrors oracle/hf_gen.h bit for bit; it is used to
build small inputs in tests without touching C.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_u16p = ctypes.POINTER(ctypes.c_uint16)

KIND_X, KIND_ROUTER, KIND_BIAS, KIND_GATE, KIND_UP, KIND_DOWN = range(6)
_M64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


class HfoDims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("num_experts", ctypes.c_int),
                ("top_k", ctypes.c_int), ("inter", ctypes.c_int),
                ("shared_inter", ctypes.c_int), ("scale", ctypes.c_float),
                ("norm_topk", ctypes.c_int)]


@dataclass(frozen=True)
class Dims:
    hidden: int
    num_experts: int
    top_k: int
    inter: int
    shared_inter: int
    scale: float = 2.5
    norm_topk: bool = True

    def c(self) -> HfoDims:
        return HfoDims(self.hidden, self.num_experts, self.top_k, self.inter,
                       self.shared_inter, self.scale, int(self.norm_topk))


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def _load(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (run __graft_entry__.build())")
    return ctypes.CDLL(path)


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = _load(os.path.join(_HERE, "liboracle.so"))
        L.hfo_gemv_bf16_f32.argtypes = [_c_u16p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_float]
        L.hfo_topk_scores.argtypes = [_c_f32p, ctypes.c_int, _c_f32p, ctypes.c_int,
                                      ctypes.c_float, ctypes.c_int, _c_i32p, _c_f32p, _c_f32p]
        L.hfo_topk_scores.restype = ctypes.c_int
        L.hfo_router_scores.argtypes = [_c_u16p, _c_f32p, ctypes.c_int, ctypes.c_int, _c_f32p]
        L.hfo_expert_ffn.argtypes = [_c_u16p, _c_u16p, _c_u16p, _c_f32p, _c_f32p, ctypes.c_int,
                                     ctypes.c_int]
        L.hfo_rmsnorm.argtypes = [_c_f32p, _c_u16p, ctypes.c_float, ctypes.c_int, _c_f32p]
        L.hfo_residual_add.argtypes = [_c_f32p, _c_f32p, ctypes.c_int, _c_f32p]
        L.hfo_permute.argtypes = [_c_i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  _c_i32p, _c_i32p, _c_i32p]
        L.hfo_moe_layer_synth.argtypes = [ctypes.POINTER(HfoDims), ctypes.c_uint64,
                                          ctypes.c_uint32, _c_f32p, _c_f32p, ctypes.c_int,
                                          _c_f32p, _c_i32p, _c_f32p, _c_f32p, _c_f32p]
        L.hfo_moe_layer_synth.restype = ctypes.c_int
        L.hfo_moe_layer.argtypes = [ctypes.POINTER(HfoDims), _c_u16p, _c_f32p,
                                    ctypes.POINTER(_c_u16p), _c_u16p, _c_f32p, ctypes.c_int,
                                    _c_f32p, _c_i32p, _c_f32p, _c_f32p, _c_f32p]
        L.hfo_moe_layer.restype = ctypes.c_int
        L.hfo_gen_bf16_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.c_double, ctypes.c_uint64,
                                          _c_u16p]
        L.hfo_gen_f32_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                          ctypes.c_uint64, _c_f32p]
        L.hfo_gen_expert.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                     ctypes.c_int, ctypes.c_int, _c_u16p]
        L.hfo_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_available(flavour: str = "avx2") -> bool:
    return os.path.exists(os.path.join(_HERE, "_ref", f"libhfref_{flavour}.so"))


_ref_libs: dict = {}


def ref_lib(flavour: str = "avx2"):
    """The reference's own cpu_kernels.cpp (+ moeLayer glue), `avx2` or `scalar` build."""
    if flavour not in _ref_libs:
        L = _load(os.path.join(_HERE, "_ref", f"libhfref_{flavour}.so"))
        L.hfr_gemv_bf16_f32.argtypes = [_c_u16p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_float]
        L.hfr_topk_scores.argtypes = [_c_f32p, ctypes.c_int, _c_f32p, ctypes.c_int,
                                      ctypes.c_float, ctypes.c_int, _c_i32p, _c_f32p]
        L.hfr_topk_scores.restype = ctypes.c_int
        L.hfr_threads.restype = ctypes.c_int
        L.hfr_layer_create.argtypes = [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int,
                                                             ctypes.c_uint64, ctypes.c_uint32,
                                                             _c_f32p]
        L.hfr_layer_create.restype = ctypes.c_void_p
        L.hfr_layer_destroy.argtypes = [ctypes.c_void_p]
        L.hfr_layer_prepare.argtypes = [ctypes.c_void_p, _c_f32p, ctypes.c_int]
        L.hfr_layer_forward.argtypes = [ctypes.c_void_p, _c_f32p, ctypes.c_int, _c_f32p,
                                        _c_i32p, _c_f32p, _c_f32p]
        L.hfr_layer_forward.restype = ctypes.c_double
        _ref_libs[flavour] = L
    return _ref_libs[flavour]


# ---------------------------------------------------------------- generator
def _mix64(z: np.ndarray) -> np.ndarray:
    z = z ^ (z >> np.uint64(30))
    z = z * np.uint64(0xBF58476D1CE4E5B9)
    z = z ^ (z >> np.uint64(27))
    z = z * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _mix64_int(z: int) -> int:
    z &= _M64
    z ^= z >> 30
    z = (z * 0xBF58476D1CE4E5B9) & _M64
    z ^= z >> 27
    z = (z * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def key(seed: int, layer: int, kind: int, expert: int) -> int:
    k = _mix64_int((seed + GOLDEN) & _M64)
    return _mix64_int(k ^ ((layer << 40) | (kind << 32) | expert))


def _bits(k: int, n: int, start: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        idx = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        return _mix64(np.uint64(k) + idx * np.uint64(GOLDEN))


def normal_scale(sigma: float) -> np.float32:
    return np.float32(sigma / np.sqrt(1431655765.0))


def gen_normal_f32(seed, layer, kind, expert, sigma, n) -> np.ndarray:
    b = _bits(key(seed, layer, kind, expert), n)
    s = ((b & np.uint64(0xFFFF)) + ((b >> np.uint64(16)) & np.uint64(0xFFFF)) +
         ((b >> np.uint64(32)) & np.uint64(0xFFFF)) + (b >> np.uint64(48))).astype(np.int64)
    c = (s - 131070).astype(np.float32)
    return c * normal_scale(sigma)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """BFloat16::fromF32 (compute/dtype_bf16.h:27-33)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return (r & np.uint64(0xFFFF)).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def gen_bf16_normal(seed, layer, kind, expert, sigma, n) -> np.ndarray:
    return f32_to_bf16(gen_normal_f32(seed, layer, kind, expert, sigma, n))


def gen_f32_uniform(seed, layer, kind, expert, lo, hi, n) -> np.ndarray:
    b = _bits(key(seed, layer, kind, expert), n)
    t = (b >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
    w = np.float32(hi) - np.float32(lo)
    return np.float32(lo) + w * t


def gen_x_bf16(seed: int, T: int, H: int) -> np.ndarray:
    """Activations ~N(0,1) BF16, [T x H] (kind X, layer 0, expert 0)."""
    return gen_bf16_normal(seed, 0, KIND_X, 0, 1.0, T * H).reshape(T, H)


def gen_x_bf16_c(seed: int, T: int, H: int) -> np.ndarray:
    """gen_x_bf16 through the C generator (multi-threaded; same bits)."""
    out = np.empty(T * H, np.uint16)
    lib().hfo_gen_bf16_normal(seed, 0, KIND_X, 0, 1.0, T * H, _p(out, _c_u16p))
    return out.reshape(T, H)


def gen_x_rows_bf16(seed: int, rows, H: int) -> np.ndarray:
    """Rows `rows` of gen_x_bf16(seed, T, H) for any T above them (element
    t*H + j of the stream), without generating the other rows."""
    k = key(seed, 0, KIND_X, 0)
    out = np.empty((len(rows), H), np.uint16)
    sc = normal_scale(1.0)
    for i, t in enumerate(rows):
        b = _bits(k, H, int(t) * H)
        s = ((b & np.uint64(0xFFFF)) + ((b >> np.uint64(16)) & np.uint64(0xFFFF)) +
             ((b >> np.uint64(32)) & np.uint64(0xFFFF)) + (b >> np.uint64(48))).astype(np.int64)
        out[i] = f32_to_bf16((s - 131070).astype(np.float32) * sc)
    return out


# ---------------------------------------------------------------- wrappers
def gemv_bf16_f32(A_bf16, x, y=None, alpha=1.0, beta=0.0):
    A = np.ascontiguousarray(A_bf16, dtype=np.uint16)
    M, K = A.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(M, np.float32) if y is None else np.array(y, dtype=np.float32)
    lib().hfo_gemv_bf16_f32(_p(A, _c_u16p), _p(x, _c_f32p), _p(y, _c_f32p), M, K, alpha, beta)
    return y


def rmsnorm(x, w_bf16=None, eps=1e-5):
    """GLMForward::rmsNorm (glm_forward.cpp:185-197) on each row of x [T x H]."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    w = None if w_bf16 is None else np.ascontiguousarray(w_bf16, dtype=np.uint16)
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        lib().hfo_rmsnorm(_p(x[t], _c_f32p), _p(w, _c_u16p), eps, x.shape[1], _p(out[t], _c_f32p))
    return out


def residual_add(x, mlp_out):
    """glm_forward.cpp:795-796: hidden = residual + mlpOut, per row."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    m = np.ascontiguousarray(np.atleast_2d(mlp_out), dtype=np.float32)
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        lib().hfo_residual_add(_p(x[t], _c_f32p), _p(m[t], _c_f32p), x.shape[1],
                               _p(out[t], _c_f32p))
    return out


def router_scores(router_bf16, x_f32):
    """Router GEMV + sigmoid for one token (glm_forward.cpp:519-524)."""
    W = np.ascontiguousarray(router_bf16, dtype=np.uint16)
    E, H = W.shape
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    s = np.zeros(E, np.float32)
    lib().hfo_router_scores(_p(W, _c_u16p), _p(x, _c_f32p), E, H, _p(s, _c_f32p))
    return s


def route_synth(d: Dims, wseed: int, layer: int, x_f32, bias=None):
    """Router + top-k for every token on generated router weights.
    Returns (ids [T x k], weights [T x k], margins [T])."""
    router = gen_bf16_normal(wseed, layer, KIND_ROUTER, 0, 0.02, d.num_experts * d.hidden)
    router = router.reshape(d.num_experts, d.hidden)
    if bias is None:
        bias = gen_f32_uniform(wseed, layer, KIND_BIAS, 0, -0.1, 0.1, d.num_experts)
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    T = x.shape[0]
    k = min(d.top_k, d.num_experts)
    ids = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    mg = np.zeros(T, np.float32)
    for t in range(T):
        i, ww, m = topk_scores(router_scores(router, x[t]), bias, d.top_k, d.scale, d.norm_topk)
        ids[t], w[t], mg[t] = i, ww, m
    return ids, w, mg


def topk_scores(scores, bias, top_k, scale=2.5, norm=True):
    s = np.ascontiguousarray(scores, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    idx = np.zeros(8, np.int32)
    w = np.zeros(8, np.float32)
    m = np.zeros(1, np.float32)
    k = lib().hfo_topk_scores(_p(s, _c_f32p), len(s), _p(b, _c_f32p), top_k, scale, int(norm),
                              _p(idx, _c_i32p), _p(w, _c_f32p), _p(m, _c_f32p))
    return idx[:k].copy(), w[:k].copy(), float(m[0])


def permute(ids, E, has_shared=True):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, k = ids.shape
    counts = np.zeros(E + 1, np.int32)
    offsets = np.zeros(E + 2, np.int32)
    perm = np.zeros(T * k + T, np.int32)
    lib().hfo_permute(_p(ids, _c_i32p), T, k, E, int(has_shared), _p(counts, _c_i32p),
                      _p(offsets, _c_i32p), _p(perm, _c_i32p))
    n = T * k + (T if has_shared else 0)
    return counts, offsets, perm[:n]


def moe_layer_synth(d: Dims, wseed: int, layer: int, x_f32, bias=None, want_slots=False):
    """Oracle MoE layer on generated weights. Returns dict(out, ids, w, margins[, slots])."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    T = x.shape[0]
    k = min(d.top_k, d.num_experts)
    out = np.zeros((T, d.hidden), np.float32)
    ids = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    mg = np.zeros(T, np.float32)
    slots = np.zeros((T * k + T, d.hidden), np.float32) if want_slots else None
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    dc = d.c()
    rc = lib().hfo_moe_layer_synth(ctypes.byref(dc), wseed, layer, _p(b, _c_f32p),
                                   _p(x, _c_f32p), T, _p(out, _c_f32p), _p(ids, _c_i32p),
                                   _p(w, _c_f32p), _p(mg, _c_f32p), _p(slots, _c_f32p))
    if rc != 0:
        raise ValueError("oracle rejected the layer shape")
    r = dict(out=out, ids=ids, w=w, margins=mg)
    if want_slots:
        r["slots"] = slots
    return r


def gen_expert(wseed, layer, expert, H, I) -> np.ndarray:
    out = np.zeros(3 * H * I, np.uint16)
    lib().hfo_gen_expert(wseed, layer, expert, H, I, _p(out, _c_u16p))
    return out


class RefLayer:
    """The reference's own CPU moeLayer math on generated weights (oracle/_ref)."""

    def __init__(self, d: Dims, wseed: int, layer: int = 0, bias=None, flavour="avx2"):
        self.L = ref_lib(flavour)
        self.d = d
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self.h = self.L.hfr_layer_create(d.hidden, d.num_experts, d.top_k, d.inter,
                                         d.shared_inter, d.scale, int(d.norm_topk), wseed, layer,
                                         _p(b, _c_f32p))
        if not self.h:
            raise ValueError("reference harness rejected the layer shape")

    def prepare(self, x_f32):
        x = np.ascontiguousarray(x_f32, dtype=np.float32)
        self.L.hfr_layer_prepare(self.h, _p(x, _c_f32p), x.shape[0])

    def forward(self, x_f32, want_slots=False):
        x = np.ascontiguousarray(x_f32, dtype=np.float32)
        T, H = x.shape
        k = self.d.top_k
        out = np.zeros((T, H), np.float32)
        ids = np.zeros((T, k), np.int32)
        w = np.zeros((T, k), np.float32)
        slots = np.zeros((T, k + 1, H), np.float32) if want_slots else None
        sec = self.L.hfr_layer_forward(self.h, _p(x, _c_f32p), T, _p(out, _c_f32p),
                                       _p(ids, _c_i32p), _p(w, _c_f32p), _p(slots, _c_f32p))
        return dict(out=out, ids=ids, w=w, seconds=sec, slots=slots)

    def close(self):
        if self.h:
            self.L.hfr_layer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
