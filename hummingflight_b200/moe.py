"""Host-side mirror of HummingFlight's MoE-layer interface over libhf_moe.so.

Names and argument meaning follow the reference:

* :class:`MoELayer` ~ ``GLMForward::moeLayer`` (model/glm_forward.cpp:509-661)
  plus the weight provider ``Scheduler::getExpertPtr`` ([gate|up|down] BF16,
  engine/scheduler.h:80-84) and ``getSharedProjectionPtr`` (three pointers,
  :93-96). ``moe_layer(layer, input, output)`` is the per-token, fp32-host
  entry with the reference's signature; ``forward`` runs T tokens on device.
* :func:`gemv_bf16_f32` ~ ``gemv_bf16_f32`` (compute/cpu_kernels.h:16-17).
* :func:`top_k_scores` ~ ``topKScores`` (compute/moe_router.h:29-57).

Errors raise :class:`HfError` carrying the C status; nothing falls back to the
CPU. Torch supplies device memory and the current CUDA stream only.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from ._lib import (HF_BF16, HF_F32, HF_MEM_DEVICE, HF_MEM_HOST, HF_PATH_AUTO, HF_PATH_GEMM,
                   HF_PATH_GEMV, HfError, HfMoeConfig, HfMoeRouting, call)
from .configs import GLM, LayerShape

_PATHS = {"auto": HF_PATH_AUTO, "gemv": HF_PATH_GEMV, "gemm": HF_PATH_GEMM}
_ACT = {"f32": HF_F32, "bf16": HF_BF16}


def _torch():
    import torch
    return torch


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


def _kind(t) -> int:
    return HF_MEM_HOST if isinstance(t, np.ndarray) or not t.is_cuda else HF_MEM_DEVICE


def _dtype_code(t) -> int:
    torch = _torch()
    if isinstance(t, np.ndarray):
        if t.dtype == np.float32:
            return HF_F32
        if t.dtype == np.uint16:
            return HF_BF16
    elif t.dtype == torch.float32:
        return HF_F32
    elif t.dtype in (torch.bfloat16, torch.int16, torch.uint16):
        return HF_BF16
    raise TypeError("activations must be bfloat16 (or raw uint16/int16 bits) or float32")


def _host_u16(a):
    if isinstance(a, np.ndarray):
        return np.ascontiguousarray(a).view(np.uint16)
    return a


class MoELayer:
    """Resident MoE layers on one device (a drop-in for the reference's moeLayer)."""

    def __init__(self, shape: LayerShape = GLM, num_layers: int = 1, max_tokens: int = 64,
                 device: int = 0, path: str = "auto", gemv_max_tokens: int = 0,
                 ep_rank: int = 0, ep_world: int = 1, ep_unique_id: Optional[bytes] = None):
        """ep_world > 1: this rank holds experts [ep_rank*E/W, (ep_rank+1)*E/W)
        and exchanges token rows with the other ranks (ep_unique_id from
        hummingflight_b200.ep.unique_id() on rank 0, shared with all ranks)."""
        self.shape = shape
        self.num_layers = num_layers
        self.max_tokens = max_tokens
        self.device = device
        self.k = min(shape.top_k, shape.num_experts)
        self.ep_rank, self.ep_world = ep_rank, ep_world
        uid = None
        if ep_world > 1:
            if ep_unique_id is None or len(ep_unique_id) != 128:
                raise ValueError("ep_unique_id (128 bytes) is required when ep_world > 1")
            uid = ctypes.create_string_buffer(bytes(ep_unique_id), 128)
        cfg = HfMoeConfig(shape.hidden, shape.num_experts, shape.top_k, shape.inter,
                          shape.shared_inter, shape.scale, int(shape.norm_topk), num_layers,
                          max_tokens, device, _PATHS[path], gemv_max_tokens, ep_rank, ep_world,
                          ctypes.cast(uid, ctypes.c_void_p) if uid is not None else None)
        h = ctypes.c_void_p()
        call("hf_moe_create", ctypes.byref(h), ctypes.byref(cfg))
        self._h = h

    # ---------------------------------------------------------------- weights
    def set_router(self, layer: int, router_bf16, bias=None):
        """mlp.gate.weight [E x H] BF16 bits + e_score_correction_bias [E] fp32."""
        r = _host_u16(router_bf16)
        b = np.ascontiguousarray(bias, np.float32) if isinstance(bias, np.ndarray) else bias
        kind = _kind(r)
        call("hf_moe_set_router", self._h, layer, _ptr(r), _ptr(b), kind)

    def set_expert(self, layer: int, eid: int, gate_up_down):
        """One expert in getExpertPtr's [gate | up | down] layout (BF16 bits)."""
        w = _host_u16(gate_up_down)
        call("hf_moe_set_expert", self._h, layer, eid, _ptr(w), _kind(w))

    def set_shared(self, layer: int, gate, up, down):
        g, u, d = _host_u16(gate), _host_u16(up), _host_u16(down)
        call("hf_moe_set_shared", self._h, layer, _ptr(g), _ptr(u), _ptr(d), _kind(g))

    def synth_layer(self, layer: int, seed: int, gen_layer: int = 0, bias=None, stream=None):
        """Seeded synthetic weights written in place (include/hf_synth.h)."""
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        call("hf_moe_synth_layer", self._h, layer, seed, gen_layer, _ptr(b), _stream(stream))

    def set_expert_parts(self, layer: int, eid: int, gate, up, down):
        """One expert from its three checkpoint tensors (experts.<e>.{gate,up,down}_proj)."""
        g, u, d = _host_u16(gate), _host_u16(up), _host_u16(down)
        call("hf_moe_set_expert_parts", self._h, layer, eid, _ptr(g), _ptr(u), _ptr(d), _kind(g))

    def load_safetensors(self, layer: int, shard_paths, model_layer: Optional[int] = None):
        """Makes `layer` resident from safetensors shards holding model layer
        `model_layer` (default: the same index); returns the ingest stats."""
        from ._lib import HfIngestStats
        from .safetensors import shard_paths_arg
        paths = [str(p) for p in shard_paths]
        st = HfIngestStats()
        call("hf_moe_load_safetensors", self._h, layer,
             layer if model_layer is None else model_layer, shard_paths_arg(paths), len(paths),
             ctypes.byref(st))
        return {n: getattr(st, n) for n, _ in HfIngestStats._fields_}

    def load_checkpoint_layer(self, layer: int, checkpoint_dir: str, model_layer: int):
        """load_safetensors over the shards of `checkpoint_dir` that hold model
        layer `model_layer` (see hummingflight_b200.safetensors.layer_shards)."""
        from .safetensors import layer_shards
        return self.load_safetensors(layer, layer_shards(checkpoint_dir, model_layer), model_layer)

    def expert_device_ptr(self, layer: int, eid: int) -> int:
        p = ctypes.c_void_p()
        call("hf_moe_expert_device_ptr", self._h, layer, eid, ctypes.byref(p))
        return p.value

    def router_device_ptrs(self, layer: int):
        r, b = ctypes.c_void_p(), ctypes.c_void_p()
        call("hf_moe_router_device_ptr", self._h, layer, ctypes.byref(r), ctypes.byref(b))
        return r.value, b.value

    # ---------------------------------------------------------------- forward
    def forward(self, layer: int, x, out=None, routing: bool = False, slot_out: bool = False,
                stream=None):
        """MoE layer over x [T x H] (device, bf16 or fp32) -> fp32 [T x H].

        With routing=True also returns a dict of device tensors: topk_ids,
        topk_weights, margins, counts [E+1], offsets [E+2], perm [T*k+T] (and
        slot_out [(T*k+T) x H] when slot_out=True)."""
        torch = _torch()
        T, H = x.shape
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        r, rs = self._routing_bufs(T, x.device, routing, slot_out)
        call("hf_moe_forward", self._h, layer, _ptr(x), _dtype_code(x), T, _ptr(out),
             ctypes.byref(rs) if rs is not None else None, _stream(stream))
        return (out, r) if routing else out

    def block_forward(self, layer: int, hidden, norm_weight=None, eps: float = 1e-5,
                      act_dtype: str = "f32", out=None, routing: bool = False,
                      slot_out: bool = False, stream=None):
        """The MLP residual block (glm_forward.cpp:785-796): returns
        hidden + moeLayer(rmsNorm(norm_weight, hidden)) as fp32 [T x H].

        hidden: device fp32 [T x H]; norm_weight: device BF16 bits [H] or None;
        act_dtype "f32" (the reference's hand-off) or "bf16"; out may be
        `hidden` itself (in place, as the reference updates hiddenStates)."""
        torch = _torch()
        T, H = hidden.shape
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=hidden.device)
        r, rs = self._routing_bufs(T, hidden.device, routing, slot_out)
        call("hf_moe_block_forward", self._h, layer, _ptr(hidden), _ptr(out), _ptr(norm_weight),
             eps, _ACT[act_dtype], T, ctypes.byref(rs) if rs is not None else None,
             _stream(stream))
        return (out, r) if routing else out

    def route(self, layer: int, x, stream=None):
        torch = _torch()
        T, _ = x.shape
        r, rs = self._routing_bufs(T, x.device, True, False)
        call("hf_moe_route", self._h, layer, _ptr(x), _dtype_code(x), T, ctypes.byref(rs),
             _stream(stream))
        return r

    def _routing_bufs(self, T, device, routing, slot_out):
        if not routing and not slot_out:
            return None, None
        torch = _torch()
        E, k, H = self.shape.num_experts, self.k, self.shape.hidden
        ns = T * k + (T if self.shape.shared_inter else 0)
        r = dict(topk_ids=torch.empty((T, k), dtype=torch.int32, device=device),
                 topk_weights=torch.empty((T, k), dtype=torch.float32, device=device),
                 margins=torch.empty(T, dtype=torch.float32, device=device),
                 counts=torch.empty(E + 1, dtype=torch.int32, device=device),
                 offsets=torch.empty(E + 2, dtype=torch.int32, device=device),
                 perm=torch.empty(ns, dtype=torch.int32, device=device))
        if slot_out:
            r["slot_out"] = torch.empty((T * k + T, H), dtype=torch.float32, device=device)
        rs = HfMoeRouting(*[_ptr(r.get(n)) for n in ("topk_ids", "topk_weights", "margins",
                                                      "counts", "offsets", "perm", "slot_out")])
        return r, rs

    def forward_host(self, layer: int, x_host: np.ndarray, out_host: Optional[np.ndarray] = None,
                     stream=None) -> np.ndarray:
        """Host buffers in and out (H2D, layer, D2H, wait); pinned numpy views
        make the copies asynchronous DMA."""
        T, H = x_host.shape
        if out_host is None:
            out_host = np.empty((T, H), np.float32)
        code = HF_F32 if x_host.dtype == np.float32 else HF_BF16
        call("hf_moe_forward_host", self._h, layer, x_host.ctypes.data, code, T,
             out_host.ctypes.data, _stream(stream) if stream is not None else None)
        return out_host

    def moe_layer(self, layer: int, input: np.ndarray, output: Optional[np.ndarray] = None):
        """GLMForward::moeLayer(layer, input, output): one token, fp32 host vectors."""
        inp = np.ascontiguousarray(input, np.float32)
        if output is None:
            output = np.empty(self.shape.hidden, np.float32)
        call("hf_moe_layer", self._h, layer, inp.ctypes.data, output.ctypes.data)
        return output

    def synchronize(self):
        """Wait for the last forward; raises HfError(HF_ERR_TIMEOUT) when a
        bounded device wait gave up in one of the forwards since the last check."""
        call("hf_moe_synchronize", self._h)

    def set_placement(self, layer: int, order):
        """Expert placement of a layer (hf_moe_set_placement): rank r owns the
        experts order[r*E/W:(r+1)*E/W]. Set the layer's weights afterwards."""
        o = None if order is None else np.ascontiguousarray(order, np.int32)
        call("hf_moe_set_placement", self._h, layer, _ptr(o))

    EP_TRANSPORTS = {0: "none", 1: "peer", 2: "nccl_slabs", 3: "nccl_sized"}

    def ep_transport(self) -> str:
        """The exchange the ranks agreed on at create (hf_moe_ep_transport)."""
        v = ctypes.c_int()
        call("hf_moe_ep_transport", self._h, ctypes.byref(v))
        return self.EP_TRANSPORTS[v.value]

    def ep_resync(self):
        """Every rank, between forwards, after a forward some rank skipped."""
        call("hf_moe_ep_resync", self._h)

    def set_wait_timeout(self, ns: int):
        call("hf_moe_set_wait_timeout", self._h, ns)

    def debug_stall(self, enable: bool):
        """Test hook: tensor-core kernels wait on a barrier nothing signals."""
        call("hf_moe_debug_stall", self._h, int(enable))

    def last_stats(self):
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        call("hf_moe_last_stats", self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return dict(active_experts=a.value, gemv_segments=b.value, gemm_segments=c.value)

    PHASES = ("router", "route", "gemv_gate_up", "gemv_down", "gemm_gate_up", "gemm_down",
              "combine", "ep_dispatch", "ep_return", "norm")

    def profile(self, enable: bool = True):
        call("hf_moe_profile", self._h, int(enable))

    def profile_read(self):
        """{phase: (ms, launches)} since the previous read (waits for the work)."""
        ms = (ctypes.c_double * len(self.PHASES))()
        ln = (ctypes.c_longlong * len(self.PHASES))()
        call("hf_moe_profile_read", self._h, ms, ln)
        return {p: (ms[i], ln[i]) for i, p in enumerate(self.PHASES)}

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().hf_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def balanced_placement(load, world: int) -> np.ndarray:
    """hf_ep_balanced_placement: an expert order for set_placement that
    balances `load` [E] (e.g. calibration token counts) over `world` ranks."""
    ld = np.ascontiguousarray(load, np.int64)
    order = np.empty(ld.size, np.int32)
    call("hf_ep_balanced_placement", int(ld.size), int(world), _ptr(ld), _ptr(order))
    return order


def gemv_bf16_f32(A, x, y, M: int, K: int, alpha: float = 1.0, beta: float = 0.0, stream=None):
    """y = alpha * A x + beta * y on device (A BF16 bits [M x K], x/y fp32)."""
    call("hf_gemv_bf16_f32", _ptr(A), _ptr(x), _ptr(y), M, K, alpha, beta, _stream(stream))
    return y


def top_k_scores(scores, bias, top_k: int, routed_scaling_factor: float, norm_topk_prob: bool,
                 stream=None):
    """topKScores over rows of scores [T x E] (device fp32) -> (indices, weights)."""
    torch = _torch()
    T, E = scores.shape
    k = min(top_k, E)
    idx = torch.empty((T, k), dtype=torch.int32, device=scores.device)
    w = torch.empty((T, k), dtype=torch.float32, device=scores.device)
    call("hf_topk_scores", _ptr(scores), T, E, _ptr(bias), top_k, routed_scaling_factor,
         int(norm_topk_prob), _ptr(idx), _ptr(w), _stream(stream))
    return idx, w


def dense_mlp_workspace_size(T: int, H: int, I: int) -> int:
    return int(_lib.lib().hf_dense_mlp_workspace_size(T, H, I))


def dense_mlp_forward(gate, up, down, x, out=None, workspace=None, stream=None):
    """denseMlp (glm_forward.cpp:411-432) over the rows of x [T x H] (device
    bf16 or fp32): out = Wd (silu(Wg x) * (Wu x)), fp32 [T x H]. gate/up are
    BF16 bits [I x H], down [H x I], each its own device tensor."""
    torch = _torch()
    T, H = x.shape
    I = gate.shape[0]
    if tuple(gate.shape) != (I, H) or tuple(up.shape) != (I, H) or tuple(down.shape) != (H, I):
        raise ValueError("dense_mlp_forward: gate/up must be [I x H] and down [H x I]")
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
    need = dense_mlp_workspace_size(T, H, I)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    call("hf_dense_mlp_forward", _ptr(gate), _ptr(up), _ptr(down), _ptr(x), _dtype_code(x), T, H,
         I, _ptr(out), _ptr(workspace), workspace.numel(), _stream(stream))
    return out, workspace


def dense_block_forward(gate, up, down, hidden, norm_weight=None, eps: float = 1e-5,
                        act_dtype: str = "f32", out=None, workspace=None, stream=None):
    """The dense layers' MLP residual block (glm_forward.cpp:785-796 with
    denseMlp): hidden + denseMlp(rmsNorm(norm_weight, hidden)), fp32 [T x H].
    out may be `hidden` itself."""
    torch = _torch()
    T, H = hidden.shape
    I = gate.shape[0]
    if tuple(gate.shape) != (I, H) or tuple(up.shape) != (I, H) or tuple(down.shape) != (H, I):
        raise ValueError("dense_block_forward: gate/up must be [I x H] and down [H x I]")
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=hidden.device)
    need = dense_mlp_workspace_size(T, H, I)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=hidden.device)
    call("hf_dense_block_forward", _ptr(gate), _ptr(up), _ptr(down), _ptr(norm_weight), eps,
         _ACT[act_dtype], _ptr(hidden), _ptr(out), T, H, I, _ptr(workspace), workspace.numel(),
         _stream(stream))
    return out, workspace


def rmsnorm(x, weight=None, eps: float = 1e-5, out_dtype: str = "f32", out=None, stream=None):
    """GLMForward::rmsNorm (glm_forward.cpp:185-197) over the rows of x [T x H]
    (device fp32); weight: device BF16 bits [H] or None. Returns fp32 or bf16."""
    torch = _torch()
    T, H = x.shape
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32 if out_dtype == "f32" else torch.bfloat16,
                          device=x.device)
    call("hf_rmsnorm", _ptr(x), _ptr(weight), eps, T, H, _ptr(out), _ACT[out_dtype],
         _stream(stream))
    return out


def dense_mlp_status(workspace, stream=None):
    """Waits for the stream; raises HfError (HF_ERR_TIMEOUT) if the last dense
    forward on this workspace hit a bounded-wait timeout."""
    call("hf_dense_mlp_status", _ptr(workspace), _stream(stream))


def synth_bf16_normal(dst, seed: int, layer: int, kind: int, expert: int, sigma: float,
                      stream=None):
    call("hf_synth_bf16_normal", _ptr(dst), dst.numel(), seed, layer, kind, expert, sigma,
         _stream(stream))
    return dst


def synth_f32_uniform(dst, seed: int, layer: int, kind: int, expert: int, lo: float, hi: float,
                      stream=None):
    call("hf_synth_f32_uniform", _ptr(dst), dst.numel(), seed, layer, kind, expert, lo, hi,
         _stream(stream))
    return dst


__all__ = ["MoELayer", "balanced_placement", "gemv_bf16_f32", "top_k_scores", "dense_mlp_forward",
           "dense_mlp_workspace_size", "dense_mlp_status", "dense_block_forward", "rmsnorm",
           "synth_bf16_normal",
           "synth_f32_uniform", "HfError", "HF_BF16", "HF_F32"]
