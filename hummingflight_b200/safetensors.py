"""Safetensors shards and checkpoint ingest (include/hf_ingest.h).

``SafeTensors(path)`` is the reference's SafeTensorsFile
(model/safetensors.h:64-80): the header is parsed and validated by
libhf_moe.so with the checkpoint loader's strict options unless others are
given; ``tensors()`` lists the accepted ones, ``read()`` returns a tensor's
bytes, ``upload()`` sends them to device memory through the pinned ring.
``MoELayer.load_safetensors`` (hummingflight_b200.moe) makes a whole MoE
layer resident from its shards.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import HfStOptions, HfStStats, call

_NP = {"BF16": np.uint16, "F32": np.float32, "F16": np.float16, "F64": np.float64,
       "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8, "U64": np.uint64,
       "U32": np.uint32, "U16": np.uint16, "U8": np.uint8, "BOOL": np.bool_}


@dataclass
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    file_offset: int
    nbytes: int


def options(require_bf16=True, allow_f32=("e_score_correction_bias",), aligned_header=True,
            aligned_data=True) -> HfStOptions:
    """SafeTensorsOptions (model/safetensors.h:38-48)."""
    arr = (ctypes.c_char_p * max(1, len(allow_f32)))(*[s.encode() for s in allow_f32])
    o = HfStOptions(int(require_bf16), ctypes.cast(arr, ctypes.POINTER(ctypes.c_char_p)),
                    len(allow_f32), int(aligned_header), int(aligned_data))
    o._keep = arr  # the fragments must outlive the call
    return o


class SafeTensors:
    def __init__(self, path: str, opts: Optional[HfStOptions] = None):
        self.path = path
        self.stats = HfStStats()
        h = ctypes.c_void_p()
        call("hf_st_open", path.encode(), ctypes.byref(opts) if opts is not None else None,
             ctypes.byref(h), ctypes.byref(self.stats))
        self._h = h

    def stats_dict(self) -> Dict[str, int]:
        return {n: int(getattr(self.stats, n)) for n, _ in HfStStats._fields_}

    def __len__(self) -> int:
        return int(_lib.lib().hf_st_count(self._h))

    def info(self, i: int) -> TensorInfo:
        """Tensor i. Names are the header's bytes; bytes that are not UTF-8
        become surrogate escapes, so find(name) still matches them."""
        name, dtype = ctypes.c_char_p(), ctypes.c_char_p()
        nd = ctypes.c_int()
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        cap = 8
        while True:
            shape = (ctypes.c_int64 * cap)()
            call("hf_st_tensor", self._h, i, ctypes.byref(name), ctypes.byref(dtype),
                 ctypes.byref(nd), shape, cap, ctypes.byref(off), ctypes.byref(nb))
            if nd.value <= cap:
                break
            cap = nd.value  # more dimensions than the buffer: ask again with room for all
        return TensorInfo(name.value.decode("utf-8", "surrogateescape"),
                          dtype.value.decode("utf-8", "surrogateescape"),
                          tuple(shape[d] for d in range(nd.value)), off.value, nb.value)

    def tensors(self) -> List[TensorInfo]:
        return [self.info(i) for i in range(len(self))]

    def find(self, name: str) -> int:
        return int(_lib.lib().hf_st_find(self._h, name.encode("utf-8", "surrogateescape")))

    def read(self, name: str) -> np.ndarray:
        i = self.find(name)
        if i < 0:
            raise KeyError(name)
        t = self.info(i)
        out = np.empty(t.shape, _NP[t.dtype])
        call("hf_st_read", self._h, i, out.ctypes.data, out.nbytes)
        return out

    def upload(self, name: str, dst, device: int = 0):
        """Copies tensor `name` into device tensor `dst` (at least as many bytes)."""
        i = self.find(name)
        if i < 0:
            raise KeyError(name)
        nbytes = dst.numel() * dst.element_size()
        call("hf_st_upload", self._h, i, dst.data_ptr(), nbytes, device)
        return dst

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().hf_st_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def layer_shards(checkpoint_dir: str, model_layer: int) -> List[str]:
    """The shards of a checkpoint directory holding model layer `model_layer`'s
    MLP tensors (hf_st_layer_shards: the index's weight_map when present, else
    every *.safetensors file, sorted)."""
    n = ctypes.c_int()
    size = 1 << 16
    while True:
        buf = ctypes.create_string_buffer(size)
        st = _lib.lib().hf_st_layer_shards(checkpoint_dir.encode(), model_layer, buf, size,
                                           ctypes.byref(n))
        if st == _lib.HF_OK:
            break
        if n.value and size < (1 << 26):  # the buffer was too small: retry larger
            size *= 8
            continue
        _lib.check(st, "hf_st_layer_shards")
    parts = buf.raw.split(b"\0")[:n.value]
    return [p.decode() for p in parts]


def shard_paths_arg(paths: Sequence[str]):
    arr = (ctypes.c_char_p * len(paths))(*[p.encode() for p in paths])
    return arr


__all__ = ["SafeTensors", "TensorInfo", "options", "layer_shards", "shard_paths_arg"]
