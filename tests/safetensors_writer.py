"""Writes safetensors files (tensors of numpy arrays), streaming each tensor's
bytes after the JSON header: 8-byte little-endian header length, the header
padded with spaces to a multiple of 8, tensor data 8-byte aligned -- the layout
the checkpoint loader's strict options require (model/safetensors.h:32-48).
Used to build checkpoints for the tests and for `bench.py --probe ingest`.
"""
from __future__ import annotations

import json
import struct
from typing import Iterable, Sequence, Tuple

import numpy as np

_SIZES = {"BF16": 2, "F16": 2, "F32": 4, "F64": 8, "I64": 8, "I32": 4, "I16": 2, "I8": 1,
          "U64": 8, "U32": 4, "U8": 1, "BOOL": 1}


def write_file(path: str, tensors: Iterable[Tuple[str, str, Sequence[int], np.ndarray]],
               metadata=None) -> None:
    """tensors: (name, dtype, shape, array) with array.nbytes == prod(shape) * size(dtype)."""
    tensors = list(tensors)
    hdr, off = {}, 0
    if metadata is not None:
        hdr["__metadata__"] = metadata
    for name, dtype, shape, arr in tensors:
        n = int(np.prod(shape)) * _SIZES[dtype]
        if arr.nbytes != n:
            raise ValueError(f"{name}: {arr.nbytes} bytes for shape {tuple(shape)} {dtype}")
        off += -off % 8
        hdr[name] = {"dtype": dtype, "shape": [int(s) for s in shape],
                     "data_offsets": [off, off + n]}
        off += n
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        pos = 0
        for name, dtype, shape, arr in tensors:
            pad = -pos % 8
            f.write(b"\0" * pad)
            pos += pad
            f.write(memoryview(np.ascontiguousarray(arr)).cast("B"))
            pos += arr.nbytes
