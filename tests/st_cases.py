"""Safetensors test files: a small writer and the parser cases shared by
tests/test_safetensors_cpu.py and tests/golden/make_st_golden.py.

Each case is (name, options, bytes): `options` is "strict" (the checkpoint
loader's SafeTensorsOptions, weight_index.cpp:20-27) or "loose" (no dtype or
alignment requirement). The files are built deterministically, so the golden
results the reference's own parser produced for them (tests/golden/
st_cases.json) stay valid.
"""
from __future__ import annotations

import json
import struct
from typing import List, Optional, Sequence, Tuple

import numpy as np

Entry = Tuple[str, str]   # (JSON-encoded key, JSON text of the value)


def entry(name: str, dtype=None, shape=None, offsets=None, raw: Optional[str] = None,
          key: Optional[str] = None) -> Entry:
    """One header entry; fields left as None are omitted, `raw` replaces the value."""
    if raw is None:
        d = {}
        if dtype is not None:
            d["dtype"] = dtype
        if shape is not None:
            d["shape"] = shape
        if offsets is not None:
            d["data_offsets"] = offsets
        raw = json.dumps(d)
    return (key if key is not None else json.dumps(name), raw)


def header_text(entries: Sequence[Entry], metadata: Optional[dict] = None) -> str:
    items = []
    if metadata is not None:
        items.append('"__metadata__": ' + json.dumps(metadata))
    items += [f"{k}: {v}" for k, v in entries]
    return "{" + ", ".join(items) + "}"


def build(header: str, data: bytes, pad: int = 8, hlen: Optional[int] = None) -> bytes:
    h = header.encode()
    if pad:
        h += b" " * (-len(h) % pad)
    return struct.pack("<Q", len(h) if hlen is None else hlen) + h + data


def tensors_file(tensors: Sequence[Tuple[str, str, Sequence[int], bytes]],
                 metadata: Optional[dict] = None) -> bytes:
    """A valid file: tensors packed in order, each start 8-byte aligned."""
    ents, data = [], b""
    for name, dtype, shape, raw in tensors:
        data += b"\0" * (-len(data) % 8)
        ents.append(entry(name, dtype, list(shape), [len(data), len(data) + len(raw)]))
        data += raw
    return build(header_text(ents, metadata), data)


def _bytes(n: int, seed: int) -> bytes:
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


def cases() -> List[Tuple[str, str, bytes]]:
    out = []
    bias = "model.layers.3.mlp.gate.e_score_correction_bias"
    valid = tensors_file([
        ("model.layers.3.mlp.gate.weight", "BF16", [4, 8], _bytes(64, 1)),
        (bias, "F32", [4], _bytes(16, 2)),
        ("model.layers.3.mlp.experts.0.gate_proj.weight", "BF16", [2, 3], _bytes(12, 3)),
    ], metadata={"format": "pt"})
    out += [("valid", "strict", valid), ("valid_loose", "loose", valid)]

    d = _bytes(256, 4)
    dt = [entry("a.bf16", "BF16", [4], [0, 8]), entry("b.f16", "F16", [4], [8, 16]),
          entry("c.f32", "F32", [2], [16, 24]), entry("d.q4", "Q4", [8], [24, 32]),
          entry("e.e_score_correction_bias", "F32", [2], [32, 40]),
          entry("f.nodtype", None, [4], [40, 48]), entry("g.i64", "I64", [1], [48, 56]),
          entry("h.u16", "U16", [4], [56, 64])]
    out += [("dtype", "strict", build(header_text(dt), d)),
            ("dtype_loose", "loose", build(header_text(dt), d))]

    sh = [entry("ok", "BF16", [4], [0, 8]), entry("empty", "BF16", [], [8, 16]),
          entry("neg", "BF16", [-4], [16, 24]), entry("frac", "BF16", [2.5], [24, 32]),
          entry("intfloat", "BF16", [4.0], [32, 40]), entry("str", "BF16", ["4"], [40, 48]),
          entry("huge", "BF16", [(1 << 30) + 1, 1], [48, 56]), entry("noshape", "BF16", None, [56, 64]),
          entry("notobj", raw="5"), entry("nine_dims", "BF16", [1] * 8 + [4], [64, 72]),
          entry("negzero", "BF16", [4], [72, 80], raw=None)]
    sh[-1] = ("\"negzero\"", '{"dtype": "BF16", "shape": [-0, 4], "data_offsets": [80, 80]}')
    out.append(("shape", "strict", build(header_text(sh), d)))

    of = [entry("ok", "BF16", [4], [0, 8]), entry("empty", "BF16", [4], [8, 8]),
          entry("reversed", "BF16", [4], [24, 16]), entry("one", "BF16", [4], [8]),
          entry("none", "BF16", [4], None), entry("past_end", "BF16", [4], [250, 258]),
          entry("float_offsets", "BF16", [4], [16.0, 24.0]),
          entry("str_offsets", "BF16", [4], ["24", "32"])]
    out.append(("offsets", "strict", build(header_text(of), d)))

    al = [entry("aligned", "BF16", [4], [0, 8]), entry("odd", "BF16", [4], [10, 18]),
          entry("mismatch", "BF16", [4, 4], [24, 40]), entry("short", "BF16", [4], [40, 44])]
    out += [("align_bytes", "strict", build(header_text(al), d)),
            ("align_bytes_loose", "loose", build(header_text(al), d))]

    dup = [entry("t", "BF16", [4], [0, 8]), entry("t", "BF16", [4], [8, 16])]
    out.append(("duplicate", "strict", build(header_text(dup), d)))

    good = header_text([entry("t", "BF16", [4], [0, 8])])
    out += [("header_unaligned", "strict", build(good, d, pad=0)),
            ("header_unaligned_loose", "loose", build(good, d, pad=0)),
            ("header_past_end", "strict", build(good, d[:8], hlen=4096)),
            ("no_data_after_header", "strict", build(header_text([]), b"")),
            ("bad_json", "strict", build('{"t": {"dtype": "BF16",', d)),
            ("not_object", "strict", build("[1, 2, 3]", d)),
            ("empty_object", "strict", build("{}", d)),
            ("trailing_text", "strict", build(good + " x", d))]

    esc = [entry("café.weight", "BF16", [4], [0, 8]),
           entry("quote\"d", "BF16", [4], [8, 16]),
           entry("_private", "BF16", [4], [16, 24])]
    meta = {"format": "pt", "nested": {"a": [1, 2, {"b": None}], "t": True}}
    out.append(("escapes_metadata", "strict", build(header_text(esc, meta), d)))
    return out
