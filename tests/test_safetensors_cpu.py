"""The safetensors parser of libhf_moe.so (include/hf_ingest.h) against the
reference's own parser (model/safetensors.cpp:52-223).

tests/golden/st_cases.json holds what the reference's SafeTensorsFile::open,
compiled unmodified (oracle/st_harness.cpp, tests/golden/make_st_golden.py),
accepted and counted on each file of tests/st_cases.py: valid files, every
rejection class (dtype, shape, offsets, bounds, alignment, byte span), header
errors, JSON escapes and metadata, duplicate keys, trailing text. Ours must
open the same files, accept the same tensors with the same dtypes, shapes,
offsets and sizes, and report the same counters. No GPU.
"""
import json
import os

import numpy as np
import pytest

from st_cases import cases, tensors_file

G = os.path.join(os.path.dirname(__file__), "golden")


def st():
    from hummingflight_b200 import safetensors as S
    return S


def open_case(tmp_path, name, opts, blob):
    from hummingflight_b200._lib import HfError
    S = st()
    p = tmp_path / (name + ".safetensors")
    p.write_bytes(blob)
    o = None if opts == "strict" else S.options(require_bf16=False, allow_f32=(),
                                                  aligned_header=False, aligned_data=False)
    try:
        return S.SafeTensors(str(p), o)
    except HfError:
        return None


@pytest.mark.parametrize("case", cases(), ids=lambda c: c[0])
def test_parser_matches_reference(tmp_path, case):
    name, opts, blob = case
    with open(os.path.join(G, "st_cases.json")) as f:
        want = json.load(f)[name]
    f = open_case(tmp_path, name, opts, blob)
    assert (f is not None) == want["ok"], name
    if f is None:
        return
    assert f.stats_dict() == want["stats"], name
    got = {t.name: t for t in f.tensors()}
    assert sorted(got) == sorted(t["name"] for t in want["tensors"])
    for t in want["tensors"]:
        g = got[t["name"]]
        assert (g.dtype, list(g.shape), g.file_offset, g.nbytes) == \
            (t["dtype"], t["shape"], t["offset"], t["bytes"]), t["name"]
    f.close()


def test_shape_product_past_64_bits_is_rejected(tmp_path):
    """A shape whose element count wraps 64 bits to a small number that matches
    the byte span (641 * 6700417 * 65535 * 65537 = 2^64 - 1, squared = 1 mod
    2^64, times 4 elements = the 8 bytes given) is rejected as a shape error.
    The reference's parser multiplies in size_t without this guard
    (safetensors.cpp:153-164, 208) and would accept it, so this case is not in
    the reference-generated golden set."""
    from st_cases import build, entry, header_text
    S = st()
    wrap = [641, 6700417, 65535, 65537] * 2 + [4]
    good = entry("ok.weight", "BF16", [4], [8, 16])
    bad = entry("wrapped.weight", "BF16", wrap, [0, 8])
    blob = build(header_text([bad, good]), bytes(16))
    f = open_case(tmp_path, "wrapped", "strict", blob)
    assert f is not None
    assert [t.name for t in f.tensors()] == ["ok.weight"]
    assert f.stats_dict()["shape_rejected"] == 1
    f.close()


def test_read_returns_the_file_bytes(tmp_path):
    S = st()
    rng = np.random.default_rng(9)
    w = rng.integers(0, 1 << 16, (6, 10), dtype=np.uint16)
    b = rng.standard_normal(6).astype(np.float32)
    blob = tensors_file([("model.layers.0.mlp.gate.weight", "BF16", w.shape, w.tobytes()),
                         ("model.layers.0.mlp.gate.e_score_correction_bias", "F32", b.shape,
                          b.tobytes())])
    p = tmp_path / "x.safetensors"
    p.write_bytes(blob)
    with S.SafeTensors(str(p)) as f:
        assert len(f) == 2
        assert np.array_equal(f.read("model.layers.0.mlp.gate.weight"), w)
        assert np.array_equal(f.read("model.layers.0.mlp.gate.e_score_correction_bias"), b)
        assert f.find("missing") == -1
        with pytest.raises(KeyError):
            f.read("missing")


def test_open_missing_file_fails():
    from hummingflight_b200._lib import HfError
    with pytest.raises(HfError):
        st().SafeTensors("/nonexistent/x.safetensors")


def test_package_writer_round_trip(tmp_path):
    """tests/safetensors_writer.py output passes the strict checks."""
    from safetensors_writer import write_file
    S = st()
    rng = np.random.default_rng(11)
    a = rng.integers(0, 1 << 16, (5, 7), dtype=np.uint16)      # 70 bytes: the next start pads
    b = rng.standard_normal(3).astype(np.float32)
    c = rng.integers(0, 1 << 16, (2, 2, 2), dtype=np.uint16)
    p = tmp_path / "w.safetensors"
    write_file(str(p), [("a.weight", "BF16", a.shape, a),
                        ("b.e_score_correction_bias", "F32", b.shape, b),
                        ("c.weight", "BF16", c.shape, c)], metadata={"format": "pt"})
    with S.SafeTensors(str(p)) as f:
        assert f.stats_dict()["accepted"] == 3 and f.stats_dict()["rejected"] == 0
        assert all(t.file_offset % 8 == 0 for t in f.tensors())
        assert np.array_equal(f.read("a.weight"), a)
        assert np.array_equal(f.read("b.e_score_correction_bias"), b)
        assert np.array_equal(f.read("c.weight"), c)
    with pytest.raises(ValueError):
        write_file(str(tmp_path / "bad.safetensors"), [("x", "BF16", (3,), a)])


def test_layer_shards_follow_the_index(tmp_path):
    """hf_st_layer_shards: every *.safetensors file (sorted) without an index;
    with model.safetensors.index.json only the shards its weight_map names for
    model.layers.<L>.mlp.* (WeightIndex::build, weight_index.cpp:79-130)."""
    import json as js
    from hummingflight_b200._lib import HfError
    S = st()
    for n in ("model-00002-of-00003.safetensors", "model-00001-of-00003.safetensors",
              "model-00003-of-00003.safetensors", "notes.txt"):
        (tmp_path / n).write_bytes(b"")
    all3 = [str(tmp_path / f"model-0000{i}-of-00003.safetensors") for i in (1, 2, 3)]
    assert S.layer_shards(str(tmp_path), 3) == all3
    import ctypes
    from hummingflight_b200 import _lib
    n = ctypes.c_int()
    small = ctypes.create_string_buffer(8)
    assert _lib.lib().hf_st_layer_shards(str(tmp_path).encode(), 3, small, 8,
                                         ctypes.byref(n)) == _lib.HF_ERR_ARG
    assert n.value == 3                               # the count even when the buffer is short
    wm = {"model.layers.3.mlp.gate.weight": "model-00002-of-00003.safetensors",
          "model.layers.3.mlp.experts.0.up_proj.weight": "model-00003-of-00003.safetensors",
          "model.layers.3.mlp.experts.1.up_proj.weight": "model-00002-of-00003.safetensors",
          "model.layers.3.self_attn.o_proj.weight": "model-00001-of-00003.safetensors",
          "model.layers.30.mlp.gate.weight": "model-00001-of-00003.safetensors"}
    idx = tmp_path / "model.safetensors.index.json"
    idx.write_text(js.dumps({"metadata": {"total_size": 1}, "weight_map": wm}))
    assert S.layer_shards(str(tmp_path), 3) == all3[1:]
    assert S.layer_shards(str(tmp_path), 30) == all3[:1]
    with pytest.raises(HfError, match="names no tensor of model.layers.7.mlp"):
        S.layer_shards(str(tmp_path), 7)              # a wrong layer number is an error
    wm["model.layers.7.mlp.gate.weight"] = "model-00009-of-00009.safetensors"
    idx.write_text(js.dumps({"weight_map": wm}))
    with pytest.raises(HfError, match="missing shard"):
        S.layer_shards(str(tmp_path), 7)
    idx.write_text("{not json")                      # unreadable index: every shard
    assert S.layer_shards(str(tmp_path), 3) == all3
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(HfError, match="no .safetensors"):
        S.layer_shards(str(empty), 3)
