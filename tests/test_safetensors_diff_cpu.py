"""Differential test of the safetensors parser against the reference's own.

oracle/_ref/st_harness is the reference's SafeTensorsFile::open
(model/safetensors.cpp:52-223 with its vendored picojson), compiled unmodified
from the reference tree by `make -C oracle st`. This test mutates the parser
cases of tests/st_cases.py with a seeded generator -- bit flips, JSON
punctuation, truncations, repeated spans, rewritten header lengths, number
spellings picojson accepts or refuses ("08", "16.", "-.5", "1e2", "1e", ".5",
"+4", ...), string escapes (surrogate pairs, lone surrogates, bad \\u digits,
raw control and non-UTF-8 bytes), junk after the header -- and opens every mutant with both parsers
under the strict and the loose options. Both must agree on whether the file
opens, on every counter, and on every accepted tensor (name, dtype, shape,
absolute offset, byte size).

Two kinds of mutant are left out of the comparison, each counted:
* the reference process aborts (an uncaught std::length_error for a header
  length near 2^64, std::overflow_error from picojson for a number beyond the
  double range): our parser must then refuse the file;
* the header holds a number the reference converts with undefined behaviour
  (a shape entry at or past 2^31 through int(double), a data offset at or
  below -1 or at or past 2^64 through uint64_t(double)) and the two disagree:
  there the accepted tensors still agree and only the rejection counter that
  a tensor lands in can differ.

Needs the reference build (this test is skipped where oracle/_ref is absent).
No GPU.
"""
import json
import os
import random
import re
import struct
import subprocess

import pytest

from st_cases import cases

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "st_harness")

PUNCT = b'{}[]":,0123456789-.eE\\u \t\n'
NUMBERS = [b"08", b"16.", b"-.5", b"1e2", b"4.0", b"-0", b"0.5", b"16.9", b"1E1", b"007", b"2e-1",
           b"8.", b"-0.0", b"1.e1", b"0e0", b"24.99", b"1e+1", b"-", b"1e", b".5", b"+4", b"1-2",
           b"1..2", b"0x8", b"1e1e1"]
ESCAPES = [b"\\u00e9", b"\\ud83d\\ude00", b"\\ud83d", b"\\udc00", b"\\ud83dx", b"\\x", b"\\/",
           b"\\b", b"\\u12", b"\\uZZZZ", b"\x01", b"\x7f", b"\xc3\xa9", b"\xff", b'\\"', b"\\\\",
           b"\\u0000", b"\\ud800\\u0041"]
NUM = re.compile(rb"[0-9-][0-9+\-eE.]*")


def mutate(blob: bytes, rng: random.Random) -> bytes:
    b = bytearray(blob)
    for _ in range(1 + rng.randrange(4)):
        n = len(b)
        op = rng.randrange(8)
        if op == 0 and n:
            b[rng.randrange(n)] ^= 1 << rng.randrange(8)
        elif op == 1 and n:
            b[rng.randrange(n)] = PUNCT[rng.randrange(len(PUNCT))]
        elif op == 2 and n:
            del b[rng.randrange(n):]
        elif op == 3 and n >= 2:
            a = rng.randrange(n)
            span = b[a:a + 1 + rng.randrange(min(64, n - a))]
            at = rng.randrange(n)
            b[at:at] = span
        elif op == 4 and n >= 8:
            h = struct.unpack("<Q", bytes(b[:8]))[0]
            b[:8] = struct.pack("<Q", (h + rng.randrange(33) - 16) % 2**64)
        elif op == 5:
            b += bytes(rng.randrange(256) for _ in range(rng.randrange(16)))
        elif op == 6:
            digits = [i for i in range(8, n) if 48 <= b[i] <= 57]
            if digits:
                i = rng.choice(digits)
                b[i:i + 1] = rng.choice(NUMBERS)
        elif op == 7:
            quotes = [i for i in range(8, n) if b[i] == 0x22]
            if quotes:
                i = rng.choice(quotes) + 1
                b[i:i] = rng.choice(ESCAPES)
    return bytes(b)


def ub_territory(blob: bytes) -> bool:
    """True when the header holds a shape entry >= 2^31 or a data offset <= -1
    or >= 2^64 (found by key in the raw text)."""
    if len(blob) < 8:
        return False
    h = blob[8:8 + struct.unpack("<Q", blob[:8])[0]]
    for key, lo, hi in ((rb'"shape"', None, 2.0**31), (rb'"data_offsets"', -1.0, 2.0**64)):
        for m in re.finditer(key + rb"\s*:\s*\[([^\]]*)\]", h):
            for t in NUM.findall(m.group(1)):
                try:
                    v = float(t)
                except ValueError:
                    continue
                if v >= hi or (lo is not None and v <= lo):
                    return True
    return False


def ours(path, opts):
    from hummingflight_b200 import safetensors as S
    from hummingflight_b200._lib import HfError
    o = None if opts == "strict" else S.options(require_bf16=False, allow_f32=(),
                                                  aligned_header=False, aligned_data=False)
    try:
        f = S.SafeTensors(path, o)
    except HfError:
        return {"ok": False}
    r = {"ok": True, "stats": f.stats_dict(),
         "tensors": sorted((t.name, t.dtype, list(t.shape), t.file_offset, t.nbytes)
                           for t in f.tensors())}
    f.close()
    return r


def reference(path, opts):
    p = subprocess.run([HARNESS, path, opts], capture_output=True, timeout=60)
    out = p.stdout.decode("utf-8", "surrogateescape").strip()
    if p.returncode != 0 or not out:
        return {"abort": p.returncode}
    j = json.loads(out.splitlines()[-1])
    if not j["ok"]:
        return {"ok": False}
    # names come back through the C ABI as C strings: one holding \u0000 ends there
    return {"ok": True, "stats": j["stats"],
            "tensors": sorted((t["name"].split("\0")[0], t["dtype"], t["shape"], t["offset"],
                               t["bytes"]) for t in j["tensors"])}


@pytest.mark.parametrize("seed", [11, 12, 13])
def test_parser_agrees_with_reference_on_mutants(tmp_path, seed):
    if not os.path.exists(HARNESS):
        pytest.skip("the reference's parser is not built (oracle/_ref/st_harness)")
    rng = random.Random(seed)
    seeds = cases()
    path = str(tmp_path / "mutant.safetensors")
    n, opened, aborts, ub = 2000, 0, 0, 0
    bad = []
    for i in range(n):
        name, _opts, blob = seeds[rng.randrange(len(seeds))]
        m = mutate(blob, rng)
        with open(path, "wb") as f:
            f.write(m)
        for opts in ("strict", "loose"):
            a, b = ours(path, opts), reference(path, opts)
            opened += a["ok"]
            if "abort" in b:
                aborts += 1
                if a["ok"]:
                    bad.append((i, name, opts, "the reference aborts but ours opens the file"))
                continue
            if a == b:
                continue
            if ub_territory(m) and a["ok"] and b["ok"] and a["tensors"] == b["tensors"]:
                ub += 1
                continue
            bad.append((i, name, opts, a, b))
    assert not bad, bad[:3]
    assert opened > n // 2            # the mutants reach the accepting paths too
    assert aborts + ub < n // 20, (aborts, ub)
