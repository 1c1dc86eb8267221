"""Golden results of the reference's own safetensors parser on tests/st_cases.py.

Builds oracle/_ref/st_harness (the reference's model/safetensors.cpp, compiled
unmodified, with oracle/st_harness.cpp), writes every case file to a temporary
directory, runs the harness on it and stores the results in
tests/golden/st_cases.json. Run by hand with the reference tree present:

    python tests/golden/make_st_golden.py [--ref PATH]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from st_cases import cases  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HF_REFERENCE_SRC", ""))
    a = ap.parse_args()
    if not a.ref:
        raise SystemExit("--ref <reference source tree> is required")
    subprocess.check_call(["make", "-C", os.path.join(ROOT, "oracle"), "st", f"REF={a.ref}"])
    exe = os.path.join(ROOT, "oracle", "_ref", "st_harness")
    res = {}
    with tempfile.TemporaryDirectory() as td:
        for name, opts, blob in cases():
            p = os.path.join(td, name + ".safetensors")
            with open(p, "wb") as f:
                f.write(blob)
            res[name] = json.loads(subprocess.check_output([exe, p, opts]).decode())
    with open(os.path.join(HERE, "st_cases.json"), "w") as f:
        json.dump(res, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
