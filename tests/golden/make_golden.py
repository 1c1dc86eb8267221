"""Regenerate tests/golden/ from the reference's own code.

Needs the reference source tree (``--ref``, default from $HF_REFERENCE_SRC) and
is run by hand, never by the tests. It

1. compiles tests/golden/ref_kat.cpp against the reference's unmodified
   compute/cpu_kernels.cpp twice (the Linux scalar build and the AVX2 build the
   reference only enables under _MSC_VER) into oracle/_ref/, runs both and
   stores ref_kat_{scalar,avx2}.json: the inputs and outputs of the reference's
   own self-tests (src/self_test.cpp:73-103, :180-200) and of its expert-FFN
   parity case (compute/cuda_backend.cpp:497-520);
2. runs the reference's GLMForward::moeLayer math (oracle/_ref, see
   oracle/ref_harness.cpp) on seeded layers of several shapes and stores
   ids / weights / outputs / per-slot expert outputs as moe_*.npz.

Usage: python tests/golden/make_golden.py [--ref PATH]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from hummingflight_b200.configs import GLM, WORKLOADS, zipf_bias  # noqa: E402

# (name, dims, weight seed, x seed, T, bias) -- small shapes cover the edge
# cases (no shared expert, k > E, shared inter != routed inter, skewed bias).
SMALL = [
    ("moe_small", O.Dims(64, 16, 4, 32, 32), 7, 8, 8, None),
    ("moe_mid", O.Dims(512, 64, 8, 128, 256), 11, 12, 32, None),
    ("moe_noshared", O.Dims(64, 8, 2, 32, 0), 13, 14, 5, None),
    ("moe_k_gt_e", O.Dims(32, 4, 8, 16, 16), 15, 16, 3, None),
    ("moe_zipf", O.Dims(256, 64, 8, 64, 64), 17, 18, 64, "zipf"),
]


def build_kat(ref: str) -> None:
    out_dir = os.path.join(ROOT, "oracle", "_ref")
    os.makedirs(out_dir, exist_ok=True)
    src = os.path.join(ref, "src", "compute", "cpu_kernels.cpp")
    for flavour, extra in (("scalar", []), ("avx2", ["-mavx2", "-mfma", "-D_MSC_VER=1930"])):
        exe = os.path.join(out_dir, f"ref_kat_{flavour}")
        obj = os.path.join(out_dir, f"ref_kat_cpu_kernels_{flavour}.o")
        base = ["g++", "-O3", "-std=c++20", "-fopenmp", "-w", f"-I{ref}/src"]
        subprocess.check_call(base + extra + ["-c", src, "-o", obj])
        subprocess.check_call(base + [os.path.join(HERE, "ref_kat.cpp"), obj, "-o", exe])
        txt = subprocess.check_output([exe]).decode()
        json.loads(txt)  # validate
        with open(os.path.join(HERE, f"ref_kat_{flavour}.json"), "w") as f:
            f.write(txt)


def small_fixture(name, d, wseed, xseed, T, bias_kind) -> None:
    x = O.bf16_to_f32(O.gen_x_bf16(xseed, T, d.hidden))
    bias = zipf_bias(d.num_experts, wseed) if bias_kind == "zipf" else None
    res = {}
    for flavour in ("scalar", "avx2"):
        R = O.RefLayer(d, wseed, 0, bias=bias, flavour=flavour)
        r = R.forward(x, want_slots=True)
        R.close()
        res[flavour] = r
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        dims=np.array([d.hidden, d.num_experts, d.top_k, d.inter, d.shared_inter], np.int32),
        scale=np.float32(d.scale), wseed=np.int64(wseed), xseed=np.int64(xseed),
        bias=(bias if bias is not None else np.zeros(0, np.float32)),
        ids=res["scalar"]["ids"], w=res["scalar"]["w"], out=res["scalar"]["out"],
        slots=res["scalar"]["slots"], out_avx2=res["avx2"]["out"], ids_avx2=res["avx2"]["ids"])


def glm_fixture(name, cfg, ntok) -> None:
    wl = WORKLOADS[cfg]
    s = GLM
    d = O.Dims(s.hidden, s.num_experts, s.top_k, s.inter, s.shared_inter, s.scale, s.norm_topk)
    x = O.bf16_to_f32(O.gen_x_bf16(wl.x_seed, wl.tokens, s.hidden))[:ntok]
    res = {}
    for flavour in ("scalar", "avx2"):
        R = O.RefLayer(d, wl.weight_seeds[0], 0, flavour=flavour)
        R.prepare(x)
        res[flavour] = R.forward(x, want_slots=(flavour == "scalar"))
        R.close()
    o = O.moe_layer_synth(d, wl.weight_seeds[0], 0, x)
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"), config=np.int32(cfg), tokens=np.int32(ntok),
        ids=res["scalar"]["ids"], w=res["scalar"]["w"], out=res["scalar"]["out"],
        slots=res["scalar"]["slots"], out_avx2=res["avx2"]["out"], margins=o["margins"])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HF_REFERENCE_SRC", ""))
    a = ap.parse_args()
    if not a.ref or not os.path.isdir(os.path.join(a.ref, "src", "compute")):
        sys.exit("reference source tree not found (pass --ref)")
    subprocess.check_call(["make", "-C", os.path.join(ROOT, "oracle"), "all", "ref",
                           f"REF={a.ref}"])
    build_kat(a.ref)
    for spec in SMALL:
        small_fixture(*spec)
    glm_fixture("moe_cfg0", 0, 1)
    glm_fixture("moe_cfg1_head", 1, 2)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
