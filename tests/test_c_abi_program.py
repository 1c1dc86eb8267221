"""The layer from plain C++ through the C ABI (tests/c_abi_program.cpp): no
PyTorch and no CUDA headers in the caller, host buffers, weights set from the
checkpoint's per-projection tensors, the per-token moeLayer drop-in and the
batched host entry checked against the oracle at the north-star bars.

Built here with g++ against include/ and linked with libhf_moe.so and
oracle/liboracle.so. On a machine without a GPU the program must fail loudly
(HF_ERR_UNSUPPORTED from hf_moe_create: there is no CPU fallback); on a GPU it
must pass.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def build(tmp_path):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("g++ not available")
    lib_dir = os.path.join(ROOT, "hummingflight_b200")
    oracle_dir = os.path.join(ROOT, "oracle")
    for f in (os.path.join(lib_dir, "libhf_moe.so"), os.path.join(oracle_dir, "liboracle.so")):
        if not os.path.exists(f):
            pytest.skip(f"{f} is not built")
    exe = str(tmp_path / "c_abi_program")
    cmd = [gxx, "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I", oracle_dir,
           os.path.join(HERE, "c_abi_program.cpp"), "-o", exe, "-L", lib_dir, "-lhf_moe",
           "-L", oracle_dir, "-loracle", f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{oracle_dir}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def test_c_abi_program_builds_and_fails_loudly_without_a_device(tmp_path):
    exe = build(tmp_path)
    if has_gpu():
        pytest.skip("a GPU is present (the gpu test runs the program)")
    p = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert p.returncode != 0
    assert "HF_ERR_UNSUPPORTED" in p.stdout or "HF_ERR_CUDA" in p.stdout, p.stdout


@pytest.mark.gpu
def test_c_abi_program_matches_oracle(tmp_path):
    if not has_gpu():
        pytest.skip("no CUDA device")
    exe = build(tmp_path)
    p = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0 and p.stdout.startswith("OK"), p.stdout + p.stderr
