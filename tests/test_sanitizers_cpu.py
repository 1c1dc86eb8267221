"""The library's host code under AddressSanitizer and UndefinedBehaviorSanitizer.

Every CUDA source is compiled again with the sanitizers on its host side (its
device side only as PTX, which nothing here runs) and linked with
tests/host_fuzz.cpp: the safetensors parser on the reference-pinned parser
cases of tests/st_cases.py and on seeded mutations of them, hf_st_layer_shards
on mutated checkpoint indexes, and the expert-parallel planners
(hf_ep_balanced_placement, hf_ep_plan) on random loads and counts with their
invariants checked. Checkpoint files are untrusted input, so the parser must
reject anything malformed without reading or writing out of bounds. No GPU:
none of these paths touches a device.
"""
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "hummingflight_b200", "csrc")
SAN = ["-fsanitize=address", "-fsanitize=undefined", "-fno-omit-frame-pointer"]
PTX_ONLY = ["-gencode", "arch=compute_100a,code=compute_100a"]


@pytest.fixture(scope="module")
def host_fuzz(tmp_path_factory):
    from hummingflight_b200.build import nvcc
    gxx = shutil.which("g++")
    try:
        cc = nvcc()
    except RuntimeError:
        pytest.skip("nvcc not available")
    if not gxx:
        pytest.skip("g++ not available")
    d = tmp_path_factory.mktemp("san")
    host = [a for f in SAN for a in ("-Xcompiler", f)]
    jobs = []
    for s in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        o = str(d / (os.path.basename(s)[:-3] + ".o"))
        jobs.append((o, [cc, "-O1", "-g", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                         "-I", CSRC, "--expt-relaxed-constexpr"] + host + PTX_ONLY +
                     ["-c", s, "-o", o]))
    main_o = str(d / "host_fuzz.o")
    jobs.append((main_o, [gxx, "-std=c++17", "-O1", "-g", "-Wall", "-I", os.path.join(ROOT, "include")]
                 + SAN + ["-c", os.path.join(HERE, "host_fuzz.cpp"), "-o", main_o]))
    with cf.ThreadPoolExecutor(max_workers=8) as ex:
        for r in ex.map(lambda j: subprocess.run(j[1], capture_output=True, text=True), jobs):
            assert r.returncode == 0, r.stdout + r.stderr
    exe = str(d / "host_fuzz")
    r = subprocess.run([cc] + PTX_ONLY + host + [o for o, _ in jobs] + ["-o", exe],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return exe


@pytest.mark.parametrize("seed", [1, 2])
def test_host_code_under_sanitizers(host_fuzz, tmp_path, seed):
    from st_cases import cases
    corpus = tmp_path / "corpus"
    scratch = tmp_path / "scratch"
    corpus.mkdir()
    scratch.mkdir()
    for name, _opts, blob in cases():
        (corpus / (name + ".safetensors")).write_bytes(blob)
    env = dict(os.environ, ASAN_OPTIONS="halt_on_error=1:detect_leaks=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    p = subprocess.run([host_fuzz, str(corpus), str(scratch), "20000", str(seed)],
                       capture_output=True, text=True, timeout=600, env=env)
    assert p.returncode == 0 and p.stdout.startswith("OK"), p.stdout + p.stderr[-4000:]
    assert "runtime error" not in p.stderr, p.stderr[-4000:]
