"""Builds hummingflight_b200/libhf_moe.so for sm_100a (B200) with nvcc.

Every CUDA source under csrc/ is compiled to an object in _build/ (skipped
when up to date), then linked into one shared library next to this file.
Run ``python -m hummingflight_b200.build [-v]``; ``-v`` adds ``-Xptxas -v``
(registers, spills, shared memory per kernel).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libhf_moe.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _flags(ptxas_verbose: bool) -> list:
    f = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC, "--expt-relaxed-constexpr"] + ARCH
    if ptxas_verbose:
        f += ["-Xptxas", "-v"]
    return f


def _deps() -> list:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, sources: list) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = _deps()
    cc = nvcc()
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or verbose or _stale(o, [s] + deps):
            jobs.append([cc] + _flags(verbose) + ["-c", s, "-o", o])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError("nvcc failed on: " + ", ".join(failed))
    if force or jobs or _stale(LIB, objs):
        cmd = [cc, "-shared"] + ARCH + ["-o", LIB] + objs + ["-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(verbose=v, force="-f" in sys.argv))
