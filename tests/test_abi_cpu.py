"""C-ABI checks that need no GPU: the library loads, exports every entry point
declared in include/*.h, and reports errors through statuses (no device here
means HF_ERR_UNSUPPORTED, never a silent fallback)."""
import ctypes
import os
import re

import pytest

from hummingflight_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("hf_moe.h", "hf_synth.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(hf_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 20
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # and the ctypes table covers them all
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_abi_version_and_status_strings():
    L = _lib.lib()
    assert L.hf_abi_version() == 1
    assert L.hf_status_string(_lib.HF_ERR_TIMEOUT) == b"HF_ERR_TIMEOUT"


def test_create_without_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    cfg = _lib.HfMoeConfig(64, 8, 2, 32, 32, 2.5, 1, 1, 4, 0, 0, 0, 0, 1, None)
    h = ctypes.c_void_p()
    st = _lib.lib().hf_moe_create(ctypes.byref(h), ctypes.byref(cfg))
    assert st == _lib.HF_ERR_UNSUPPORTED
    assert b"device" in _lib.lib().hf_last_error()


def test_create_rejects_bad_shapes_before_touching_a_device():
    L = _lib.lib()
    h = ctypes.c_void_p()
    for bad in [dict(hidden=60), dict(k=9), dict(k=0), dict(inter=30), dict(E=0), dict(layers=0)]:
        p = dict(hidden=64, E=8, k=2, inter=32, layers=1)
        p.update(bad)
        cfg = _lib.HfMoeConfig(p["hidden"], p["E"], p["k"], p["inter"], 32, 2.5, 1, p["layers"],
                               4, 0, 0, 0, 0, 1, None)
        assert L.hf_moe_create(ctypes.byref(h), ctypes.byref(cfg)) == _lib.HF_ERR_ARG, bad


def test_null_arguments_are_rejected():
    L = _lib.lib()
    assert L.hf_gemv_bf16_f32(None, None, None, 4, 4, 1.0, 0.0, None) == _lib.HF_ERR_ARG
    assert L.hf_topk_scores(None, 1, 8, None, 9, 1.0, 1, None, None, None) == _lib.HF_ERR_ARG
    assert L.hf_moe_forward(None, 0, None, 0, 1, None, None, None) == _lib.HF_ERR_ARG


def test_dense_mlp_arguments_checked_before_any_device_call():
    """hf_dense_mlp_forward validates shape, pointers, alignment and workspace
    size on the host; these cases return HF_ERR_ARG without touching CUDA (the
    pointers below are never dereferenced)."""
    L = _lib.lib()
    T, H, I = 4, 256, 384
    need = L.hf_dense_mlp_workspace_size(T, H, I)
    assert need > 0 and L.hf_dense_mlp_workspace_size(0, H, I) == 0
    assert L.hf_dense_mlp_workspace_size(2 * T, H, I) > need
    p, ws = 0x10000, 0x100000   # fake, aligned
    ok = [p, p, p, p, _lib.HF_BF16, T, H, I, p, ws, need, None]

    def call(**kw):
        a = list(ok)
        for k, v in kw.items():
            a[["gate", "up", "down", "x", "dt", "T", "H", "I", "out", "ws", "nb", "st"].index(k)] = v
        return L.hf_dense_mlp_forward(*a)

    assert call(T=-1) == _lib.HF_ERR_ARG
    assert call(up=None) == _lib.HF_ERR_ARG
    assert call(dt=7) == _lib.HF_ERR_ARG
    assert call(H=250) == _lib.HF_ERR_ARG          # not a multiple of 8
    assert call(x=p + 2) == _lib.HF_ERR_ARG        # not 16-byte aligned
    assert call(ws=ws + 16) == _lib.HF_ERR_ARG     # workspace not 256-byte aligned
    assert call(nb=need - 1) == _lib.HF_ERR_ARG    # workspace too small
    assert call(T=0) == _lib.HF_OK                 # nothing to do
    assert L.hf_dense_mlp_status(None, None) == _lib.HF_ERR_ARG


def test_block_and_rmsnorm_arguments_checked_before_any_device_call():
    """hf_dense_block_forward, hf_moe_block_forward and hf_rmsnorm validate on
    the host (the fake pointers below are never dereferenced)."""
    L = _lib.lib()
    T, H, I = 4, 256, 384
    need = L.hf_dense_mlp_workspace_size(T, H, I)
    p, q, ws = 0x10000, 0x20000, 0x100000
    ok = [p, p, p, p, 1e-5, _lib.HF_F32, p, q, T, H, I, ws, need, None]
    names = ["gate", "up", "down", "nw", "eps", "dt", "hin", "hout", "T", "H", "I", "ws", "nb",
             "st"]

    def dense(**kw):
        a = list(ok)
        for k, v in kw.items():
            a[names.index(k)] = v
        return L.hf_dense_block_forward(*a)

    assert dense(T=-1) == _lib.HF_ERR_ARG
    assert dense(hin=None) == _lib.HF_ERR_ARG
    assert dense(dt=7) == _lib.HF_ERR_ARG
    assert dense(nw=p + 8) == _lib.HF_ERR_ARG          # norm weight not 16-byte aligned
    assert dense(hout=p + 16) == _lib.HF_ERR_ARG       # overlaps hidden_in, not the same buffer
    assert dense(nb=need - 1) == _lib.HF_ERR_ARG
    assert dense(T=0) == _lib.HF_OK

    assert L.hf_moe_block_forward(None, 0, p, p, None, 1e-5, _lib.HF_F32, T, None,
                                  None) == _lib.HF_ERR_ARG
    assert L.hf_rmsnorm(p, None, 1e-5, T, 250, q, _lib.HF_F32, None) == _lib.HF_ERR_ARG
    assert L.hf_rmsnorm(None, None, 1e-5, T, H, q, _lib.HF_F32, None) == _lib.HF_ERR_ARG
    assert L.hf_rmsnorm(p, None, 1e-5, T, H, q, 7, None) == _lib.HF_ERR_ARG
    assert L.hf_rmsnorm(p + 4, None, 1e-5, T, H, q, _lib.HF_F32, None) == _lib.HF_ERR_ARG
    assert L.hf_rmsnorm(p, None, 1e-5, 0, H, q, _lib.HF_F32, None) == _lib.HF_OK


def test_route_noalloc_arguments_checked_before_any_device_call():
    """hf_moe_route_noalloc rejects sizes beyond its fixed in-library scratch
    (T <= 128, E <= 256, k <= 8) and bad arguments on the host, before it looks
    up the scratch array's device address (the fake pointers below are never
    dereferenced)."""
    L = _lib.lib()
    p = 0x10000
    names = ["router", "bias", "x", "dt", "T", "H", "E", "k", "scale", "norm", "shared",
             "ids", "w", "counts", "offsets", "perm", "st"]
    ok = [p, None, p, _lib.HF_BF16, 16, 256, 64, 8, 2.5, 1, 1, p, p, p, p, p, None]

    def call(**kw):
        a = list(ok)
        for k, v in kw.items():
            a[names.index(k)] = v
        return L.hf_moe_route_noalloc(*a)

    for bad in (dict(T=129), dict(T=-1), dict(E=257), dict(E=0)):
        assert call(**bad) == _lib.HF_ERR_ARG, bad
        assert b"static scratch" in L.hf_last_error(), bad
    assert call(k=9) == _lib.HF_ERR_ARG
    assert call(k=0) == _lib.HF_ERR_ARG
    assert call(H=60) == _lib.HF_ERR_ARG              # not a multiple of 8
    assert call(dt=7) == _lib.HF_ERR_ARG
    assert call(perm=None) == _lib.HF_ERR_ARG
    assert call(router=None) == _lib.HF_ERR_ARG
    assert call(x=p + 8) == _lib.HF_ERR_ARG           # not 16-byte aligned
