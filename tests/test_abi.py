"""The C-ABI library loads and exports every entry point include/fme.h declares; host-side argument checks
that need no GPU (CPU only)."""
import ctypes
import os
import re

import numpy as np
import pytest
from conftest import ROOT, fme

from fast_mario_env_b200 import _native as N


def declared_functions():
    src = open(os.path.join(ROOT, "include", "fme.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fme_[a-z_0-9]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(N.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = N.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert b"sm_100a" in L.fme_version()


def test_palette_and_gray_lut_match_oracle(oracle):
    assert np.array_equal(fme.palette_rgb(), oracle.palette_rgb())
    assert np.array_equal(fme.gray_lut(), oracle.gray_lut())


def test_create_rejects_bad_arguments_before_touching_a_device(rom):
    L = N.lib()
    n = 2
    lv = np.array([1, 1, 1] * n, np.int32)
    lut = fme.gray_lut()
    rng = np.zeros(6 * n, np.uint64)
    h = ctypes.c_void_p()
    romb = np.frombuffer(rom, np.uint8).copy()
    cfg = N.FmeConfig(n_envs=n, skip=0, max_steps=10, noop_max=0, maxpool=0, frame_stack=4, sticky=0.0, device=0)
    assert L.fme_create(ctypes.byref(cfg), N.ptr(romb), len(romb), N.ptr(lv), N.ptr(lut), N.ptr(rng), ctypes.byref(h)) == -1
    assert "skip" in N.last_error()
    cfg.skip = 4
    bad = np.frombuffer(b"NES\x1a" + bytes([2, 1, 0x10, 0]) + bytes(8) + rom[16:], np.uint8).copy()  # mapper 1
    assert L.fme_create(ctypes.byref(cfg), N.ptr(bad), len(bad), N.ptr(lv), N.ptr(lut), N.ptr(rng), ctypes.byref(h)) == -2
    short = romb[:1000].copy()
    assert L.fme_create(ctypes.byref(cfg), N.ptr(short), len(short), N.ptr(lv), N.ptr(lut), N.ptr(rng), ctypes.byref(h)) == -2
    cfg.frame_stack = 0
    assert L.fme_create(ctypes.byref(cfg), N.ptr(romb), len(romb), N.ptr(lv), N.ptr(lut), N.ptr(rng), ctypes.byref(h)) == -1
    assert L.fme_create(None, N.ptr(romb), len(romb), N.ptr(lv), N.ptr(lut), N.ptr(rng), ctypes.byref(h)) == -1
    assert not h.value


def test_rng_state_matches_numpy():
    for seed in (0, 7, 1000 * 3 + 5):
        w = fme.rng_state(seed)
        st = np.random.default_rng(seed).bit_generator.state
        assert (w[0] << 64 | w[1]) == st["state"]["state"] and (w[2] << 64 | w[3]) == st["state"]["inc"]
        assert w[4] == st["has_uint32"] and w[5] == st["uinteger"]


def test_python_api_validates_before_device(rom):
    with pytest.raises(ValueError):
        fme.CudaVecEnv("1-1", 2, skip=0, rom=rom)
    with pytest.raises(ValueError):
        fme.CudaVecEnv("1-1", 2, frame_stack=0, rom=rom)
    with pytest.raises(ValueError):
        fme.CudaVecEnv("1-1", 2, device="cpu", rom=rom)
