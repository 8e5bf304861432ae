"""TEST ORACLE ONLY. ctypes access to the plain-C restatement (oracle/fme_oracle.c -> oracle/_ref/libfme_oracle.so).
Same call shapes as oracle/ref.py so tests can run either; only tests/ and bench.py's CPU-baseline leg use it."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from ref import gray_lut, rng_state  # noqa: F401  (same seeding / LUT helpers)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libfme_oracle.so")
_P = ctypes.c_void_p
_lib = None


def available() -> bool:
    return os.path.isfile(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB_PATH)
        i64, i32, dbl = ctypes.c_int64, ctypes.c_int, ctypes.c_double
        L.orc_create.restype = _P
        L.orc_create.argtypes = [_P, i64, i32, _P, _P, i32, i32, dbl, i32, i32, i32, _P, i32]
        L.orc_reset.argtypes = [_P, _P]
        L.orc_step.argtypes = [_P] * 10
        L.orc_ram.argtypes = [_P, i32, _P]
        L.orc_frames.restype = L.orc_bad_ops.restype = i64
        L.orc_frames.argtypes = L.orc_bad_ops.argtypes = [_P]
        L.orc_destroy.argtypes = [_P]
        L.orc_resize.argtypes = [_P, _P]
        L.orc_raw_create.restype = _P
        L.orc_raw_create.argtypes = [_P, i64]
        L.orc_raw_frame.argtypes = [_P, i32, i32]
        L.orc_raw_ram.restype = L.orc_raw_screen.restype = _P
        L.orc_raw_ram.argtypes = L.orc_raw_screen.argtypes = [_P]
        L.orc_raw_backup.argtypes = L.orc_raw_restore.argtypes = L.orc_raw_destroy.argtypes = [_P]
        L.orc_raw_bad_ops.restype = i64
        L.orc_raw_bad_ops.argtypes = [_P]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(_P)


def resize(img):
    out = np.zeros((84, 84), np.uint8)
    lib().orc_resize(_ptr(np.ascontiguousarray(img, np.uint8)), _ptr(out))
    return out


class PortRaw:
    def __init__(self, rom: bytes):
        L = lib()
        self._rom = np.frombuffer(rom, np.uint8).copy()
        self.h = L.orc_raw_create(_ptr(self._rom), len(self._rom))
        if not self.h:
            raise ValueError("ROM rejected")
        u8p = ctypes.POINTER(ctypes.c_uint8)
        self.ram = np.ctypeslib.as_array(ctypes.cast(L.orc_raw_ram(self.h), u8p), (0x800,))
        self.screen = np.ctypeslib.as_array(ctypes.cast(L.orc_raw_screen(self.h), u8p), (240, 256))

    def frame(self, buttons, render=True):
        lib().orc_raw_frame(self.h, int(buttons), int(bool(render)))

    def backup(self):
        lib().orc_raw_backup(self.h)

    def restore(self):
        lib().orc_raw_restore(self.h)

    def bad_ops(self):
        return int(lib().orc_raw_bad_ops(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_raw_destroy(self.h)
            self.h = None


class PortVecEnv:
    """Sequential restatement of the reference FastVecEnv (same constructor shape as ref.RefVecEnv)."""

    def __init__(self, rom: bytes, levels, n: int, seed=0, skip=4, max_steps=2000, sticky=0.0, noop_max=0,
                 maxpool=False, frame_stack=4, env_offset=0, boot_cap=20000, **_):
        L = lib()
        self.n, self.k = n, frame_stack
        self._lv = np.array([tuple(levels)] * n if isinstance(levels[0], int) else list(levels), np.int32).reshape(-1)
        self._rng = np.array([rng_state(seed * 1000 + env_offset + i) for i in range(n)], np.uint64).reshape(-1)
        self._rom = np.frombuffer(rom, np.uint8).copy()
        self._lut = gray_lut()
        self.h = L.orc_create(_ptr(self._rom), len(self._rom), n, _ptr(self._lv), _ptr(self._lut), skip, max_steps,
                              float(sticky), int(noop_max), int(bool(maxpool)), frame_stack, _ptr(self._rng), boot_cap)
        if not self.h:
            raise RuntimeError("orc_create failed")
        self.obs = np.zeros((n, frame_stack, 84, 84), np.uint8)
        self.fin = np.zeros_like(self.obs)
        self.rew = np.zeros(n, np.float32)
        self.term = np.zeros(n, np.uint8)
        self.trunc = np.zeros(n, np.uint8)
        self.info = np.zeros((n, 10), np.int64)
        self.ep_ret = np.zeros(n, np.float64)
        self.ep_len = np.zeros(n, np.int64)

    def reset(self):
        lib().orc_reset(self.h, _ptr(self.obs))
        return self.obs

    def step(self, actions):
        a = np.ascontiguousarray(np.asarray(actions).reshape(-1), np.int64)
        lib().orc_step(self.h, _ptr(a), _ptr(self.obs), _ptr(self.fin), _ptr(self.rew), _ptr(self.term), _ptr(self.trunc),
                       _ptr(self.info), _ptr(self.ep_ret), _ptr(self.ep_len))
        return self.obs, self.rew, self.term.astype(bool), self.trunc.astype(bool), self.info

    def ram(self, i):
        out = np.zeros(0x800, np.uint8)
        lib().orc_ram(self.h, int(i), _ptr(out))
        return out

    @property
    def frames(self):
        return int(lib().orc_frames(self.h))

    def bad_ops(self):
        return int(lib().orc_bad_ops(self.h))

    def close(self):
        if self.h:
            lib().orc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
