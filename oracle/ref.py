"""TEST ORACLE ONLY. ctypes access to the reference's own C++ core, built from its sources by oracle/Makefile
into oracle/_ref/libfastmario.so. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module; the product never imports it.

The C ABI bound here is the reference's `extern "C"` block (csrc/fastmario.cpp:562-674); the argument lists
follow its ctypes declarations (src/fast_mario_env/_native.py:35-58). Seeding follows env.py:50-55
(`rng_state`) and env.py:155-156 (`seed*1000 + env_offset + i`).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libfastmario.so")
INFO_FIELDS = ("x_pos", "flag_get", "life", "score", "time", "world", "stage", "coins", "y_pos", "status")
_P = ctypes.c_void_p
_lib = None


def available() -> bool:
    return os.path.isfile(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"reference oracle not built: {LIB_PATH} (run `make -C oracle ref`)")
        L = ctypes.CDLL(LIB_PATH)
        i64, i32, dbl = ctypes.c_int64, ctypes.c_int, ctypes.c_double
        L.fm_create.restype = _P
        L.fm_create.argtypes = [_P, i64, i32, _P, _P, i32, i32, dbl, i32, i32, i32, _P, i32]
        L.fm_set_buffers.argtypes = [_P] * 9
        for f in ("fm_reset", "fm_step_wait", "fm_destroy"):
            getattr(L, f).argtypes = [_P]
        L.fm_step_async.argtypes = [_P, _P]
        L.fm_frames.restype = L.fm_bad_ops.restype = i64
        L.fm_frames.argtypes = L.fm_bad_ops.argtypes = [_P]
        L.fm_env_ram.argtypes = [_P, i32, _P]
        L.fm_state_bytes.restype = i64
        L.fm_palette.argtypes = [_P]
        L.fm_resize_ref.argtypes = [_P, i32, i32, _P, i32, i32]
        L.fm_resize_fast.argtypes = [_P, _P]
        L.fm_raw_create.restype = _P
        L.fm_raw_create.argtypes = [_P, i64]
        L.fm_raw_frame.argtypes = [_P, i32, i32]
        L.fm_raw_ram.restype = L.fm_raw_screen.restype = _P
        L.fm_raw_ram.argtypes = L.fm_raw_screen.argtypes = [_P]
        L.fm_raw_backup.argtypes = L.fm_raw_restore.argtypes = L.fm_raw_destroy.argtypes = [_P]
        L.fm_raw_bad_ops.restype = i64
        L.fm_raw_bad_ops.argtypes = [_P]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def palette_rgb() -> np.ndarray:
    p = np.zeros(64, np.uint32)
    lib().fm_palette(_ptr(p))
    return np.stack([(p >> 16) & 255, (p >> 8) & 255, p & 255], -1).astype(np.uint8)


def gray_lut() -> np.ndarray:
    """cv2 RGB2GRAY fixed point over the reference palette (env.py:42-47)."""
    rgb = palette_rgb().astype(np.int64)
    g = (rgb[:, 0] * 4899 + rgb[:, 1] * 9617 + rgb[:, 2] * 1868 + (1 << 13)) >> 14
    return np.ascontiguousarray(g[np.arange(256) & 63], np.uint8)


def rng_state(seed: int) -> list[int]:
    st = np.random.default_rng(seed).bit_generator.state
    s, inc = st["state"]["state"], st["state"]["inc"]
    m = (1 << 64) - 1
    return [s >> 64, s & m, inc >> 64, inc & m, st["has_uint32"], st["uinteger"]]


def resize_ref(img: np.ndarray) -> np.ndarray:
    out = np.zeros((84, 84), np.uint8)
    g = np.ascontiguousarray(img, np.uint8)
    lib().fm_resize_ref(_ptr(g), 256, 240, _ptr(out), 84, 84)
    return out


class RefRaw:
    """One reference console (fm_raw_*): frame stepping, RAM and the palette-value screen."""

    def __init__(self, rom: bytes):
        L = lib()
        self._rom = np.frombuffer(rom, np.uint8).copy()
        self.h = L.fm_raw_create(_ptr(self._rom), len(self._rom))
        if not self.h:
            raise ValueError("reference rejected the ROM")
        u8p = ctypes.POINTER(ctypes.c_uint8)
        self.ram = np.ctypeslib.as_array(ctypes.cast(L.fm_raw_ram(self.h), u8p), (0x800,))
        self.screen = np.ctypeslib.as_array(ctypes.cast(L.fm_raw_screen(self.h), u8p), (240, 256))

    def frame(self, buttons: int, render: bool = True):
        lib().fm_raw_frame(self.h, int(buttons), int(bool(render)))

    def backup(self):
        lib().fm_raw_backup(self.h)

    def restore(self):
        lib().fm_raw_restore(self.h)

    def bad_ops(self) -> int:
        return int(lib().fm_raw_bad_ops(self.h))

    def close(self):
        if self.h:
            lib().fm_raw_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def smb_time(ram: np.ndarray) -> int:
    """int(''.join(map(str, ram[0x7f8:0x7fb]))) as fastmario.cpp:205-212 computes it."""
    v = 0
    for b in ram[0x7F8:0x7FB]:
        b = int(b)
        v = v * (1000 if b >= 100 else 100 if b >= 10 else 10) + b
    return v


def boot_frames_bounded(rom: bytes, level=(1, 1, 1), cap: int = 4000) -> int:
    """Replays the reference boot protocol (fastmario.cpp:422-445) on RefRaw with a frame cap, so a ROM whose
    boot would never terminate is caught before fm_create (which has no cap) ever runs it. Returns the number
    of frames boot takes; raises RuntimeError past `cap`."""
    r = RefRaw(rom)
    n = 0

    def fa(b):
        nonlocal n
        r.frame(b, True)
        n += 1
        if n > cap:
            raise RuntimeError(f"boot did not finish within {cap} frames")

    w, s, a = level
    fa(8)
    fa(0)
    while smb_time(r.ram) == 0:
        fa(8)
        r.ram[0x75F] = w - 1
        r.ram[0x75C] = s - 1
        r.ram[0x760] = a - 1
        fa(0)
        r.ram[0x7A0] = 0
    tl = smb_time(r.ram)
    while smb_time(r.ram) >= tl:
        tl = smb_time(r.ram)
        fa(8)
        fa(0)
    r.close()
    return n


class RefVecEnv:
    """The reference FastVecEnv engine (fm_create ...) driven directly, with numpy output buffers.

    Matches FastVecEnv's constructor semantics (env.py:140-184): levels as (world, stage, area) triples, env i
    seeded with rng_state(seed*1000 + env_offset + i), the cv2 gray LUT.
    """

    def __init__(self, rom: bytes, levels, n: int, seed=0, skip=4, max_steps=2000, sticky=0.0, noop_max=0,
                 maxpool=False, frame_stack=4, n_threads=0, env_offset=0, env_ids=None):
        """env_ids: global indices of the n envs of a larger run (any order, not necessarily contiguous); env k
        is then seeded as env env_ids[k] of that run, default_rng(seed*1000 + env_ids[k]). Without it the envs
        are env_offset .. env_offset + n - 1, as in the reference."""
        L = lib()
        self.n, self.k = n, frame_stack
        lv = np.array([tuple(levels)] * n if isinstance(levels[0], int) else list(levels), np.int32).reshape(-1)
        assert lv.size == 3 * n
        self._lv = lv
        ids = [env_offset + i for i in range(n)] if env_ids is None else [int(i) for i in env_ids]
        assert len(ids) == n
        self._rng = np.array([rng_state(seed * 1000 + i) for i in ids], np.uint64).reshape(-1)
        self._rom = np.frombuffer(rom, np.uint8).copy()
        self._lut = gray_lut()
        self.h = L.fm_create(_ptr(self._rom), len(self._rom), n, _ptr(self._lv), _ptr(self._lut), skip, max_steps,
                             float(sticky), int(noop_max), int(bool(maxpool)), frame_stack, _ptr(self._rng),
                             int(n_threads))
        if not self.h:
            raise RuntimeError("fm_create failed")
        self.obs = np.zeros((n, frame_stack, 84, 84), np.uint8)
        self.fin = np.zeros_like(self.obs)
        self.rew = np.zeros(n, np.float32)
        self.term = np.zeros(n, np.uint8)
        self.trunc = np.zeros(n, np.uint8)
        self.info = np.zeros((n, 10), np.int64)
        self.ep_ret = np.zeros(n, np.float64)
        self.ep_len = np.zeros(n, np.int64)
        L.fm_set_buffers(self.h, *[_ptr(x) for x in (self.obs, self.fin, self.rew, self.term, self.trunc, self.info,
                                                    self.ep_ret, self.ep_len)])
        self._act = np.zeros(n, np.int64)

    def reset(self) -> np.ndarray:
        lib().fm_reset(self.h)
        return self.obs

    def step(self, actions):
        self._act = np.ascontiguousarray(np.asarray(actions).reshape(-1), np.int64)
        lib().fm_step_async(self.h, _ptr(self._act))
        lib().fm_step_wait(self.h)
        return self.obs, self.rew, self.term.astype(bool), self.trunc.astype(bool), self.info

    def ram(self, i: int) -> np.ndarray:
        out = np.zeros(0x800, np.uint8)
        lib().fm_env_ram(self.h, int(i), _ptr(out))
        return out

    @property
    def frames(self) -> int:
        return int(lib().fm_frames(self.h))

    def bad_ops(self) -> int:
        return int(lib().fm_bad_ops(self.h))

    def close(self):
        if self.h:
            lib().fm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
