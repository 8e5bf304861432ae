"""ctypes binding of libfme_cuda.so (the C ABI declared in include/fme.h).

The library is built in-tree by build.py (nvcc, sm_100a). There is no CPU fallback: if the library is missing
or cannot be loaded, every entry point raises. The reference's binding pattern is _native.py
(src/fast_mario_env/_native.py:16-65): one lazily loaded CDLL with explicit argtypes.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ENV_VAR = "FME_B200_LIB"
LIB_NAME = "libfme_cuda.so"

_P = ctypes.c_void_p
_i32, _i64, _u32, _dbl = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_double
_lib = None

# status bits (include/fme.h)
ST_LOG_OVERFLOW = 1
ST_HACK_CAP = 2
ST_BOOT_CAP = 4
ST_BAD_ACTION = 8
# capacity of the allocation-free raw frame call (include/fme.h FME_STATIC_*)
FME_STATIC_MAX_CONSOLES = 64
FME_STATIC_LOG_CAPACITY = 2048
STATUS_NAMES = {ST_LOG_OVERFLOW: "PPU log overflow (raise log_capacity)",
                ST_HACK_CAP: "busy-state skip loop exceeded hack_cap frames",
                ST_BOOT_CAP: "level boot exceeded boot_cap frames",
                ST_BAD_ACTION: "action outside 0..6"}

# declared entry points: name -> (restype, argtypes); tests check the library exports all of them
SIGNATURES = {
    "fme_create": (_i32, [_P, _P, _i64, _P, _P, _P, _P]),
    "fme_set_buffers": (_i32, [_P, _P]),
    "fme_reset": (_i32, [_P, _P]),
    "fme_step": (_i32, [_P, _P, _P]),
    "fme_poll_error": (_i32, [_P, _P]),
    "fme_env_ram": (_i32, [_P, _i32, _P]),
    "fme_ram_all": (_i32, [_P, _P, _P]),
    "fme_frames": (_i32, [_P, _P]),
    "fme_bad_ops": (_i32, [_P, _P]),
    "fme_work_counters": (_i32, [_P, _P, _P]),
    "fme_env_bytes": (_i64, [_P]),
    "fme_destroy": (None, [_P]),
    "fme_raw_create": (_i32, [_P, _i64, _i32, _i32, _i32, _P]),
    "fme_raw_frame": (_i32, [_P, _P, _i32, _P]),
    "fme_raw_ram": (_i32, [_P, _P, _P]),
    "fme_raw_screen": (_i32, [_P, _P, _P]),
    "fme_raw_backup": (_i32, [_P, _P]),
    "fme_raw_restore": (_i32, [_P, _P]),
    "fme_raw_bad_ops": (_i32, [_P, _P]),
    "fme_raw_poll_error": (_i32, [_P, _P]),
    "fme_raw_destroy": (None, [_P]),
    "fme_raw_frame_static": (_i32, [_P, _P, _P, _i32, _P]),
    "fme_step_marked": (_i32, [_P, _P, _P, _P]),
    "fme_step_to_host": (_i32, [_P, _P, _P, _P]),
    "fme_gae": (_i32, [_P, _P, _P, _P, _P, _i32, _i32, ctypes.c_float, ctypes.c_float, _P, _P, _P]),
    "fme_adv_norm": (_i32, [_P, _P, _i32, _P]),
    "fme_replay_add": (_i32, [_P, _P, _P, _i32, _P, _P, _P, _P, _P]),
    "fme_replay_gather": (_i32, [_P, _P, _P, _i32, _i32, _i32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "fme_palette": (None, [_P]),
    "fme_resize": (_i32, [_P, _P, _i32, _P]),
    "fme_state_bytes": (_i64, []),
    "fme_last_error": (ctypes.c_char_p, []),
    "fme_version": (ctypes.c_char_p, []),
}


class FmeConfig(ctypes.Structure):
    _fields_ = [("n_envs", _i32), ("skip", _i32), ("max_steps", _i32), ("noop_max", _i32), ("maxpool", _i32),
                ("frame_stack", _i32), ("sticky", _dbl), ("device", _i32), ("log_capacity", _i32),
                ("hack_cap", _i32), ("boot_cap", _i32)]


FME_HOST_OBS_IN_PLACE = 1


class FmeHostOut(ctypes.Structure):
    _fields_ = [(f, _P) for f in ("obs", "rew", "term", "trunc", "info", "ep_ret", "ep_len")] + [("flags", _u32)]


class FmeReplayBufs(ctypes.Structure):
    _fields_ = [(f, _P) for f in ("frames", "age", "act", "rew", "flags", "ptr", "new_ep")] + \
               [("n_envs", _i32), ("capacity", _i32)]


class FmeBuffers(ctypes.Structure):
    _fields_ = [(f, _P) for f in ("obs", "final_obs", "rew", "term", "trunc", "info", "ep_ret", "ep_len")]


class FmeError(RuntimeError):
    pass


def lib_path() -> str:
    p = os.environ.get(LIB_ENV_VAR)
    return p if p else os.path.join(HERE, LIB_NAME)


def lib():
    """Load (once) and return the CDLL. Raises ImportError if the CUDA library is not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.isfile(path):
        raise ImportError(f"fast-mario-env_b200: {path} not found; build it with `python fast-mario-env_b200/build.py` "
                          "(nvcc, sm_100a). There is no CPU fallback.")
    L = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    m = lib().fme_last_error()
    return m.decode() if m else ""


def check(rc: int, what: str):
    if rc != 0:
        raise FmeError(f"{what} failed ({rc}): {last_error()}")


def status_text(st: int) -> str:
    return "; ".join(msg for bit, msg in STATUS_NAMES.items() if st & bit) or "ok"


def ptr(a) -> ctypes.c_void_p:
    """Address of a numpy array's data or a torch tensor's storage as a void pointer."""
    if hasattr(a, "data_ptr"):
        return ctypes.c_void_p(a.data_ptr())
    return a.ctypes.data_as(_P)
