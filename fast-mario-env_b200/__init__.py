"""fast-mario-env_b200: the batched NES / SMB-style env step of fast-mario-env, rebuilt for B200 (sm_100a).

    from fast_mario_env_b200 import CudaVecEnv, FastVecEnv, RawNES
    from fast_mario_env_b200.synth_rom import build_rom

The engine is libfme_cuda.so (C ABI in include/fme.h), built by build.py; Python reaches the kernels only through
that ABI. See env.py for the API.
"""
from .env import (INFO_FIELDS, INFO_KEYS, N_ACTIONS, OBS_HW, SIMPLE_MOVEMENT, CudaVecEnv, FastVecEnv, MonitorCSV,
                  RawNES, RawNESBatch, gray_lut, palette_rgb, resize_area, rng_state)
from .rom import ALL_LEVELS, ROM_ENV_VAR, RomNotFoundError, check_rom, decode_level, find_rom, load_rom

__version__ = "0.1.0"

__all__ = ["CudaVecEnv", "FastVecEnv", "RawNES", "RawNESBatch", "MonitorCSV", "palette_rgb", "gray_lut", "rng_state",
           "resize_area", "find_rom", "load_rom", "check_rom", "decode_level", "RomNotFoundError", "ROM_ENV_VAR",
           "ALL_LEVELS", "OBS_HW", "N_ACTIONS", "SIMPLE_MOVEMENT", "INFO_FIELDS", "INFO_KEYS", "__version__"]
