"""ROM lookup / validation and level-name decoding, with the reference's rules (src/fast_mario_env/rom.py).

No ROM ships with this package. `load_rom` takes an explicit path, then the FAST_MARIO_ENV_ROM variable
(rom.py:16, 46-61); `check_rom` applies the reference's header checks (rom.py:73-82); `decode_level` maps
'w-s' to (world, stage, area) with the extra intro area of stage >= 2 in worlds 1, 2, 4 and 7
(rom.py:88-103). The gym-super-mario-bros package lookup is not available here (not installed).
"""
from __future__ import annotations

import os

ROM_ENV_VAR = "FAST_MARIO_ENV_ROM"
ALL_LEVELS = tuple(f"{w}-{s}" for w in range(1, 9) for s in range(1, 5))


class RomNotFoundError(FileNotFoundError):
    pass


def find_rom(rom_path=None) -> str:
    for cand, src in ((rom_path, "rom_path"), (os.environ.get(ROM_ENV_VAR) or None, ROM_ENV_VAR)):
        if cand is not None:
            cand = os.path.expanduser(os.fspath(cand))
            if not os.path.isfile(cand):
                raise RomNotFoundError(f"{src} points to {cand!r}, which is not a file")
            return cand
    raise RomNotFoundError("no ROM given: pass rom=bytes, rom_path=..., or set FAST_MARIO_ENV_ROM "
                           "(a synthetic image is available from fast_mario_env_b200.synth_rom.build_rom)")


def check_rom(data: bytes, name: str = "ROM") -> None:
    if len(data) < 16 or data[:4] != b"NES\x1a":
        raise ValueError(f"{name}: not an iNES ROM image (bad header)")
    mapper = (data[6] >> 4) | (data[7] & 0xF0)
    prg, chr_ = data[4], data[5]
    if mapper != 0 or prg not in (1, 2) or chr_ != 1:
        raise ValueError(f"{name}: unsupported ROM (mapper {mapper}, {prg}x16K PRG, {chr_}x8K CHR); "
                         "only NROM images are supported")
    if len(data) < 16 + prg * 0x4000 + 0x2000:
        raise ValueError(f"{name}: truncated ROM image")


def load_rom(rom_path=None) -> bytes:
    path = find_rom(rom_path)
    with open(path, "rb") as f:
        data = f.read()
    check_rom(data, path)
    return data


def decode_level(level) -> tuple[int, int, int]:
    if isinstance(level, str):
        try:
            w, s = (int(x) for x in level.split("-"))
        except ValueError:
            raise ValueError(f"level must look like '1-1', got {level!r}") from None
    else:
        w, s = (int(x) for x in level)
    if not (1 <= w <= 8 and 1 <= s <= 4):
        raise ValueError(f"level {level!r} out of range (worlds 1-8, stages 1-4)")
    area = s + 1 if (w in (1, 2, 4, 7) and s >= 2) else s
    return w, s, area
