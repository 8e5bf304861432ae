"""ROM lookup / validation and level-name decoding, with the reference's rules (src/fast_mario_env/rom.py).

No ROM ships with this package. `load_rom` takes an explicit path, then the FAST_MARIO_ENV_ROM variable
(rom.py:16, 46-61); `check_rom` applies the reference's header checks (rom.py:73-82); `decode_level` maps
'w-s' to (world, stage, area) with the extra intro area of stage >= 2 in worlds 1, 2, 4 and 7
(rom.py:88-103). The gym-super-mario-bros package lookup is not available here (not installed).
"""
from __future__ import annotations

import os
import re

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


# iNES acceptance rules of the reference loader: an "NES\x1a" magic, mapper 0 (NROM), one or two 16 KB PRG
# banks, exactly one 8 KB CHR bank, and enough bytes behind the header for all of them.
_MAGIC = b"NES\x1a"
_PRG_BANK, _CHR_BANK = 0x4000, 0x2000


def check_rom(data: bytes, name: str = "ROM") -> None:
    """Raise ValueError unless `data` is an NROM iNES image this engine (and the reference) can run."""
    head = bytes(data[:16])
    if len(head) != 16 or head[:4] != _MAGIC:
        raise ValueError(f"{name}: the first bytes are not an iNES header")
    n_prg, n_chr = head[4], head[5]
    mapper_id = (head[7] & 0xF0) | (head[6] >> 4)
    if mapper_id != 0 or n_chr != 1 or n_prg not in (1, 2):
        raise ValueError(f"{name}: only NROM images run here (this one: mapper {mapper_id}, "
                         f"{n_prg} PRG bank(s) of 16 KB, {n_chr} CHR bank(s) of 8 KB)")
    need = len(head) + n_prg * _PRG_BANK + _CHR_BANK
    if len(data) < need:
        raise ValueError(f"{name}: image ends after {len(data)} bytes, its header promises {need}")


def load_rom(rom_path=None) -> bytes:
    path = find_rom(rom_path)
    with open(path, "rb") as f:
        data = f.read()
    check_rom(data, path)
    return data


# Worlds whose stages 2-4 sit one area later in the game's level table: their stage 2 opens with a separate
# pipe-intro area (world 1, 2, 4 and 7 of Super Mario Bros).
_INTRO_AREA_WORLDS = frozenset((1, 2, 4, 7))
_LEVEL_RE = re.compile(r"^\s*(\d+)\s*-\s*(\d+)\s*$")


def decode_level(level) -> tuple[int, int, int]:
    """Level name 'w-s' (or a (w, s) pair) -> the (world, stage, area) numbers written into RAM at boot."""
    if isinstance(level, str):
        m = _LEVEL_RE.match(level)
        if m is None:
            raise ValueError(f"a level is named 'world-stage' such as '1-1'; got {level!r}")
        world, stage = int(m.group(1)), int(m.group(2))
    else:
        world, stage = (int(v) for v in level)
    if world not in range(1, 9) or stage not in range(1, 5):
        raise ValueError(f"no level {level!r}: worlds run 1..8 and stages 1..4")
    shift = 1 if (stage >= 2 and world in _INTRO_AREA_WORLDS) else 0
    return world, stage, stage + shift
