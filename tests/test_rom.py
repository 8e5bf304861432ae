"""Synthetic NROM generator: deterministic, valid iNES, and it satisfies the reference's termination hazards
(boot protocol and busy-state loops) on the oracle, with frame caps (CPU only)."""
import os

import numpy as np
import pytest
from conftest import fme

from fast_mario_env_b200 import synth_rom
from fast_mario_env_b200.asm6502 import OPCODES, Asm

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_rom_is_deterministic_and_pinned(rom, rom_div):
    import zlib
    g = np.load(os.path.join(GOLD, "rom_seed0.npz"))
    assert zlib.crc32(rom) == int(g["crc"])
    assert zlib.crc32(rom_div) == int(g["crc_div"])
    assert synth_rom.build_rom(0) == rom
    assert synth_rom.build_rom(1) != rom


def test_rom_header(rom):
    assert len(rom) == 16 + 0x8000 + 0x2000
    assert rom[:4] == b"NES\x1a" and rom[4] == 2 and rom[5] == 1 and rom[6] == 1 and rom[7] == 0
    fme.check_rom(rom)
    chr_ = rom[16 + 0x8000:]
    for bank in (0, 0x1000):
        assert chr_[bank + 0xFF * 16: bank + 0x100 * 16] == b"\xff" * 16  # opaque sprite-0 tile


@pytest.mark.parametrize("level", [(1, 1, 1), (4, 2, 3), (8, 4, 4)])
def test_boot_terminates_on_oracle(oracle, rom, rom_div, level):
    assert oracle.boot_frames_bounded(rom, level, cap=500) < 100
    assert oracle.boot_frames_bounded(rom_div, level, cap=500) < 100


def test_rom_runs_without_bad_ops(oracle, rom_div):
    r = oracle.RefRaw(rom_div)
    rng = np.random.default_rng(0)
    for _ in range(300):
        r.frame(int(rng.integers(0, 256)), False)
    assert r.bad_ops() == 0


def test_four_idle_loop_image(oracle, rom):
    """The test image with four `JMP *` loops: only the code after the main loop and the NMI tail differ, it
    boots and runs on the reference engine without unimplemented opcodes."""
    r4 = synth_rom.build_rom(0, idle_loops=4)
    assert len(r4) == len(rom) and r4[:16] == rom[:16] and r4 != rom
    assert oracle.boot_frames_bounded(r4, (1, 1, 1), cap=500) < 100
    r = oracle.RefRaw(r4)
    rng = np.random.default_rng(0)
    for _ in range(300):
        r.frame(int(rng.integers(0, 256)), False)
    assert r.bad_ops() == 0
    with pytest.raises(ValueError):
        synth_rom.build_rom(0, idle_loops=3)


def test_asm_encodings():
    a = Asm()
    a.label("top")
    a.op("lda", "imm", 0x12)
    a.op("sta", "abs", 0x2000)
    a.op("bne", "rel", "top")
    a.op("jmp", "abs", "top")
    prg = a.assemble()
    assert prg[:10] == bytes([0xA9, 0x12, 0x8D, 0x00, 0x20, 0xD0, 0xF9, 0x4C, 0x00, 0x80])
    assert len(OPCODES) == 151  # every official (mnemonic, mode) pair
    with pytest.raises(ValueError):
        a.op("sta", "imm", 1)


def test_decode_level_and_rom_checks(tmp_path, monkeypatch):
    assert fme.decode_level("1-1") == (1, 1, 1)
    assert fme.decode_level("1-2") == (1, 2, 3)
    assert fme.decode_level((4, 4)) == (4, 4, 5)
    assert fme.decode_level("3-2") == (3, 2, 2)
    for bad in ("0-1", "9-1", "1-5", "x"):
        with pytest.raises(ValueError):
            fme.decode_level(bad)
    with pytest.raises(ValueError, match="iNES"):
        fme.check_rom(b"not a rom" * 100)
    monkeypatch.setenv(fme.ROM_ENV_VAR, str(tmp_path / "nope.nes"))
    with pytest.raises(fme.RomNotFoundError):
        fme.find_rom()
