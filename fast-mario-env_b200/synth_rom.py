"""Deterministic synthetic NROM image that stands in for the Super Mario Bros ROM (none ships anywhere).

The program is shaped like SMB's engine so that every part of the env path is exercised:

* iNES header: mapper 0, vertical mirroring, 2 x 16 KB PRG, 1 x 8 KB CHR (passes the reference's
  `check_rom`, rom.py:73-82, and `cart_load`, nes_core.hpp:67-75).
* CHR: 8 KB of uniform random bytes from ``numpy.random.default_rng(seed)``; tiles $FE/$FF of both pattern
  tables are made fully opaque so the sprite-0 split always hits.
* Reset handler: stack init, two vblank waits, random palette writes to $3F00-$3F1F, a seeded nametable
  fill through $2006/$2007, then NMI + background + sprites on, and the main loop idles in ``JMP *`` (the
  reference's idle-loop fast-forward, nes_core.hpp:1176-1193, applies to it exactly as to SMB).
* NMI handler (SMB order): OAM DMA from $0200, a VRAM column update with +32 increment, palette cycling,
  status-bar scroll, controller strobe + 8 serial reads of $4016 into $00F7, the first part of the seeded
  basic blocks, the sprite-0 poll split (``BIT $2002 / BVS`` then ``BVC``), the game scroll, the rest of
  the blocks and the game logic.
* 256 seeded basic blocks of ALU, load/store, stack and bounded-branch ops mutating scratch zero page and
  $0220-$06CF (random sprites 8-63 included). With ``divergence=True`` (the divergence-stress image) about a
  third of the blocks also branch on the controller byte $00F7 or the LFSR in $00F0, and some run LFSR-counted
  loops. Both images keep the NMI handler inside one frame, so the game runs at one NMI per frame.
* Game logic on the SMB RAM map: x_pos $006D/$0086, player state $000E (8 = normal, 7 = busy for a
  number of frames, $0B = dying, 6 = dead), $00B5, lives $075A, world/stage/area $075F/$075C/$0760, time
  digits $07F8-$07FA, score $07DE-$07E3, coins $07ED-$07EE, stage-over flag via $001D/$0016, $06DE area
  hack byte. Title mode ($0770 = 0) waits for Start; the level then starts with time 400, which counts
  down every 24 frames, so the reference boot protocol (fastmario.cpp:422-445) terminates. A 64-frame grace
  period keeps random events out of the boot snapshot. Random events come from a 16-bit LFSR mixed with the
  controller byte, so envs with different actions diverge.

The generator itself checks nothing about termination; `oracle`-side tests run the image on the reference
core with frame caps before any GPU run.
"""
from __future__ import annotations

import numpy as np

try:
    from .asm6502 import Asm
except ImportError:  # loaded as a plain module
    from asm6502 import Asm

# ---- RAM map ---------------------------------------------------------------------------------------
PLAYER_STATE = 0x0E
STAGE_FLOAT = 0x1D
ENEMY0 = 0x16
PTR = 0x40            # (zp),Y pointer -> $0400
XHI, XLO = 0x6D, 0x86
YVIEW = 0xB5
LFSR_LO, LFSR_HI = 0xF0, 0xF1
FRAMES = 0xF2
TSUB = 0xF3
TMP = 0xF4
SCROLL = 0xF5
BUSY = 0xF6
JOY = 0xF7
GRACE = 0xF8
DTIMER = 0xF9
MODECNT = 0xFA
PREVJOY = 0xFB
JUMP = 0xFC
XSCORE = 0xFD
TMP2 = 0xFE
IDLE_TMP = 0xFF       # idle_loops > 1 only
STATUS = 0x0756
LIVES = 0x075A
STAGE = 0x075C
WORLD = 0x075F
AREA = 0x0760
OPER = 0x0770
SCRTIMER = 0x07A0
SCORE = 0x07DE
COINS = 0x07ED
TIME = 0x07F8
YPOS = 0x03B8
AREAHACK = 0x06DE

SCRATCH_ZP = [a for a in range(0x20, 0x40)] + [a for a in range(0x42, 0x60)] + \
             [a for a in range(0x90, 0xB0)] + [a for a in range(0xC0, 0xF0)]
SCRATCH_ABS_LO, SCRATCH_ABS_HI = 0x0220, 0x06CF
ABSX_BASES = [0x0400, 0x0500, 0x0300]  # + X/Y (<= 255) stays inside scratch (or $03xx, which holds only y_pos)


def _scratch_abs(rng) -> int:
    while True:
        a = int(rng.integers(SCRATCH_ABS_LO, SCRATCH_ABS_HI + 1))
        if a != YPOS and not (0x03B0 <= a <= 0x03BF):
            return a


def _rmw_block_target(rng):
    if rng.random() < 0.6:
        return "zp", int(rng.choice(SCRATCH_ZP))
    return "abs", _scratch_abs(rng)


def _emit_block(a: Asm, rng, divergence: bool, sub_label: str):
    """One seeded basic block: 2-6 operations (each 1-5 instructions) with bounded branches / tiny loops."""
    n = int(rng.integers(2, 7))
    for _ in range(n):
        k = int(rng.integers(0, 20))
        if k <= 3:  # load
            mode = rng.choice(["imm", "zp", "abs", "zpx", "absy", "indy"])
            reg = rng.choice(["lda", "ldx", "ldy"]) if mode in ("imm", "zp", "abs") else "lda"
            if mode == "imm":
                a.op(reg, "imm", int(rng.integers(0, 256)))
            elif mode == "zp":
                a.op(reg, "zp", int(rng.choice(SCRATCH_ZP)))
            elif mode == "abs":
                a.op(reg, "abs", _scratch_abs(rng) if rng.random() < 0.8 else int(rng.integers(0x8000, 0x10000)))
            elif mode == "zpx":
                a.op("lda", "zpx", int(rng.choice(SCRATCH_ZP)))
            elif mode == "absy":
                a.op("lda", "absy", int(rng.choice(ABSX_BASES)) + int(rng.integers(0, 0x80)))
            else:
                a.op("lda", "indy", PTR)
        elif k <= 6:  # store (scratch only)
            mode = rng.choice(["zp", "abs", "absx", "indy", "zpx"])
            if mode == "zp":
                a.op(rng.choice(["sta", "stx", "sty"]), "zp", int(rng.choice(SCRATCH_ZP)))
            elif mode == "abs":
                a.op(rng.choice(["sta", "stx", "sty"]), "abs", _scratch_abs(rng))
            elif mode == "absx":
                a.op("sta", rng.choice(["absx", "absy"]), int(rng.choice(ABSX_BASES[:2])))
            elif mode == "indy":
                a.op("sta", "indy", PTR)
            else:  # zp,X with X masked: keep inside $20-$3F
                a.op("txa")
                a.op("and", "imm", 0x1F)
                a.op("tax")
                a.op("sta", "zpx", 0x20)
        elif k <= 10:  # ALU on A
            mn = rng.choice(["adc", "sbc", "and", "ora", "eor", "cmp"])
            mode = rng.choice(["imm", "zp", "abs", "absx"])
            if mode == "imm":
                a.op(mn, "imm", int(rng.integers(0, 256)))
            elif mode == "zp":
                a.op(mn, "zp", int(rng.choice(SCRATCH_ZP)))
            elif mode == "abs":
                a.op(mn, "abs", _scratch_abs(rng))
            else:
                a.op(mn, "absx", int(rng.choice(ABSX_BASES)))
        elif k <= 12:  # read-modify-write
            mn = rng.choice(["asl", "lsr", "rol", "ror", "inc", "dec"])
            if rng.random() < 0.25 and mn in ("asl", "lsr", "rol", "ror"):
                a.op(mn, "acc")
            else:
                md, addr = _rmw_block_target(rng)
                a.op(mn, md, addr)
        elif k == 13:  # register shuffles
            a.op(rng.choice(["tax", "tay", "txa", "tya", "inx", "iny", "dex", "dey", "clc", "sec", "clv"]))
        elif k == 14:  # balanced stack use
            if rng.random() < 0.5:
                a.op("pha")
                a.op("eor", "imm", int(rng.integers(0, 256)))
                a.op("sta", "zp", int(rng.choice(SCRATCH_ZP)))
                a.op("pla")
            else:
                a.op("php")
                a.op("adc", "imm", int(rng.integers(0, 256)))
                a.op("plp")
        elif k == 15:  # bounded forward branch over 1-3 instructions
            br = rng.choice(["beq", "bne", "bcc", "bcs", "bmi", "bpl", "bvc", "bvs"])
            skip = a.fresh()
            a.op(br, "rel", skip)
            for _ in range(int(rng.integers(1, 4))):
                a.op(rng.choice(["inc", "dec"]), "zp", int(rng.choice(SCRATCH_ZP)))
            a.label(skip)
        elif k == 16:  # tiny counted loop
            a.op("ldx", "imm", int(rng.integers(1, 5)))
            top = a.label()
            a.op("lda", "zpx", int(rng.choice(SCRATCH_ZP[:24])))
            a.op("adc", "zp", int(rng.choice(SCRATCH_ZP)))
            a.op("sta", "absx", 0x0400)
            a.op("dex")
            a.op("bne", "rel", top)
        elif k == 17:
            a.op("jsr", "abs", sub_label)
        elif k == 18:
            a.op("bit", rng.choice(["zp", "abs"]), int(rng.choice(SCRATCH_ZP)) if rng.random() < 0.5 else 0)
        else:
            a.op(rng.choice(["cpx", "cpy"]), "imm", int(rng.integers(0, 256)))
    if divergence and rng.random() < 0.3:
        # data-dependent control flow on the controller byte or the LFSR
        src = JOY if rng.random() < 0.5 else LFSR_LO
        skip = a.fresh()
        a.op("lda", "zp", src)
        a.op("and", "imm", int(1 << int(rng.integers(0, 8))))
        a.op("beq", "rel", skip)
        for _ in range(int(rng.integers(1, 4))):
            md, addr = _rmw_block_target(rng)
            a.op(rng.choice(["inc", "dec", "asl", "lsr"]), md, addr)
        a.label(skip)
    if divergence and rng.random() < 0.05:
        # a data-dependent loop count (1..4) from the LFSR
        a.op("lda", "zp", LFSR_HI)
        a.op("and", "imm", 3)
        a.op("tax")
        a.op("inx")
        top = a.label()
        a.op("lda", "zpx", 0x20)
        a.op("eor", "zp", JOY)
        a.op("sta", "zpx", 0x20)
        a.op("dex")
        a.op("bne", "rel", top)


def _lfsr_step(a: Asm):
    # 16-bit Galois LFSR (taps $B400) in $F0/$F1, then the controller byte is mixed in.
    a.op("lsr", "zp", LFSR_HI)
    a.op("ror", "zp", LFSR_LO)
    skip = a.fresh()
    a.op("bcc", "rel", skip)
    a.op("lda", "zp", LFSR_HI)
    a.op("eor", "imm", 0xB4)
    a.op("sta", "zp", LFSR_HI)
    a.label(skip)
    a.op("lda", "zp", JOY)
    a.op("eor", "zp", LFSR_LO)
    a.op("sta", "zp", LFSR_LO)
    nz = a.fresh()
    a.op("ora", "zp", LFSR_HI)
    a.op("bne", "rel", nz)
    a.op("lda", "imm", 0xE1)     # never let the LFSR stall at zero
    a.op("sta", "zp", LFSR_LO)
    a.label(nz)


def _event(a: Asm, mask_lo: int, mask_hi: int, value_lo: int, body):
    """Run `body` when (LFSR & mask) == value (probability 2^-popcount(mask))."""
    skip = a.fresh()
    a.op("lda", "zp", LFSR_LO)
    a.op("and", "imm", mask_lo)
    a.op("cmp", "imm", value_lo)
    a.op("bne", "rel", skip)
    a.op("lda", "zp", LFSR_HI)
    a.op("and", "imm", mask_hi)
    a.op("bne", "rel", skip)
    body()
    a.label(skip)


def _add_digits(a: Asm, base: int, ndig: int, pos: int, amount: int):
    """Decimal add of `amount` (0-9) at digit `pos` of the ndig-byte digit string at `base`; the carry moves
    toward lower addresses (the most significant digit is first, as in SMB's score/coin strings)."""
    assert 0 <= pos < ndig
    done = a.fresh()
    for p in range(pos, -1, -1):
        a.op("lda", "abs", base + p)
        a.op("clc")
        a.op("adc", "imm", amount if p == pos else 1)
        carry = a.fresh()
        a.op("cmp", "imm", 10)
        a.op("bcs", "rel", carry)
        a.op("sta", "abs", base + p)
        a.op("jmp", "abs", done)
        a.label(carry)
        a.op("sbc", "imm", 10)   # C=1 from CMP, so this subtracts exactly 10
        a.op("sta", "abs", base + p)
    a.label(done)


def build_rom(seed: int = 0, divergence: bool = False, n_blocks: int = 256, pre_blocks: int = 96,
              idle_loops: int = 1) -> bytes:
    """Return the iNES image (16 + 32768 + 8192 bytes).

    idle_loops=4 (test image): the main thread idles in one of four ``JMP *`` loops; at the end of every NMI
    the handler rewrites the interrupted return address to loop (LFSR ^ controller) & 3, so envs wait in
    different idle loops from frame to frame. The default image (1 loop) is unchanged by this option."""
    if idle_loops not in (1, 4):
        raise ValueError("idle_loops must be 1 or 4")
    rng = np.random.default_rng(seed)
    chr_ = bytearray(rng.integers(0, 256, 0x2000, dtype=np.uint8).tobytes())
    for bank in (0x0000, 0x1000):
        for tile in (0xFE, 0xFF):
            chr_[bank + tile * 16: bank + tile * 16 + 16] = b"\xff" * 16
    prng = np.random.default_rng(seed + 0x5EED)
    palette = [int(v) for v in prng.integers(0, 64, 32)]
    nt = bytearray(prng.integers(0, 256, 0x800, dtype=np.uint8).tobytes())
    # status bar rows 0-4 of nametable 0: sprite-0 landing tile at row 3, columns 10-13 (under x = 88..95)
    for col in range(10, 14):
        nt[3 * 32 + col] = 0xFF
    a = Asm()
    brng = np.random.default_rng(seed + 0xB10C)

    # ------------------------------------------------------------------ reset
    a.label("reset")
    a.op("sei")
    a.op("cld")
    a.op("ldx", "imm", 0xFF)
    a.op("txs")
    a.op("lda", "imm", 0)
    a.op("sta", "abs", 0x2000)
    a.op("sta", "abs", 0x2001)
    for _ in range(2):
        w = a.label()
        a.op("lda", "abs", 0x2002)
        a.op("bpl", "rel", w)
    # palette
    a.op("lda", "abs", 0x2002)
    a.op("lda", "imm", 0x3F)
    a.op("sta", "abs", 0x2006)
    a.op("lda", "imm", 0x00)
    a.op("sta", "abs", 0x2006)
    a.op("ldx", "imm", 0)
    pl = a.label()
    a.op("lda", "absx", "pal_data")
    a.op("sta", "abs", 0x2007)
    a.op("inx")
    a.op("cpx", "imm", 32)
    a.op("bne", "rel", pl)
    # nametables $2000-$27FF from nt_data via (PTR),Y
    a.op("lda", "abs", 0x2002)
    a.op("lda", "imm", 0x20)
    a.op("sta", "abs", 0x2006)
    a.op("lda", "imm", 0x00)
    a.op("sta", "abs", 0x2006)
    a.op("lda", "imm", "<nt_data")
    a.op("sta", "zp", PTR)
    a.op("lda", "imm", ">nt_data")
    a.op("sta", "zp", PTR + 1)
    a.op("ldx", "imm", 8)
    a.op("ldy", "imm", 0)
    ntl = a.label()
    a.op("lda", "indy", PTR)
    a.op("sta", "abs", 0x2007)
    a.op("iny")
    a.op("bne", "rel", ntl)
    a.op("inc", "zp", PTR + 1)
    a.op("dex")
    a.op("bne", "rel", ntl)
    # (zp),Y scratch pointer -> $0400
    a.op("lda", "imm", 0x00)
    a.op("sta", "zp", PTR)
    a.op("lda", "imm", 0x04)
    a.op("sta", "zp", PTR + 1)
    # sprite 0 over the opaque status-bar tiles; sprites 1-7 parked off screen
    for off, v in ((0, 23), (1, 0xFF), (2, 0x00), (3, 88)):
        a.op("lda", "imm", v)
        a.op("sta", "abs", 0x0200 + off)
    a.op("lda", "imm", 0xF8)
    for s in range(1, 8):
        a.op("sta", "abs", 0x0200 + 4 * s)
    a.op("lda", "imm", 0xE1)
    a.op("sta", "zp", LFSR_LO)
    a.op("lda", "imm", 0xAC)
    a.op("sta", "zp", LFSR_HI)
    a.op("lda", "imm", 2)
    a.op("sta", "abs", LIVES)
    a.op("lda", "imm", 0x90)   # NMI on, background from $1000, 8x8 sprites from $0000
    a.op("sta", "abs", 0x2000)
    a.op("lda", "imm", 0x1E)
    a.op("sta", "abs", 0x2001)
    a.label("main")
    a.op("jmp", "abs", "main")   # idle: the reference fast-forwards JMP-to-self exactly
    if idle_loops > 1:           # three more idle loops right after it (3 bytes each, one page)
        for k in range(1, idle_loops):
            a.label(f"main{k}")
            a.op("jmp", "abs", f"main{k}")
        if (a.labels["main"] & 0xFF) > 0x100 - 3 * idle_loops:
            raise ValueError("idle loops cross a page")

    # ------------------------------------------------------------------ shared subroutine for blocks
    a.label("sub")
    a.op("lda", "zp", 0x21)
    a.op("eor", "zp", 0x33)
    a.op("sta", "zp", 0x21)
    a.op("rol", "zp", 0x34)
    a.op("rts")

    # ------------------------------------------------------------------ NMI
    a.label("nmi")
    a.op("pha")
    a.op("txa")
    a.op("pha")
    a.op("tya")
    a.op("pha")
    a.op("lda", "imm", 0x10)   # NMI off while the handler runs (as SMB does)
    a.op("sta", "abs", 0x2000)
    # OAM DMA
    a.op("lda", "imm", 0x00)
    a.op("sta", "abs", 0x2003)
    a.op("lda", "imm", 0x02)
    a.op("sta", "abs", 0x4014)
    # VRAM column update: 8 tiles down a column of rows 8..15, with +32 increment
    a.op("lda", "imm", 0x14)
    a.op("sta", "abs", 0x2000)
    a.op("lda", "abs", 0x2002)
    a.op("lda", "zp", FRAMES)
    a.op("and", "imm", 0x04)          # alternate nametable 0 / 1
    a.op("ora", "imm", 0x21)          # $2100 / $2500: row 8
    a.op("sta", "abs", 0x2006)
    a.op("lda", "zp", FRAMES)
    a.op("and", "imm", 0x1F)
    a.op("sta", "abs", 0x2006)
    a.op("ldx", "imm", 0)
    vl = a.label()
    a.op("lda", "zpx", 0x20)
    a.op("sta", "abs", 0x2007)
    a.op("inx")
    a.op("cpx", "imm", 8)
    a.op("bne", "rel", vl)
    # status bar digits (time) at nametable 0 row 1 with +1 increment
    a.op("lda", "imm", 0x10)
    a.op("sta", "abs", 0x2000)
    a.op("lda", "imm", 0x20)
    a.op("sta", "abs", 0x2006)
    a.op("lda", "imm", 0x3A)
    a.op("sta", "abs", 0x2006)
    for i in range(3):
        a.op("lda", "abs", TIME + i)
        a.op("sta", "abs", 0x2007)
    # palette cycling every 8th frame
    skp = a.fresh()
    a.op("lda", "zp", FRAMES)
    a.op("and", "imm", 0x07)
    a.op("bne", "rel", skp)
    a.op("lda", "imm", 0x3F)
    a.op("sta", "abs", 0x2006)
    a.op("lda", "zp", FRAMES)
    a.op("lsr", "acc")
    a.op("lsr", "acc")
    a.op("and", "imm", 0x0E)
    a.op("ora", "imm", 0x01)
    a.op("sta", "abs", 0x2006)
    a.op("lda", "zp", 0x22)
    a.op("and", "imm", 0x3F)
    a.op("sta", "abs", 0x2007)
    a.label(skp)
    # mask: hide the left 8 pixels in frames with bit 5 set
    a.op("lda", "zp", FRAMES)
    a.op("and", "imm", 0x20)
    a.op("lsr", "acc")
    a.op("lsr", "acc")
    a.op("lsr", "acc")
    a.op("lsr", "acc")                # 0 or 2
    a.op("eor", "imm", 0x1E)          # $1E or $1C ... use $1C (bg edge hidden, sprite edge shown)
    a.op("sta", "abs", 0x2001)
    # status-bar scroll (0, 0), nametable 0; 8x16 sprites in frames with bit 6 set
    a.op("lda", "abs", 0x2002)
    a.op("lda", "imm", 0)
    a.op("sta", "abs", 0x2005)
    a.op("sta", "abs", 0x2005)
    a.op("lda", "zp", FRAMES)
    a.op("and", "imm", 0x40)
    a.op("lsr", "acc")
    a.op("ora", "imm", 0x10)
    a.op("sta", "zp", TMP2)           # ctrl without NMI
    a.op("sta", "abs", 0x2000)
    # controller
    a.op("lda", "zp", JOY)
    a.op("sta", "zp", PREVJOY)
    a.op("lda", "imm", 1)
    a.op("sta", "abs", 0x4016)
    a.op("lda", "imm", 0)
    a.op("sta", "abs", 0x4016)
    a.op("ldx", "imm", 8)
    jl = a.label()
    a.op("lda", "abs", 0x4016)
    a.op("lsr", "acc")
    a.op("rol", "zp", JOY)
    a.op("dex")
    a.op("bne", "rel", jl)
    _lfsr_step(a)
    a.op("inc", "zp", FRAMES)

    # first part of the blocks
    blocks = []
    for b in range(n_blocks):
        blocks.append(b)
    for b in blocks[:pre_blocks]:
        _emit_block(a, brng, divergence, "sub")

    # sprite-0 split: wait for the flag to clear, then to set (SMB's status-bar split)
    s0c = a.label()
    a.op("bit", "abs", 0x2002)
    a.op("bvs", "rel", s0c)
    s0s = a.label()
    a.op("bit", "abs", 0x2002)
    a.op("bvc", "rel", s0s)
    # game scroll: x = x_pos low byte, nametable from x_pos bit 8
    a.op("lda", "zp", XLO)
    a.op("sta", "abs", 0x2005)
    a.op("lda", "imm", 0)
    a.op("sta", "abs", 0x2005)
    a.op("lda", "zp", XHI)
    a.op("and", "imm", 1)
    a.op("ora", "zp", TMP2)
    a.op("sta", "abs", 0x2000)

    for b in blocks[pre_blocks:]:
        _emit_block(a, brng, divergence, "sub")
    a.op("jsr", "abs", "game")

    # restore and return; NMI back on
    a.op("lda", "zp", TMP2)
    a.op("ora", "imm", 0x80)
    a.op("sta", "abs", 0x2000)
    if idle_loops > 1:
        # stack: $101+S = Y, X, A, P, PCL, PCH; an interrupted idle loop returns to loop (LFSR ^ JOY) & 3
        a.op("tsx")
        a.op("lda", "absx", 0x0106)
        a.op("cmp", "imm", ">main")
        a.op("bne", "rel", "nmi_keep")
        a.op("lda", "absx", 0x0105)
        a.op("sec")
        a.op("sbc", "imm", "<main")
        a.op("cmp", "imm", 3 * idle_loops)
        a.op("bcs", "rel", "nmi_keep")
        a.op("lda", "zp", LFSR_LO)
        a.op("eor", "zp", JOY)
        a.op("and", "imm", idle_loops - 1)
        a.op("sta", "zp", IDLE_TMP)
        a.op("asl", "acc")
        a.op("clc")
        a.op("adc", "zp", IDLE_TMP)
        a.op("clc")
        a.op("adc", "imm", "<main")
        a.op("sta", "absx", 0x0105)
        a.label("nmi_keep")
    a.op("pla")
    a.op("tay")
    a.op("pla")
    a.op("tax")
    a.op("pla")
    a.label("irq")
    a.op("rti")

    # ------------------------------------------------------------------ game logic (JSR'd from NMI)
    a.label("game")
    a.op("lda", "abs", OPER)
    a.op("bne", "rel", "g_play")
    # title mode: Start (bit 4 of the serial byte) begins the level after a short countdown
    a.op("lda", "zp", MODECNT)
    a.op("bne", "rel", "g_count")
    a.op("lda", "zp", JOY)
    a.op("and", "imm", 0x10)
    a.op("beq", "rel", "g_ret0")
    a.op("lda", "imm", 3)
    a.op("sta", "zp", MODECNT)
    a.label("g_ret0")
    a.op("rts")
    a.label("g_count")
    a.op("dec", "zp", MODECNT)
    a.op("bne", "rel", "g_ret0")
    a.op("jsr", "abs", "level_init")
    a.op("lda", "imm", 1)
    a.op("sta", "abs", OPER)
    a.op("rts")

    a.label("g_play")
    # grace counter (saturating)
    gsat = a.fresh()
    a.op("lda", "zp", GRACE)
    a.op("cmp", "imm", 0xFF)
    a.op("beq", "rel", gsat)
    a.op("inc", "zp", GRACE)
    a.label(gsat)
    # time: every 24 frames, decrement the 3-digit time
    a.op("inc", "zp", TSUB)
    a.op("lda", "zp", TSUB)
    a.op("cmp", "imm", 24)
    a.op("bcc", "rel", "g_state")
    a.op("lda", "imm", 0)
    a.op("sta", "zp", TSUB)
    a.op("jsr", "abs", "time_dec")
    a.label("g_state")
    a.op("lda", "zp", PLAYER_STATE)
    a.op("cmp", "imm", 7)
    a.op("bne", "rel", "g_notbusy")
    # busy: the screen timer $07A0 runs first, then the busy counter
    a.op("lda", "abs", SCRTIMER)
    a.op("beq", "rel", "g_busy2")
    a.op("dec", "abs", SCRTIMER)
    a.op("rts")
    a.label("g_busy2")
    a.op("dec", "zp", BUSY)
    a.op("bne", "rel", "g_ret1")
    a.op("lda", "imm", 8)
    a.op("sta", "zp", PLAYER_STATE)
    a.label("g_ret1")
    a.op("rts")
    a.label("g_notbusy")
    a.op("cmp", "imm", 8)
    a.op("beq", "rel", "g_normal")
    # dying / dead: after 40 frames respawn (or back to title when out of lives)
    a.op("inc", "zp", DTIMER)
    a.op("lda", "zp", DTIMER)
    a.op("cmp", "imm", 40)
    a.op("bcc", "rel", "g_ret1")
    a.op("lda", "imm", 0)
    a.op("sta", "zp", DTIMER)
    a.op("sta", "zp", YVIEW)
    a.op("dec", "abs", LIVES)
    a.op("bpl", "rel", "g_respawn")
    a.op("lda", "imm", 0)
    a.op("sta", "abs", OPER)
    a.op("lda", "imm", 2)
    a.op("sta", "abs", LIVES)
    a.op("rts")
    a.label("g_respawn")
    a.op("jsr", "abs", "place_player")
    a.op("rts")

    a.label("g_normal")
    # stage over: after the flag, wait 64 frames then start the next stage
    a.op("lda", "zp", STAGE_FLOAT)
    a.op("cmp", "imm", 3)
    a.op("bne", "rel", "g_move")
    a.op("inc", "zp", DTIMER)
    a.op("lda", "zp", DTIMER)
    a.op("cmp", "imm", 64)
    a.op("bcc", "rel", "g_ret1")
    a.op("lda", "imm", 0)
    a.op("sta", "zp", DTIMER)
    a.op("sta", "zp", STAGE_FLOAT)
    a.op("sta", "zp", ENEMY0)
    a.op("inc", "abs", STAGE)
    a.op("jsr", "abs", "place_player")
    a.op("rts")

    a.label("g_move")
    # right (bit 0): +1, +1 more with B (bit 6); left (bit 1): -1 while x_pos >= $0010
    nr = a.fresh()
    a.op("lda", "zp", JOY)
    a.op("and", "imm", 0x01)
    a.op("beq", "rel", nr)
    a.op("jsr", "abs", "x_inc")
    a.op("lda", "zp", JOY)
    a.op("and", "imm", 0x40)
    a.op("beq", "rel", nr)
    a.op("jsr", "abs", "x_inc")
    a.label(nr)
    nl = a.fresh()
    a.op("lda", "zp", JOY)
    a.op("and", "imm", 0x02)
    a.op("beq", "rel", nl)
    a.op("lda", "zp", XHI)
    a.op("bne", "rel", "g_left")
    a.op("lda", "zp", XLO)
    a.op("cmp", "imm", 0x10)
    a.op("bcc", "rel", nl)
    a.label("g_left")
    a.op("lda", "zp", XLO)
    a.op("sec")
    a.op("sbc", "imm", 1)
    a.op("sta", "zp", XLO)
    a.op("lda", "zp", XHI)
    a.op("sbc", "imm", 0)
    a.op("sta", "zp", XHI)
    a.label(nl)
    # jump on A (bit 7): 16-frame arc in $00FC; y_pos = 176 - arc
    nj = a.fresh()
    a.op("lda", "zp", JUMP)
    a.op("bne", "rel", "g_air")
    a.op("lda", "zp", JOY)
    a.op("and", "imm", 0x80)
    a.op("beq", "rel", nj)
    a.op("lda", "imm", 16)
    a.op("sta", "zp", JUMP)
    a.label("g_air")
    a.op("dec", "zp", JUMP)
    a.label(nj)
    a.op("lda", "zp", JUMP)
    a.op("asl", "acc")
    a.op("sta", "zp", TMP)
    a.op("lda", "imm", 176)
    a.op("sec")
    a.op("sbc", "zp", TMP)
    a.op("sta", "abs", YPOS)
    # player sprites 1-4 follow the player
    a.op("sta", "abs", 0x0204)
    a.op("sta", "abs", 0x0208)
    a.op("clc")
    a.op("adc", "imm", 8)
    a.op("sta", "abs", 0x020C)
    a.op("sta", "abs", 0x0210)
    a.op("lda", "zp", XLO)
    a.op("and", "imm", 0x7F)
    a.op("adc", "imm", 40)
    a.op("sta", "abs", 0x0207)
    a.op("sta", "abs", 0x020F)
    a.op("adc", "imm", 8)
    a.op("sta", "abs", 0x020B)
    a.op("sta", "abs", 0x0213)
    a.op("lda", "zp", FRAMES)
    a.op("and", "imm", 0x03)
    a.op("sta", "abs", 0x0206)
    a.op("sta", "abs", 0x020A)
    # score: +50 whenever x_pos crosses a 16-pixel boundary
    nsc = a.fresh()
    a.op("lda", "zp", XLO)
    a.op("lsr", "acc")
    a.op("lsr", "acc")
    a.op("lsr", "acc")
    a.op("lsr", "acc")
    a.op("cmp", "zp", XSCORE)
    a.op("beq", "rel", nsc)
    a.op("sta", "zp", XSCORE)
    _add_digits(a, SCORE, 6, 4, 5)
    a.label(nsc)
    # flag: x_pos >= $0C00 -> stage over ($001D = 3, enemy slot 0 = $31)
    nf = a.fresh()
    a.op("lda", "zp", XHI)
    a.op("cmp", "imm", 0x0C)
    a.op("bcc", "rel", nf)
    a.op("lda", "imm", 3)
    a.op("sta", "zp", STAGE_FLOAT)
    a.op("lda", "imm", 0x31)
    a.op("sta", "zp", ENEMY0)
    a.op("lda", "imm", 0)
    a.op("sta", "zp", DTIMER)
    a.op("rts")
    a.label(nf)
    # random events only after the grace period
    a.op("lda", "zp", GRACE)
    a.op("cmp", "imm", 64)
    a.op("bcs", "rel", "g_events")
    a.op("rts")
    a.label("g_events")

    def coin():
        _add_digits(a, COINS, 2, 1, 1)

    def busy():
        a.op("lda", "imm", 7)
        a.op("sta", "zp", PLAYER_STATE)
        a.op("lda", "zp", LFSR_HI)
        a.op("and", "imm", 0x0F)
        a.op("ora", "imm", 0x04)
        a.op("sta", "zp", BUSY)
        a.op("lda", "imm", 2)
        a.op("sta", "abs", SCRTIMER)

    def dying():
        a.op("lda", "imm", 0x0B)
        a.op("sta", "zp", PLAYER_STATE)
        a.op("lda", "imm", 0)
        a.op("sta", "zp", DTIMER)

    def dead():
        a.op("lda", "imm", 0x06)
        a.op("sta", "zp", PLAYER_STATE)
        a.op("lda", "imm", 0)
        a.op("sta", "zp", DTIMER)

    def pit():
        a.op("lda", "imm", 2)
        a.op("sta", "zp", YVIEW)
        dying()

    def lifeloss():
        nz = a.fresh()
        a.op("lda", "abs", LIVES)
        a.op("beq", "rel", nz)
        a.op("dec", "abs", LIVES)
        a.label(nz)

    def teleport():
        a.op("lda", "zp", XLO)
        a.op("clc")
        a.op("adc", "imm", 64)
        a.op("sta", "zp", XLO)
        a.op("lda", "zp", XHI)
        a.op("adc", "imm", 0)
        a.op("sta", "zp", XHI)

    def areahack():
        a.op("lda", "imm", 5)
        a.op("sta", "abs", AREAHACK)

    def status():
        a.op("inc", "abs", STATUS)

    _event(a, 0x3F, 0x00, 0x11, coin)           # 1/64
    _event(a, 0xFF, 0x01, 0x2A, busy)           # 1/512
    _event(a, 0xFF, 0x07, 0x5C, dying)          # 1/2048
    _event(a, 0xFF, 0x1F, 0x77, dead)           # 1/8192
    _event(a, 0xFF, 0x0F, 0x93, lifeloss)       # 1/4096
    _event(a, 0xFF, 0x1F, 0xC4, pit)            # 1/8192
    _event(a, 0xFF, 0x00, 0x3B, teleport)       # 1/256
    _event(a, 0x7F, 0x00, 0x05, areahack)       # 1/128
    _event(a, 0xFF, 0x03, 0xE8, status)         # 1/1024
    a.op("rts")

    # ------------------------------------------------------------------ helpers
    a.label("x_inc")
    a.op("inc", "zp", XLO)
    nz = a.fresh()
    a.op("bne", "rel", nz)
    a.op("inc", "zp", XHI)
    a.label(nz)
    a.op("rts")

    a.label("place_player")
    a.op("lda", "imm", 8)
    a.op("sta", "zp", PLAYER_STATE)
    a.op("lda", "imm", 0x28)
    a.op("sta", "zp", XLO)
    a.op("lda", "imm", 0)
    a.op("sta", "zp", XHI)
    a.op("sta", "zp", JUMP)
    a.op("sta", "zp", YVIEW)
    a.op("sta", "zp", GRACE)
    a.op("rts")

    a.label("level_init")
    a.op("jsr", "abs", "place_player")
    a.op("lda", "imm", 4)
    a.op("sta", "abs", TIME)
    a.op("lda", "imm", 0)
    a.op("sta", "abs", TIME + 1)
    a.op("sta", "abs", TIME + 2)
    a.op("sta", "zp", TSUB)
    a.op("sta", "zp", STAGE_FLOAT)
    a.op("sta", "zp", ENEMY0)
    a.op("lda", "imm", 2)
    a.op("sta", "abs", LIVES)
    # LFSR seeded from the level (world/stage/area written by the boot protocol)
    a.op("lda", "abs", WORLD)
    a.op("asl", "acc")
    a.op("asl", "acc")
    a.op("asl", "acc")
    a.op("asl", "acc")
    a.op("ora", "abs", STAGE)
    a.op("eor", "imm", 0xE1)
    a.op("sta", "zp", LFSR_LO)
    a.op("lda", "abs", AREA)
    a.op("eor", "imm", 0xAC)
    a.op("sta", "zp", LFSR_HI)
    a.op("rts")

    a.label("time_dec")
    # decrement the 3 time digits; at 000 the player dies (time up)
    a.op("ldx", "imm", 2)
    tl_ = a.label()
    a.op("lda", "absx", TIME)
    a.op("bne", "rel", "td_dec")
    a.op("lda", "imm", 9)
    a.op("sta", "absx", TIME)
    a.op("dex")
    a.op("bpl", "rel", tl_)
    # wrapped below 000: clamp to 000 and die
    a.op("lda", "imm", 0)
    a.op("sta", "abs", TIME)
    a.op("sta", "abs", TIME + 1)
    a.op("sta", "abs", TIME + 2)
    dying()
    a.op("rts")
    a.label("td_dec")
    a.op("sec")
    a.op("sbc", "imm", 1)
    a.op("sta", "absx", TIME)
    a.op("rts")

    # ------------------------------------------------------------------ data + vectors
    a.label("pal_data")
    a.byte(*palette)
    a.label("nt_data")
    a.byte(*nt)
    if a.pc > 0xFFFA:
        raise ValueError(f"program too large ({a.pc:#x})")
    a.org(0xFFFA)
    a.word_label("nmi")
    a.word_label("reset")
    a.word_label("irq")
    prg = a.assemble()
    header = b"NES\x1a" + bytes([2, 1, 0x01, 0x00]) + bytes(8)
    return header + prg + bytes(chr_)


def code_size(seed: int = 0, divergence: bool = False) -> int:
    a_rom = build_rom(seed, divergence)
    prg = a_rom[16:16 + 0x8000]
    return len(prg.rstrip(b"\x00"))


if __name__ == "__main__":  # pragma: no cover
    import sys
    rom = build_rom(int(sys.argv[1]) if len(sys.argv) > 1 else 0)
    sys.stdout.buffer.write(rom)
