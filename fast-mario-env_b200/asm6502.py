"""A small two-pass 6502 assembler used to build the synthetic NROM test images.

Only official opcodes are emitted. Labels are resolved at `assemble()` time; branches are checked to be in
range. The output is the 32 KB PRG image mapped at $8000-$FFFF.
"""
from __future__ import annotations

# (mnemonic, mode) -> opcode.  Modes: imp, acc, imm, zp, zpx, zpy, abs, absx, absy, ind, indx, indy, rel.
_OPS = {}


def _def(mn, **modes):
    for md, op in modes.items():
        _OPS[(mn, md)] = op


for _mn, _base in (("ora", 0x00), ("and", 0x20), ("eor", 0x40), ("adc", 0x60), ("lda", 0xA0), ("cmp", 0xC0),
                   ("sbc", 0xE0)):
    _def(_mn, indx=_base | 0x01, zp=_base | 0x05, imm=_base | 0x09, abs=_base | 0x0D, indy=_base | 0x11,
         zpx=_base | 0x15, absy=_base | 0x19, absx=_base | 0x1D)
_def("sta", indx=0x81, zp=0x85, abs=0x8D, indy=0x91, zpx=0x95, absy=0x99, absx=0x9D)
for _mn, _base in (("asl", 0x00), ("rol", 0x20), ("lsr", 0x40), ("ror", 0x60)):
    _def(_mn, zp=_base | 0x06, acc=_base | 0x0A, abs=_base | 0x0E, zpx=_base | 0x16, absx=_base | 0x1E)
_def("dec", zp=0xC6, abs=0xCE, zpx=0xD6, absx=0xDE)
_def("inc", zp=0xE6, abs=0xEE, zpx=0xF6, absx=0xFE)
_def("ldx", imm=0xA2, zp=0xA6, abs=0xAE, zpy=0xB6, absy=0xBE)
_def("ldy", imm=0xA0, zp=0xA4, abs=0xAC, zpx=0xB4, absx=0xBC)
_def("stx", zp=0x86, abs=0x8E, zpy=0x96)
_def("sty", zp=0x84, abs=0x8C, zpx=0x94)
_def("cpx", imm=0xE0, zp=0xE4, abs=0xEC)
_def("cpy", imm=0xC0, zp=0xC4, abs=0xCC)
_def("bit", zp=0x24, abs=0x2C)
_def("jmp", abs=0x4C, ind=0x6C)
_def("jsr", abs=0x20)
for _mn, _op in (("bpl", 0x10), ("bmi", 0x30), ("bvc", 0x50), ("bvs", 0x70), ("bcc", 0x90), ("bcs", 0xB0),
                 ("bne", 0xD0), ("beq", 0xF0)):
    _def(_mn, rel=_op)
for _mn, _op in (("brk", 0x00), ("php", 0x08), ("clc", 0x18), ("plp", 0x28), ("sec", 0x38), ("rti", 0x40),
                 ("pha", 0x48), ("cli", 0x58), ("rts", 0x60), ("pla", 0x68), ("sei", 0x78), ("dey", 0x88),
                 ("txa", 0x8A), ("tya", 0x98), ("txs", 0x9A), ("tay", 0xA8), ("tax", 0xAA), ("clv", 0xB8),
                 ("tsx", 0xBA), ("iny", 0xC8), ("dex", 0xCA), ("cld", 0xD8), ("inx", 0xE8), ("nop", 0xEA),
                 ("sed", 0xF8)):
    _def(_mn, imp=_op)

_LEN = {"imp": 1, "acc": 1, "imm": 2, "zp": 2, "zpx": 2, "zpy": 2, "indx": 2, "indy": 2, "rel": 2,
        "abs": 3, "absx": 3, "absy": 3, "ind": 3}

OPCODES = dict(_OPS)


class Asm:
    """Emit code at increasing addresses in $8000-$FFFF; `label()` marks the current address."""

    def __init__(self, org: int = 0x8000):
        self.prg = bytearray(0x8000)
        self.pc = org
        self.labels: dict[str, int] = {}
        self.fix: list[tuple[int, str, str]] = []  # (address, label, kind: 'abs' | 'rel' | 'lo' | 'hi')
        self._anon = 0

    # ---------------------------------------------------------------- layout
    def label(self, name: str | None = None) -> str:
        if name is None:
            self._anon += 1
            name = f"_L{self._anon}"
        if name in self.labels:
            raise ValueError(f"duplicate label {name}")
        self.labels[name] = self.pc
        return name

    def fresh(self) -> str:
        self._anon += 1
        return f"_F{self._anon}"

    def org(self, addr: int):
        if addr < self.pc:
            raise ValueError(f"org {addr:#x} below current pc {self.pc:#x}")
        self.pc = addr

    def byte(self, *vals):
        for v in vals:
            self._put(int(v) & 0xFF)

    def word_label(self, name: str):
        self.fix.append((self.pc, name, "abs"))
        self._put(0)
        self._put(0)

    def _put(self, b: int):
        if not 0x8000 <= self.pc <= 0xFFFF:
            raise ValueError(f"PRG overflow at {self.pc:#x}")
        self.prg[self.pc - 0x8000] = b
        self.pc += 1

    # ---------------------------------------------------------------- instructions
    def op(self, mn: str, mode: str = "imp", arg=None):
        """Emit `mn` in addressing `mode`. `arg` is an int, or a label name for abs/rel/imm('<lab'/'>lab')."""
        key = (mn, mode)
        if key not in _OPS:
            raise ValueError(f"no opcode for {mn} {mode}")
        self._put(_OPS[key])
        n = _LEN[mode] - 1
        if n == 0:
            return
        if mode == "rel":
            if isinstance(arg, str):
                self.fix.append((self.pc, arg, "rel"))
                self._put(0)
            else:
                self._put(int(arg) & 0xFF)
            return
        if isinstance(arg, str):
            if mode == "imm":
                kind = "lo" if arg.startswith("<") else "hi"
                self.fix.append((self.pc, arg[1:], kind))
                self._put(0)
            else:
                self.fix.append((self.pc, arg, "abs"))
                self._put(0)
                self._put(0)
            return
        v = int(arg)
        if n == 1:
            if not 0 <= v <= 0xFF:
                raise ValueError(f"{mn} {mode}: operand {v:#x} out of range")
            self._put(v)
        else:
            if not 0 <= v <= 0xFFFF:
                raise ValueError(f"{mn} {mode}: operand {v:#x} out of range")
            self._put(v & 0xFF)
            self._put(v >> 8)

    def __getattr__(self, mn):
        # a.lda("imm", 5) style shortcuts
        if (mn, "imp") in _OPS or any(k[0] == mn for k in _OPS):
            return lambda mode="imp", arg=None: self.op(mn, mode, arg)
        raise AttributeError(mn)

    # ---------------------------------------------------------------- finish
    def assemble(self) -> bytes:
        for addr, name, kind in self.fix:
            if name not in self.labels:
                raise ValueError(f"undefined label {name}")
            tgt = self.labels[name]
            i = addr - 0x8000
            if kind == "abs":
                self.prg[i] = tgt & 0xFF
                self.prg[i + 1] = tgt >> 8
            elif kind == "lo":
                self.prg[i] = tgt & 0xFF
            elif kind == "hi":
                self.prg[i] = tgt >> 8
            else:
                off = tgt - (addr + 1)
                if not -128 <= off <= 127:
                    raise ValueError(f"branch to {name} out of range ({off})")
                self.prg[i] = off & 0xFF
        return bytes(self.prg)
