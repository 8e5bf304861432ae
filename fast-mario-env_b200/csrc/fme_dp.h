// fme_dp.h - the data-driven 6502 datapath: every lane executes its own instruction in the same code.
//
// The exact interpreter (fme_fast.h hot_step + Core) dispatches on a handler id, so a warp can only run the
// lanes that sit at one PC; the kernels therefore vote for the warp's minimum PC every instruction, and an
// instruction costs a vote, an indirect branch and a chain of dependent handler steps with one warp per
// scheduler. Here an instruction is instead described by a datapath micro-op (the "dop", built once per ROM
// on the host by build_dops from the exact micro-ops): an addressing mode, an ALU function with its operand
// selects, a destination, a flag mask, a stack delta and a next-pc mode. One straight-line routine evaluates
// any dop, with predicated loads and stores into the lane's own RAM words, so the 32 lanes of a warp each
// run a different instruction at the same time: no vote, no dispatch branch, no divergence.
//
// Which instructions take it: every one whose memory accesses are RAM or PRG only (the same set the exact
// fast path executes, fme_fast.h Fast::exec, minus BRK, RTI, JMP (ind) and undefined opcodes), with the
// semantics of Core::execute_op (nes_core.hpp:645-1163): nes-py's flag layout (N = bit 0 ... C = bit 7),
// page-cross penalties with the decode cascade's quirks (the (zp,X) penalty tests the high byte of the
// address itself), taken-branch costs 1 or 3, writes into ROM ignored. A lane whose next instruction is not
// of that kind (I/O operand, the controller ports, the PPU catch-up or NMI due, the `JMP *` idle loop, the
// frame end) stops and waits for the exact path. A computed address that lands in I/O space is found only
// while executing; then nothing is committed and the lane waits as well.
#pragma once
#include "fme_fast.h"

namespace fme {

// ---------------------------------------------------------------- dop layout (2 words per PRG address)
// word 0: W (16 bits: static address, immediate or ROM operand value, jump / branch target)
//         | cycles<<16 (3) | len<<19 (2) | PEN<<21 | IX<<22 (index X) | IY<<23 (index Y) | ZW<<24 (address wraps
//         in page 0) | IND<<25 (pointer in page 0) | INX<<26 (pointer at W+X) | CMPA<<27 (computed address: I/O
//         test, page penalty, ROM read) | PULL<<28 | PUSH<<29 | IMM<<30 | OK<<31
// word 1: SEL (8: byte-permute nibbles of the ALU operands L and R in {A, X, Y, SP, M, 1, $FF, P}; for a
//         branch or a flag operation: flag bit index (3) | value<<3) | FMASK<<8 (8: the flags the ALU result
//         sets, in nes-py's layout) | CLS<<16 (2: logic, add, shift left, shift right) | LOP<<18 (2: pass R, or,
//         and, eor) | BITF<<20 | INV<<21 | CIN<<22 (2: 0, 1, C) | DST<<24 (3) | PCM<<27 (2) | PF<<29 | JSR<<30
//         | BX<<31
constexpr uint32_t D_PEN = 1u << 21, D_IX = 1u << 22, D_IY = 1u << 23, D_ZW = 1u << 24, D_IND = 1u << 25,
                   D_INX = 1u << 26, D_CMPA = 1u << 27, D_PULL = 1u << 28, D_PUSH = 1u << 29, D_IMM = 1u << 30,
                   D_OK = 1u << 31;
enum DCls : uint32_t { CL_LOGIC = 0, CL_ADD, CL_SHL, CL_SHR };
enum DLop : uint32_t { LO_PASS = 0, LO_OR, LO_AND, LO_EOR };
enum DByte : uint32_t { B_A = 0, B_X, B_Y, B_SP, B_M, B_ONE, B_FF, B_P };
enum DCin : uint32_t { CI_0 = 0, CI_1, CI_C };
enum DDst : uint32_t { DS_NONE = 0, DS_A, DS_X, DS_Y, DS_SP, DS_MEM, DS_P };
enum DPcm : uint32_t { PC_NEXT = 0, PC_JUMP, PC_BRANCH, PC_RTS };
constexpr uint32_t D_BITF = 1u << 20, D_INV = 1u << 21, D_PF = 1u << 29, D_JSR = 1u << 30, D_BX = 1u << 31;
enum DAm : uint32_t { AM_NONE = 0, AM_IMM, AM_DIR, AM_ZPX, AM_ZPY, AM_ABX, AM_ABY, AM_INX, AM_INY, AM_PULL, AM_PUSH };
// flag masks in nes-py's layout
constexpr uint32_t PN = F_N, PV = F_V, PZ = F_Z, PC_ = F_C;

// Addressing-mode flags of word 0.
inline uint32_t dop_am(uint32_t am) {
    switch (am) {
        case AM_IMM: return D_IMM;
        case AM_ZPX: return D_IX | D_ZW;
        case AM_ZPY: return D_IY | D_ZW;
        case AM_ABX: return D_IX | D_CMPA;
        case AM_ABY: return D_IY | D_CMPA;
        case AM_INX: return D_IND | D_INX | D_CMPA;
        case AM_INY: return D_IND | D_IY | D_CMPA;
        case AM_PULL: return D_PULL;
        case AM_PUSH: return D_PUSH;
        default: return 0u;  // AM_NONE, AM_DIR (W is the address)
    }
}
inline uint32_t dop_x(uint32_t w, uint32_t am, uint32_t cyc, uint32_t len, bool pen) {
    return (w & 0xffffu) | ((cyc & 7u) << 16) | ((len & 3u) << 19) | (pen ? D_PEN : 0u) | dop_am(am) | D_OK;
}
inline uint32_t dop_y(uint32_t sel, uint32_t fmask, uint32_t cls, uint32_t lop, bool bitf, bool inv, uint32_t cin,
                      uint32_t dst, uint32_t pcm, bool pf, bool jsr, bool bx) {
    return (sel & 0xffu) | (fmask << 8) | (cls << 16) | (lop << 18) | (bitf ? D_BITF : 0u) | (inv ? D_INV : 0u) |
           (cin << 22) | (dst << 24) | (pcm << 27) | (pf ? D_PF : 0u) | (jsr ? D_JSR : 0u) | (bx ? D_BX : 0u);
}
inline uint32_t lr(uint32_t l, uint32_t r) { return l | (r << 4); }

// The datapath micro-op of the instruction the exact micro-op (ux, uy) at a PRG address describes
// (fme_tables.h build_uops). Not-OK dops leave the instruction to the exact path. Host only (build time).
inline uint2 make_dop(uint32_t ux, uint32_t uy) {
    const uint32_t hid = ux & 0xffu, pen = (ux >> 21) & 1u, len = (ux >> 22) & 3u;
    const uint32_t w = uy & 0xffffu, cyc = (uy >> 16) & 0xffu, extra = uy >> 24;
    uint2 d;
    d.x = 0u;  // not OK
    d.y = 0u;
    if ((ux & UOP_IDLE) || cyc < 1u || cyc > 7u) return d;
    // the read operations (R_ORA .. R_CPY)
    auto rd = [&](uint32_t op, uint32_t am, uint32_t wv) {
        static const uint8_t kCls[12] = {CL_LOGIC, CL_LOGIC, CL_LOGIC, CL_ADD, CL_LOGIC, CL_ADD, CL_ADD, CL_LOGIC,
                                         CL_LOGIC, CL_LOGIC, CL_ADD, CL_ADD};
        static const uint8_t kLop[12] = {LO_OR, LO_AND, LO_EOR, 0, LO_PASS, 0, 0, LO_AND, LO_PASS, LO_PASS, 0, 0};
        static const uint8_t kLs[12] = {B_A, B_A, B_A, B_A, B_A, B_A, B_A, B_A, B_A, B_A, B_X, B_Y};
        static const uint8_t kInv[12] = {0, 0, 0, 0, 0, 1, 1, 0, 0, 0, 1, 1};
        static const uint8_t kCin[12] = {CI_0, CI_0, CI_0, CI_C, CI_0, CI_1, CI_C, CI_0, CI_0, CI_0, CI_1, CI_1};
        static const uint8_t kDst[12] = {DS_A, DS_A, DS_A, DS_A, DS_A, DS_NONE, DS_A, DS_NONE, DS_X, DS_Y, DS_NONE,
                                         DS_NONE};
        static const uint8_t kFm[12] = {PN | PZ, PN | PZ, PN | PZ, PN | PZ | PC_ | PV, PN | PZ, PN | PZ | PC_,
                                        PN | PZ | PC_ | PV, PN | PZ | PV, PN | PZ, PN | PZ, PN | PZ | PC_, PN | PZ | PC_};
        d.x = dop_x(wv, am, cyc, len, pen != 0);
        d.y = dop_y(lr(kLs[op], B_M), kFm[op], kCls[op], kLop[op], op == R_BIT, kInv[op] != 0, kCin[op], kDst[op],
                    PC_NEXT, false, false, false);
    };
    auto st = [&](uint32_t op, uint32_t am, uint32_t wv) {  // W_STA / W_STX / W_STY
        d.x = dop_x(wv, am, cyc, len, pen != 0);
        d.y = dop_y(lr(B_A, op == W_STA ? B_A : op == W_STX ? B_X : B_Y), 0, CL_LOGIC, LO_PASS, false, false, CI_0,
                    DS_MEM, PC_NEXT, false, false, false);
    };
    auto rmw = [&](uint32_t op, uint32_t am, uint32_t wv, bool acc) {  // X_ASL .. X_INC on memory or A
        static const uint8_t kCls[6] = {CL_SHL, CL_SHL, CL_SHR, CL_SHR, CL_ADD, CL_ADD};
        static const uint8_t kRs[6] = {B_M, B_M, B_M, B_M, B_FF, B_ONE};
        static const uint8_t kCin[6] = {CI_0, CI_C, CI_0, CI_C, CI_0, CI_0};
        const uint32_t fm = op >= X_DEC ? (PN | PZ) : (PN | PZ | PC_);
        d.x = dop_x(wv, am, cyc, len, pen != 0);
        d.y = dop_y(lr(acc ? B_A : B_M, kRs[op]), fm, kCls[op], 0, false, false, kCin[op], acc ? DS_A : DS_MEM,
                    PC_NEXT, false, false, false);
    };
    if (hid >= H_X_RDIX && hid < H_X_RDIX + 12) { rd(hid - H_X_RDIX, AM_INX, w); return d; }
    if (hid >= H_X_RDIY && hid < H_X_RDIY + 12) { rd(hid - H_X_RDIY, AM_INY, w); return d; }
    if (hid >= H_X_RDAY && hid < H_X_RDAY + 12) { rd(hid - H_X_RDAY, AM_ABY, w); return d; }
    if (hid >= H_X_RDAX && hid < H_X_RDAX + 12) { rd(hid - H_X_RDAX, AM_ABX, w); return d; }
    if (hid >= H_X_RDZX && hid < H_X_RDZX + 12) { rd(hid - H_X_RDZX, AM_ZPX, w); return d; }
    if (hid >= H_X_RD && hid < H_X_RD + 12) { rd(hid - H_X_RD, AM_IMM, w); return d; }
    if (hid >= H_X_RD + 16 && hid < H_X_RD + 28) { rd(hid - H_X_RD - 16, AM_DIR, w); return d; }
    if (hid >= H_X_ST && hid < H_X_ST + 3) { st(hid - H_X_ST, AM_DIR, w); return d; }
    if (hid >= H_X_RMW && hid < H_X_RMW + 6) { rmw(hid - H_X_RMW, AM_DIR, w, false); return d; }
    if (hid >= H_X_ACC && hid < H_X_ACC + 6) { rmw(hid - H_X_ACC, AM_NONE, 0, true); return d; }
    const uint32_t op = (ux >> 16) & 31u;
    switch (hid) {
        case H_RD_ZPY: if (op < 12) rd(op, AM_ZPY, w); return d;
        case H_ST_ZPX: st(op, AM_ZPX, w); return d;
        case H_ST_ZPY: st(op, AM_ZPY, w); return d;
        case H_ST_ABSX: st(op, AM_ABX, w); return d;
        case H_ST_ABSY: st(op, AM_ABY, w); return d;
        case H_ST_INDX: st(op, AM_INX, w); return d;
        case H_ST_INDY: st(op, AM_INY, w); return d;
        case H_RMW_ZPX: if (op < 6) rmw(op, AM_ZPX, w, false); return d;
        case H_RMW_ABSX: if (op < 6) rmw(op, AM_ABX, w, false); return d;
        case H_NOPW:
            d.x = dop_x(0, AM_NONE, cyc, len, false);
            d.y = dop_y(lr(B_A, B_A), 0, CL_LOGIC, LO_PASS, false, false, CI_0, DS_NONE, PC_NEXT, false, false, false);
            return d;
        case H_BRANCH:
            d.x = dop_x(w, AM_NONE, cyc, len, false);
            d.y = dop_y((op & 7u) | (((op >> 3) & 1u) << 3), 0, CL_LOGIC, LO_PASS, false, false, CI_0, DS_NONE,
                        PC_BRANCH, false, false, extra > 1u);
            return d;
        default: break;
    }
    if (hid < H_X_IMPL || hid >= H_X_IMPL + 28) return d;  // exact path
    const uint32_t io = hid - H_X_IMPL;
    const uint32_t NZ = PN | PZ;
    auto impl = [&](uint32_t am, uint32_t y_) {
        d.x = dop_x(w, am, cyc, len, false);
        d.y = y_;
    };
    auto reg = [&](uint32_t cls, uint32_t ls, uint32_t rs, uint32_t dst, uint32_t fm) {
        impl(AM_NONE, dop_y(lr(ls, rs), fm, cls, LO_PASS, false, false, CI_0, dst, PC_NEXT, false, false, false));
    };
    auto flag = [&](uint32_t bit, uint32_t v) {
        impl(AM_NONE, dop_y(bit | (v << 3), 0, CL_LOGIC, LO_PASS, false, false, CI_0, DS_NONE, PC_NEXT, true, false,
                            false));
    };
    auto stk = [&](uint32_t am, uint32_t rs, uint32_t dst, uint32_t fm, uint32_t pcm, bool jsr) {
        impl(am, dop_y(lr(B_A, rs), fm, CL_LOGIC, LO_PASS, false, false, CI_0, dst, pcm, false, jsr, false));
    };
    switch (io) {
        case I_CLC: flag(7, 0); break;
        case I_JSR: stk(AM_NONE, B_A, DS_NONE, 0, PC_JUMP, true); break;
        case I_SEC: flag(7, 1); break;
        case I_PHA: stk(AM_PUSH, B_A, DS_MEM, 0, PC_NEXT, false); break;
        case I_PHP: stk(AM_PUSH, B_P, DS_MEM, 0, PC_NEXT, false); break;   // the status byte as stored
        case I_PLP: stk(AM_PULL, B_M, DS_P, 0, PC_NEXT, false); break;     // the pulled byte, unchanged
        case I_JMP: stk(AM_NONE, B_A, DS_NONE, 0, PC_JUMP, false); break;
        case I_CLI: flag(5, 0); break;
        case I_RTS: stk(AM_PULL, B_M, DS_NONE, 0, PC_RTS, false); break;
        case I_PLA: stk(AM_PULL, B_M, DS_A, NZ, PC_NEXT, false); break;
        case I_SEI: flag(5, 1); break;
        case I_DEY: reg(CL_ADD, B_Y, B_FF, DS_Y, NZ); break;
        case I_TXA: reg(CL_LOGIC, B_A, B_X, DS_A, NZ); break;
        case I_TYA: reg(CL_LOGIC, B_A, B_Y, DS_A, NZ); break;
        case I_TXS: reg(CL_LOGIC, B_A, B_X, DS_SP, 0); break;
        case I_TAY: reg(CL_LOGIC, B_A, B_A, DS_Y, NZ); break;
        case I_TAX: reg(CL_LOGIC, B_A, B_A, DS_X, NZ); break;
        case I_CLV: flag(1, 0); break;
        case I_TSX: reg(CL_LOGIC, B_A, B_SP, DS_X, NZ); break;
        case I_INY: reg(CL_ADD, B_Y, B_ONE, DS_Y, NZ); break;
        case I_DEX: reg(CL_ADD, B_X, B_FF, DS_X, NZ); break;
        case I_CLD: flag(4, 0); break;
        case I_INX: reg(CL_ADD, B_X, B_ONE, DS_X, NZ); break;
        case I_NOP: stk(AM_NONE, B_A, DS_NONE, 0, PC_NEXT, false); break;
        case I_SED: flag(4, 1); break;
        default: break;  // BRK, RTI, JMP (ind): exact path
    }
    return d;
}

// A, X, Y and SP as the bytes of one word (the datapath's register file) and back.
FME_HD void rf_pack(Hot& h) { h.rf = h.a | (h.x << 8) | (h.y << 16) | (h.sp << 24); }
FME_HD void rf_unpack(Hot& h) {
    h.a = h.rf & 0xffu; h.x = (h.rf >> 8) & 0xffu; h.y = (h.rf >> 16) & 0xffu; h.sp = h.rf >> 24;
}
// Bytes (s & 7) and ((s >> 4) & 7) of the 8-byte value hi:lo as bytes 0 and 1 of the result (upper bytes
// unspecified): the device's byte permute with the selector taken from the micro-op.
FME_HD uint32_t byte_sel2(uint32_t lo, uint32_t hi, uint32_t s) {
#if defined(__CUDA_ARCH__)
    return __byte_perm(lo, hi, s);
#else
    const uint64_t v = ((uint64_t)hi << 32) | lo;
    return (uint32_t)((v >> (8u * (s & 7u))) & 0xffu) | ((uint32_t)((v >> (8u * ((s >> 4) & 7u))) & 0xffu) << 8);
#endif
}

FME_HD uint2 dop_load(const uint32_t* dops, uint32_t pc) {
    const uint32_t i = pc & 0x7fffu;
#if defined(__CUDA_ARCH__)
    uint2 u = __ldg(reinterpret_cast<const uint2*>(dops) + i);
#else
    uint2 u;
    u.x = dops[2 * i]; u.y = dops[2 * i + 1];
#endif
    if (pc < 0x8000u) { u.x = 0u; u.y = 0u; }   // code outside PRG: the exact path
    return u;
}
// Datapath micro-op of the lane's pc into h.ux / h.uy (in the datapath loop they hold the dop; the exact path
// fetches its own micro-op before it runs).
FME_HD void dfetch(Hot& h, const uint32_t* dops) {
    const uint2 u = dop_load(dops, h.pc);
    h.ux = u.x; h.uy = u.y;
}

// Run limit of the datapath for the lane's current timing state: it may run the instruction at exec_at J while
// J < lim, i.e. before the frame end and with no PPU catch-up or NMI due (3 (J + 1) < nmi_thresh, the test of
// hot_step's common case). Recomputed whenever the exact path has run (it moves the threshold).
FME_HD int32_t dp_limit(const Hot& h) {
    const int32_t t = h.thresh >= 3 ? (h.thresh - 1) / 3 : 0;
    return t < FRAME_ITERS ? t : FRAME_ITERS;
}
FME_HD bool dp_ready(const Hot& h, int32_t lim) { return (h.ux & D_OK) && h.exec_at < lim; }

// Execute the instruction at h.pc from its dop (h.ux, h.uy; registers in h.rf) and load the dop of the next
// pc, if `run`. Every lane of a warp evaluates the same straight-line code whatever its instruction (a lane
// that does not run computes on its current dop and commits nothing): all state updates and memory writes
// are predicated, so the whole instruction is one block of code the compiler can schedule freely. Returns
// whether the instruction was committed; false with `run` means a computed address is an I/O address (the
// exact path must run it) and nothing was changed.
FME_HD bool dp_exec(Hot& h, const Fast& f, const uint32_t* dops, bool run = true) {
    const uint32_t dx = h.ux, dy = h.uy, rf = h.rf, P = h.p;
    const uint32_t W = dx & 0xffffu;
    const uint32_t X = (rf >> 8) & 0xffu, SP = rf >> 24;
    // the two pre-reads: the pointer of (zp,X) / (zp),Y, or the two bytes above the stack pointer
    const bool pull = (dx & D_PULL) != 0u;
    const uint32_t zb = (W + ((dx & D_INX) ? X : 0u)) & 0xffu;
    const uint32_t a0 = pull ? (0x100u | ((SP + 1u) & 0xffu)) : zb;
    const uint32_t a1 = pull ? (0x100u | ((SP + 2u) & 0xffu)) : ((zb + 1u) & 0xffu);
    const uint32_t p0 = f.Rz(a0), p1 = f.Rz(a1);
    const uint32_t ptr = p0 | (p1 << 8);
    // next pc, and its dop loaded right away (branches test the flags before this instruction)
    const uint32_t pcm = (dy >> 27) & 3u;
    const uint32_t npc = (h.pc + ((dx >> 19) & 3u)) & 0xffffu;
    const bool taken = pcm == PC_BRANCH && ((P >> (dy & 7u)) & 1u) == ((dy >> 3) & 1u);
    const uint32_t pc = (pcm == PC_JUMP || taken) ? W : pcm == PC_RTS ? ((ptr + 1u) & 0xffffu) : npc;
    const uint2 nd = dop_load(dops, pc);
    // effective address; the RAM and the PRG byte there are both read (one of them may be the operand)
    const uint32_t idx = (dx & D_IX) ? X : (dx & D_IY) ? ((rf >> 16) & 0xffu) : 0u;
    const uint32_t base = (dx & D_IND) ? ptr : (dx & D_PUSH) ? (0x100u | SP) : W;
    const uint32_t ea = (base + idx) & ((dx & D_ZW) ? 0xffu : 0xffffu);
    const bool cmpa = (dx & D_CMPA) != 0u;
    const bool ok = run && !(cmpa && Fast::io(ea));
    const uint32_t mram = f.R(ea), mrom = f.P(ea);
    // operand: immediate, pulled byte, or memory (a ROM byte only at a computed address: static ROM operands
    // are immediates by now)
    const uint32_t m = (dx & D_IMM) ? W : pull ? p0 : (cmpa && ea >= 0x8000u) ? mrom : mram;
    // ALU: L and R are bytes of {A, X, Y, SP, M, 1, $FF, P}
    const uint32_t ops = byte_sel2(rf, m | 0x00ff0100u | (P << 24), dy);
    const uint32_t L = ops & 0xffu, R = (ops >> 8) & 0xffu;
    const uint32_t Ri = R ^ ((dy & D_INV) ? 0xffu : 0u);
    const uint32_t cm = (dy >> 22) & 3u;
    const uint32_t cin = cm == CI_C ? (P >> 7) : cm;
    const uint32_t sum = L + Ri + cin;
    const uint32_t lop = (dy >> 18) & 3u, cls = (dy >> 16) & 3u;
    const uint32_t rl = (lop & 2u) ? ((lop & 1u) ? (L ^ R) : (L & R)) : ((lop & 1u) ? (L | R) : R);
    const uint32_t r = (cls & 2u) ? ((cls & 1u) ? ((L >> 1) | (cin << 7)) : (((L << 1) | cin) & 0xffu))
                                  : ((cls & 1u) ? (sum & 0xffu) : rl);
    const uint32_t cout = (cls & 2u) ? ((cls & 1u) ? L : (L >> 7)) : (sum >> 8);
    // flags in nes-py's layout (N bit 0, V bit 1, Z bit 6, C bit 7); BIT takes N and V from the operand
    const bool bitf = (dy & D_BITF) != 0u;
    const uint32_t nf = bitf ? ((R >> 7) & 1u) : ((r >> 7) & 1u);
    const uint32_t vf = bitf ? ((R >> 6) & 1u) : ((((L ^ sum) & (Ri ^ sum)) >> 7) & 1u);
    const uint32_t fl = nf | (vf << 1) | (r == 0u ? PZ : 0u) | ((cout & 1u) << 7);
    const uint32_t fmask = (dy >> 8) & 0xffu;
    const uint32_t bitm = (dy & D_PF) ? (1u << (dy & 7u)) : 0u;   // flag set / clear (bit index and value
    const uint32_t p = (((P & ~fmask) | (fl & fmask)) & ~bitm) | ((dy & 8u) ? bitm : 0u);  // in the select byte)
    // cycles (the (zp,X) penalty tests the address's own high byte)
    const uint32_t penb = (dx & D_INX) ? 0u : base;
    const int32_t S = (int32_t)((dx >> 16) & 7u) + (((dx & D_PEN) && cmpa && ((penb ^ ea) & 0xff00u)) ? 1 : 0) +
                      (taken ? ((dy & D_BX) ? 3 : 1) : 0);
    // memory writes (RAM only; writes into ROM are ignored)
    const uint32_t dst = (dy >> 24) & 7u;
    const bool jsr = (dy & D_JSR) != 0u;
    if (ok && dst == DS_MEM && ea < 0x2000u) f.W(ea, r);
    const uint32_t ret = (npc + 1u) & 0xffffu;
    if (ok && jsr) f.Wz(0x100u | SP, ret >> 8);
    if (ok && jsr) f.Wz(0x100u | ((SP - 1u) & 0xffu), ret & 0xffu);
    // registers: the destination byte of the register file, then the stack pointer change in its top byte
    const uint32_t sh = 8u * ((dst - DS_A) & 3u);
    const uint32_t nrf = (dst >= DS_A && dst <= DS_SP) ? ((rf & ~(0xffu << sh)) | (r << sh)) : rf;
    const uint32_t spd = (dx & D_PUSH) ? 0xffu : jsr ? 0xfeu : pull ? (pcm == PC_RTS ? 2u : 1u) : 0u;
    h.rf = ok ? nrf + (spd << 24) : rf;
    h.p = ok ? (dst == DS_P ? r : p) : P;   // PLP loads the status byte whole
    h.pc = ok ? pc : h.pc;
    h.ux = ok ? nd.x : dx;
    h.uy = ok ? nd.y : dy;
    h.exec_at += ok ? S : 0;      // datapath instructions take 2..7 cycles, so the exact path's max(S, 1) is S
    h.zero_skip = ok ? 0u : h.zero_skip;   // and its zero-skip flag (S <= 0) is clear
    h.icount += ok ? 1u : 0u;
    return ok;
}

// One scheduling unit of one lane: its next instruction in the datapath when it can run there, else the exact
// path (hot_step). This is what the kernels' two-phase warp loop does for each lane, written for one lane (the
// host build of the engine steps consoles with it). On entry and return h.ux/h.uy hold the dop of h.pc and
// h.rf the registers. Returns false at the frame end, with nothing changed.
FME_HD bool lane_step(Hot& h, Core& c, const Fast& f, const uint32_t* dops) {
    if (dp_ready(h, dp_limit(h)) && dp_exec(h, f, dops)) return true;
    rf_unpack(h);
    fetch(h, f);
    const bool more = hot_step(h, c, f);
    rf_pack(h);
    dfetch(h, dops);
    return more;
}

}  // namespace fme
