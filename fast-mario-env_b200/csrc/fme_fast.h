// fme_fast.h - register-resident fast path of the 6502 interpreter.
//
// The full console (`Core`, fme_core.h) is the exact model; its I/O, PPU and NMI code is large and rarely
// needed per instruction. Keeping the whole object in registers is not possible once that code is out of
// line, so the loop works on `Hot`: the 6502 registers, the frame clock and the NMI threshold, held by value
// (its address is never taken, so it stays in registers). Instructions are executed from per-PC micro-ops
// built once per ROM (fme_tables.h build_uops): every instruction whose memory accesses are RAM or PRG only
// runs here with the semantics of Core::execute_op (nes_core.hpp:645-1163); an instruction that would touch
// $2000-$7FFF (PPU registers, joypads, OAM DMA), or code outside PRG, is handed to the exact Core path with
// Hot written back first. Nothing here has side effects before that decision.
#pragma once
#include "fme_core.h"

namespace fme {

struct Hot {
    uint32_t pc, a, x, y, sp, p;
    int32_t exec_at, thresh;
    uint32_t zero_skip, bad;
    uint32_t ux, uy;  // micro-op of the instruction at pc (fme_defs.h); zero outside PRG
    uint32_t icount;  // instructions executed since hot_init (emulated-work counter)
    uint32_t rf;      // A | X<<8 | Y<<16 | SP<<24 while the datapath (fme_dp.h) owns the registers
};

// Exact slow paths (the Core methods), out of line so the hot loop stays small.
FME_NI void slow_presync(Core& c, int32_t J) {
    c.cur = J;
    c.sync_to(3 * (J + 1));
}
FME_NI int32_t slow_execute(Core& c, int32_t J, uint32_t opc) {
    c.cur = J;
    const int32_t D = (opc == 0x2Cu || opc == 0xADu) ? c.poll_skip(J, opc) : 0;  // sets cur = J + D
    return D + (opc <= 0xffu ? c.execute_op(opc) : c.execute_op(c.rd(c.pc)));
}

struct Fast {
    uint8_t* ram;            // lane base of the RAM slab
    uint8_t* ramh;           // lane base for addresses >= ram_end
    uint32_t ram_end;
    const uint8_t* prg;
    const uint32_t* uop;     // per-PC micro-ops, 2 words per address $8000-$FFFF

    FME_HD uint32_t P(uint32_t a) const { return FME_LDG(prg + (a & 0x7fffu)); }
    FME_HD uint8_t* at(uint32_t a) const {
        const uint32_t m = a & 0x7ffu;
        return (m < ram_end ? ram : ramh) + il(m);
    }
    FME_HD uint32_t R(uint32_t a) const { return *at(a); }
    FME_HD void W(uint32_t a, uint32_t v) const { *at(a) = (uint8_t)v; }
    // zero page and stack ($0000-$01FF, below every boundary): no base select
    FME_HD uint32_t Rz(uint32_t a) const { return ram[il(a & 0x1ffu)]; }
    FME_HD void Wz(uint32_t a, uint32_t v) const { ram[il(a & 0x1ffu)] = (uint8_t)v; }
    // side-effect-free read of an address outside $2000-$7FFF
    FME_HD uint32_t M(uint32_t a) const { return a >= 0x8000u ? P(a) : R(a); }
    FME_HD static bool io(uint32_t a) { return a >= 0x2000u && a < 0x8000u; }
    // micro-op of PRG address pc (masked like every PRG access, so any pc indexes inside the table)
    FME_HD uint2 U(uint32_t pc) const {
        const uint32_t i = pc & 0x7fffu;
#if defined(__CUDA_ARCH__)
        return __ldg(reinterpret_cast<const uint2*>(uop) + i);
#else
        uint2 u;
        u.x = uop[2 * i]; u.y = uop[2 * i + 1];
        return u;
#endif
    }

    FME_HD static void zn(Hot& h, uint32_t v) {
        v &= 0xffu;
        h.p = (h.p & ~(F_Z | F_N)) | (v ? 0u : F_Z) | ((v & 0x80u) ? F_N : 0u);
    }
    FME_HD static void setf(Hot& h, uint32_t f, bool on) { h.p = on ? (h.p | f) : (h.p & ~f); }

    FME_HD static void alu_read(Hot& h, uint32_t op, uint32_t m) {
        switch (op) {
            case R_ORA: h.a |= m; zn(h, h.a); break;
            case R_AND: h.a &= m; zn(h, h.a); break;
            case R_EOR: h.a ^= m; zn(h, h.a); break;
            case R_ADC: {
                uint32_t sum = h.a + m + ((h.p & F_C) ? 1u : 0u);
                setf(h, F_C, sum & 0x100u);
                setf(h, F_V, (h.a ^ sum) & (m ^ sum) & 0x80u);
                h.a = sum & 0xffu; zn(h, h.a);
                break;
            }
            case R_LDA: h.a = m; zn(h, h.a); break;
            case R_CMP: { uint32_t t = (h.a - m) & 0xffffu; setf(h, F_C, !(t & 0x100u)); zn(h, t); break; }
            case R_SBC: {
                uint32_t t = (h.a - m - ((h.p & F_C) ? 0u : 1u)) & 0xffffu;
                setf(h, F_C, !(t & 0x100u));
                setf(h, F_V, (h.a ^ t) & (~m ^ t) & 0x80u);
                h.a = t & 0xffu; zn(h, t);
                break;
            }
            case R_BIT: setf(h, F_Z, !(h.a & m)); setf(h, F_V, m & 0x40u); setf(h, F_N, m & 0x80u); break;
            case R_LDX: h.x = m; zn(h, h.x); break;
            case R_LDY: h.y = m; zn(h, h.y); break;
            case R_CPX: { uint32_t t = (h.x - m) & 0xffffu; setf(h, F_C, !(t & 0x100u)); zn(h, t); break; }
            default:    { uint32_t t = (h.y - m) & 0xffffu; setf(h, F_C, !(t & 0x100u)); zn(h, t); break; }
        }
    }
    FME_HD static uint32_t alu_rmw(Hot& h, uint32_t op, uint32_t m) {
        const uint32_t c = (h.p & F_C) ? 1u : 0u;
        switch (op) {
            case X_ASL: setf(h, F_C, m & 0x80u); m = (m << 1) & 0xffu; break;
            case X_ROL: setf(h, F_C, m & 0x80u); m = ((m << 1) | c) & 0xffu; break;
            case X_LSR: setf(h, F_C, m & 1u); m >>= 1; break;
            case X_ROR: setf(h, F_C, m & 1u); m = (m >> 1) | (c << 7); break;
            case X_DEC: m = (m - 1) & 0xffu; break;
            default: m = (m + 1) & 0xffu; break;
        }
        zn(h, m);
        return m;
    }

    // Execute the instruction at h.pc from its micro-op (h.ux, h.uy; not H_SLOW) with the semantics of
    // Core::execute_op. Returns the skip-cycle count, or -1 if a computed address is an I/O address and the
    // exact path must run it instead (nothing was changed then).
    FME_HD int32_t exec(Hot& h) const {
        const uint32_t hid = h.ux & 0xffu, op = (h.ux >> 16) & 31u, pen = (h.ux >> 21) & 1u;
        const uint32_t w = h.uy & 0xffffu;
        int32_t skip = (int32_t)((h.uy >> 16) & 0xffu);
        uint32_t npc = (h.pc + ((h.ux >> 22) & 3u)) & 0xffffu;
        uint32_t loc = 0, base = 0;
        int cls = 3;  // 0 read m, 1 store to loc, 2 read-modify-write loc, 3 done
        uint32_t m = 0;
        switch (hid) {
#define FME_X_RD(OP)                                                                          \
            case H_X_RD + OP: alu_read(h, OP, w); h.pc = npc; return skip;                    \
            case H_X_RD + 16 + OP: alu_read(h, OP, R(w)); h.pc = npc; return skip;
            FME_X_RD(R_ORA) FME_X_RD(R_AND) FME_X_RD(R_EOR) FME_X_RD(R_ADC) FME_X_RD(R_LDA) FME_X_RD(R_CMP)
            FME_X_RD(R_SBC) FME_X_RD(R_BIT) FME_X_RD(R_LDX) FME_X_RD(R_LDY) FME_X_RD(R_CPX) FME_X_RD(R_CPY)
#undef FME_X_RD
#define FME_X_RDI(OP)                                                                                          \
            case H_X_RDZX + OP: alu_read(h, OP, R((w + h.x) & 0xffu)); h.pc = npc; return skip;                \
            case H_X_RDAX + OP: {                                                                              \
                const uint32_t l = (w + h.x) & 0xffffu;                                                        \
                if (io(l)) return -1;                                                                          \
                if (pen && ((w ^ l) & 0xff00u)) skip += 1;                                                     \
                alu_read(h, OP, M(l)); h.pc = npc; return skip;                                                \
            }                                                                                                  \
            case H_X_RDAY + OP: {                                                                              \
                const uint32_t l = (w + h.y) & 0xffffu;                                                        \
                if (io(l)) return -1;                                                                          \
                if (pen && ((w ^ l) & 0xff00u)) skip += 1;                                                     \
                alu_read(h, OP, M(l)); h.pc = npc; return skip;                                                \
            }                                                                                                  \
            case H_X_RDIY + OP: {                                                                              \
                const uint32_t b = R(w) | (R((w + 1) & 0xffu) << 8), l = (b + h.y) & 0xffffu;                  \
                if (io(l)) return -1;                                                                          \
                if (pen && ((b ^ l) & 0xff00u)) skip += 1;                                                     \
                alu_read(h, OP, M(l)); h.pc = npc; return skip;                                                \
            }                                                                                                  \
            case H_X_RDIX + OP: {                                                                              \
                const uint32_t za = (h.x + w) & 0xffu, l = R(za) | (R((za + 1) & 0xffu) << 8);                 \
                if (io(l)) return -1;                                                                          \
                if (pen && (l & 0xff00u)) skip += 1;                                                           \
                alu_read(h, OP, M(l)); h.pc = npc; return skip;                                                \
            }
            FME_X_RDI(R_ORA) FME_X_RDI(R_AND) FME_X_RDI(R_EOR) FME_X_RDI(R_ADC) FME_X_RDI(R_LDA) FME_X_RDI(R_CMP)
            FME_X_RDI(R_SBC) FME_X_RDI(R_BIT) FME_X_RDI(R_LDX) FME_X_RDI(R_LDY) FME_X_RDI(R_CPX) FME_X_RDI(R_CPY)
#undef FME_X_RDI
            case H_X_ST + W_STA: W(w, h.a); h.pc = npc; return skip;
            case H_X_ST + W_STX: W(w, h.x); h.pc = npc; return skip;
            case H_X_ST + W_STY: W(w, h.y); h.pc = npc; return skip;
#define FME_X_RMW(OP)                                                                         \
            case H_X_RMW + OP: W(w, alu_rmw(h, OP, R(w))); h.pc = npc; return skip;           \
            case H_X_ACC + OP: h.a = alu_rmw(h, OP, h.a); h.pc = npc; return skip;
            FME_X_RMW(X_ASL) FME_X_RMW(X_ROL) FME_X_RMW(X_LSR) FME_X_RMW(X_ROR) FME_X_RMW(X_DEC) FME_X_RMW(X_INC)
#undef FME_X_RMW
            case H_X_IMPL + I_BRK: {
                uint32_t r = npc + 1;  // BRK skips its padding byte
                W(0x100u | h.sp, (r >> 8) & 0xffu); h.sp = (h.sp - 1) & 0xffu;
                W(0x100u | h.sp, r & 0xffu); h.sp = (h.sp - 1) & 0xffu;
                W(0x100u | h.sp, h.p | 0x30u); h.sp = (h.sp - 1) & 0xffu;
                h.p |= F_I;
                h.pc = P(0xfffe) | (P(0xffff) << 8);
                return skip + 7;
            }
            case H_X_IMPL + I_PHP: W(0x100u | h.sp, h.p); h.sp = (h.sp - 1) & 0xffu; h.pc = npc; return skip;
            case H_X_IMPL + I_CLC: setf(h, F_C, false); h.pc = npc; return skip;
            case H_X_IMPL + I_JSR: {
                uint32_t r = (npc + 1) & 0x1ffffu;
                W(0x100u | h.sp, (r >> 8) & 0xffu); h.sp = (h.sp - 1) & 0xffu;
                W(0x100u | h.sp, r & 0xffu); h.sp = (h.sp - 1) & 0xffu;
                h.pc = w;
                return skip;
            }
            case H_X_IMPL + I_PLP: h.sp = (h.sp + 1) & 0xffu; h.p = R(0x100u | h.sp); h.pc = npc; return skip;
            case H_X_IMPL + I_SEC: setf(h, F_C, true); h.pc = npc; return skip;
            case H_X_IMPL + I_RTI: {
                h.sp = (h.sp + 1) & 0xffu; h.p = R(0x100u | h.sp);
                h.sp = (h.sp + 1) & 0xffu; uint32_t lo = R(0x100u | h.sp);
                h.sp = (h.sp + 1) & 0xffu; h.pc = lo | (R(0x100u | h.sp) << 8);
                return skip;
            }
            case H_X_IMPL + I_PHA: W(0x100u | h.sp, h.a); h.sp = (h.sp - 1) & 0xffu; h.pc = npc; return skip;
            case H_X_IMPL + I_JMP: h.pc = w; return skip;
            case H_X_IMPL + I_CLI: setf(h, F_I, false); h.pc = npc; return skip;
            case H_X_IMPL + I_RTS: {
                h.sp = (h.sp + 1) & 0xffu; uint32_t lo = R(0x100u | h.sp);
                h.sp = (h.sp + 1) & 0xffu; h.pc = ((lo | (R(0x100u | h.sp) << 8)) + 1) & 0xffffu;
                return skip;
            }
            case H_X_IMPL + I_PLA: h.sp = (h.sp + 1) & 0xffu; h.a = R(0x100u | h.sp); zn(h, h.a); h.pc = npc; return skip;
            case H_X_IMPL + I_JMPI: {  // the builder routed I/O pointer addresses to the exact path
                const uint32_t hiad = (w & 0xff00u) | ((w + 1) & 0xffu);
                h.pc = M(w) | (M(hiad) << 8);
                return skip;
            }
            case H_X_IMPL + I_SEI: setf(h, F_I, true); h.pc = npc; return skip;
            case H_X_IMPL + I_DEY: h.y = (h.y - 1) & 0xffu; zn(h, h.y); h.pc = npc; return skip;
            case H_X_IMPL + I_TXA: h.a = h.x; zn(h, h.a); h.pc = npc; return skip;
            case H_X_IMPL + I_TYA: h.a = h.y; zn(h, h.a); h.pc = npc; return skip;
            case H_X_IMPL + I_TXS: h.sp = h.x; h.pc = npc; return skip;
            case H_X_IMPL + I_TAY: h.y = h.a; zn(h, h.y); h.pc = npc; return skip;
            case H_X_IMPL + I_TAX: h.x = h.a; zn(h, h.x); h.pc = npc; return skip;
            case H_X_IMPL + I_CLV: setf(h, F_V, false); h.pc = npc; return skip;
            case H_X_IMPL + I_TSX: h.x = h.sp; zn(h, h.x); h.pc = npc; return skip;
            case H_X_IMPL + I_INY: h.y = (h.y + 1) & 0xffu; zn(h, h.y); h.pc = npc; return skip;
            case H_X_IMPL + I_DEX: h.x = (h.x - 1) & 0xffu; zn(h, h.x); h.pc = npc; return skip;
            case H_X_IMPL + I_CLD: setf(h, F_D, false); h.pc = npc; return skip;
            case H_X_IMPL + I_INX: h.x = (h.x + 1) & 0xffu; zn(h, h.x); h.pc = npc; return skip;
            case H_X_IMPL + I_NOP: h.pc = npc; return skip;
            case H_X_IMPL + I_SED: setf(h, F_D, true); h.pc = npc; return skip;
            // indexed and indirect forms: address first (I/O check below), then the operation
            case H_RD_ZPY: m = R((w + h.y) & 0xffu); cls = 0; break;
            case H_ST_ZPX: loc = (w + h.x) & 0xffu; cls = 1; break;
            case H_ST_ZPY: loc = (w + h.y) & 0xffu; cls = 1; break;
            case H_ST_ABSX: base = w; loc = (w + h.x) & 0xffffu; cls = 5; break;
            case H_ST_ABSY: base = w; loc = (w + h.y) & 0xffffu; cls = 5; break;
            case H_ST_INDX: { const uint32_t za = (h.x + w) & 0xffu; loc = R(za) | (R((za + 1) & 0xffu) << 8); cls = 5; break; }
            case H_ST_INDY: base = R(w) | (R((w + 1) & 0xffu) << 8); loc = (base + h.y) & 0xffffu; cls = 5; break;
            case H_NOPW: break;
            case H_RMW_ZPX: loc = (w + h.x) & 0xffu; cls = 2; break;
            case H_RMW_ABSX: base = w; loc = (w + h.x) & 0xffffu; cls = 6; break;
            case H_BRANCH:
                if (((h.p >> (op & 7u)) & 1u) == ((op >> 3) & 1u)) { skip += (int32_t)(h.uy >> 24); npc = w; }
                break;
            case H_JOY_RD: case H_JOY_ST: return -1;  // hot_step's controller path
            case H_BAD_ABSX:
                if (((w + h.x) ^ w) & 0xff00u) skip += 1;
                h.bad++;
                break;
            default: h.bad++; break;  // H_BAD
        }
        if (cls >= 4) {  // computed address: I/O goes to the exact path, then the page-cross penalty
            if (io(loc)) return -1;
            if (pen && ((base ^ loc) & 0xff00u)) skip += 1;
            cls -= 4;
            if (cls == 0) m = M(loc);
        }
        if (cls == 0) {
            alu_read(h, op, m);
        } else if (cls == 1) {
            if (loc < 0x2000u) W(loc, op == W_STA ? h.a : op == W_STX ? h.x : h.y);  // ROM writes are ignored
        } else if (cls == 2) {
            const uint32_t r = alu_rmw(h, op, M(loc));
            if (loc < 0x2000u) W(loc, r);
        }
        h.pc = npc;
        return skip;
    }
};

// Micro-op of the instruction at the new pc: the next iteration's scheduler vote, idle test and decode
// read it, so the load overlaps the loop head instead of following it.
FME_HD void fetch(Hot& h, const Fast& f) {
    if (h.pc >= 0x8000u) { const uint2 u = f.U(h.pc); h.ux = u.x; h.uy = u.y; }
    else { h.ux = 0u; h.uy = 0u; }
}
FME_HD bool idle_loop(const Hot& h) { return (h.ux & UOP_IDLE) != 0u; }  // `JMP *` (rd_prg_fast bytes)
FME_HD void hot_out(const Hot& h, Core& c) {
    c.pc = h.pc; c.a = h.a; c.x = h.x; c.y = h.y; c.sp = h.sp; c.p = h.p;
    c.exec_at = h.exec_at; c.nmi_thresh = h.thresh; c.zero_skip = h.zero_skip != 0; c.bad_ops = h.bad;
}
FME_HD void hot_in(Hot& h, const Core& c, const Fast& f) {
    h.pc = c.pc; h.a = c.a; h.x = c.x; h.y = c.y; h.sp = c.sp; h.p = c.p;
    h.exec_at = c.exec_at; h.thresh = c.nmi_thresh; h.zero_skip = c.zero_skip ? 1u : 0u; h.bad = c.bad_ops;
    fetch(h, f);
}

// Controller port access (Core::joy_read and the $4016 strobe of Core::wr_io): the only console state it
// touches is the controller's, which Hot does not hold, so the registers stay in Hot.
FME_HD int32_t joy_exec(Hot& h, Core& c) {
    const uint32_t op = (h.ux >> 16) & 31u;
    if ((h.ux & 0xffu) == H_JOY_RD) {
        Fast::alu_read(h, op, c.joy_read((int)(h.uy & 1u)));
    } else {
        const uint32_t v = op == W_STA ? h.a : op == W_STX ? h.x : h.y;
        for (int i = 0; i < 2; i++) {
            c.joy_strobe[i] = v & 1u;
            if (!c.joy_strobe[i]) c.joy_bits[i] = c.joy_buttons[i];
        }
    }
    h.pc = (h.pc + 3u) & 0xffffu;
    return (int32_t)((h.uy >> 16) & 0xffu);
}

// One scheduling unit of the frame loop (the body of nes_core.hpp:1169-1201) on the register state.
// Returns false when exec_at reached the frame end (the caller then runs Core::end_frame via hot_out).
FME_HD bool hot_step(Hot& h, Core& c, const Fast& f) {
    const int32_t J = h.exec_at;
    if (J >= FRAME_ITERS) return false;
    int32_t S;
    // common case, tested with one branch: no PPU catch-up due, no idle loop, a fast-path micro-op
    const bool common = (3 * (J + 1) < h.thresh) & ((h.ux & UOP_IDLE) == 0u) & ((h.ux & 0xffu) != H_SLOW);
    if (common) {
        S = f.exec(h);
    } else {
        if (3 * (J + 1) >= h.thresh) {
            hot_out(h, c);
            slow_presync(c, J);
            hot_in(h, c, f);
            if (h.exec_at != J) return true;  // an NMI was taken before this instruction
        }
        // idle-loop test with rd_prg_fast semantics (0xff outside PRG, nes_core.hpp:153, 1178)
        if (idle_loop(h)) {
            int32_t lim_end = FRAME_ITERS - J;
            int32_t lim_nmi = h.thresh - 3 * (J + 1);
            int32_t k1 = lim_end > 0 ? (lim_end + 2) / 3 : 0;
            int32_t k2 = lim_nmi > 0 ? (lim_nmi + 8) / 9 : 0;
            int32_t k = k1 < k2 ? k1 : k2;
            if (k > 1) {
                h.exec_at = J + 3 * (k - 1);
                h.zero_skip = 0;
                return true;
            }
        }
        S = (h.ux & 0xffu) != H_SLOW ? f.exec(h) : -1;
    }
    if (S < 0 && ((h.ux & 0xffu) == H_JOY_RD || (h.ux & 0xffu) == H_JOY_ST)) {
        S = joy_exec(h, c);
        fetch(h, f);
    } else if (S < 0) {
        const uint32_t opc = h.pc >= 0x8000u ? (h.ux >> 8) & 0xffu : 0x100u;
        hot_out(h, c);
        S = slow_execute(c, J, opc);
        hot_in(h, c, f);
    } else {
        fetch(h, f);
    }
    h.exec_at = J + (S >= 1 ? S : 1);
    h.zero_skip = S <= 0 ? 1u : 0u;
    h.icount++;
    return true;
}

}  // namespace fme
