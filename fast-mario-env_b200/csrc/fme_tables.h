// fme_tables.h - host-side constant tables: nes-py's cycle table and palette, SIMPLE_MOVEMENT, the opcode
// decode table (nes-py's decode cascade evaluated once per opcode) and OpenCV's area-resize taps.
#pragma once
#include <math.h>
#include <string.h>
#include <algorithm>
#include <vector>
#include "fme_defs.h"
#include "fme_render.h"
#include "fme_dp.h"

namespace fme {
namespace tables {

// nes-py's per-opcode base cycle table (OPERATION_CYCLES); 0 for opcodes nes-py does not time.
static const uint8_t kCycles[256] = {
    7, 6, 0, 0, 0, 3, 5, 0, 3, 2, 2, 0, 0, 4, 6, 0, 2, 5, 0, 0, 0, 4, 6, 0, 2, 4, 0, 0, 0, 4, 7, 0,
    6, 6, 0, 0, 3, 3, 5, 0, 4, 2, 2, 0, 4, 4, 6, 0, 2, 5, 0, 0, 0, 4, 6, 0, 2, 4, 0, 0, 0, 4, 7, 0,
    6, 6, 0, 0, 0, 3, 5, 0, 3, 2, 2, 0, 3, 4, 6, 0, 2, 5, 0, 0, 0, 4, 6, 0, 2, 4, 0, 0, 0, 4, 7, 0,
    6, 6, 0, 0, 0, 3, 5, 0, 4, 2, 2, 0, 5, 4, 6, 0, 2, 5, 0, 0, 0, 4, 6, 0, 2, 4, 0, 0, 0, 4, 7, 0,
    0, 6, 0, 0, 3, 3, 3, 0, 2, 0, 2, 0, 4, 4, 4, 0, 2, 6, 0, 0, 4, 4, 4, 0, 2, 5, 2, 0, 0, 5, 0, 0,
    2, 6, 2, 0, 3, 3, 3, 0, 2, 2, 2, 0, 4, 4, 4, 0, 2, 5, 0, 0, 4, 4, 4, 0, 2, 4, 2, 0, 4, 4, 4, 0,
    2, 6, 0, 0, 3, 3, 5, 0, 2, 2, 2, 0, 4, 4, 6, 0, 2, 5, 0, 0, 0, 4, 6, 0, 2, 4, 0, 0, 0, 4, 7, 0,
    2, 6, 0, 0, 3, 3, 5, 0, 2, 2, 2, 2, 4, 4, 6, 0, 2, 5, 0, 0, 0, 4, 6, 0, 2, 4, 0, 0, 0, 4, 7, 0,
};

// nes-py master palette (0xRRGGBB)
static const uint32_t kPalette[64] = {
    0x7C7C7C, 0x0000FC, 0x0000BC, 0x4428BC, 0x940084, 0xA80020, 0xA81000, 0x881400,
    0x503000, 0x007800, 0x006800, 0x005800, 0x004058, 0x000000, 0x000000, 0x000000,
    0xBCBCBC, 0x0078F8, 0x0058F8, 0x6844FC, 0xD800CC, 0xE40058, 0xF83800, 0xE45C10,
    0xAC7C00, 0x00B800, 0x00A800, 0x00A844, 0x008888, 0x000000, 0x000000, 0x000000,
    0xF8F8F8, 0x3CBCFC, 0x6888FC, 0x9878F8, 0xF878F8, 0xF85898, 0xF87858, 0xFCA044,
    0xF8B800, 0xB8F818, 0x58D854, 0x58F898, 0x00E8D8, 0x787878, 0x000000, 0x000000,
    0xFCFCFC, 0xA4E4FC, 0xB8B8F8, 0xD8B8F8, 0xF8B8F8, 0xF8A4C0, 0xF0D0B0, 0xFCE0A8,
    0xF8D878, 0xD8F878, 0xB8F8B8, 0xB8F8D8, 0x00FCFC, 0xF8D8F8, 0x000000, 0x000000};

// gym-super-mario-bros SIMPLE_MOVEMENT as nes-py controller bytes (bit 7 right, 6 left, 1 B, 0 A)
static const uint8_t kSimple[8] = {0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40, 0x00};

inline uint32_t enc(uint32_t kind, uint32_t mode, uint32_t op, uint32_t pen, uint32_t cyc) {
    return kind | (mode << 4) | (op << 8) | (pen << 13) | (cyc << 16);
}

// nes-py's decode cascade (nes_core.hpp:645-900), evaluated once per opcode on the host:
// implied -> branch -> type1 (op&3==1) -> type2 (op&3==2) -> type0 (op&3==0) -> unimplemented.
inline void build_dtab(uint32_t* t) {
    static const int kImplied[] = {0x00, 0x08, 0x18, 0x20, 0x28, 0x38, 0x40, 0x48, 0x4C, 0x58, 0x60, 0x68, 0x6C, 0x78,
                                   0x88, 0x8A, 0x98, 0x9A, 0xA8, 0xAA, 0xB8, 0xBA, 0xC8, 0xCA, 0xD8, 0xE8, 0xEA, 0xF8};
    for (int opc = 0; opc < 256; opc++) {
        const uint32_t cyc = kCycles[opc];
        int impl = -1;
        for (int k = 0; k < 28; k++) if (kImplied[k] == opc) impl = k;
        if (impl >= 0) { t[opc] = enc(K_IMPL, M_NONE, (uint32_t)impl, 0, cyc); continue; }
        if ((opc & 0x1f) == 0x10) {
            static const uint32_t kFlagBit[4] = {0, 1, 7, 6};  // N, V, C, Z in the reversed flag byte
            uint32_t field = kFlagBit[opc >> 6] | ((uint32_t)((opc >> 5) & 1) << 3);
            t[opc] = enc(K_BRANCH, M_NONE, field, 0, cyc);
            continue;
        }
        const int mode = (opc >> 2) & 7, opn = opc >> 5;
        if ((opc & 3) == 1) {
            static const uint32_t kM1[8] = {M_INDX, M_ZP, M_IMM, M_ABS, M_INDY, M_ZPX, M_ABSY, M_ABSX};
            static const uint32_t kR1[8] = {R_ORA, R_AND, R_EOR, R_ADC, 0, R_LDA, R_CMP, R_SBC};
            uint32_t pen = ((mode == 4 || mode == 6 || mode == 7) && opn != 4) ? 1u : 0u;
            t[opc] = opn == 4 ? enc(K_STORE, kM1[mode], W_STA, pen, cyc) : enc(K_READ, kM1[mode], kR1[opn], pen, cyc);
            continue;
        }
        if ((opc & 3) == 2) {
            const bool yidx = opn == 4 || opn == 5;  // STX / LDX index with Y
            uint32_t md = 0;
            bool ok = true;
            switch (mode) {
                case 0: md = M_IMM; break;
                case 1: md = M_ZP; break;
                case 2: md = M_NONE; break;
                case 3: md = M_ABS; break;
                case 5: md = yidx ? M_ZPY : M_ZPX; break;
                case 7: md = yidx ? M_ABSY : M_ABSX; break;
                default: ok = false;
            }
            if (!ok) { t[opc] = enc(K_BAD, 0, 0, 0, 0); continue; }
            uint32_t pen = mode == 7 ? 1u : 0u;
            static const uint32_t kRmw[8] = {X_ASL, X_ROL, X_LSR, X_ROR, 0, 0, X_DEC, X_INC};
            if (mode == 2) t[opc] = enc(K_ACC, M_NONE, kRmw[opn], 0, cyc);  // only ASL/ROL/LSR/ROR reach here
            else if (opn == 4) t[opc] = enc(K_STORE, md, W_STX, pen, cyc);
            else if (opn == 5) t[opc] = enc(K_READ, md, R_LDX, pen, cyc);
            else t[opc] = enc(K_RMW, md, kRmw[opn], pen, cyc);
            continue;
        }
        if ((opc & 3) == 0) {
            uint32_t md = 0;
            bool ok = true;
            switch (mode) {
                case 0: md = M_IMM; break;
                case 1: md = M_ZP; break;
                case 3: md = M_ABS; break;
                case 5: md = M_ZPX; break;
                case 7: md = M_ABSX; break;
                default: ok = false;
            }
            if (!ok) { t[opc] = enc(K_BAD, 0, 0, 0, 0); continue; }
            uint32_t pen = mode == 7 ? 1u : 0u;
            switch (opn) {
                case 1: t[opc] = enc(K_READ, md, R_BIT, pen, cyc); break;
                case 4: t[opc] = enc(K_STORE, md, W_STY, pen, cyc); break;
                case 5: t[opc] = enc(K_READ, md, R_LDY, pen, cyc); break;
                case 6: t[opc] = enc(K_READ, md, R_CPY, pen, cyc); break;
                case 7: t[opc] = enc(K_READ, md, R_CPX, pen, cyc); break;
                default:  // addressing already consumed its operands when the operation is found missing
                    t[opc] = enc(md == M_ABS ? K_BAD_ABS : md == M_ABSX ? K_BAD_ABSX : K_BAD_ZP, 0, 0, 0, 0);
            }
            continue;
        }
        t[opc] = enc(K_BAD, 0, 0, 0, 0);
    }
}

// OpenCV's area-resize tap table (cv::computeResizeAreaTab, the published algorithm), double precision.
struct Tap { int d, s; float w; };
inline std::vector<Tap> area_taps(int ssize, int dsize) {
    std::vector<Tap> out;
    const double scale = 1.0 / ((double)dsize / ssize);
    for (int dx = 0; dx < dsize; dx++) {
        double f1 = dx * scale, f2 = f1 + scale;
        double cell = std::min(scale, ssize - f1);
        int s1 = (int)std::ceil(f1), s2 = (int)std::floor(f2);
        s2 = std::min(s2, ssize - 1);
        s1 = std::min(s1, s2);
        if (s1 - f1 > 1e-3) out.push_back({dx, s1 - 1, (float)((s1 - f1) / cell)});
        for (int sx = s1; sx < s2; sx++) out.push_back({dx, sx, (float)(1.0 / cell)});
        if (f2 - s2 > 1e-3) out.push_back({dx, s2, (float)(std::min(std::min(f2 - s2, 1.), cell) / cell)});
    }
    return out;
}
// Per-PC micro-ops of the fast path (fme_fast.h): the decode of the instruction at every PRG address, with
// what the ROM fixes already resolved (static addresses, immediate and ROM operands, branch targets and
// their page-cross cost). Addresses whose instruction needs the exact path get H_SLOW.
inline bool io_addr(uint32_t a) { return a >= 0x2000u && a < 0x8000u; }
inline void build_uops(const uint8_t* prg, const uint32_t* dtab, uint32_t* out /* 2 x 32768 words */) {
    auto P = [&](uint32_t a) -> uint32_t { return prg[a & 0x7fffu]; };
    auto pf = [&](uint32_t a) -> uint32_t { a &= 0xffffu; return a >= 0x8000u ? P(a) : 0xffu; };
    for (uint32_t a = 0x8000u; a <= 0xffffu; a++) {
        const uint32_t opc = P(a), d = dtab[opc];
        const uint32_t kind = d_kind(d), mode = d_mode(d), op = d_op(d), pen = d_pen(d);
        const uint32_t b1 = pf(a + 1), b2 = pf(a + 2), w16 = b1 | (b2 << 8);
        const uint32_t cyc = kind >= K_IMPL ? d_cycles(d) : 0u;
        const bool idle = opc == 0x4Cu && w16 == a;  // `JMP *` with rd_prg_fast operand bytes
        uint32_t hid = H_SLOW, len = 1, w = 0, extra = 0;
        if (a <= 0xfffdu) {  // operand bytes inside PRG
            const uint32_t mlen = (mode == M_ABS || mode == M_ABSX || mode == M_ABSY) ? 3u : (mode == M_NONE ? 1u : 2u);
            switch (kind) {
                case K_READ:
                    len = mlen;
                    switch (mode) {
                        case M_IMM: hid = H_RD_IMM; w = b1; break;
                        case M_ZP: hid = H_RD_ZP; w = b1; break;
                        case M_ZPX: hid = H_RD_ZPX; w = b1; break;
                        case M_ZPY: hid = H_RD_ZPY; w = b1; break;
                        case M_ABS:
                            if (w16 < 0x2000u) { hid = H_RD_ABS; w = w16; }
                            else if (w16 >= 0x8000u) { hid = H_RD_IMM; w = P(w16); }  // ROM operand
                            else if ((w16 | 1u) == 0x4017u) { hid = H_JOY_RD; w = w16 & 1u; }
                            break;
                        case M_ABSX: hid = H_RD_ABSX; w = w16; break;
                        case M_ABSY: hid = H_RD_ABSY; w = w16; break;
                        case M_INDX: hid = H_RD_INDX; w = b1; break;
                        case M_INDY: hid = H_RD_INDY; w = b1; break;
                        default: break;
                    }
                    break;
                case K_STORE:
                    len = mlen;
                    switch (mode) {
                        case M_IMM: hid = H_NOPW; break;                          // writes into ROM: no effect
                        case M_ZP: hid = H_ST_ZP; w = b1; break;
                        case M_ZPX: hid = H_ST_ZPX; w = b1; break;
                        case M_ZPY: hid = H_ST_ZPY; w = b1; break;
                        case M_ABS:
                            if (w16 < 0x2000u) { hid = H_ST_ABS; w = w16; }
                            else if (w16 >= 0x8000u) hid = H_NOPW;
                            else if (w16 == 0x4016u) hid = H_JOY_ST;
                            break;
                        case M_ABSX: hid = H_ST_ABSX; w = w16; break;
                        case M_ABSY: hid = H_ST_ABSY; w = w16; break;
                        case M_INDX: hid = H_ST_INDX; w = b1; break;
                        case M_INDY: hid = H_ST_INDY; w = b1; break;
                        default: break;
                    }
                    break;
                case K_RMW:
                    len = mlen;
                    switch (mode) {
                        case M_ZP: hid = H_RMW_ZP; w = b1; break;
                        case M_ZPX: hid = H_RMW_ZPX; w = b1; break;
                        case M_ABS: if (w16 < 0x2000u) { hid = H_RMW_ABS; w = w16; } break;
                        case M_ABSX: hid = H_RMW_ABSX; w = w16; break;
                        default: break;  // immediate / ROM targets: exact path
                    }
                    break;
                case K_ACC: hid = H_ACC; break;
                case K_BRANCH: {
                    len = 2;
                    const uint32_t npc = (a + 2u) & 0xffffu;
                    const uint32_t t = (uint32_t)((int32_t)npc + (int32_t)(int8_t)(uint8_t)b1) & 0xffffu;
                    hid = H_BRANCH; w = t; extra = 1u + (((t ^ npc) & 0xff00u) ? 2u : 0u);
                    break;
                }
                case K_IMPL:
                    hid = H_IMPL; w = w16;
                    if (op == I_JMPI) {
                        const uint32_t hiad = (w16 & 0xff00u) | ((w16 + 1u) & 0xffu);
                        if (io_addr(w16) || io_addr(hiad)) hid = H_SLOW;
                    }
                    break;
                case K_BAD_ZP: hid = H_BAD; len = 2; break;
                case K_BAD_ABS: hid = H_BAD; len = 3; break;
                case K_BAD_ABSX: hid = H_BAD_ABSX; len = 3; w = w16; break;
                default: hid = H_BAD; len = 1; break;
            }
        }
        if (hid == H_SLOW) { len = 0; w = w16; }  // operand kept for diagnostics only
        {  // the forms whose operation is folded into the handler id (an operation outside its family's range
           // would alias another handler: such an instruction takes the exact path)
            uint32_t base = 0, nops = 0;
            switch (hid) {
                case H_RD_IMM: base = H_X_RD; nops = 12; break;
                case H_RD_ZP: case H_RD_ABS: base = H_X_RD + 16; nops = 12; break;
                case H_ST_ZP: case H_ST_ABS: base = H_X_ST; nops = 3; break;
                case H_RMW_ZP: case H_RMW_ABS: base = H_X_RMW; nops = 6; break;
                case H_ACC: base = H_X_ACC; nops = 6; break;
                case H_IMPL: base = H_X_IMPL; nops = 28; break;
                case H_RD_ZPX: base = H_X_RDZX; nops = 12; break;
                case H_RD_ABSX: base = H_X_RDAX; nops = 12; break;
                case H_RD_ABSY: base = H_X_RDAY; nops = 12; break;
                case H_RD_INDY: base = H_X_RDIY; nops = 12; break;
                case H_RD_INDX: base = H_X_RDIX; nops = 12; break;
                default: break;
            }
            if (nops) hid = op < nops ? base + op : (uint32_t)H_SLOW;
            if (hid == H_SLOW) { len = 0; w = w16; }
        }
        out[2 * (a - 0x8000u)] = hid | (opc << 8) | (op << 16) | (pen << 21) | (len << 22) | ((idle ? 1u : 0u) << 24);
        out[2 * (a - 0x8000u) + 1] = (w & 0xffffu) | (cyc << 16) | (extra << 24);
    }
}

// Datapath micro-ops (fme_dp.h) of every PRG address, from the exact micro-op table (2 x 32768 words each).
inline void build_dops(const uint32_t* uops, uint32_t* out) {
    for (uint32_t i = 0; i < 0x8000u; i++) {
        const uint2 d = make_dop(uops[2 * i], uops[2 * i + 1]);
        out[2 * i] = d.x;
        out[2 * i + 1] = d.y;
    }
}

inline bool build_area(AreaTabs& T) {
    memset(&T, 0, sizeof(T));
    int cnt[OBS];
    for (int pass = 0; pass < 2; pass++) {
        std::vector<Tap> taps = area_taps(pass == 0 ? SCREEN_W : SCREEN_H, OBS);
        for (int d = 0; d < OBS; d++) cnt[d] = 0;
        for (const Tap& tp : taps) {
            if (cnt[tp.d] >= 6) return false;
            if (pass == 0) { T.xs[cnt[tp.d]][tp.d] = tp.s; T.xw[cnt[tp.d]][tp.d] = tp.w; }
            else { T.ys[cnt[tp.d]][tp.d] = tp.s; T.yw[cnt[tp.d]][tp.d] = tp.w; }
            cnt[tp.d]++;
        }
    }
    return true;
}


}  // namespace tables
}  // namespace fme
