// fme_render.h - replay of one frame's log into a 240x256 framebuffer, and the 256x240 -> 84x84 area resize.
//
// Pixel semantics follow the reference's render path (nes_core.hpp:422-513): background pattern/attribute
// per dot with the dot's own v (coarse-x increments inside a segment), left-edge hiding, the first opaque
// sprite of the line's list per dot with its priority bit, palette lookup, then either the palette value
// (raw screen, nes_core.hpp:503-506) or the cv2 gray value (507-512).
//
// Layout of the work: a warp renders one env-frame at a time. Records are read by all lanes (broadcast
// loads); a segment's dots are split 8 per lane; palette/VRAM/OAM writes and DMA payloads are applied to the
// warp's shared-memory copies in record order, so every segment sees exactly the contents the PPU saw.
// When a frame is max-pooled with the previous one, the only row the frame can draw twice (the row of its
// first segment, because an emulated frame is 1-2 PPU calls longer than a PPU frame) is staged separately so
// "later write wins" inside the frame and "max" applies only across frames.
//
// The area resize reproduces OpenCV's float INTER_AREA in the operation order of the reference's fast
// resizer (fastmario.cpp:157-201): per source row the horizontal taps are summed from 0.f in tap order,
// then the vertical taps, no fused multiply-add, round-half-even and saturation.
#pragma once
#include "fme_defs.h"

#if defined(__CUDA_ARCH__)
#define FME_LDG(p) __ldg(p)
#else
#ifndef FME_LDG
#define FME_LDG(p) (*(p))
#endif
#endif

namespace fme {

constexpr int AREA_XTAPS = 4;  // 256 -> 84 columns: at most 4 taps each, consecutive source dots
struct AreaTabs {           // per output column / row up to 6 (index, weight) taps, zero-weight padded
    int32_t xs[6][OBS];
    float xw[6][OBS];
    int32_t ys[6][OBS];
    float yw[6][OBS];
};

// Render state of the warp (all pointers into shared memory except chr).
struct RState {
    uint8_t* vram;   // 2048
    uint8_t* pal;    // 32
    uint8_t* oam;    // 256
    const uint8_t* chr;
    uint32_t ntm;    // nametable t maps to VRAM offset ((ntm >> t) & 1) * 0x400 (a bit mask, so it stays in a register)
    // current explicit list (used by segments without a pending evaluation)
    uint32_t nsl, sl_lo, sl_hi;
};
FME_HD uint32_t nt_base(uint32_t ntm, uint32_t t) { return ((ntm >> t) & 1u) << 10; }

FME_HD uint32_t r_pb_read(const RState& s, uint32_t addr) {
    if (addr < 0x2000) return FME_LDG(s.chr + addr);
    if (addr < 0x3eff) {
        uint32_t tsel = addr < 0x2400 ? 0u : addr < 0x2800 ? 1u : addr < 0x2c00 ? 2u : 3u;
        return s.vram[nt_base(s.ntm, tsel) + (addr & 0x3ffu)];
    }
    if (addr < 0x3fff) return s.pal[addr & 0x1fu];
    return 0;
}

FME_HD int inc_count_fx(uint32_t fine_x, int x0, int x1) {
    int r = (7 - (int)fine_x) & 7;
    return (x1 - r + 7) / 8 - (x0 - r + 7) / 8;
}

// One line of a segment record: decode_seg gives its first line, seg_next_line steps to the next one.
struct Seg {
    int y, x0, x1;          // this line and its dots [x0, x1)
    uint32_t v, fine_x, flags;
    uint32_t pend, ev_y, oam_addr;
    int y1, xe;             // last line of the record and its end dot
    uint32_t tx;            // t's x bits (coarse x, nametable x), copied into v at dot 258
};
FME_HD Seg decode_seg(uint4 r) {
    Seg s;
    s.y = (int)((r.x >> 4) & 0xffu); s.x0 = (int)((r.x >> 12) & 0x1ffu); s.xe = (int)((r.x >> 21) & 0x1ffu);
    s.v = r.y & 0xffffu; s.fine_x = (r.y >> 16) & 7u; s.flags = (r.y >> 19) & 0x7fu;
    s.pend = r.z & 1u; s.ev_y = (r.z >> 1) & 0xffu; s.oam_addr = (r.z >> 9) & 0xffu;
    s.tx = ((r.z >> 17) & 0x1fu) | (((r.z >> 22) & 1u) << 10);
    s.y1 = (int)(r.w & 0xffu) > s.y ? (int)(r.w & 0xffu) : s.y;
    s.x1 = s.y1 == s.y ? s.xe : 256;
    return s;
}
// v from the line's first dot to the next line's dot 0 (nes_core.hpp:310-334: coarse-x increments of the
// remaining dots, fine-y at 257, copy of t's x bits at 258), and that line's list (evaluation of this one).
FME_HD void seg_next_line(Seg& g) {
    if (g.flags & RF_SHOW_BG) {
        uint32_t v = g.v;
        const int n = inc_count_fx(g.fine_x, g.x0, 256);
        uint32_t tot = (v & 0x1fu) + (uint32_t)n;
        v = (v & ~0x1fu & 0xffffu) | (tot & 31u);
        if ((tot >> 5) & 1u) v ^= 0x0400u;
        v = fine_y_add(v, 1);
        if (g.flags & RF_SHOW_SPR) v = (v & ~0x041fu & 0xffffu) | g.tx;
        g.v = v;
    }
    g.pend = 1u; g.ev_y = (uint32_t)g.y;
    g.y++; g.x0 = 0; g.x1 = g.y == g.y1 ? g.xe : 256;
}
// L >= 1 applications of seg_next_line in closed form (whole lines after the first add 32 coarse-x
// increments, one fine-y increment and the copy of t's x bits each).
FME_HD void seg_skip_lines(Seg& g, int L) {
    if (L == 1) { seg_next_line(g); return; }
    if (g.flags & RF_SHOW_BG) {
        uint32_t v = g.v;
        const uint32_t tot = (v & 0x1fu) + (uint32_t)inc_count_fx(g.fine_x, g.x0, 256);
        v = (v & ~0x1fu & 0xffffu) | (tot & 31u);
        if ((tot >> 5) & 1u) v ^= 0x0400u;
        if (g.flags & RF_SHOW_SPR) {
            v = fine_y_add(v, L);
            v = (v & ~0x041fu & 0xffffu) | g.tx;
        } else {
            if ((L - 1) & 1) v ^= 0x0400u;
            v = fine_y_add(v, L);
        }
        g.v = v;
    }
    g.y += L;
    g.pend = 1u; g.ev_y = (uint32_t)(g.y - 1);
    g.x0 = 0; g.x1 = g.y == g.y1 ? g.xe : 256;
}

// v after n coarse-x increments (nes_core.hpp:310-315 applied n times in closed form)
FME_HD uint32_t v_after(uint32_t v, int n) {
    if (n <= 0) return v;
    uint32_t tot = (v & 0x1fu) + (uint32_t)n;
    uint32_t r = (v & ~0x1fu & 0xffffu) | (tot & 31u);
    // each wrap of the 5-bit coarse x toggles the nametable bit
    if (((tot >> 5) & 1u)) r ^= 0x0400u;
    return r;
}

// 2-bit sprite pattern (exact integer semantics of nes_core.hpp:368-387) using the segment's flags
FME_HD uint32_t r_spr_bits(const RState& s, uint32_t flags, int i, int xx, int yy) {
    int spr_x = (int)s.oam[i * 4 + 3];
    int spr_y = (int)((s.oam[i * 4 + 0] + 1u) & 0xffu);
    int tile = (int)s.oam[i * 4 + 1], attribute = (int)s.oam[i * 4 + 2];
    bool lng = (flags & RF_LONG) != 0;
    int length = lng ? 16 : 8;
    int x_shift = (xx - spr_x) % 8, y_offset = (yy - spr_y) % length;
    if ((attribute & 0x40) == 0) x_shift ^= 7;
    if ((attribute & 0x80) != 0) y_offset ^= (length - 1);
    uint32_t address;
    if (!lng) {
        address = (uint32_t)(tile * 16 + y_offset) & 0xffffu;
        if (flags & RF_SPR_PAGE) address = (address + 0x1000u) & 0xffffu;
    } else {
        y_offset = (y_offset & 7) | ((y_offset & 8) << 1);
        address = (uint32_t)((tile >> 1) * 32 + y_offset) & 0xffffu;
        address |= (uint32_t)(tile & 1) << 12;
    }
    uint32_t c = (r_pb_read(s, address) >> x_shift) & 1u;
    c |= ((r_pb_read(s, (address + 8u) & 0xffffu) >> x_shift) & 1u) << 1;
    return c;
}

// sprite list of a segment whose evaluation is still pending (nes_core.hpp:336-349), scalar form
FME_HD void r_eval_scalar(const RState& s, const Seg& g, uint32_t& nsl, uint32_t& lo, uint32_t& hi) {
    uint32_t n = 0; lo = 0; hi = 0;
    int range = (g.flags & RF_LONG) ? 16 : 8;
    for (int i = (int)(g.oam_addr >> 2); i < 64; ++i) {
        int diff = (int)g.ev_y - (int)s.oam[i * 4];
        if (0 <= diff && diff < range) {
            if (n < 4) lo |= (uint32_t)i << (8 * n); else hi |= (uint32_t)i << (8 * (n - 4));
            if (++n >= 8) break;
        }
    }
    nsl = n;
}

// palette address (0..31) of dot x of segment g, with sprite list (nsl, lo, hi)
FME_HD uint32_t seg_dot_pa(const RState& s, const Seg& g, int xx, uint32_t nsl, uint32_t lo, uint32_t hi) {
    uint32_t pa = 0;
    if (g.flags & RF_SHOW_BG) {
        uint32_t vx = v_after(g.v, inc_count_fx(g.fine_x, g.x0, xx));
        uint32_t xf = (g.fine_x + (uint32_t)xx) & 7u;
        uint32_t tile = s.vram[nt_base(s.ntm, ((0x2000u | (vx & 0x0fffu)) >> 10) & 3u) + (vx & 0x3ffu)];
        uint32_t addr = (((tile * 16u) + ((vx >> 12) & 7u)) | ((g.flags & RF_BG_PAGE) ? 0x1000u : 0u)) & 0xffffu;
        uint32_t b = (FME_LDG(s.chr + (addr & 0x1fffu)) >> (7u ^ xf)) & 1u;
        b |= ((FME_LDG(s.chr + ((addr + 8u) & 0x1fffu)) >> (7u ^ xf)) & 1u) << 1;
        if (b) {
            uint32_t aaddr = 0x23C0u | (vx & 0x0C00u) | ((vx >> 4) & 0x38u) | ((vx >> 2) & 0x07u);
            uint32_t attr = s.vram[nt_base(s.ntm, (aaddr >> 10) & 3u) + (aaddr & 0x3ffu)];
            uint32_t shift = ((vx >> 4) & 4u) | (vx & 2u);
            pa = b | (((attr >> shift) & 3u) << 2);
        }
        if ((g.flags & RF_HIDE_BG) && xx < 8) pa = 0;
    }
    if ((g.flags & RF_SHOW_SPR) && nsl && !((g.flags & RF_HIDE_SPR) && xx < 8)) {
        for (uint32_t k = 0; k < nsl; k++) {
            int i = (int)(((k < 4 ? lo >> (8 * k) : hi >> (8 * (k - 4)))) & 0xffu);
            int sx = (int)s.oam[i * 4 + 3];
            if (xx < sx || xx >= sx + 8) continue;
            uint32_t c = r_spr_bits(s, g.flags, i, xx, g.y);
            if (!c) continue;
            uint32_t attribute = s.oam[i * 4 + 2];
            uint32_t col = c | 0x10u | ((attribute & 3u) << 2);
            bool front = !(attribute & 0x20u);
            if (!(pa & 3u) || front) pa = col;
            break;  // the first opaque sprite of the list decides this dot
        }
    }
    return pa;
}

// ---------------------------------------------------------------- area resize (portable, one output pixel)
FME_HD uint8_t sat_round(float v) {
#if defined(__CUDA_ARCH__)
    int iv = __float2int_rn(v);
#else
    int iv = (int)__builtin_lrintf(v);
#endif
    return (uint8_t)(iv < 0 ? 0 : iv > 255 ? 255 : iv);
}
FME_HD float fmul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
FME_HD float fadd(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}
FME_HD uint8_t area_pixel(const uint8_t* fb, const AreaTabs& T, int dy, int dx) {
    float sacc = 0.f;
    for (int m = 0; m < 6; m++) {
        float wy = T.yw[m][dy];
        if (wy == 0.f) break;
        const uint8_t* row = fb + T.ys[m][dy] * SCREEN_W;
        float b = 0.f;
        for (int k = 0; k < 6; k++) {
            float wx = T.xw[k][dx];
            if (wx == 0.f) break;
            b = fadd(b, fmul((float)row[T.xs[k][dx]], wx));
        }
        sacc = fadd(sacc, fmul(wy, b));
    }
    return sat_round(sacc);
}

// ---------------------------------------------------------------- 8-dot span form used by the renderers
FME_HD uint32_t brev8(uint32_t b) {
#if defined(__CUDA_ARCH__)
    return __brev(b) >> 24;
#else
    b = ((b & 0xF0u) >> 4) | ((b & 0x0Fu) << 4);
    b = ((b & 0xCCu) >> 2) | ((b & 0x33u) << 2);
    return ((b & 0xAAu) >> 1) | ((b & 0x55u) << 1);
#endif
}

// Row of sprite i on line y as MSB-first pattern bytes (column 0 = bit 7), with the exact address arithmetic
// of nes_core.hpp:368-387 (negative line offsets of stale lists included). Packed: lo | hi<<8.
FME_HD uint32_t sprite_row(const RState& rs, uint32_t flags, int i, int y) {
    int spr_y = (int)((rs.oam[i * 4 + 0] + 1u) & 0xffu);
    int tile = (int)rs.oam[i * 4 + 1], attribute = (int)rs.oam[i * 4 + 2];
    bool lng = (flags & RF_LONG) != 0;
    int length = lng ? 16 : 8;
    int y_offset = (y - spr_y) % length;
    if ((attribute & 0x80) != 0) y_offset ^= (length - 1);
    uint32_t address;
    if (!lng) {
        address = (uint32_t)(tile * 16 + y_offset) & 0xffffu;
        if (flags & RF_SPR_PAGE) address = (address + 0x1000u) & 0xffffu;
    } else {
        y_offset = (y_offset & 7) | ((y_offset & 8) << 1);
        address = (uint32_t)((tile >> 1) * 32 + y_offset) & 0xffffu;
        address |= (uint32_t)(tile & 1) << 12;
    }
    uint32_t lo = r_pb_read(rs, address), hi = r_pb_read(rs, (address + 8u) & 0xffffu);
    if (attribute & 0x40) { lo = brev8(lo); hi = brev8(hi); }
    return lo | (hi << 8);
}
// x | (0x10 | palette<<2) << 8 | front << 13 of sprite i (the part of nes_core.hpp:426-429 that is per sprite)
FME_HD uint32_t sprite_info(const RState& rs, int i) {
    uint32_t attribute = rs.oam[i * 4 + 2];
    return rs.oam[i * 4 + 3] | ((0x10u | ((attribute & 3u) << 2)) << 8) | ((attribute & 0x20u) ? 0u : (1u << 13));
}

// background tile of v: pattern bytes (MSB = leftmost dot) and the 2 palette-select bits (nes_core.hpp:453-464)
FME_HD void bg_tile(const RState& rs, uint32_t v, uint32_t bg_page, uint32_t& lo, uint32_t& hi, uint32_t& at) {
    uint32_t tile = rs.vram[nt_base(rs.ntm, (v >> 10) & 3u) + (v & 0x3ffu)];
    uint32_t addr = ((tile * 16u) + ((v >> 12) & 7u)) | (bg_page << 12);
    lo = FME_LDG(rs.chr + (addr & 0x1fffu));
    hi = FME_LDG(rs.chr + ((addr + 8u) & 0x1fffu));
    uint32_t aaddr = 0x23C0u | (v & 0x0C00u) | ((v >> 4) & 0x38u) | ((v >> 2) & 0x07u);
    uint32_t attr = rs.vram[nt_base(rs.ntm, (aaddr >> 10) & 3u) + (aaddr & 0x3ffu)];
    at = (attr >> (((v >> 4) & 4u) | (v & 2u))) & 3u;
}

// bit k of n (k < 4) -> byte k
FME_HD uint32_t expand4(uint32_t n) { return (n * 0x00204081u) & 0x01010101u; }

// The 8 output values of dots xa..xa+7 of segment g (bytes j of out[0..1]; dots outside the segment are
// computed but must not be stored). srow/sinfo: the line's sprite rows (list order); cand: bit k set for each
// list entry k that may cover one of the dots (every sprite that does is included). gv: the
// output value of each of the 32 palette addresses (palette entry, through the gray LUT unless raw).
// Per-dot decisions of nes_core.hpp:422-513 are made on 8-bit planes (bit 7-j = dot xa+j): background
// pattern bits and palette select, left-edge hiding, first opaque sprite of the list, and its priority.
FME_HD void render8(const RState& rs, const Seg& g, int xa, uint32_t cand, const uint32_t* srow, const uint32_t* sinfo,
                    const uint8_t* gv, uint32_t* out) {
    const uint32_t keep = xa >= 8 ? 0xffu : (1u << xa) - 1u;   // dots at x >= 8 (for left-edge hiding)
    uint32_t wlo = 0, whi = 0, am0 = 0, am1 = 0;
    if (g.flags & RF_SHOW_BG) {
        const int tx0 = ((int)g.fine_x + g.x0) >> 3;
        const int t0 = ((int)g.fine_x + xa) >> 3;
        const uint32_t s = ((uint32_t)g.fine_x + (uint32_t)xa) & 7u;
        const uint32_t bgp = (g.flags & RF_BG_PAGE) ? 1u : 0u;
        uint32_t lo0, hi0, at0, lo1 = 0, hi1 = 0, at1;
        bg_tile(rs, v_after(g.v, t0 - tx0), bgp, lo0, hi0, at0);
        at1 = at0;
        if (s) bg_tile(rs, v_after(g.v, t0 + 1 - tx0), bgp, lo1, hi1, at1);
        wlo = (((lo0 << 8) | lo1) >> (8u - s)) & 0xffu;
        whi = (((hi0 << 8) | hi1) >> (8u - s)) & 0xffu;
        const uint32_t first = (0xffu << s) & 0xffu;           // dots of the first tile
        am0 = ((at0 & 1u) ? first : 0u) | ((at1 & 1u) ? (~first & 0xffu) : 0u);
        am1 = ((at0 & 2u) ? first : 0u) | ((at1 & 2u) ? (~first & 0xffu) : 0u);
        if (g.flags & RF_HIDE_BG) { wlo &= keep; whi &= keep; }
    }
    const uint32_t bo = wlo | whi;                               // opaque background dots
    am0 &= bo; am1 &= bo;
    uint32_t filled = 0, front_m = 0, p0 = 0, p1 = 0, q0 = 0, q1 = 0;
    if ((g.flags & RF_SHOW_SPR) && cand) {
        for (uint32_t m = cand; m; m &= m - 1u) {   // list order: the lowest entry first
#if defined(__CUDA_ARCH__)
            const uint32_t k = (uint32_t)__ffs((int)m) - 1u;
#else
            const uint32_t k = (uint32_t)__builtin_ctz(m);
#endif
            const uint32_t inf = sinfo[k];
            const int o = xa - (int)(inf & 0xffu);
            if (o <= -8 || o >= 8) continue;
            const uint32_t rl = srow[k] & 0xffu, rh = (srow[k] >> 8) & 0xffu;
            const uint32_t al = o >= 0 ? (rl << o) & 0xffu : rl >> (-o);
            const uint32_t ah = o >= 0 ? (rh << o) & 0xffu : rh >> (-o);
            const uint32_t nw = (al | ah) & ~filled;             // dots this sprite is the first opaque one
            if (!nw) continue;
            filled |= nw;
            if (inf & (1u << 13)) front_m |= nw;
            p0 |= al & nw; p1 |= ah & nw;
            if (inf & (1u << 10)) q0 |= nw;                     // sprite palette bits (address bits 2, 3)
            if (inf & (1u << 11)) q1 |= nw;
        }
        if (g.flags & RF_HIDE_SPR) filled &= keep;
    }
    const uint32_t W = filled & (~bo | front_m);               // dots where the sprite is drawn
    const uint32_t P0 = brev8((wlo & ~W) | (p0 & W)), P1 = brev8((whi & ~W) | (p1 & W));
    const uint32_t P2 = brev8((am0 & ~W) | (q0 & W)), P3 = brev8((am1 & ~W) | (q1 & W)), P4 = brev8(W);
    // palette address of dot j in byte j
    const uint32_t alo = expand4(P0 & 15u) | (expand4(P1 & 15u) << 1) | (expand4(P2 & 15u) << 2) |
                         (expand4(P3 & 15u) << 3) | (expand4(P4 & 15u) << 4);
    const uint32_t ahi = expand4(P0 >> 4) | (expand4(P1 >> 4) << 1) | (expand4(P2 >> 4) << 2) |
                         (expand4(P3 >> 4) << 3) | (expand4(P4 >> 4) << 4);
    out[0] = (uint32_t)gv[alo & 0xffu] | ((uint32_t)gv[(alo >> 8) & 0xffu] << 8) |
             ((uint32_t)gv[(alo >> 16) & 0xffu] << 16) | ((uint32_t)gv[alo >> 24] << 24);
    out[1] = (uint32_t)gv[ahi & 0xffu] | ((uint32_t)gv[(ahi >> 8) & 0xffu] << 8) |
             ((uint32_t)gv[(ahi >> 16) & 0xffu] << 16) | ((uint32_t)gv[ahi >> 24] << 24);
}

}  // namespace fme
