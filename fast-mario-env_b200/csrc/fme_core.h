// fme_core.h - the NES console (6502 CPU, catch-up PPU, NROM bus) for one env per CUDA lane.
//
// Semantics follow the reference core exactly (csrc/nes_core.hpp, itself nes-py 8.2.1-exact): the
// instruction-atomic CPU with skip cycles (nes_core.hpp:901-1163), the decode cascade and its quirks
// (645-893), the catch-up PPU that advances whole scanline segments (534-616), NMI scheduling through
// `exec_at` / `zero_skip` (520-531, 1166-1204), the exact sprite-0 hit (390-413) and the `JMP *` idle-loop
// fast-forward (1176-1193). The structure is our own and built for the GPU:
//  * CPU/PPU scalars live in registers for a whole agent step; 6502 RAM, OAM and palette live in shared
//    memory in the lane-interleaved layout (fme_defs.h), VRAM in HBM.
//  * Frame-relative 32-bit time (iter/exec_at/ppu_calls/nmi_thresh minus the frame base) instead of
//    64-bit counters; the 64-bit base is kept for the OAM-DMA parity and for export.
//  * No pixels are produced here. Every PPU catch-up over visible dots appends a compact segment record
//    (line, dot range, v, fine_x, render flags, sprite-list state) to a per-frame log, together with the
//    VRAM/palette/OAM writes; the warp-cooperative renderer (fme_render.h) replays the log later.
//  * Sprite evaluation is lazy: the end-of-line evaluation only records the line; the 8-entry list is
//    materialised when an input of the evaluation is about to change ($2000 8x16 bit, $2003, $2004,
//    $4014) or when the state is saved. The sprite-0-in-list test needs only OAM[0] and oam_addr.
// The code is host/device portable so the same source can be exercised on a CPU during development.
#pragma once
#include "fme_defs.h"

#if defined(__CUDA_ARCH__)
#define FME_LDG(p) __ldg(p)
#else
#define FME_LDG(p) (*(p))
#endif

namespace fme {

// Decode table lookup: the kernels define FME_DTAB to read their __constant__ copy.
#ifndef FME_DTAB
extern uint32_t g_host_dtab[256];
#define FME_DTAB(op) (::fme::g_host_dtab[(op)])
#endif

FME_HD uint32_t il(uint32_t a) { return ((a & ~3u) << 5) | (a & 3u); }  // lane-interleaved byte offset

struct Cart {
    const uint8_t* prg;   // 32 KB ($8000-$FFFF; 16 KB images mirrored at load)
    const uint8_t* chr;   // 8 KB
    uint32_t nt[4];       // nametable offsets into VRAM (mirroring)
};

struct Core {
    // ---- CPU
    uint32_t pc, a, x, y, sp, p;
    bool zero_skip;
    // ---- time, relative to the frame base (`base` = nes-py CPU iteration at the frame start)
    int64_t base;
    int32_t exec_at, ppu_calls, nmi_thresh;
    int32_t cur;     // iteration of the instruction being executed
    int32_t skip;    // skip cycles accumulated by the executing instruction
    // ---- controllers
    uint32_t joy_strobe[2], joy_buttons[2], joy_bits[2];
    // ---- PPU
    uint32_t pstate, scanline, pcyc, fine_x, first_write, vblank, s0hit, even, inc;
    uint32_t v, t, data_buffer, oam_addr;
    uint32_t show_bg, show_spr, hide_bg, hide_spr, long_spr, nmi_en, bg_page, spr_page;
    uint32_t nsl, sl_lo, sl_hi;      // materialised sprite list (byte k of sl_lo|sl_hi<<32)
    bool ev_pend;                    // an end-of-line evaluation is recorded but not materialised
    uint32_t ev_y;                   // scanline of that evaluation
    // ---- memory
    uint8_t* ram;   // lane base of the RAM slab (shared memory on the device)
    uint8_t* ramh;  // lane base for addresses >= ram_end (== ram when the whole RAM is in one place)
    uint32_t ram_end;
    uint8_t* oam;
    uint8_t* pal;
    uint8_t* vram;  // this env's 2 KB VRAM (global)
    Cart cart;
    // ---- frame log
    uint4* rec;     // record area of the current slot
    int32_t nrec, cap;
    bool seg_open;        // the last segment may still be extended by later dots
    uint32_t seg_w0;
    uint32_t seg_y1;      // its last line
    int32_t seg_idx;      // record index of that segment
    uint32_t seg_reads;   // TOUCH_* inputs its pixels depend on
    int32_t vram_burst;   // VRAM write records since the last segment that reads VRAM
    bool vram_dirty;      // writes were not logged one by one; snapshot VRAM before the next such segment
    uint32_t bad_ops;
    uint32_t status;

    // ================================================================ memory helpers
    FME_HD uint8_t* ram_at(uint32_t a) const {
        const uint32_t m = a & 0x7ffu;
        return (m < ram_end ? ram : ramh) + il(m);
    }
    FME_HD uint32_t RAM(uint32_t a) const { return *ram_at(a); }
    FME_HD void RAMW(uint32_t a, uint32_t v_) { *ram_at(a) = (uint8_t)v_; }
    FME_HD uint32_t OAM(uint32_t i) const { return oam[il(i & 0xffu)]; }
    FME_HD void OAMW(uint32_t i, uint32_t v_) { oam[il(i & 0xffu)] = (uint8_t)v_; }
    FME_HD uint32_t PAL(uint32_t i) const { return pal[il(i & 0x1fu)]; }
    FME_HD void PALW(uint32_t i, uint32_t v_) { pal[il(i & 0x1fu)] = (uint8_t)v_; }
    FME_HD uint32_t prg(uint32_t a) const { return FME_LDG(cart.prg + (a & 0x7fffu)); }
    FME_HD uint32_t chr(uint32_t a) const { return FME_LDG(cart.chr + (a & 0x1fffu)); }

    // ================================================================ state import / export
    FME_HD void load_scalars(const uint32_t* w) {
        pc = w[S_CPU0] & 0xffffu; a = (w[S_CPU0] >> 16) & 0xffu; x = w[S_CPU0] >> 24;
        y = w[S_CPU1] & 0xffu; sp = (w[S_CPU1] >> 8) & 0xffu; p = (w[S_CPU1] >> 16) & 0xffu;
        zero_skip = (w[S_CPU1] >> 24) & 1u;
        base = (int64_t)((uint64_t)w[S_ITER_LO] | ((uint64_t)w[S_ITER_HI] << 32));
        exec_at = (int32_t)w[S_EXEC]; ppu_calls = (int32_t)w[S_PPUC]; nmi_thresh = (int32_t)w[S_THRESH];
        joy_strobe[0] = w[S_JOY] & 1u; joy_strobe[1] = (w[S_JOY] >> 1) & 1u;
        joy_buttons[0] = (w[S_JOY] >> 8) & 0xffu; joy_buttons[1] = (w[S_JOY] >> 16) & 0xffu;
        joy_bits[0] = w[S_JOYB] & 0xffu; joy_bits[1] = (w[S_JOYB] >> 8) & 0xffu;
        uint32_t q = w[S_PPU0];
        pstate = q & 3u; scanline = (q >> 2) & 0x3ffu; pcyc = (q >> 12) & 0x3ffu; fine_x = (q >> 22) & 7u;
        first_write = (q >> 25) & 1u; vblank = (q >> 26) & 1u; s0hit = (q >> 27) & 1u; even = (q >> 28) & 1u;
        inc = ((q >> 29) & 1u) ? 32u : 1u;
        v = w[S_PPU1] & 0xffffu; t = w[S_PPU1] >> 16;
        q = w[S_PPU2];
        data_buffer = q & 0xffu; oam_addr = (q >> 8) & 0xffu;
        uint32_t f = (q >> 16) & 0xffu;
        show_bg = f & PF_SHOW_BG ? 1u : 0u; show_spr = f & PF_SHOW_SPR ? 1u : 0u;
        hide_bg = f & PF_HIDE_BG ? 1u : 0u; hide_spr = f & PF_HIDE_SPR ? 1u : 0u;
        long_spr = f & PF_LONG ? 1u : 0u; nmi_en = f & PF_NMI ? 1u : 0u;
        bg_page = f & PF_BG_PAGE ? 1u : 0u; spr_page = f & PF_SPR_PAGE ? 1u : 0u;
        nsl = q >> 24; sl_lo = w[S_SL0]; sl_hi = w[S_SL1];
        ev_pend = false; ev_y = 0;
    }
    FME_HD uint32_t reg_flags() const {
        return (show_bg ? PF_SHOW_BG : 0u) | (show_spr ? PF_SHOW_SPR : 0u) | (hide_bg ? PF_HIDE_BG : 0u) |
               (hide_spr ? PF_HIDE_SPR : 0u) | (long_spr ? PF_LONG : 0u) | (nmi_en ? PF_NMI : 0u) |
               (bg_page ? PF_BG_PAGE : 0u) | (spr_page ? PF_SPR_PAGE : 0u);
    }
    // Caller must have materialised a pending evaluation (so nsl/sl are the exact reference values).
    FME_HD void store_scalars(uint32_t* w) const {
        w[S_CPU0] = pc | (a << 16) | (x << 24);
        w[S_CPU1] = y | (sp << 8) | (p << 16) | ((zero_skip ? 1u : 0u) << 24);
        w[S_ITER_LO] = (uint32_t)(uint64_t)base; w[S_ITER_HI] = (uint32_t)((uint64_t)base >> 32);
        w[S_EXEC] = (uint32_t)exec_at; w[S_PPUC] = (uint32_t)ppu_calls; w[S_THRESH] = (uint32_t)nmi_thresh;
        w[S_JOY] = joy_strobe[0] | (joy_strobe[1] << 1) | (joy_buttons[0] << 8) | (joy_buttons[1] << 16);
        w[S_JOYB] = joy_bits[0] | (joy_bits[1] << 8);
        w[S_PPU0] = pstate | (scanline << 2) | (pcyc << 12) | (fine_x << 22) | (first_write << 25) |
                    (vblank << 26) | (s0hit << 27) | (even << 28) | ((inc == 32u ? 1u : 0u) << 29);
        w[S_PPU1] = v | (t << 16);
        w[S_PPU2] = data_buffer | (oam_addr << 8) | (reg_flags() << 16) | (nsl << 24);
        w[S_SL0] = sl_lo; w[S_SL1] = sl_hi;
    }

    // ================================================================ power-on (nes_core.hpp:128-147)
    FME_NI void power_on() {
        for (uint32_t i = 0; i < RAM_BYTES; i++) RAMW(i, 0);
        for (uint32_t i = 0; i < OAM_BYTES; i++) OAMW(i, 0);
        for (uint32_t i = 0; i < PAL_BYTES; i++) PALW(i, 0);
        for (uint32_t i = 0; i < VRAM_BYTES; i++) vram[i] = 0;
        a = x = y = 0; sp = 0; p = 0; zero_skip = false;
        base = 0; exec_at = ppu_calls = nmi_thresh = 0; cur = 0; skip = 0;
        joy_strobe[0] = joy_strobe[1] = 1; joy_buttons[0] = joy_buttons[1] = 0; joy_bits[0] = joy_bits[1] = 0;
        fine_x = first_write = vblank = s0hit = even = 0; data_buffer = oam_addr = 0;
        show_bg = show_spr = hide_bg = hide_spr = long_spr = nmi_en = bg_page = spr_page = 0;
        nsl = 0; sl_lo = sl_hi = 0; ev_pend = false; ev_y = 0;
        // CPU::reset + PPU::reset
        p = 0x34; pc = prg(0xfffc) | (prg(0xfffd) << 8); sp = 0xfd;
        show_bg = 1; show_spr = 1; even = 1; first_write = 1; v = 0; t = 0; pcyc = 0; scanline = 0;
        inc = 1; pstate = PS_PRE;
        update_nmi_thresh();
    }

    // ================================================================ log
    FME_HD void emit(uint32_t w0, uint32_t w1 = 0, uint32_t w2 = 0, uint32_t w3 = 0) {
        if (nrec < cap) {
            uint4 r; r.x = w0; r.y = w1; r.z = w2; r.w = w3;
            rec[nrec] = r;
            nrec++;
        } else {
            status |= ST_LOG_OVERFLOW;
        }
    }
    // An event changed some render input: the open segment must end if its pixels depend on that input
    // (later dots then start a new segment that sees the change). Inputs: TOUCH_ALL (palette, mask),
    // TOUCH_BG (v, fine_x, background page), TOUCH_SPR (OAM, sprite list, sprite size/page),
    // TOUCH_VRAM (read by the background, and by sprites through out-of-range pattern addresses).
    FME_HD void touch(uint32_t what) {
        if (seg_open && (seg_reads & what)) seg_open = false;
    }
    FME_HD uint32_t render_flags() const {
        return (show_bg ? RF_SHOW_BG : 0u) | (show_spr ? RF_SHOW_SPR : 0u) | (hide_bg ? RF_HIDE_BG : 0u) |
               (hide_spr ? RF_HIDE_SPR : 0u) | (long_spr ? RF_LONG : 0u) | (bg_page ? RF_BG_PAGE : 0u) |
               (spr_page ? RF_SPR_PAGE : 0u);
    }
    // visible dots [x0, x1) of the current scanline are about to be produced with the current state
    FME_NI void log_vram_snapshot() {
        emit(REC_VSNAP);
        const uint4* src = reinterpret_cast<const uint4*>(vram);
        for (int k = 0; k < VRAM_BYTES / 16; k++) { uint4 q = src[k]; emit(q.x, q.y, q.z, q.w); }
        vram_dirty = false;
    }
    FME_HD uint32_t reads_now() const {
        return TOUCH_ALL | (show_bg ? (TOUCH_BG | TOUCH_VRAM) : 0u) | (show_spr ? (TOUCH_SPR | TOUCH_VRAM) : 0u);
    }
    FME_HD void log_seg(uint32_t x0, uint32_t x1) {
        if (seg_open) {
            const uint32_t end = seg_w0 >> 21;
            if (seg_y1 == scanline && end == x0) {                    // continues on the same line
                seg_w0 = (seg_w0 & ~(0x1ffu << 21)) | (x1 << 21);
                rec[seg_idx].x = seg_w0;
                return;
            }
            if (seg_y1 + 1 == scanline && end == 256u && x0 == 0) {  // continues on the next line
                seg_w0 = (seg_w0 & ~(0x1ffu << 21)) | (x1 << 21);
                seg_y1 = scanline;
                rec[seg_idx].x = seg_w0;
                rec[seg_idx].w = seg_y1;
                return;
            }
        }
        const uint32_t rd_ = reads_now();
        if (rd_ & TOUCH_VRAM) {
            if (vram_dirty) log_vram_snapshot();
            vram_burst = 0;
        }
        uint32_t w0 = REC_SEG | (scanline << 4) | (x0 << 12) | (x1 << 21);
        uint32_t w1 = v | (fine_x << 16) | (render_flags() << 19);
        uint32_t w2 = (ev_pend ? 1u : 0u) | (ev_y << 1) | (oam_addr << 9) | ((t & 0x1fu) << 17) | (((t >> 10) & 1u) << 22);
        const bool room = nrec < cap;
        emit(w0, w1, w2, scanline);
        seg_open = room;
        seg_w0 = w0; seg_y1 = scanline; seg_idx = nrec - 1; seg_reads = rd_;
    }

    // ================================================================ sprite evaluation (nes_core.hpp:336-349)
    FME_NI void eval_now(uint32_t line) {
        uint32_t n = 0, lo = 0, hi = 0;
        int range = long_spr ? 16 : 8;
        for (int i = (int)(oam_addr >> 2); i < 64; ++i) {
            int diff = (int)line - (int)OAM(i * 4);
            if (0 <= diff && diff < range) {
                if (n < 4) lo |= (uint32_t)i << (8 * n); else hi |= (uint32_t)i << (8 * (n - 4));
                if (++n >= 8) break;
            }
        }
        nsl = n; sl_lo = lo; sl_hi = hi;
    }
    // materialise a recorded evaluation before one of its inputs changes
    FME_NI void materialise() {
        if (!ev_pend) return;
        eval_now(ev_y);
        ev_pend = false;
        touch(TOUCH_SPR);
        emit(REC_LIST | (nsl << 4), sl_lo, sl_hi);
    }
    FME_HD uint32_t sl(uint32_t k) const { return ((k < 4 ? sl_lo >> (8 * k) : sl_hi >> (8 * (k - 4)))) & 0xffu; }
    FME_HD bool s0_in_list() const {
        if (ev_pend) {
            int diff = (int)ev_y - (int)OAM(0);
            return oam_addr < 4 && 0 <= diff && diff < (long_spr ? 16 : 8);
        }
        return nsl > 0 && sl(0) == 0;
    }

    // ================================================================ picture bus (nes_core.hpp:263-285)
    FME_HD uint32_t nt_index(uint32_t addr) const {  // addr in [0x2000, 0x3eff)
        uint32_t tsel = addr < 0x2400 ? 0u : addr < 0x2800 ? 1u : addr < 0x2c00 ? 2u : 3u;
        return cart.nt[tsel] + (addr & 0x3ffu);
    }
    FME_HD uint32_t pb_read(uint32_t addr) const {
        if (addr < 0x2000) return chr(addr);
        if (addr < 0x3eff) return vram[nt_index(addr)];
        if (addr < 0x3fff) return PAL(addr & 0x1fu);
        return 0;
    }
    FME_HD void pb_write(uint32_t addr, uint32_t val) {
        if (addr < 0x2000) return;
        if (addr < 0x3eff) {
            uint32_t i = nt_index(addr);
            vram[i] = (uint8_t)val;
            touch(TOUCH_VRAM);
            if (vram_dirty) return;
            if (vram_burst < VRAM_BURST_MAX) { emit(REC_VRAM | (i << 4) | (val << 16)); vram_burst++; }
            else vram_dirty = true;
        } else if (addr < 0x3fff) {
            uint32_t i = addr == 0x3f10 ? 0u : (addr & 0x1fu);
            PALW(i, val);
            touch(TOUCH_ALL);
            emit(REC_PAL | (i << 4) | (val << 16));
        }
    }
    FME_HD uint32_t nt_read(uint32_t addr) const {  // addr in [0x2000, 0x2fff]
        return vram[cart.nt[(addr >> 10) & 3u] + (addr & 0x3ffu)];
    }

    // ================================================================ PPU registers (nes_core.hpp:211-260)
    FME_HD void ppu_control(uint32_t c) {
        uint32_t nl = (c & 0x20) ? 1u : 0u;
        if (nl != long_spr) materialise();
        nmi_en = (c & 0x80) ? 1u : 0u;
        long_spr = nl;
        bg_page = (c & 0x10) ? 1u : 0u;
        spr_page = (c & 0x08) ? 1u : 0u;
        inc = (c & 0x04) ? 32u : 1u;
        t = (t & ~0xc00u & 0xffffu) | ((c & 3u) << 10);
        touch(TOUCH_BG | TOUCH_SPR);
    }
    FME_HD void ppu_mask(uint32_t m) {
        hide_bg = (m & 2) ? 0u : 1u;
        hide_spr = (m & 4) ? 0u : 1u;
        show_bg = (m & 8) ? 1u : 0u;
        show_spr = (m & 16) ? 1u : 0u;
        touch(TOUCH_ALL);
    }
    FME_HD uint32_t ppu_status() {
        uint32_t st = (s0hit << 6) | (vblank << 7);
        vblank = 0;
        first_write = 1;
        return st;
    }
    FME_HD void ppu_addr(uint32_t val) {
        if (first_write) {
            const uint32_t nt_ = (t & 0x00ffu) | ((val & 0x3fu) << 8);
            if ((nt_ ^ t) & 0x0400u) touch(TOUCH_BG);  // t's x bits reach v at the next dot-258 copy
            t = nt_; first_write = 0;
        }
        else { t = (t & 0xff00u) | val; v = t; first_write = 1; touch(TOUCH_BG); }
    }
    FME_HD uint32_t ppu_get_data() {
        uint32_t d = pb_read(v);
        v = (v + inc) & 0xffffu;
        if (v < 0x3f00) { uint32_t tmp = d; d = data_buffer; data_buffer = tmp; }
        touch(TOUCH_BG);
        return d;
    }
    FME_HD void ppu_set_data(uint32_t d) {
        pb_write(v, d);
        v = (v + inc) & 0xffffu;
        touch(TOUCH_BG);
    }
    FME_HD void ppu_scroll(uint32_t sc) {
        if (first_write) { t = (t & ~0x1fu & 0xffffu) | ((sc >> 3) & 0x1fu); fine_x = sc & 7u; first_write = 0; touch(TOUCH_BG); }
        else { t = (t & ~0x73e0u & 0xffffu) | ((sc & 7u) << 12) | ((sc & 0xf8u) << 2); first_write = 1; }
    }

    // ================================================================ PPU timing (nes_core.hpp:289-334)
    FME_HD void update_nmi_thresh() {
        int line = pstate == PS_PRE ? -1 : pstate == PS_POST ? 240 : (int)scanline;
        int P = (line + 1) * 341 + ((int)pcyc - 1);
        const int PN = 242 * 341;
        int d = P <= PN ? PN - P + 1 : (262 * 341 - P) + PN + 1;
        nmi_thresh = ppu_calls + d - 8;
    }
    FME_HD void sync_to(int32_t target) {
        if (target > ppu_calls) {
            ppu_run(target - ppu_calls);
            update_nmi_thresh();
        }
    }
    FME_HD void sync() { sync_to(3 * (cur + 1)); }

    FME_HD void coarse_x_inc_n(int n) {
        if (n <= 0) return;
        uint32_t tot = (v & 0x1fu) + (uint32_t)n;
        v = (v & ~0x1fu & 0xffffu) | (tot & 31u);
        if ((tot >> 5) & 1u) v ^= 0x0400u;
    }
    FME_HD int inc_count(int x0, int x1) const {  // x in [x0, x1) with (fine_x + x) % 8 == 7
        int r = (7 - (int)fine_x) & 7;
        return (x1 - r + 7) / 8 - (x0 - r + 7) / 8;
    }
    FME_HD void fine_y_inc() {
        if ((v & 0x7000u) != 0x7000u) {
            v = (v + 0x1000u) & 0xffffu;
        } else {
            v &= ~0x7000u & 0xffffu;
            uint32_t yy = (v & 0x03e0u) >> 5;
            if (yy == 29) { yy = 0; v ^= 0x0800u; }
            else if (yy == 31) yy = 0;
            else yy += 1;
            v = (v & ~0x03e0u & 0xffffu) | (yy << 5);
        }
    }
    FME_HD void hcopy() { v = (v & ~0x41fu & 0xffffu) | (t & 0x41fu); }
    FME_HD void vcopy() { v = (v & ~0x7be0u & 0xffffu) | (t & 0x7be0u); }

    // background opacity at dot x for the current v (nes_core.hpp:352-366, opaque part only)
    FME_HD bool bg_opaque(int xx) const {
        uint32_t xf = (fine_x + (uint32_t)xx) & 7u;
        uint32_t tile = nt_read(0x2000u | (v & 0x0fffu));
        uint32_t addr = ((tile * 16u) + ((v >> 12) & 7u)) | (bg_page << 12);
        addr &= 0xffffu;
        uint32_t c = (chr(addr) >> (7u ^ xf)) & 1u;
        c |= ((chr(addr + 8u) >> (7u ^ xf)) & 1u) << 1;
        return c != 0;
    }
    // 2-bit pattern of sprite i at (x, y); exact C integer semantics of nes_core.hpp:368-387
    FME_HD uint32_t spr_bits(int i, int xx, int yy) const {
        int spr_x = (int)OAM(i * 4 + 3);
        int spr_y = (int)((OAM(i * 4 + 0) + 1u) & 0xffu);
        int tile = (int)OAM(i * 4 + 1), attribute = (int)OAM(i * 4 + 2);
        int length = long_spr ? 16 : 8;
        int x_shift = (xx - spr_x) % 8, y_offset = (yy - spr_y) % length;
        if ((attribute & 0x40) == 0) x_shift ^= 7;
        if ((attribute & 0x80) != 0) y_offset ^= (length - 1);
        uint32_t address;
        if (!long_spr) {
            address = (uint32_t)(tile * 16 + y_offset) & 0xffffu;
            if (spr_page) address = (address + 0x1000u) & 0xffffu;
        } else {
            y_offset = (y_offset & 7) | ((y_offset & 8) << 1);
            address = (uint32_t)((tile >> 1) * 32 + y_offset) & 0xffffu;
            address |= (uint32_t)(tile & 1) << 12;
        }
        uint32_t c = (pb_read(address) >> x_shift) & 1u;
        c |= ((pb_read((address + 8u) & 0xffffu) >> x_shift) & 1u) << 1;
        return c;
    }

    // visible dots [x0, x1): only CPU-visible state (scroll increments, exact sprite-0 hit), plus the log
    FME_HD void dots(int x0, int x1) {
        log_seg((uint32_t)x0, (uint32_t)x1);
        if (!show_bg) return;
        if (!s0hit && show_spr && s0_in_list()) {
            int sx = (int)OAM(3);
            int lo = x0 > sx ? x0 : sx;
            int hi = x1 < sx + 8 ? x1 : sx + 8;
            if (hide_spr && lo < 8) lo = 8;
            if (lo < hi) {
                coarse_x_inc_n(inc_count(x0, lo));
                int yy = (int)scanline;
                for (int xx = lo; xx < hi; xx++) {
                    if (!s0hit && (!hide_bg || xx >= 8)) {
                        if (bg_opaque(xx) && spr_bits(0, xx, yy)) s0hit = 1;
                    }
                    if ((((int)fine_x + xx) & 7) == 7) coarse_x_inc_n(1);
                }
                coarse_x_inc_n(inc_count(hi, x1));
                return;
            }
        }
        coarse_x_inc_n(inc_count(x0, x1));
    }

    // CPU::interrupt(NMI) with nes-py's skip-cycle bookkeeping (nes_core.hpp:520-531)
    FME_NI void nmi(int32_t call_index) {
        int32_t m = (call_index - 1) / 3;
        push(pc >> 8);
        push(pc & 0xffu);
        push(p | 0x20u);
        p |= F_I;
        pc = prg(0xfffa) | (prg(0xfffb) << 8);
        int32_t vv = (zero_skip && m == exec_at) ? 0 : (exec_at - m + 1);
        exec_at = m + vv + 6;
        zero_skip = false;
    }

    // How many of the next `avail` whole visible lines (from dot 1 of the current line) can be advanced in
    // closed form: all of them unless a line could test sprite-0 pixels, which must then run dot by dot.
    FME_HD int bulk_lines(int avail) const {
        int L = avail < 240 - (int)scanline ? avail : 240 - (int)scanline;
        if (L <= 0 || !show_bg || !show_spr || s0hit) return L;
        if (s0_in_list()) return 0;                    // this line's list (as evaluated so far) holds sprite 0
        if (oam_addr >= 4) return L;                   // later lists start past sprite 0
        const int range = long_spr ? 16 : 8;
        const int c0 = (int)OAM(0) + 1, c1 = (int)OAM(0) + range;   // lines whose list (line-1) holds sprite 0
        const int y_lo = (int)scanline + 1 > c0 ? (int)scanline + 1 : c0;
        const int y_hi = (int)scanline + L - 1 < c1 ? (int)scanline + L - 1 : c1;
        if (y_lo <= y_hi) L = y_lo - (int)scanline;
        return L;
    }
    // L >= 1 whole visible lines without sprite-0 tests: one segment (extended), the scroll increments of
    // dots 1-256, the dot-257 fine-y increment and the dot-258 copy, the lazy evaluation of the last line.
    FME_HD void run_lines(int L) {
        log_seg(0, 256);
        if (L > 1 && seg_open) { seg_y1 = scanline + (uint32_t)L - 1u; rec[seg_idx].w = seg_y1; }
        if (L > 1 && !seg_open) status |= ST_LOG_OVERFLOW;  // the per-line records would not have fit either
        if (show_bg) {
            if (show_spr) v = (v & ~0x041fu & 0xffffu) | (t & 0x041fu);
            else if (L & 1) v ^= 0x0400u;                 // 32 coarse-x increments per line
            v = fine_y_add(v, L);
        }
        ev_pend = true; ev_y = scanline + (uint32_t)L - 1u;
        scanline += (uint32_t)L;
        ppu_calls += 341 * L;
        if (scanline >= 240) pstate = PS_POST;
    }

    // advance the PPU by n PPU::cycle calls (semantics of nes_core.hpp:534-616)
    FME_NI void ppu_run(int32_t n) {
        while (n > 0) {
            int c = (int)pcyc;
            if (pstate == PS_RENDER) {
                if (c == 1 && n >= 341) {
                    const int L = bulk_lines(n / 341);
                    if (L > 0) { run_lines(L); n -= 341 * L; continue; }
                }
                if (c >= 1 && c <= 256) {
                    int k = n < 257 - c ? n : 257 - c;
                    dots(c - 1, c - 1 + k);
                    pcyc += (uint32_t)k; ppu_calls += k; n -= k;
                } else if (c == 257) {
                    if (show_bg) fine_y_inc();
                    pcyc++; ppu_calls++; n--;
                } else if (c == 258) {
                    if (show_bg && show_spr) hcopy();
                    pcyc++; ppu_calls++; n--;
                } else if (c > 258 && c < 341) {
                    int k = n < 341 - c ? n : 341 - c;
                    pcyc += (uint32_t)k; ppu_calls += k; n -= k;
                } else if (c >= 341) {
                    ev_pend = true; ev_y = scanline;   // end-of-line sprite evaluation (lazy)
                    ++scanline;
                    pcyc = 1; ppu_calls++; n--;
                    if (scanline >= 240) pstate = PS_POST;
                } else {  // c == 0: not reachable from a reference state; kept for exactness
                    pcyc++; ppu_calls++; n--;
                }
            } else if (pstate == PS_PRE) {
                bool rend = show_bg && show_spr;
                int end = 341 - ((!even && rend) ? 1 : 0);
                int k = c >= end ? 1 : (n < end - c ? n : end - c);
                int a0 = c, b0 = c + k;
                if (a0 <= 1 && 1 < b0) { vblank = 0; s0hit = 0; }
                if (rend) {
                    if (a0 <= 258 && 258 < b0) hcopy();
                    if (a0 <= 304 && 281 < b0) vcopy();
                }
                ppu_calls += k; n -= k;
                if (b0 - 1 >= end) { pstate = PS_RENDER; scanline = 0; pcyc = 1; }
                else pcyc = (uint32_t)b0;
            } else if (pstate == PS_POST) {
                if (c >= 341) {
                    ++scanline; pcyc = 1; pstate = PS_VBLANK;
                    ppu_calls++; n--;
                } else {
                    int k = n < 341 - c ? n : 341 - c;
                    pcyc += (uint32_t)k; ppu_calls += k; n -= k;
                }
            } else if (!(c == 1 && scanline == 241) && c >= 1 && c <= 341 && scanline >= 241 && scanline <= 260) {
                // vertical blank after the flag dot: nothing happens until the pre-render line, so advance
                // by position (each line is dots 1..340 and its line end, 341 calls)
                const int end = 20 * 341;
                int pos = ((int)scanline - 241) * 341 + (c - 1);
                const int k = n < end - pos ? n : end - pos;
                pos += k; ppu_calls += k; n -= k;
                if (pos >= end) { pstate = PS_PRE; scanline = 0; pcyc = 1; even = even ? 0u : 1u; }
                else { scanline = 241u + (uint32_t)(pos / 341); pcyc = (uint32_t)(pos % 341) + 1u; }
            } else {  // vertical blank
                if (c >= 341) {
                    ++scanline;
                    pcyc = 1;
                    if (scanline >= 261) { pstate = PS_PRE; scanline = 0; even = even ? 0u : 1u; }
                    ppu_calls++; n--;
                } else if (c == 1 && scanline == 241) {
                    vblank = 1;
                    ppu_calls++; n--;
                    pcyc = 2;
                    if (nmi_en) nmi(ppu_calls);
                } else {
                    int lim = 341 - c;
                    if (scanline == 241 && c < 1) lim = 1 - c;
                    int k = n < lim ? n : lim;
                    pcyc += (uint32_t)k; ppu_calls += k; n -= k;
                }
            }
        }
    }

    // ================================================================ CPU bus (nes_core.hpp:150-208)
    FME_HD uint32_t joy_read(int i) {
        uint32_t r;
        if (joy_strobe[i]) r = joy_buttons[i] & 1u;
        else { r = joy_bits[i] & 1u; joy_bits[i] >>= 1; }
        return r | 0x40u;
    }
    FME_NI uint32_t rd_io(uint32_t addr) {
        if (addr < 0x4000) {
            switch (addr & 0x2007u) {
                case 0x2002: sync(); return ppu_status();
                case 0x2007: sync(); return ppu_get_data();
                case 0x2004: return OAM(oam_addr);
                default: return 0;
            }
        }
        if (addr == 0x4016) return joy_read(0);
        if (addr == 0x4017) return joy_read(1);
        return 0;
    }
    FME_HD uint32_t rd(uint32_t addr) {
        if (addr >= 0x8000) return prg(addr);
        if (addr < 0x2000) return RAM(addr);
        return rd_io(addr);
    }
    FME_NI void wr_io(uint32_t addr, uint32_t val) {
        if (addr < 0x4000) {
            switch (addr & 0x2007u) {
                case 0x2000: sync(); ppu_control(val); break;
                case 0x2001: sync(); ppu_mask(val); break;
                case 0x2003: sync(); materialise(); oam_addr = val; touch(TOUCH_SPR); break;
                case 0x2004:
                    sync(); materialise();
                    OAMW(oam_addr, val);
                    touch(TOUCH_SPR);
                    emit(REC_OAM | (oam_addr << 4) | (val << 16));
                    oam_addr = (oam_addr + 1) & 0xffu;
                    break;
                case 0x2005: sync(); ppu_scroll(val); break;
                case 0x2006: sync(); ppu_addr(val); break;
                case 0x2007: sync(); ppu_set_data(val); break;
                default: break;
            }
            return;
        }
        if (addr == 0x4014) {  // OAM DMA
            sync();
            skip += 513 + (int32_t)((uint64_t)(base + cur + 1) & 1u);
            materialise();
            uint32_t src = val << 8;
            if (src < 0x2000) {
                for (uint32_t k = 0; k < 256; k++) OAMW(oam_addr + k, RAM(src + k));
            }
            touch(TOUCH_SPR);
            emit(REC_DMA);
            for (uint32_t k = 0; k < 16; k++) {
                uint32_t w[4];
                for (uint32_t q = 0; q < 4; q++) {
                    uint32_t o = 16 * k + 4 * q;
                    w[q] = OAM(o) | (OAM(o + 1) << 8) | (OAM(o + 2) << 16) | (OAM(o + 3) << 24);
                }
                emit(w[0], w[1], w[2], w[3]);
            }
            return;
        }
        if (addr == 0x4016) {
            for (int i = 0; i < 2; i++) {
                joy_strobe[i] = val & 1u;
                if (!joy_strobe[i]) joy_bits[i] = joy_buttons[i];
            }
        }
    }
    FME_HD void wr(uint32_t addr, uint32_t val) {
        if (addr < 0x2000) { RAMW(addr, val); return; }
        wr_io(addr, val);
    }

    // ================================================================ CPU (nes_core.hpp:619-1163)
    FME_HD void set_zn(uint32_t val) {
        val &= 0xffu;
        p = (p & ~(F_Z | F_N)) | (val ? 0u : F_Z) | ((val & 0x80u) ? F_N : 0u);
    }
    FME_HD void setf(uint32_t f, bool on) { p = on ? (p | f) : (p & ~f); }
    FME_HD uint32_t getf(uint32_t f) const { return (p & f) ? 1u : 0u; }
    FME_HD void push(uint32_t val) { RAMW(0x100u | sp, val); sp = (sp - 1) & 0xffu; }
    FME_HD uint32_t pop() { sp = (sp + 1) & 0xffu; return RAM(0x100u | sp); }
    FME_HD uint32_t read_address(uint32_t addr) {
        uint32_t lo = rd(addr & 0xffffu);
        uint32_t hi = rd((addr + 1) & 0xffffu);
        return lo | (hi << 8);
    }
    FME_HD void page_pen(uint32_t a0, uint32_t b0, int pen) {
        if ((a0 & 0xff00u) != (b0 & 0xff00u)) skip += pen;
    }
    // effective address of an addressing mode (operand bytes consumed exactly as the reference does)
    FME_HD uint32_t ea(uint32_t mode, uint32_t pen) {
        uint32_t loc = 0;
        switch (mode) {
            case M_IMM: loc = pc; pc = (pc + 1) & 0xffffu; break;
            case M_ZP: loc = rd(pc); pc = (pc + 1) & 0xffffu; break;
            case M_ZPX: loc = (rd(pc) + x) & 0xffu; pc = (pc + 1) & 0xffffu; break;
            case M_ZPY: loc = (rd(pc) + y) & 0xffu; pc = (pc + 1) & 0xffffu; break;
            case M_ABS: loc = read_address(pc); pc = (pc + 2) & 0xffffu; break;
            case M_ABSX: case M_ABSY: {
                uint32_t b = read_address(pc); pc = (pc + 2) & 0xffffu;
                uint32_t idx = mode == M_ABSX ? x : y;
                loc = (b + idx) & 0xffffu;
                if (pen) page_pen(b, loc, 1);
                break;
            }
            case M_INDX: {
                uint32_t za = (x + rd(pc)) & 0xffu; pc = (pc + 1) & 0xffffu;
                uint32_t lo = rd(za), hi = rd((za + 1) & 0xffu);
                loc = lo | (hi << 8);
                break;
            }
            case M_INDY: {
                uint32_t za = rd(pc); pc = (pc + 1) & 0xffffu;
                uint32_t lo = rd(za), hi = rd((za + 1) & 0xffu);
                uint32_t b = lo | (hi << 8);
                loc = (b + y) & 0xffffu;
                if (pen) page_pen(b, loc, 1);
                break;
            }
            default: break;
        }
        return loc;
    }
    FME_HD void alu_read(uint32_t op, uint32_t m) {
        switch (op) {
            case R_ORA: a |= m; set_zn(a); break;
            case R_AND: a &= m; set_zn(a); break;
            case R_EOR: a ^= m; set_zn(a); break;
            case R_ADC: {
                uint32_t sum = a + m + getf(F_C);
                setf(F_C, sum & 0x100u);
                setf(F_V, (a ^ sum) & (m ^ sum) & 0x80u);
                a = sum & 0xffu; set_zn(a);
                break;
            }
            case R_LDA: a = m; set_zn(a); break;
            case R_CMP: { uint32_t d = (a - m) & 0xffffu; setf(F_C, !(d & 0x100u)); set_zn(d); break; }
            case R_SBC: {
                uint32_t d = (a - m - (getf(F_C) ? 0u : 1u)) & 0xffffu;
                setf(F_C, !(d & 0x100u));
                setf(F_V, (a ^ d) & (~m ^ d) & 0x80u);
                a = d & 0xffu; set_zn(d);
                break;
            }
            case R_BIT: setf(F_Z, !(a & m)); setf(F_V, m & 0x40u); setf(F_N, m & 0x80u); break;
            case R_LDX: x = m; set_zn(x); break;
            case R_LDY: y = m; set_zn(y); break;
            case R_CPX: { uint32_t d = (x - m) & 0xffffu; setf(F_C, !(d & 0x100u)); set_zn(d); break; }
            default:    { uint32_t d = (y - m) & 0xffffu; setf(F_C, !(d & 0x100u)); set_zn(d); break; }  // CPY
        }
    }
    FME_HD uint32_t alu_rmw(uint32_t op, uint32_t m) {
        uint32_t c = getf(F_C);
        switch (op) {
            case X_ASL: setf(F_C, m & 0x80u); m = (m << 1) & 0xffu; break;
            case X_ROL: setf(F_C, m & 0x80u); m = ((m << 1) | c) & 0xffu; break;
            case X_LSR: setf(F_C, m & 1u); m >>= 1; break;
            case X_ROR: setf(F_C, m & 1u); m = (m >> 1) | (c << 7); break;
            case X_DEC: m = (m - 1) & 0xffu; break;
            default: m = (m + 1) & 0xffu; break;  // INC
        }
        set_zn(m);
        return m;
    }
    FME_HD void implied(uint32_t op) {
        switch (op) {
            case I_BRK:
                pc = (pc + 1) & 0xffffu;
                push(pc >> 8); push(pc & 0xffu); push(p | 0x30u);
                p |= F_I;
                pc = read_address(0xfffe);
                skip += 7;
                break;
            case I_PHP: push(p); break;
            case I_CLC: setf(F_C, false); break;
            case I_JSR: {
                uint32_t r = (pc + 1) & 0x1ffffu;
                push((r >> 8) & 0xffu); push(r & 0xffu);
                pc = read_address(pc);
                break;
            }
            case I_PLP: p = pop(); break;
            case I_SEC: setf(F_C, true); break;
            case I_RTI: p = pop(); pc = pop(); pc |= pop() << 8; break;
            case I_PHA: push(a); break;
            case I_JMP: pc = read_address(pc); break;
            case I_CLI: setf(F_I, false); break;
            case I_RTS: pc = pop(); pc |= pop() << 8; pc = (pc + 1) & 0xffffu; break;
            case I_PLA: a = pop(); set_zn(a); break;
            case I_JMPI: {
                uint32_t loc = read_address(pc);
                uint32_t page = loc & 0xff00u;
                uint32_t lo = rd(loc);
                uint32_t hi = rd(page | ((loc + 1) & 0xffu));
                pc = lo | (hi << 8);
                break;
            }
            case I_SEI: setf(F_I, true); break;
            case I_DEY: y = (y - 1) & 0xffu; set_zn(y); break;
            case I_TXA: a = x; set_zn(a); break;
            case I_TYA: a = y; set_zn(a); break;
            case I_TXS: sp = x; break;
            case I_TAY: y = a; set_zn(y); break;
            case I_TAX: x = a; set_zn(x); break;
            case I_CLV: setf(F_V, false); break;
            case I_TSX: x = sp; set_zn(x); break;
            case I_INY: y = (y + 1) & 0xffu; set_zn(y); break;
            case I_DEX: x = (x - 1) & 0xffu; set_zn(x); break;
            case I_CLD: setf(F_D, false); break;
            case I_INX: x = (x + 1) & 0xffu; set_zn(x); break;
            case I_NOP: break;
            default: setf(F_D, true); break;  // SED
        }
    }
    // one instruction whose opcode byte was already read from `pc`; returns the reference's skip-cycle count
    FME_HD int32_t execute_op(uint32_t opc) {
        skip = 0;
        pc = (pc + 1) & 0xffffu;
        uint32_t d = FME_DTAB(opc);
        uint32_t kind = d_kind(d);
        switch (kind) {
            case K_READ: {
                uint32_t loc = ea(d_mode(d), d_pen(d));
                alu_read(d_op(d), rd(loc));
                break;
            }
            case K_STORE: {
                uint32_t loc = ea(d_mode(d), d_pen(d));
                uint32_t op = d_op(d);
                wr(loc, op == W_STA ? a : op == W_STX ? x : y);
                break;
            }
            case K_RMW: {
                uint32_t loc = ea(d_mode(d), d_pen(d));
                uint32_t m = rd(loc);
                wr(loc, alu_rmw(d_op(d), m));
                break;
            }
            case K_ACC: a = alu_rmw(d_op(d), a); break;
            case K_BRANCH: {
                uint32_t op = d_op(d);  // flag mask | want<<8 packed by the host table (see fme_host)
                uint32_t f = (p >> (op & 7u)) & 1u;
                uint32_t want = (op >> 3) & 1u;
                if (f == want) {
                    int32_t off = (int32_t)(int8_t)(uint8_t)rd(pc);
                    pc = (pc + 1) & 0xffffu;
                    skip += 1;
                    uint32_t np = (uint32_t)((int32_t)pc + off) & 0xffffu;
                    page_pen(pc, np, 2);
                    pc = np;
                } else {
                    pc = (pc + 1) & 0xffffu;
                }
                break;
            }
            case K_IMPL: implied(d_op(d)); break;
            case K_BAD_ZP: rd(pc); pc = (pc + 1) & 0xffffu; bad_ops++; break;
            case K_BAD_ABS: read_address(pc); pc = (pc + 2) & 0xffffu; bad_ops++; break;
            case K_BAD_ABSX: {
                uint32_t b = read_address(pc); pc = (pc + 2) & 0xffffu;
                page_pen(b, (b + x) & 0xffffu, 1);
                bad_ops++;
                break;
            }
            default: bad_ops++; break;
        }
        if (kind >= K_IMPL) skip += (int32_t)d_cycles(d);
        return skip;
    }

    // ================================================================ sprite-0 busy-wait
    // Last PPU call count up to which the sprite-0 flag keeps its current value while no register is written:
    // the flag is set only by a pixel test on a line whose sprite list holds sprite 0 (`dots`) and cleared at
    // dot 1 of the pre-render line. Conservative: never later than the true value, ppu_calls when unsure.
    FME_HD int32_t s0_steady_until() const {
        const int32_t FAR = 0x3fffffff;
        const int c = (int)pcyc;
        if (s0hit) {
            if (pstate == PS_VBLANK && scanline >= 241 && scanline <= 260 && c >= 1 && c <= 341)
                return ppu_calls + (20 * 341 - (((int)scanline - 241) * 341 + (c - 1)));  // to the pre-render line
            if (pstate == PS_RENDER || pstate == PS_POST) return FAR;  // the clear comes after the next vblank
            return ppu_calls;
        }
        if (!show_bg || !show_spr) return FAR;                        // no pixel test runs
        if (s0_in_list()) return ppu_calls;                           // the current / next line may test
        if (oam_addr >= 4) return FAR;                                // later lists start past sprite 0
        const int range = long_spr ? 16 : 8;
        const int y_first = (int)OAM(0) + 1, y_last = (int)OAM(0) + range;   // lines whose list (line-1) holds it
        if (pstate == PS_RENDER && c >= 1 && c <= 341) {
            const int y = (int)scanline + 1 > y_first ? (int)scanline + 1 : y_first;
            if (y > y_last || y > 239) return FAR;
            return ppu_calls + (y - (int)scanline) * 341 - (c - 1);  // dot 1 of line y not yet processed
        }
        if (pstate == PS_PRE && c >= 1 && c <= 341) {
            const int y = y_first > 1 ? y_first : 1;                  // line 0 uses the state checked above
            if (y > y_last || y > 239) return FAR;
            return ppu_calls + (341 - c) + y * 341;                   // shortest (odd-frame) pre-render line
        }
        return ppu_calls;
    }
    // The instruction at pc (executing at iteration J) may open a loop that polls $2002 until bit 6 (the
    // sprite-0 flag) changes: `BIT $2002 / BVC|BVS *-3` or `LDA $2002 / AND #$40 / BEQ|BNE *-5`. Once vblank
    // is clear and the address latch reset, another read of $2002 only catches the PPU up, and the loop's
    // other instructions are plain register work that the exiting iteration overwrites (A, N, V, Z). So the
    // iterations whose read still sees the waiting value are replaced by their PPU catch-ups; the read that
    // ends the loop runs as usual. Iterations are skipped only while the next read stays before the NMI
    // pre-sync and the frame end, where the frame loop has work of its own. Returns the skipped cycles.
    FME_NI int32_t poll_skip(int32_t J, uint32_t opc) {
        if (vblank || !first_write || pc < 0x8000u || pc > 0xfff8u) return 0;
        if (prg(pc + 1) != 0x02u || prg(pc + 2) != 0x20u) return 0;
        uint32_t br, br_pc, exit_bit;
        int32_t it;
        if (opc == 0x2Cu) {                                   // BIT $2002 / BVC|BVS back
            br = prg(pc + 3);
            if ((br != 0x50u && br != 0x70u) || prg(pc + 4) != 0xFBu) return 0;
            exit_bit = br == 0x50u ? 1u : 0u;
            br_pc = pc + 3;
            it = (int32_t)d_cycles(FME_DTAB(0x2Cu));
        } else {                                              // LDA $2002 / AND #$40 / BEQ|BNE back
            if (prg(pc + 3) != 0x29u || prg(pc + 4) != 0x40u) return 0;
            br = prg(pc + 5);
            if ((br != 0xF0u && br != 0xD0u) || prg(pc + 6) != 0xF9u) return 0;
            exit_bit = br == 0xF0u ? 1u : 0u;
            br_pc = pc + 5;
            it = (int32_t)d_cycles(FME_DTAB(0xADu)) + (int32_t)d_cycles(FME_DTAB(0x29u));
        }
        it += (int32_t)d_cycles(FME_DTAB(br)) + 1 + ((((br_pc + 2u) ^ pc) & 0xff00u) ? 2 : 0);  // taken branch
        int32_t D = 0;
        if (s0hit != exit_bit) {
            // reads whose catch-up target stays within the flag's steady span see the waiting value: skip them
            // without catching up (a later catch-up reaches the same state); keep a line of margin to the NMI
            // pre-sync, whose threshold is only refreshed by a catch-up
            const int32_t S = s0_steady_until();
            for (;;) {
                const int32_t Jk = J + D, Jn = Jk + it;
                if (3 * (Jn + 1) + 2 * 341 >= nmi_thresh || Jn >= FRAME_ITERS || 3 * (Jk + 1) > S) break;
                D += it;
            }
        }
        for (;;) {
            const int32_t Jk = J + D, Jn = Jk + it;
            if (3 * (Jn + 1) >= nmi_thresh || Jn >= FRAME_ITERS) break;
            cur = Jk;
            sync();                                           // the catch-up of this iteration's read
            if (s0hit == exit_bit) break;                     // this read ends the loop
            D += it;
        }
        cur = J + D;
        return D;
    }

    // ================================================================ frame driver (nes_core.hpp:1166-1204)
    // Run until the instruction boundary test. Returns false once exec_at reached the frame end.
    // One call = one executed instruction (or an NMI / idle-loop skip).
    // byte at a for the idle-loop test: PRG, or 0xff outside it (rd_prg_fast, nes_core.hpp:153)
    FME_HD uint32_t prg_fast(uint32_t a) const { a &= 0xffffu; return a >= 0x8000u ? prg(a) : 0xffu; }
    FME_HD bool step_once() {
        if (exec_at >= FRAME_ITERS) return false;
        const int32_t J = exec_at;
        if (3 * (J + 1) >= nmi_thresh) {
            cur = J;
            sync_to(3 * (J + 1));
            if (exec_at != J) return true;  // an NMI was taken before this instruction
        }
        // the opcode byte: PRG reads have no side effects, so it is read once for the idle test and execution
        const uint32_t opc = pc >= 0x8000u ? prg(pc) : 0x100u;
        if (opc == 0x4Cu && (prg_fast(pc + 1) | (prg_fast(pc + 2) << 8)) == pc) {
            int32_t lim_end = FRAME_ITERS - J;
            int32_t lim_nmi = nmi_thresh - 3 * (J + 1);
            int32_t k1 = lim_end > 0 ? (lim_end + 2) / 3 : 0;
            int32_t k2 = lim_nmi > 0 ? (lim_nmi + 8) / 9 : 0;
            int32_t k = k1 < k2 ? k1 : k2;
            if (k > 1) {
                exec_at = J + 3 * (k - 1);
                zero_skip = false;
                return true;
            }
        }
        cur = J;
        int32_t D = (opc == 0x2Cu || opc == 0xADu) ? poll_skip(J, opc) : 0;
        int32_t S = D + execute_op(opc != 0x100u ? opc : rd(pc));
        exec_at = J + (S >= 1 ? S : 1);
        zero_skip = S <= 0;
        return true;
    }
    // after step_once() returned false: catch the PPU up to the frame end and rebase the clocks
    FME_HD void end_frame() {
        sync_to(FRAME_CALLS);
        base += FRAME_ITERS;
        exec_at -= FRAME_ITERS;
        ppu_calls -= FRAME_CALLS;
        nmi_thresh -= FRAME_CALLS;
    }
};

// ---------------------------------------------------------------- SMB RAM helpers (fastmario.cpp:205-250)
FME_HD int64_t smb_digits(const Core& c, uint32_t a0, int n) {
    int64_t v = 0;
    for (int i = 0; i < n; i++) {
        int b = (int)c.RAM(a0 + (uint32_t)i);
        v = v * (b >= 100 ? 1000 : b >= 10 ? 100 : 10) + b;
    }
    return v;
}
FME_HD int32_t smb_x_pos(const Core& c) { return (int32_t)(c.RAM(0x6d) * 0x100u + c.RAM(0x86)); }
FME_HD int64_t smb_time(const Core& c) { return smb_digits(c, 0x7f8, 3); }
FME_HD bool smb_dying(const Core& c) { return c.RAM(0x0e) == 0x0b || c.RAM(0xb5) > 1; }
FME_HD bool smb_dead(const Core& c) { return c.RAM(0x0e) == 0x06; }
FME_HD bool smb_busy(const Core& c) { uint32_t s = c.RAM(0x0e); return s <= 5 || s == 7; }
FME_HD bool smb_world_over(const Core& c) { return c.RAM(0x0770) == 2; }
FME_HD bool smb_stage_over(const Core& c) {
    for (uint32_t a0 = 0x16; a0 <= 0x1a; a0++) {
        uint32_t r = c.RAM(a0);
        if (r == 0x2d || r == 0x31) return c.RAM(0x1d) == 3;
    }
    return false;
}
FME_HD bool smb_flag(const Core& c) { return smb_world_over(c) || smb_stage_over(c); }
// the 10 info fields, in the reference's order (fastmario.cpp:213-215, 234-249)
FME_HD void smb_info(const Core& c, int64_t* out) {
    out[0] = smb_x_pos(c);
    out[1] = smb_flag(c) ? 1 : 0;
    out[2] = c.RAM(0x075a);
    out[3] = smb_digits(c, 0x7de, 6);
    out[4] = smb_time(c);
    out[5] = (int64_t)c.RAM(0x075f) + 1;
    out[6] = (int64_t)c.RAM(0x075c) + 1;
    out[7] = smb_digits(c, 0x7ed, 2);
    int yp = (int)c.RAM(0x03b8);
    out[8] = c.RAM(0x00b5) < 1 ? 255 + (255 - yp) : 255 - yp;
    uint32_t st = c.RAM(0x0756);
    out[9] = st == 0 ? 0 : st == 1 ? 1 : 2;
}

}  // namespace fme
