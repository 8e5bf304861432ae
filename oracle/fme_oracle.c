/* fme_oracle.c - TEST ORACLE ONLY: a plain-C restatement of the reference's CPU path, used by tests/ (and by
 * bench.py's CPU-baseline leg) as a checker. The product never links or calls it.
 *
 * It restates, function by function, the reference's NES core (csrc/nes_core.hpp) and env wrapper chain
 * (csrc/fastmario.cpp) in straightforward C: per-frame catch-up PPU with per-dot rendering, the nes-py decode
 * cascade, PCG64, INTER_AREA, SMB reward/info, hacks, frame skip/max-pool/sticky/no-op reset, frame stack and
 * auto-reset. Every function cites the reference lines it follows. It is pinned against the reference build
 * (oracle/_ref/libfastmario.so) and the golden fixtures in tests/golden by tests/test_oracle_port.py.
 * Build: make -C oracle port  ->  oracle/_ref/libfme_oracle.so
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ flags / constants (nes_core.hpp:36-56) */
enum { FN = 0x01, FV = 0x02, FB = 0x08, FD = 0x10, FI = 0x20, FZ = 0x40, FC = 0x80 };
enum { PRE = 0, REND = 1, POST = 2, VBL = 3 };
static const uint8_t CYC[256] = {
    7,6,0,0,0,3,5,0,3,2,2,0,0,4,6,0,2,5,0,0,0,4,6,0,2,4,0,0,0,4,7,0, 6,6,0,0,3,3,5,0,4,2,2,0,4,4,6,0,2,5,0,0,0,4,6,0,2,4,0,0,0,4,7,0,
    6,6,0,0,0,3,5,0,3,2,2,0,3,4,6,0,2,5,0,0,0,4,6,0,2,4,0,0,0,4,7,0, 6,6,0,0,0,3,5,0,4,2,2,0,5,4,6,0,2,5,0,0,0,4,6,0,2,4,0,0,0,4,7,0,
    0,6,0,0,3,3,3,0,2,0,2,0,4,4,4,0,2,6,0,0,4,4,4,0,2,5,2,0,0,5,0,0, 2,6,2,0,3,3,3,0,2,2,2,0,4,4,4,0,2,5,0,0,4,4,4,0,2,4,2,0,4,4,4,0,
    2,6,0,0,3,3,5,0,2,2,2,0,4,4,6,0,2,5,0,0,0,4,6,0,2,4,0,0,0,4,7,0, 2,6,0,0,3,3,5,0,2,2,2,2,4,4,6,0,2,5,0,0,0,4,6,0,2,4,0,0,0,4,7,0};
#define ITERS 29781

typedef struct { uint8_t prg[0x8000], chr[0x2000]; int nt[4]; } cart_t;

/* nes_core.hpp:67-87 */
static int cart_parse(cart_t* c, const uint8_t* d, size_t n) {
    if (n < 16 || memcmp(d, "NES\x1a", 4)) return -1;
    int mir = d[6] & 0xB, mapper = ((d[6] >> 4) & 0xf) | (d[7] & 0xf0), banks = d[4], vb = d[5];
    if (mapper || (d[6] & 2) || (d[6] & 4)) return -2;
    if (banks < 1 || banks > 2 || vb != 1) return -3;
    if (n < 16 + 0x4000u * banks + 0x2000u) return -4;
    memset(c, 0, sizeof *c);
    memcpy(c->prg, d + 16, 0x4000 * banks);
    if (banks == 1) memcpy(c->prg + 0x4000, d + 16, 0x4000);
    memcpy(c->chr, d + 16 + 0x4000 * banks, 0x2000);
    if (mir == 0) { c->nt[2] = c->nt[3] = 0x400; }
    else if (mir == 1) { c->nt[1] = c->nt[3] = 0x400; }
    return 0;
}

/* console state (nes_core.hpp:90-114) plus per-frame working fields */
typedef struct {
    int64_t iter, exec_at, calls, thresh;
    int zero_skip;
    uint16_t pc; uint8_t sp, a, x, y, p;
    uint8_t strobe[2], buttons[2], bits[2];
    int pstate, scanline, cyc;
    int even, vblank, s0hit, latch, dbuf, oam_addr, fine_x;
    int show_bg, show_spr, hide_bg, hide_spr, tall, nmi_on, bg_page, spr_page;
    int nsl; uint8_t sl[8];
    uint16_t v, t, inc;
    uint8_t oam[256], pal[32], vram[2048], ram[2048];
} state_t;

typedef struct {
    state_t s;
    const cart_t* cart;
    uint8_t* screen;         /* 240x256 palette values, optional */
    uint8_t* gray;           /* 240x256 gray, optional */
    const uint8_t* lut;
    int render;
    int64_t cur;             /* iteration of the executing instruction */
    int skip;
    int64_t bad_ops;
} nes_t;

static void sync_to(nes_t* m, int64_t target);

/* ------------------------------------------------------------------ picture bus (nes_core.hpp:263-285) */
static int nt_slot(uint16_t a) { return a < 0x2400 ? 0 : a < 0x2800 ? 1 : a < 0x2c00 ? 2 : 3; }
static uint8_t vram_rd(const nes_t* m, uint16_t a) {
    if (a < 0x2000) return m->cart->chr[a];
    if (a < 0x3eff) return m->s.vram[m->cart->nt[nt_slot(a)] + (a & 0x3ff)];
    if (a < 0x3fff) return m->s.pal[a & 0x1f];
    return 0;
}
static void vram_wr(nes_t* m, uint16_t a, uint8_t v) {
    if (a < 0x2000) return;
    if (a < 0x3eff) m->s.vram[m->cart->nt[nt_slot(a)] + (a & 0x3ff)] = v;
    else if (a < 0x3fff) m->s.pal[a == 0x3f10 ? 0 : (a & 0x1f)] = v;
}
static uint8_t nt_rd(const nes_t* m, uint16_t a) { return m->s.vram[m->cart->nt[(a >> 10) & 3] + (a & 0x3ff)]; }

/* ------------------------------------------------------------------ PPU timing helpers (nes_core.hpp:289-334) */
static void set_thresh(nes_t* m) {
    state_t* s = &m->s;
    int line = s->pstate == PRE ? -1 : s->pstate == POST ? 240 : s->scanline;
    int64_t P = (int64_t)(line + 1) * 341 + (s->cyc - 1), PN = 242LL * 341;
    int64_t d = P <= PN ? PN - P + 1 : (262LL * 341 - P) + PN + 1;
    s->thresh = s->calls + d - 8;
}
static void cx_inc(state_t* s, int n) {
    if (n <= 0) return;
    int tot = (s->v & 0x1f) + n;
    s->v = (uint16_t)((s->v & ~0x1f) | (tot & 31));
    if ((tot >> 5) & 1) s->v ^= 0x0400;
}
static int cx_count(const state_t* s, int a, int b) {
    int r = (7 - s->fine_x) & 7;
    return (b - r + 7) / 8 - (a - r + 7) / 8;
}
static void fy_inc(state_t* s) {
    if ((s->v & 0x7000) != 0x7000) { s->v += 0x1000; return; }
    s->v &= ~0x7000;
    int yy = (s->v & 0x03E0) >> 5;
    if (yy == 29) { yy = 0; s->v ^= 0x0800; } else if (yy == 31) yy = 0; else yy++;
    s->v = (uint16_t)((s->v & ~0x03E0) | (yy << 5));
}
static void hcopy(state_t* s) { s->v = (uint16_t)((s->v & ~0x41f) | (s->t & 0x41f)); }
static void vcopy(state_t* s) { s->v = (uint16_t)((s->v & ~0x7be0) | (s->t & 0x7be0)); }

/* nes_core.hpp:336-349 */
static void eval_sprites(state_t* s) {
    int range = s->tall ? 16 : 8;
    s->nsl = 0;
    for (int i = s->oam_addr / 4; i < 64; i++) {
        int d = s->scanline - s->oam[i * 4];
        if (d >= 0 && d < range) { s->sl[s->nsl++] = (uint8_t)i; if (s->nsl >= 8) break; }
    }
}

/* 2-bit background value (opaque part) and palette bits at dot x for the current v (nes_core.hpp:352-366) */
static uint8_t bg_px(const nes_t* m, int x, int* opaque) {
    const state_t* s = &m->s;
    int xf = (s->fine_x + x) % 8;
    uint8_t tile = nt_rd(m, (uint16_t)(0x2000 | (s->v & 0x0FFF)));
    uint16_t ad = (uint16_t)((tile * 16 + ((s->v >> 12) & 7)) | (s->bg_page << 12));
    uint8_t c = (m->cart->chr[ad] >> (7 ^ xf)) & 1;
    c |= ((m->cart->chr[ad + 8] >> (7 ^ xf)) & 1) << 1;
    *opaque = c;
    uint16_t aa = (uint16_t)(0x23C0 | (s->v & 0x0C00) | ((s->v >> 4) & 0x38) | ((s->v >> 2) & 0x07));
    int sh = ((s->v >> 4) & 4) | (s->v & 2);
    return (uint8_t)(c | (((nt_rd(m, aa) >> sh) & 3) << 2));
}
/* nes_core.hpp:368-387 */
static uint8_t spr_px(const nes_t* m, int i, int x, int y) {
    const state_t* s = &m->s;
    int sx = s->oam[i * 4 + 3], sy = (uint8_t)(s->oam[i * 4] + 1), tile = s->oam[i * 4 + 1], at = s->oam[i * 4 + 2];
    int len = s->tall ? 16 : 8;
    int xs = (x - sx) % 8, yo = (y - sy) % len;
    if (!(at & 0x40)) xs ^= 7;
    if (at & 0x80) yo ^= len - 1;
    uint16_t ad;
    if (!s->tall) { ad = (uint16_t)(tile * 16 + yo); if (s->spr_page) ad += 0x1000; }
    else { yo = (yo & 7) | ((yo & 8) << 1); ad = (uint16_t)((tile >> 1) * 32 + yo); ad |= (tile & 1) << 12; }
    uint8_t c = (vram_rd(m, ad) >> xs) & 1;
    c |= ((vram_rd(m, (uint16_t)(ad + 8)) >> xs) & 1) << 1;
    return c;
}

/* visible dots [x0, x1) of the current line. Without rendering only the scroll increments and the exact
 * sprite-0 hit matter (nes_core.hpp:390-413); with rendering every dot is produced one at a time, which is the
 * per-dot form of nes_core.hpp:467-513. */
static void dots(nes_t* m, int x0, int x1) {
    state_t* s = &m->s;
    const int y = s->scanline;
    if (!m->render) {
        if (!s->show_bg) return;
        if (!s->s0hit && s->show_spr && s->nsl > 0 && s->sl[0] == 0) {
            int sx = s->oam[3], lo = x0 > sx ? x0 : sx, hi = x1 < sx + 8 ? x1 : sx + 8;
            if (s->hide_spr && lo < 8) lo = 8;
            if (lo < hi) {
                cx_inc(s, cx_count(s, x0, lo));
                for (int x = lo; x < hi; x++) {
                    if (!s->s0hit && (!s->hide_bg || x >= 8)) {
                        int op;
                        bg_px(m, x, &op);
                        if (op && spr_px(m, 0, x, y)) s->s0hit = 1;
                    }
                    if ((s->fine_x + x) % 8 == 7) cx_inc(s, 1);
                }
                cx_inc(s, cx_count(s, hi, x1));
                return;
            }
        }
        cx_inc(s, cx_count(s, x0, x1));
        return;
    }
    for (int x = x0; x < x1; x++) {
        uint8_t pa = 0;
        int op = 0;
        if (s->show_bg) {
            uint8_t c = bg_px(m, x, &op);
            pa = op ? c : 0;
            if (s->hide_bg && x < 8) { pa = 0; op = 0; }
        }
        if (s->show_spr && s->nsl && !(s->hide_spr && x < 8)) {
            for (int k = 0; k < s->nsl; k++) {        /* first opaque sprite of the list decides the dot */
                int i = s->sl[k], sx = s->oam[i * 4 + 3];
                if (x < sx || x >= sx + 8) continue;
                uint8_t c = spr_px(m, i, x, y);
                if (!c) continue;
                uint8_t at = s->oam[i * 4 + 2];
                if (i == 0 && op && !s->s0hit && s->show_bg) s->s0hit = 1;
                if (!op || !(at & 0x20)) pa = (uint8_t)(c | 0x10 | ((at & 3) << 2));
                break;
            }
        }
        if (s->show_bg && (s->fine_x + x) % 8 == 7) cx_inc(s, 1);
        if (m->screen) m->screen[y * 256 + x] = s->pal[pa];
        if (m->gray) m->gray[y * 256 + x] = m->lut[s->pal[pa]];
    }
}

static void push(nes_t* m, uint8_t v) { m->s.ram[(0x100 | m->s.sp--) & 0x7ff] = v; }
static uint8_t pull(nes_t* m) { return m->s.ram[(0x100 | ++m->s.sp) & 0x7ff]; }

/* NMI with nes-py's skip-cycle bookkeeping (nes_core.hpp:520-531) */
static void take_nmi(nes_t* m, int64_t call) {
    state_t* s = &m->s;
    int64_t it = (call - 1) / 3;
    push(m, (uint8_t)(s->pc >> 8)); push(m, (uint8_t)s->pc); push(m, (uint8_t)(s->p | 0x20));
    s->p |= FI;
    s->pc = (uint16_t)(m->cart->prg[0x7ffa] | m->cart->prg[0x7ffb] << 8);
    int64_t w = (s->zero_skip && it == s->exec_at) ? 0 : (s->exec_at - it + 1);
    s->exec_at = it + w + 6;
    s->zero_skip = 0;
}

/* n PPU::cycle calls, scanline segment at a time (nes_core.hpp:534-616) */
static void ppu(nes_t* m, int64_t n) {
    state_t* s = &m->s;
    while (n > 0) {
        int c = s->cyc;
        if (s->pstate == PRE) {
            int on = s->show_bg && s->show_spr, end = 341 - (!s->even && on);
            int64_t k = c >= end ? 1 : (n < end - c ? n : end - c);
            int a = c, b = (int)(c + k);
            if (a <= 1 && 1 < b) s->vblank = s->s0hit = 0;
            if (on) { if (a <= 258 && 258 < b) hcopy(s); if (a <= 304 && 281 < b) vcopy(s); }
            s->calls += k; n -= k;
            if (b - 1 >= end) { s->pstate = REND; s->scanline = 0; s->cyc = 1; } else s->cyc = b;
        } else if (s->pstate == REND) {
            if (c >= 1 && c <= 256) {
                int64_t k = n < 257 - c ? n : 257 - c;
                dots(m, c - 1, (int)(c - 1 + k));
                s->cyc += (int)k; s->calls += k; n -= k;
            } else if (c == 257) { if (s->show_bg) fy_inc(s); s->cyc++; s->calls++; n--; }
            else if (c == 258) { if (s->show_bg && s->show_spr) hcopy(s); s->cyc++; s->calls++; n--; }
            else if (c > 258 && c < 341) { int64_t k = n < 341 - c ? n : 341 - c; s->cyc += (int)k; s->calls += k; n -= k; }
            else if (c >= 341) {
                eval_sprites(s);
                s->scanline++; s->cyc = 1; s->calls++; n--;
                if (s->scanline >= 240) s->pstate = POST;
            } else { s->cyc++; s->calls++; n--; }
        } else if (s->pstate == POST) {
            if (c >= 341) { s->scanline++; s->cyc = 1; s->pstate = VBL; s->calls++; n--; }
            else { int64_t k = n < 341 - c ? n : 341 - c; s->cyc += (int)k; s->calls += k; n -= k; }
        } else {
            if (c >= 341) {
                s->scanline++; s->cyc = 1;
                if (s->scanline >= 261) { s->pstate = PRE; s->scanline = 0; s->even = !s->even; }
                s->calls++; n--;
            } else if (c == 1 && s->scanline == 241) {
                s->vblank = 1; s->calls++; n--; s->cyc = 2;
                if (s->nmi_on) take_nmi(m, s->calls);
            } else {
                int lim = 341 - c;
                if (s->scanline == 241 && c < 1) lim = 1 - c;
                int64_t k = n < lim ? n : lim;
                s->cyc += (int)k; s->calls += k; n -= k;
            }
        }
    }
}
static void sync_to(nes_t* m, int64_t target) {
    if (target > m->s.calls) { ppu(m, target - m->s.calls); set_thresh(m); }
}
static void sync_now(nes_t* m) { sync_to(m, 3 * (m->cur + 1)); }

/* ------------------------------------------------------------------ CPU bus (nes_core.hpp:150-260) */
static uint8_t joy(nes_t* m, int i) {
    uint8_t r;
    if (m->s.strobe[i]) r = m->s.buttons[i] & 1;
    else { r = m->s.bits[i] & 1; m->s.bits[i] >>= 1; }
    return r | 0x40;
}
static uint8_t rd(nes_t* m, uint16_t a) {
    state_t* s = &m->s;
    if (a >= 0x8000) return m->cart->prg[a & 0x7fff];
    if (a < 0x2000) return s->ram[a & 0x7ff];
    if (a < 0x4000) {
        switch (a & 0x2007) {
            case 0x2002: { sync_now(m); uint8_t st = (uint8_t)(s->s0hit << 6 | s->vblank << 7); s->vblank = 0; s->latch = 1; return st; }
            case 0x2007: {
                sync_now(m);
                uint8_t d = vram_rd(m, s->v);
                s->v = (uint16_t)(s->v + s->inc);
                if (s->v < 0x3f00) { uint8_t t = d; d = (uint8_t)s->dbuf; s->dbuf = t; }
                return d;
            }
            case 0x2004: return s->oam[s->oam_addr];
            default: return 0;
        }
    }
    if (a == 0x4016) return joy(m, 0);
    if (a == 0x4017) return joy(m, 1);
    return 0;
}
static void wr(nes_t* m, uint16_t a, uint8_t v) {
    state_t* s = &m->s;
    if (a < 0x2000) { s->ram[a & 0x7ff] = v; return; }
    if (a < 0x4000) {
        switch (a & 0x2007) {
            case 0x2000: sync_now(m);
                s->nmi_on = (v & 0x80) != 0; s->tall = (v & 0x20) != 0; s->bg_page = (v & 0x10) ? 1 : 0;
                s->spr_page = (v & 8) ? 1 : 0; s->inc = (v & 4) ? 32 : 1;
                s->t = (uint16_t)((s->t & ~0xc00) | ((v & 3) << 10)); break;
            case 0x2001: sync_now(m);
                s->hide_bg = !(v & 2); s->hide_spr = !(v & 4); s->show_bg = (v & 8) != 0; s->show_spr = (v & 16) != 0; break;
            case 0x2003: sync_now(m); s->oam_addr = v; break;
            case 0x2004: sync_now(m); s->oam[s->oam_addr] = v; s->oam_addr = (s->oam_addr + 1) & 0xff; break;
            case 0x2005: sync_now(m);
                if (s->latch) { s->t = (uint16_t)((s->t & ~0x1f) | ((v >> 3) & 0x1f)); s->fine_x = v & 7; s->latch = 0; }
                else { s->t = (uint16_t)((s->t & ~0x73e0) | ((v & 7) << 12) | ((v & 0xf8) << 2)); s->latch = 1; }
                break;
            case 0x2006: sync_now(m);
                if (s->latch) { s->t = (uint16_t)((s->t & ~0xff00) | ((v & 0x3f) << 8)); s->latch = 0; }
                else { s->t = (uint16_t)((s->t & ~0xff) | v); s->v = s->t; s->latch = 1; }
                break;
            case 0x2007: sync_now(m); vram_wr(m, s->v, v); s->v = (uint16_t)(s->v + s->inc); break;
            default: break;
        }
        return;
    }
    if (a == 0x4014) {  /* OAM DMA, nes_core.hpp:184-195 */
        sync_now(m);
        m->skip += 513 + (int)((m->cur + 1) & 1);
        uint16_t src = (uint16_t)(v << 8);
        if (src < 0x2000)
            for (int k = 0; k < 256; k++) s->oam[(s->oam_addr + k) & 0xff] = s->ram[(src & 0x7ff) + k];
        return;
    }
    if (a == 0x4016)
        for (int i = 0; i < 2; i++) { s->strobe[i] = v & 1; if (!s->strobe[i]) s->bits[i] = s->buttons[i]; }
}

/* ------------------------------------------------------------------ CPU (nes_core.hpp:619-1163) */
static void zn(state_t* s, uint8_t v) { s->p = (uint8_t)((s->p & ~(FZ | FN)) | (v ? 0 : FZ) | ((v & 0x80) ? FN : 0)); }
static void flag(state_t* s, uint8_t f, int on) { s->p = (uint8_t)(on ? (s->p | f) : (s->p & ~f)); }
static int has(const state_t* s, uint8_t f) { return (s->p & f) != 0; }
static uint16_t rd16(nes_t* m, uint16_t a) { uint8_t lo = rd(m, a); uint8_t hi = rd(m, (uint16_t)(a + 1)); return (uint16_t)(lo | hi << 8); }
static void cross(nes_t* m, uint16_t a, uint16_t b, int inc) { if ((a & 0xff00) != (b & 0xff00)) m->skip += inc; }

static int op_implied(nes_t* m, uint8_t op) {   /* nes_core.hpp:645-689 */
    state_t* s = &m->s;
    switch (op) {
        case 0x00: s->pc++; push(m, (uint8_t)(s->pc >> 8)); push(m, (uint8_t)s->pc); push(m, (uint8_t)(s->p | 0x30));
                   s->p |= FI; s->pc = rd16(m, 0xfffe); m->skip += 7; break;
        case 0x08: push(m, s->p); break;
        case 0x18: flag(s, FC, 0); break;
        case 0x20: push(m, (uint8_t)((s->pc + 1) >> 8)); push(m, (uint8_t)(s->pc + 1)); s->pc = rd16(m, s->pc); break;
        case 0x28: s->p = pull(m); break;
        case 0x38: flag(s, FC, 1); break;
        case 0x40: s->p = pull(m); s->pc = pull(m); s->pc |= pull(m) << 8; break;
        case 0x48: push(m, s->a); break;
        case 0x4C: s->pc = rd16(m, s->pc); break;
        case 0x58: flag(s, FI, 0); break;
        case 0x60: s->pc = pull(m); s->pc |= pull(m) << 8; s->pc++; break;
        case 0x68: s->a = pull(m); zn(s, s->a); break;
        case 0x6C: { uint16_t loc = rd16(m, s->pc), pg = loc & 0xff00; uint8_t lo = rd(m, loc);
                     uint8_t hi = rd(m, (uint16_t)(pg | ((loc + 1) & 0xff))); s->pc = (uint16_t)(lo | hi << 8); break; }
        case 0x78: flag(s, FI, 1); break;
        case 0x88: s->y--; zn(s, s->y); break;
        case 0x8A: s->a = s->x; zn(s, s->a); break;
        case 0x98: s->a = s->y; zn(s, s->a); break;
        case 0x9A: s->sp = s->x; break;
        case 0xA8: s->y = s->a; zn(s, s->y); break;
        case 0xAA: s->x = s->a; zn(s, s->x); break;
        case 0xB8: flag(s, FV, 0); break;
        case 0xBA: s->x = s->sp; zn(s, s->x); break;
        case 0xC8: s->y++; zn(s, s->y); break;
        case 0xCA: s->x--; zn(s, s->x); break;
        case 0xD8: flag(s, FD, 0); break;
        case 0xE8: s->x++; zn(s, s->x); break;
        case 0xEA: break;
        case 0xF8: flag(s, FD, 1); break;
        default: return 0;
    }
    return 1;
}
static int op_branch(nes_t* m, uint8_t op) {    /* nes_core.hpp:691-710 */
    state_t* s = &m->s;
    if ((op & 0x1f) != 0x10) return 0;
    static const uint8_t fl[4] = {FN, FV, FC, FZ};
    int want = (op & 0x20) != 0;
    if (has(s, fl[op >> 6]) == want) {
        int8_t off = (int8_t)rd(m, s->pc++);
        m->skip++;
        uint16_t np = (uint16_t)(s->pc + off);
        cross(m, s->pc, np, 2);
        s->pc = np;
    } else s->pc++;
    return 1;
}
static void alu(nes_t* m, int opn, uint16_t loc) {   /* type1 operations, nes_core.hpp:791-821 */
    state_t* s = &m->s;
    switch (opn) {
        case 0: s->a |= rd(m, loc); zn(s, s->a); break;
        case 1: s->a &= rd(m, loc); zn(s, s->a); break;
        case 2: s->a ^= rd(m, loc); zn(s, s->a); break;
        case 3: { uint8_t o = rd(m, loc); uint16_t sum = (uint16_t)(s->a + o + has(s, FC));
                  flag(s, FC, sum & 0x100); flag(s, FV, (s->a ^ sum) & (o ^ sum) & 0x80); s->a = (uint8_t)sum; zn(s, s->a); break; }
        case 4: wr(m, loc, s->a); break;
        case 5: s->a = rd(m, loc); zn(s, s->a); break;
        case 6: { uint16_t d = (uint16_t)(s->a - rd(m, loc)); flag(s, FC, !(d & 0x100)); zn(s, (uint8_t)d); break; }
        default: { uint16_t sb = rd(m, loc); uint16_t d = (uint16_t)(s->a - sb - !has(s, FC));
                   flag(s, FC, !(d & 0x100)); flag(s, FV, (s->a ^ d) & (~sb ^ d) & 0x80); s->a = (uint8_t)d; zn(s, (uint8_t)d); }
    }
}
static int op_type1(nes_t* m, uint8_t op) {     /* nes_core.hpp:754-823 */
    state_t* s = &m->s;
    if ((op & 3) != 1) return 0;
    int opn = op >> 5, mode = (op >> 2) & 7;
    uint16_t loc = 0;
    switch (mode) {
        case 0: { uint8_t za = (uint8_t)(s->x + rd(m, s->pc++)); loc = (uint16_t)(rd(m, za) | rd(m, (za + 1) & 0xff) << 8); break; }
        case 1: loc = rd(m, s->pc++); break;
        case 2: loc = s->pc++; break;
        case 3: loc = rd16(m, s->pc); s->pc += 2; break;
        case 4: {
            uint8_t za = rd(m, s->pc++);
            loc = (uint16_t)(rd(m, za) | rd(m, (za + 1) & 0xff) << 8);
            if (opn != 4) cross(m, loc, (uint16_t)(loc + s->y), 1);
            loc = (uint16_t)(loc + s->y);
            break;
        }
        case 5: loc = (rd(m, s->pc++) + s->x) & 0xff; break;
        case 6: loc = rd16(m, s->pc); s->pc += 2; if (opn != 4) cross(m, loc, (uint16_t)(loc + s->y), 1); loc = (uint16_t)(loc + s->y); break;
        default: loc = rd16(m, s->pc); s->pc += 2; if (opn != 4) cross(m, loc, (uint16_t)(loc + s->x), 1); loc = (uint16_t)(loc + s->x); break;
    }
    alu(m, opn, loc);
    return 1;
}
static int op_type2(nes_t* m, uint8_t op) {     /* nes_core.hpp:825-893 */
    state_t* s = &m->s;
    if ((op & 3) != 2) return 0;
    int opn = op >> 5, mode = (op >> 2) & 7;
    uint16_t loc = 0;
    uint8_t idx = (opn == 4 || opn == 5) ? s->y : s->x;
    switch (mode) {
        case 0: loc = s->pc++; break;
        case 1: loc = rd(m, s->pc++); break;
        case 2: break;
        case 3: loc = rd16(m, s->pc); s->pc += 2; break;
        case 5: loc = (rd(m, s->pc++) + idx) & 0xff; break;
        case 7: loc = rd16(m, s->pc); s->pc += 2; cross(m, loc, (uint16_t)(loc + idx), 1); loc = (uint16_t)(loc + idx); break;
        default: return 0;
    }
    int c0 = has(s, FC);
    if (opn <= 3) {
        uint8_t v = mode == 2 ? s->a : rd(m, loc);
        if (opn <= 1) { flag(s, FC, v & 0x80); v = (uint8_t)(v << 1 | (c0 && opn == 1)); }
        else { flag(s, FC, v & 1); v = (uint8_t)(v >> 1 | ((c0 && opn == 3) << 7)); }
        zn(s, v);
        if (mode == 2) s->a = v; else wr(m, loc, v);
    } else if (opn == 4) wr(m, loc, s->x);
    else if (opn == 5) { s->x = rd(m, loc); zn(s, s->x); }
    else { uint8_t v = (uint8_t)(rd(m, loc) + (opn == 6 ? -1 : 1)); zn(s, v); wr(m, loc, v); }
    return 1;
}
static int op_type0(nes_t* m, uint8_t op) {     /* nes_core.hpp:712-752 */
    state_t* s = &m->s;
    if ((op & 3) != 0) return 0;
    uint16_t loc = 0;
    switch ((op >> 2) & 7) {
        case 0: loc = s->pc++; break;
        case 1: loc = rd(m, s->pc++); break;
        case 3: loc = rd16(m, s->pc); s->pc += 2; break;
        case 5: loc = (rd(m, s->pc++) + s->x) & 0xff; break;
        case 7: loc = rd16(m, s->pc); s->pc += 2; cross(m, loc, (uint16_t)(loc + s->x), 1); loc = (uint16_t)(loc + s->x); break;
        default: return 0;
    }
    switch (op >> 5) {
        case 1: { uint8_t o = rd(m, loc); flag(s, FZ, !(s->a & o)); flag(s, FV, o & 0x40); flag(s, FN, o & 0x80); break; }
        case 4: wr(m, loc, s->y); break;
        case 5: s->y = rd(m, loc); zn(s, s->y); break;
        case 6: { uint16_t d = (uint16_t)(s->y - rd(m, loc)); flag(s, FC, !(d & 0x100)); zn(s, (uint8_t)d); break; }
        case 7: { uint16_t d = (uint16_t)(s->x - rd(m, loc)); flag(s, FC, !(d & 0x100)); zn(s, (uint8_t)d); break; }
        default: return 0;
    }
    return 1;
}
static int step_cpu(nes_t* m) {                 /* nes_core.hpp:895-900, 901-1163 */
    m->skip = 0;
    uint8_t op = rd(m, m->s.pc++);
    if (op_implied(m, op) || op_branch(m, op) || op_type1(m, op) || op_type2(m, op) || op_type0(m, op)) m->skip += CYC[op];
    else m->bad_ops++;
    return m->skip;
}

static uint8_t prg_or_ff(const nes_t* m, uint16_t a) { return a >= 0x8000 ? m->cart->prg[a & 0x7fff] : 0xff; }

/* one emulated frame (nes_core.hpp:1166-1204) */
static void frame(nes_t* m) {
    state_t* s = &m->s;
    const int64_t end = s->iter + ITERS;
    while (s->exec_at < end) {
        const int64_t J = s->exec_at;
        if (3 * (J + 1) >= s->thresh) {
            m->cur = J;
            sync_to(m, 3 * (J + 1));
            if (s->exec_at != J) continue;
        }
        if (prg_or_ff(m, s->pc) == 0x4C &&
            (uint16_t)(prg_or_ff(m, (uint16_t)(s->pc + 1)) | prg_or_ff(m, (uint16_t)(s->pc + 2)) << 8) == s->pc) {
            int64_t le = end - J, ln = s->thresh - 3 * (J + 1);
            int64_t k1 = le > 0 ? (le + 2) / 3 : 0, k2 = ln > 0 ? (ln + 8) / 9 : 0, k = k1 < k2 ? k1 : k2;
            if (k > 1) { s->exec_at = J + 3 * (k - 1); s->zero_skip = 0; continue; }
        }
        m->cur = J;
        int S = step_cpu(m);
        s->exec_at = J + (S >= 1 ? S : 1);
        s->zero_skip = S <= 0;
    }
    sync_to(m, 3 * end);
    s->iter = end;
}

/* power-on + reset (nes_core.hpp:128-147) */
static void power_on(nes_t* m, const cart_t* c) {
    state_t* s = &m->s;
    m->cart = c;
    memset(s, 0, sizeof *s);
    s->strobe[0] = s->strobe[1] = 1;
    s->p = 0x34; s->pc = (uint16_t)(c->prg[0x7ffc] | c->prg[0x7ffd] << 8); s->sp = 0xfd;
    s->show_bg = s->show_spr = 1; s->even = 1; s->latch = 1; s->inc = 1; s->pstate = PRE;
    set_thresh(m);
}

/* ------------------------------------------------------------------ numpy PCG64 (fastmario.cpp:39-78) */
typedef struct { unsigned __int128 st, inc; int has32; uint32_t u32; } pcg_t;
static uint64_t pcg64(pcg_t* r) {
    const unsigned __int128 M = ((unsigned __int128)0x2360ED051FC65DA4ULL << 64) | 0x4385DF649FCCF645ULL;
    r->st = r->st * M + r->inc;
    uint64_t hi = (uint64_t)(r->st >> 64), lo = (uint64_t)r->st;
    unsigned rot = (unsigned)(r->st >> 122);
    uint64_t x = hi ^ lo;
    return (x >> rot) | (x << ((64 - rot) & 63));
}
static uint32_t pcg32(pcg_t* r) {
    if (r->has32) { r->has32 = 0; return r->u32; }
    uint64_t n = pcg64(r);
    r->has32 = 1; r->u32 = (uint32_t)(n >> 32);
    return (uint32_t)n;
}
static double pcg_random(pcg_t* r) { return (double)(pcg64(r) >> 11) * (1.0 / 9007199254740992.0); }
static int64_t pcg_int(pcg_t* r, int64_t high) {
    uint64_t rng = (uint64_t)(high - 1);
    if (!rng) return 0;
    if (rng == 0xFFFFFFFFULL) return pcg32(r);
    uint32_t ex = (uint32_t)rng + 1;
    uint64_t mm = (uint64_t)pcg32(r) * ex;
    uint32_t left = (uint32_t)mm;
    if (left < ex) {
        uint32_t thr = (uint32_t)((0xFFFFFFFFu - (uint32_t)rng) % ex);
        while (left < thr) { mm = (uint64_t)pcg32(r) * ex; left = (uint32_t)mm; }
    }
    return (int64_t)(mm >> 32);
}

/* ------------------------------------------------------------------ OpenCV INTER_AREA, reference order (fastmario.cpp:81-130) */
typedef struct { int d, s; float w; } tap_t;
static int area_taps(int ss, int ds, tap_t* t) {
    double scale = 1. / ((double)ds / ss);
    int k = 0;
    for (int dx = 0; dx < ds; dx++) {
        double f1 = dx * scale, f2 = f1 + scale, cell = scale < ss - f1 ? scale : ss - f1;
        int s1 = (int)ceil(f1), s2 = (int)floor(f2);
        if (s2 > ss - 1) s2 = ss - 1;
        if (s1 > s2) s1 = s2;
        if (s1 - f1 > 1e-3) { t[k].d = dx; t[k].s = s1 - 1; t[k++].w = (float)((s1 - f1) / cell); }
        for (int sx = s1; sx < s2; sx++) { t[k].d = dx; t[k].s = sx; t[k++].w = (float)(1.0 / cell); }
        if (f2 - s2 > 1e-3) {
            double r = f2 - s2 < 1. ? f2 - s2 : 1.;
            if (r > cell) r = cell;
            t[k].d = dx; t[k].s = s2; t[k++].w = (float)(r / cell);
        }
    }
    return k;
}
static uint8_t satr(float v) { int i = (int)lrintf(v); return (uint8_t)(i < 0 ? 0 : i > 255 ? 255 : i); }
void orc_resize(const uint8_t* src, uint8_t* dst) {   /* 240x256 -> 84x84, area_resize_ref order */
    tap_t xt[512], yt[480];
    int xn = area_taps(256, 84, xt), yn = area_taps(240, 84, yt);
    float buf[84], sum[84];
    memset(sum, 0, sizeof sum);
    int prev = yt[0].d;
    for (int j = 0; j < yn; j++) {
        float beta = yt[j].w;
        const uint8_t* S = src + yt[j].s * 256;
        for (int dx = 0; dx < 84; dx++) buf[dx] = 0.f;
        for (int k = 0; k < xn; k++) buf[xt[k].d] += S[xt[k].s] * xt[k].w;
        if (yt[j].d != prev) {
            for (int dx = 0; dx < 84; dx++) { dst[prev * 84 + dx] = satr(sum[dx]); sum[dx] = beta * buf[dx]; }
            prev = yt[j].d;
        } else for (int dx = 0; dx < 84; dx++) sum[dx] += beta * buf[dx];
    }
    for (int dx = 0; dx < 84; dx++) dst[prev * 84 + dx] = satr(sum[dx]);
}

/* ------------------------------------------------------------------ SMB RAM (fastmario.cpp:205-250) */
static int64_t digits(const uint8_t* r, int n) {
    int64_t v = 0;
    for (int i = 0; i < n; i++) { int b = r[i]; v = v * (b >= 100 ? 1000 : b >= 10 ? 100 : 10) + b; }
    return v;
}
static int64_t xpos(const uint8_t* r) { return (int64_t)r[0x6d] * 256 + r[0x86]; }
static int64_t tleft(const uint8_t* r) { return digits(r + 0x7f8, 3); }
static int dying(const uint8_t* r) { return r[0x0e] == 0x0b || r[0xb5] > 1; }
static int dead(const uint8_t* r) { return r[0x0e] == 0x06; }
static int busy(const uint8_t* r) { return r[0x0e] <= 5 || r[0x0e] == 7; }
static int wover(const uint8_t* r) { return r[0x770] == 2; }
static int sover(const uint8_t* r) {
    for (int a = 0x16; a <= 0x1a; a++) if (r[a] == 0x2D || r[a] == 0x31) return r[0x1d] == 3;
    return 0;
}
static void info10(const uint8_t* r, int64_t* o) {
    o[0] = xpos(r); o[1] = wover(r) || sover(r); o[2] = r[0x75a]; o[3] = digits(r + 0x7de, 6); o[4] = tleft(r);
    o[5] = r[0x75f] + 1; o[6] = r[0x75c] + 1; o[7] = digits(r + 0x7ed, 2);
    o[8] = r[0xb5] < 1 ? 255 + (255 - r[0x3b8]) : 255 - r[0x3b8];
    o[9] = r[0x756] == 0 ? 0 : r[0x756] == 1 ? 1 : 2;
}

/* ------------------------------------------------------------------ env (fastmario.cpp:252-412) */
static const uint8_t MOVES[7] = {0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40};
#define GSZ (240 * 256)
#define OSZ (84 * 84)
typedef struct { int w, s, a; state_t backup; int64_t x0, t0; uint8_t obs0[OSZ]; } level_t;
typedef struct {
    nes_t nes;
    const level_t* lvl;
    int64_t x_last, t_last;
    pcg_t rng;
    int prev, lives, t, ep_len, pooled, from_backup;
    double ep_ret;
    uint8_t g[GSZ], gprev[GSZ];
    state_t snaps[16];
    uint8_t acts[16];
    int64_t info[10];
    int64_t frames;
} env_t;
typedef struct {
    int n, K, skip, max_steps, noop_max, maxpool;
    double sticky;
    cart_t cart;
    uint8_t lut[256];
    int nl;
    level_t* levels;
    env_t* envs;
} venv_t;

static void restore(env_t* e) { e->nes.s = e->lvl->backup; e->x_last = e->lvl->x0; e->t_last = e->lvl->t0; e->from_backup = 1; }
static void emu(env_t* e, uint8_t b, int render) {     /* fastmario.cpp:297-303 */
    e->nes.s.buttons[0] = b;
    e->nes.render = render;
    e->nes.gray = render ? e->g : NULL;
    frame(&e->nes);
    e->frames++;
    if (render) e->from_backup = 0;
}
static void hacks(env_t* e, int render) {              /* fastmario.cpp:304-314 */
    uint8_t* r = e->nes.s.ram;
    if (r[0x6de] > 1 && r[0x6de] < 255) r[0x6de] = 1;
    while (busy(r) || wover(r)) { r[0x7a0] = 0; emu(e, 0, render); }
}
static double frame_step(env_t* e, uint8_t b, int render, int* done) {   /* fastmario.cpp:316-334 */
    emu(e, b, render);
    const uint8_t* r = e->nes.s.ram;
    int64_t x = xpos(r), xr = x - e->x_last;
    e->x_last = x;
    if (xr < -5 || xr > 5) xr = 0;
    int64_t tm = tleft(r), tp = tm - e->t_last;
    e->t_last = tm;
    if (tp > 0) tp = 0;
    int dy = dying(r), dd = dead(r);
    int64_t rw = xr + tp + ((dy || dd) ? -25 : 0);
    if (rw < -15) rw = -15;
    if (rw > 15) rw = 15;
    info10(r, e->info);
    *done = dy || dd || e->info[1];
    if (!*done) hacks(e, render);
    return (double)rw;
}
static double agent_step(env_t* e, const venv_t* v, int a, int want, int* term) {   /* fastmario.cpp:336-374 */
    int K = v->skip, mp = v->maxpool, done = 0, i;
    double total = 0;
    for (i = 0; i < K; i++) {
        int ae = a;
        if (v->sticky != 0.0 && pcg_random(&e->rng) < v->sticky) ae = e->prev;
        e->prev = ae;
        int render = want && (i == K - 1 || (mp && i == K - 2));
        if (want) e->snaps[i] = e->nes.s;
        e->acts[i] = (uint8_t)ae;
        total += frame_step(e, MOVES[ae], render, &done);
        if (want && mp && i == K - 2) memcpy(e->gprev, e->g, GSZ);
        if (done) break;
    }
    int last = done ? i : K - 1;
    if (want && done && last < K - 1) {
        if (mp && last >= 1) {
            e->nes.s = e->snaps[last - 1];
            emu(e, MOVES[e->acts[last - 1]], 1);
            hacks(e, 1);
            memcpy(e->gprev, e->g, GSZ);
        } else e->nes.s = e->snaps[last];
        emu(e, MOVES[e->acts[last]], 1);
    }
    if (want) e->pooled = mp && last >= 1;
    int tt = done;
    int life = (int)e->info[2];
    if (e->lives >= 0 && life < e->lives) tt = 1;
    e->lives = life;
    if (e->info[1]) tt = 1;
    *term = tt;
    return total;
}
static void make_obs(env_t* e, uint8_t* out, int pool) {   /* fastmario.cpp:377-386 */
    if (e->from_backup) { memcpy(out, e->lvl->obs0, OSZ); return; }
    if (pool && e->pooled) {
        for (int k = 0; k < GSZ; k++) if (e->g[k] > e->gprev[k]) e->gprev[k] = e->g[k];
        orc_resize(e->gprev, out);
    } else orc_resize(e->g, out);
}
static void env_reset(env_t* e, const venv_t* v, uint8_t* out) {   /* fastmario.cpp:389-401 */
    restore(e); e->prev = 0; e->lives = -1;
    if (v->noop_max) {
        int64_t k = pcg_int(&e->rng, v->noop_max + 1);
        for (int64_t j = 0; j < k; j++) {
            int term;
            agent_step(e, v, 0, j == k - 1, &term);
            if (term) { restore(e); e->prev = 0; e->lives = -1; }
        }
    }
    e->t = 0; e->ep_ret = 0; e->ep_len = 0;
    make_obs(e, out, 0);
}

/* SMB boot protocol (fastmario.cpp:422-445) with a frame cap */
static int boot(const venv_t* v, level_t* L, int cap) {
    nes_t* m = calloc(1, sizeof(nes_t));
    uint8_t* g = malloc(GSZ);
    m->lut = v->lut;
    power_on(m, &v->cart);
    int frames = 0;
#define FA(b) do { m->s.buttons[0] = (b); m->render = 1; m->gray = g; frame(m); if (++frames > cap) { free(g); free(m); return -1; } } while (0)
    FA(8); FA(0);
    while (tleft(m->s.ram) == 0) {
        FA(8);
        m->s.ram[0x75f] = (uint8_t)(L->w - 1); m->s.ram[0x75c] = (uint8_t)(L->s - 1); m->s.ram[0x760] = (uint8_t)(L->a - 1);
        FA(0);
        m->s.ram[0x7a0] = 0;
    }
    int64_t tl = tleft(m->s.ram);
    while (tleft(m->s.ram) >= tl) { tl = tleft(m->s.ram); FA(8); FA(0); }
#undef FA
    L->backup = m->s;
    L->x0 = xpos(m->s.ram);
    L->t0 = tleft(m->s.ram);
    orc_resize(g, L->obs0);
    free(g); free(m);
    return 0;
}

/* ------------------------------------------------------------------ C API (sequential; shaped like fm_*) */
void* orc_create(const uint8_t* rom, int64_t len, int n, const int* levels, const uint8_t* lut, int skip, int max_steps,
                 double sticky, int noop_max, int maxpool, int frame_stack, const uint64_t* rng, int boot_cap) {
    if (skip < 1 || skip > 16 || n < 1) return NULL;
    venv_t* v = calloc(1, sizeof(venv_t));
    if (cart_parse(&v->cart, rom, (size_t)len)) { free(v); return NULL; }
    v->n = n; v->K = frame_stack; v->skip = skip; v->max_steps = max_steps; v->sticky = sticky;
    v->noop_max = noop_max; v->maxpool = maxpool;
    memcpy(v->lut, lut, 256);
    v->levels = calloc((size_t)n, sizeof(level_t));
    v->envs = calloc((size_t)n, sizeof(env_t));
    for (int i = 0; i < n; i++) {
        int found = -1;
        for (int q = 0; q < v->nl; q++)
            if (v->levels[q].w == levels[3 * i] && v->levels[q].s == levels[3 * i + 1] && v->levels[q].a == levels[3 * i + 2]) found = q;
        if (found < 0) {
            level_t* L = &v->levels[v->nl];
            L->w = levels[3 * i]; L->s = levels[3 * i + 1]; L->a = levels[3 * i + 2];
            if (boot(v, L, boot_cap)) { free(v->levels); free(v->envs); free(v); return NULL; }
            found = v->nl++;
        }
        env_t* e = &v->envs[i];
        e->lvl = &v->levels[found];
        e->nes.cart = &v->cart; e->nes.lut = v->lut;
        restore(e);
        e->lives = -1;
        const uint64_t* r = rng + 6 * i;
        e->rng.st = ((unsigned __int128)r[0] << 64) | r[1];
        e->rng.inc = ((unsigned __int128)r[2] << 64) | r[3];
        e->rng.has32 = (int)r[4]; e->rng.u32 = (uint32_t)r[5];
    }
    return v;
}
void orc_reset(void* h, uint8_t* obs) {
    venv_t* v = h;
    uint8_t o[OSZ];
    for (int i = 0; i < v->n; i++) {
        uint8_t* st = obs + (size_t)i * v->K * OSZ;
        env_reset(&v->envs[i], v, o);
        memset(st, 0, (size_t)v->K * OSZ);
        memcpy(st + (size_t)(v->K - 1) * OSZ, o, OSZ);
    }
}
/* VecEnv::do_env (fastmario.cpp:477-504) for every env in turn */
void orc_step(void* h, const int64_t* actions, uint8_t* obs, uint8_t* fin, float* rew, uint8_t* term, uint8_t* trunc,
              int64_t* info, double* ep_ret, int64_t* ep_len) {
    venv_t* v = h;
    const int K = v->K;
    uint8_t o[OSZ];
    for (int i = 0; i < v->n; i++) {
        env_t* e = &v->envs[i];
        int te;
        double r = agent_step(e, v, (int)actions[i], 1, &te);
        e->t++;
        int tr = e->t >= v->max_steps;
        e->ep_ret += r; e->ep_len++;
        make_obs(e, o, 1);
        rew[i] = (float)r; term[i] = (uint8_t)te; trunc[i] = (uint8_t)tr;
        memcpy(info + 10 * i, e->info, sizeof e->info);
        uint8_t* st = obs + (size_t)i * K * OSZ;
        memmove(st, st + OSZ, (size_t)(K - 1) * OSZ);
        if (te || tr) {
            uint8_t* fo = fin + (size_t)i * K * OSZ;
            memcpy(fo, st, (size_t)(K - 1) * OSZ);
            memcpy(fo + (size_t)(K - 1) * OSZ, o, OSZ);
            ep_ret[i] = e->ep_ret; ep_len[i] = e->ep_len;
            env_reset(e, v, o);
            memset(st, 0, (size_t)(K - 1) * OSZ);
        }
        memcpy(st + (size_t)(K - 1) * OSZ, o, OSZ);
    }
}
void orc_ram(void* h, int i, uint8_t* out) { memcpy(out, ((venv_t*)h)->envs[i].nes.s.ram, 2048); }
int64_t orc_frames(void* h) { venv_t* v = h; int64_t f = 0; for (int i = 0; i < v->n; i++) f += v->envs[i].frames; return f; }
int64_t orc_bad_ops(void* h) { venv_t* v = h; int64_t f = 0; for (int i = 0; i < v->n; i++) f += v->envs[i].nes.bad_ops; return f; }
void orc_destroy(void* h) { venv_t* v = h; if (!v) return; free(v->levels); free(v->envs); free(v); }

/* raw console (fm_raw_*, fastmario.cpp:651-673) */
typedef struct { cart_t cart; nes_t nes; uint8_t screen[GSZ]; uint8_t ident[256]; state_t backup; } raw_t;
void* orc_raw_create(const uint8_t* rom, int64_t len) {
    raw_t* r = calloc(1, sizeof(raw_t));
    if (cart_parse(&r->cart, rom, (size_t)len)) { free(r); return NULL; }
    for (int i = 0; i < 256; i++) r->ident[i] = (uint8_t)i;
    power_on(&r->nes, &r->cart);
    return r;
}
void orc_raw_frame(void* h, int buttons, int render) {
    raw_t* r = h;
    r->nes.s.buttons[0] = (uint8_t)buttons;
    r->nes.render = render != 0;
    r->nes.screen = render ? r->screen : NULL;
    frame(&r->nes);
}
uint8_t* orc_raw_ram(void* h) { return ((raw_t*)h)->nes.s.ram; }
uint8_t* orc_raw_screen(void* h) { return ((raw_t*)h)->screen; }
void orc_raw_backup(void* h) { raw_t* r = h; r->backup = r->nes.s; }
void orc_raw_restore(void* h) { raw_t* r = h; r->nes.s = r->backup; }
int64_t orc_raw_bad_ops(void* h) { return ((raw_t*)h)->nes.bad_ops; }
void orc_raw_destroy(void* h) { free(h); }
