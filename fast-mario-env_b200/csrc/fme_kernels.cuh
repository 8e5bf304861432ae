// fme_kernels.cuh - device side: PCG64, the agent-step state machine, the warp renderer driver and kernels.
#pragma once
#include <cuda_runtime.h>
#include "fme_defs.h"

namespace fme {
__constant__ uint32_t c_dtab[256];
extern uint32_t g_host_dtab[256];
}
#if defined(__CUDA_ARCH__)
#define FME_DTAB(op) (::fme::c_dtab[(op)])
#else
#define FME_DTAB(op) (::fme::g_host_dtab[(op)])
#endif
#include "fme_core.h"
#include "fme_agent.h"
#include "fme_fast.h"
#include "fme_dp.h"
#include "fme_render.h"

namespace fme {

__constant__ AreaTabs c_area;

constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------- kernel parameters
struct Dev {
    int n, n_pad;
    uint8_t* slab;      // n_pad/32 groups x SLAB_BYTES
    uint8_t* vram;      // n_pad x 2048
    uint32_t* scal;     // S_WORDS x n_pad
    uint8_t* logs;      // n_pad x 2 slots
    int log_cap;
    const uint8_t* prg;
    const uint32_t* uop; // per-PC micro-ops (fme_tables.h build_uops), stored right after the 32 KB PRG
    const uint32_t* dop; // per-PC datapath micro-ops (fme_dp.h, build_dops), after the micro-ops
    const uint8_t* chr;
    uint32_t nt[4];
    const uint8_t* lut; // 256 gray LUT (global)
    uint32_t* err;      // global status word
};

struct StepParams {
    Dev d;
    int mode;
    int skip, max_steps, noop_max, maxpool, frame_stack;
    int sticky_on;
    uint64_t sticky_thr;  // draw counts as "repeat" when (next64 >> 11) < sticky_thr
    int hack_cap;
    uint64_t simple;      // SIMPLE_MOVEMENT controller bytes, byte k = action k
    const int64_t* actions;
    // outputs (MODE_STEP)
    uint8_t* obs; uint8_t* fin; float* rew; uint8_t* term; uint8_t* trunc; int32_t* info; double* ep_ret;
    int32_t* ep_len;
    Cache cache;
    int n_levels;
    // MODE_STEP with k_render: per-env render job word (bit 0 active, 1 pooled, 2 slot, 3 episode ended)
    uint32_t* jobs;
    int group_base;  // first group of this launch (k_step block b handles group group_base + b)
    uint32_t ram_end;   // RAM below this address in shared memory (RAM_END_DEEP / RAM_END_WIDE; 0x800 for MODE_NOOP)
    // MODE_NOOP: where to write the cache entry for this noop step
    uint8_t* out_img; uint8_t* out_obs; int32_t* out_meta; int noop_j;
    const uint8_t* level_img; const uint8_t* level_obs0; const int32_t* level_meta;  // backups (x0, t0)
};

__device__ __forceinline__ size_t slot_off(int e, int s, int cap) {
    return ((size_t)e * 2 + (size_t)s) * slot_bytes(cap);
}

// ---------------------------------------------------------------- per-lane console binding
__device__ __forceinline__ void bind_core(Core& c, const Dev& d, uint8_t* sm, int lane, int e) {
    c.ram = sm + SLAB_RAM_OFF + lane * 4;
    c.ramh = c.ram;
    c.ram_end = RAM_BYTES;
    c.oam = sm + SLAB_OAM_OFF + lane * 4;
    c.pal = sm + SLAB_PAL_OFF + lane * 4;
    c.vram = d.vram + (size_t)e * VRAM_BYTES;
    c.cart.prg = d.prg; c.cart.chr = d.chr;
    for (int i = 0; i < 4; i++) c.cart.nt[i] = d.nt[i];
    c.rec = nullptr; c.nrec = 0; c.cap = 0; c.seg_open = false; c.seg_w0 = 0; c.seg_y1 = 0; c.status = 0; c.seg_idx = 0; c.seg_reads = 0;
    c.vram_burst = 0; c.vram_dirty = false;
}

// Warp scheduling of the emulation loop: among the lanes that are about to execute an instruction only those
// at the warp's minimum PC run it, so lanes that took a shorter path wait at the join point and the warp
// re-converges on identical instructions (results cannot depend on the schedule: lanes are independent).
// Lanes spinning in a `JMP *` idle loop wait until every other lane is idle or at the frame boundary, and
// lanes at the frame boundary wait for all others: the warp then takes the idle fast-forward, the PPU catch-up
// before the NMI and the frame end together instead of one lane at a time. Returns true if this lane may step.
// sched_key + __reduce_min_sync: a lane steps when its key is the warp minimum; the minimum is 0xffffffff
// once no lane is running.
__device__ __forceinline__ uint32_t sched_key(bool running, const Hot& h) {
    uint32_t k = h.pc | ((h.ux & UOP_IDLE) ? 0x10000u : 0u);
    k = h.exec_at >= FRAME_ITERS ? 0x20000u : k;
    return running ? k : 0xffffffffu;
}
// The same key with the idle loops recognised by address (the ROM's first two `JMP *`, stored after its
// micro-op table): it does not wait for the micro-op load of the new pc, so that load overlaps the vote.
// Further idle loops only group less well; the key never changes what a lane computes.
__device__ __forceinline__ uint32_t sched_key_pc(bool running, const Hot& h, uint32_t ip0, uint32_t ip1) {
    uint32_t k = h.pc | ((h.pc == ip0) | (h.pc == ip1) ? 0x10000u : 0u);
    k = h.exec_at >= FRAME_ITERS ? 0x20000u : k;
    return running ? k : 0xffffffffu;
}
__device__ __forceinline__ bool minpc_turn(bool running, const Hot& h) {
    const uint32_t key = sched_key(running, h);
    const uint32_t mn = __reduce_min_sync(FULL, key);
    return running && key == mn;
}

// coalesced copy of a whole slab between HBM and shared memory (warp-wide)
__device__ __forceinline__ void copy_slab(uint8_t* dst, const uint8_t* src, int lane, int nbytes = SLAB_BYTES) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll 4
    for (int i = lane; i < nbytes / 16; i += 32) d[i] = s[i];
}
// k_step keeps only the group's RAM below StepParams::ram_end in shared memory (OAM, palette and the RAM above
// it stay in the HBM slab, reached through L1); this many bytes at most.
constexpr int STEP_SMEM = (int)RAM_END_DEEP * LANES;

// ---------------------------------------------------------------- warp renderer
// Shared-memory layout of the render phase (reuses the emulation slab region).
constexpr int RS_FB = 0;                         // 240 x 256
constexpr int RS_VRAM = RS_FB + SCREEN_W * SCREEN_H;
constexpr int RS_PAL = RS_VRAM + VRAM_BYTES;
constexpr int RS_OAM = RS_PAL + PAL_BYTES;
constexpr int RS_STAGE = RS_OAM + OAM_BYTES;     // one staged row (256)
constexpr int RS_OBS = RS_STAGE + SCREEN_W;      // 84 x 84 result
constexpr int RS_LUT = RS_OBS + OBS_BYTES;       // 256-entry gray LUT (identity for raw screens)
constexpr int RS_SPR = RS_LUT + 256;             // 16 words: sprite rows and infos of the current line
constexpr int RS_GV = RS_SPR + 64;               // 32 output values, one per palette address
constexpr int RS_END = RS_GV + 32;
static_assert(RS_END <= SLAB_BYTES, "render scratch must fit the slab region");

// Where a replay draws: framebuffer rows [row_lo, row_hi) (fb holds those rows only) and the warp's
// copies of the render inputs.
struct RLayout {
    uint8_t* fb; uint8_t* vram; uint8_t* pal; uint8_t* oam; uint8_t* stage; const uint8_t* lut;
    uint32_t* spr; uint8_t* gv;
    uint32_t* bmask;   // 32 words: sprites of the line's list that cover each 8-dot block (scratch of the replay)
    int row_lo, row_hi;
};
__device__ __forceinline__ RLayout full_layout(uint8_t* sm) {
    RLayout L;
    L.fb = sm + RS_FB; L.vram = sm + RS_VRAM; L.pal = sm + RS_PAL; L.oam = sm + RS_OAM; L.stage = sm + RS_STAGE;
    L.lut = sm + RS_LUT; L.spr = reinterpret_cast<uint32_t*>(sm + RS_SPR); L.gv = sm + RS_GV;
    L.bmask = reinterpret_cast<uint32_t*>(sm + RS_OBS);   // the resize output is written after the replays
    L.row_lo = 0; L.row_hi = SCREEN_H;
    return L;
}

// Replay one logged frame into the framebuffer rows of L. raw: palette values (screen) instead of gray.
// max_mode: combine with the frame already in the framebuffer by max (ALE-style max-pool).
// Work split: every record is read by all lanes; a segment's dots go 8 per lane (lane L: x0 + 8L ..);
// the line's sprite rows are fetched once per line by lanes 0..7 and broadcast through shared memory.
// Records and state changes are applied in full whatever the band; only lines inside it are drawn.
__device__ void render_slot(const uint8_t* slot, const RLayout& L, const Dev& d, bool raw, bool max_mode, int lane) {
    uint8_t* fb = L.fb - L.row_lo * SCREEN_W;  // indexed by screen row
    RState rs;
    rs.vram = L.vram; rs.pal = L.pal; rs.oam = L.oam; rs.chr = d.chr;
    rs.ntm = 0;
    for (int i = 0; i < 4; i++) rs.ntm |= (d.nt[i] >> 10 & 1u) << i;
    uint8_t* stage = L.stage;
    const uint8_t* lut = L.lut;
    {
        const uint4* hv = reinterpret_cast<const uint4*>(slot + SLOT_HDR_VRAM);
        uint4* sv = reinterpret_cast<uint4*>(rs.vram);
        for (int i = lane; i < VRAM_BYTES / 16; i += 32) sv[i] = hv[i];
        if (lane < PAL_BYTES / 4)
            reinterpret_cast<uint32_t*>(rs.pal)[lane] = reinterpret_cast<const uint32_t*>(slot + SLOT_HDR_PAL)[lane];
        for (int i = lane; i < OAM_BYTES / 4; i += 32)
            reinterpret_cast<uint32_t*>(rs.oam)[i] = reinterpret_cast<const uint32_t*>(slot + SLOT_HDR_OAM)[i];
    }
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(slot + SLOT_HDR_LIST);
    rs.nsl = lw[0] & 0xffu; rs.sl_lo = lw[1]; rs.sl_hi = lw[2];
    const int nrec = (int)lw[3] < d.log_cap ? (int)lw[3] : d.log_cap;
    const uint4* recs = reinterpret_cast<const uint4*>(slot + SLOT_HDR_BYTES);
    uint8_t* gv = L.gv;
    __syncwarp();
    {
        const uint32_t pv = rs.pal[lane];
        gv[lane] = raw ? (uint8_t)pv : lut[pv];
    }
    __syncwarp();
    int first_row = -1;
    uint32_t ver = 0;                                   // bumps on every content change (VRAM/palette/OAM)
    uint32_t lkey = 0xffffffffu, lnsl = 0, llo = 0, lhi = 0;   // cached pending-evaluation result
    uint32_t skey0 = 0xffffffffu, skey1 = 0, skey2 = 0;        // cached sprite rows of the current line
    uint32_t* srow_s = L.spr;                                   // the line's sprite rows (list order)
    uint32_t* sinfo_s = srow_s + 8;
    // records are read 32 at a time (one coalesced load, lane j holds record wb + j) and broadcast by shuffle
    int wb = -64;
    uint4 wv = make_uint4(0u, 0u, 0u, 0u);
    for (int r = 0; r < nrec; r++) {
        if (r >= wb + 32) {
            wb = r;
            if (wb + lane < nrec) wv = recs[wb + lane];
        }
        const int jw = r - wb;
        uint4 rec;
        rec.x = __shfl_sync(FULL, wv.x, jw); rec.y = __shfl_sync(FULL, wv.y, jw);
        rec.z = __shfl_sync(FULL, wv.z, jw); rec.w = __shfl_sync(FULL, wv.w, jw);
        uint32_t type = rec.x & 15u;
        if (type == REC_SEG) {
            Seg g = decode_seg(rec);
            for (;;) {  // one pass per line of the record
                if (max_mode && first_row < 0) first_row = g.y;
                if (g.y >= L.row_hi) break;                        // the rest of the record is below the band
                if (g.y < L.row_lo) {                              // above the band: jump to its first line
                    const int to = L.row_lo < g.y1 ? L.row_lo : g.y1;
                    if (to <= g.y) break;                          // the record ends above the band
                    seg_skip_lines(g, to - g.y);
                    continue;
                }
                uint32_t nsl = 0, lo = 0, hi = 0;
                if (!(g.flags & RF_SHOW_SPR)) {
                    // sprites hidden: no list needed
                } else if (g.pend) {
                    uint32_t key = g.ev_y | (g.oam_addr << 8) | ((g.flags & RF_LONG) ? 0x10000u : 0u) | (ver << 17);
                    if (key != lkey) {
                        int start = (int)(g.oam_addr >> 2);
                        int range = (g.flags & RF_LONG) ? 16 : 8;
                        int d0 = (int)g.ev_y - (int)rs.oam[lane * 4];
                        int d1 = (int)g.ev_y - (int)rs.oam[(lane + 32) * 4];
                        bool in0 = lane >= start && d0 >= 0 && d0 < range;
                        bool in1 = lane + 32 >= start && d1 >= 0 && d1 < range;
                        uint64_t m = (uint64_t)__ballot_sync(FULL, in0) | ((uint64_t)__ballot_sync(FULL, in1) << 32);
                        uint32_t n = 0, lo_ = 0, hi_ = 0;
                        while (m && n < 8) {
                            uint32_t i = (uint32_t)(__ffsll((long long)m) - 1);
                            m &= m - 1;
                            if (n < 4) lo_ |= i << (8 * n); else hi_ |= i << (8 * (n - 4));
                            n++;
                        }
                        lkey = key; lnsl = n; llo = lo_; lhi = hi_;
                    }
                    nsl = lnsl; lo = llo; hi = lhi;
                } else {
                    nsl = rs.nsl; lo = rs.sl_lo; hi = rs.sl_hi;
                }
                const bool spr_on = (g.flags & RF_SHOW_SPR) && nsl;
                if (spr_on) {
                    uint32_t k0 = (uint32_t)g.y | (nsl << 8) | ((g.flags & (RF_LONG | RF_SPR_PAGE)) << 12) | (ver << 20);
                    if (k0 != skey0 || lo != skey1 || hi != skey2) {
                        L.bmask[lane] = 0u;
                        __syncwarp();
                        if ((uint32_t)lane < nsl) {
                            int i = (int)(((lane < 4 ? lo >> (8 * lane) : hi >> (8 * (lane - 4)))) & 0xffu);
                            srow_s[lane] = sprite_row(rs, g.flags, i, g.y);
                            const uint32_t inf = sprite_info(rs, i);
                            sinfo_s[lane] = inf;
                            // the 8-dot blocks holding the sprite's dots x .. x+7 (dots past 255 do not exist)
                            const uint32_t x = inf & 0xffu, b0 = x >> 3, b1 = (x + 7u) >> 3;
                            atomicOr(&L.bmask[b0], 1u << lane);
                            if (b1 != b0 && b1 < 32u) atomicOr(&L.bmask[b1], 1u << lane);
                        }
                        skey0 = k0; skey1 = lo; skey2 = hi;
                        __syncwarp();
                    }
                }
                const bool to_stage = max_mode && g.y == first_row;
                const int xa = g.x0 + lane * 8;
                uint32_t outw[2];
                // candidates: the sprites covering either 8-dot block the lane's dots xa .. xa+7 touch (lanes
                // past the segment's end draw nothing that is stored; their block index only stays in range)
                const uint32_t cand = spr_on ? (L.bmask[(xa >> 3) & 31] | L.bmask[((xa + 7) >> 3) & 31]) : 0u;
                render8(rs, g, xa, cand, srow_s, sinfo_s, gv, outw);
                uint8_t* row = to_stage ? stage : fb + g.y * SCREEN_W;
                if (xa < g.x1) {
                    if (xa + 8 <= g.x1 && (xa & 7) == 0) {
                        uint2* dst = reinterpret_cast<uint2*>(row + xa);
                        uint2 nv = make_uint2(outw[0], outw[1]);
                        if (max_mode && !to_stage) { uint2 ov = *dst; nv.x = __vmaxu4(nv.x, ov.x); nv.y = __vmaxu4(nv.y, ov.y); }
                        *dst = nv;
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const int xx = xa + j;
                            if (xx < g.x1) {
                                uint8_t val = (uint8_t)(outw[j >> 2] >> (8 * (j & 3)));
                                if (max_mode && !to_stage) { uint8_t o = row[xx]; row[xx] = val > o ? val : o; }
                                else row[xx] = val;
                            }
                        }
                    }
                }
                if (g.y >= g.y1) break;
                seg_next_line(g);
                __syncwarp();
            }
        } else if (type == REC_DMA) {
            if (r + 16 >= nrec) break;  // truncated payload (the frame overflowed its log; status says so)
            if (lane < 16) {
                uint4 pl = recs[r + 1 + lane];
                *reinterpret_cast<uint4*>(rs.oam + 16 * lane) = pl;
            }
            r += 16;
            ver++;
        } else if (type == REC_VSNAP) {
            if (r + VRAM_BYTES / 16 >= nrec) break;
            for (int q = lane; q < VRAM_BYTES / 16; q += 32)
                reinterpret_cast<uint4*>(rs.vram)[q] = recs[r + 1 + q];
            r += VRAM_BYTES / 16;
            ver++;
        } else if (type == REC_LIST) {
            rs.nsl = (rec.x >> 4) & 0xffu; rs.sl_lo = rec.y; rs.sl_hi = rec.z;
        } else {
            if (lane == 0) {
                uint32_t idx = (rec.x >> 4) & 0x7ffu, val = (rec.x >> 16) & 0xffu;
                if (type == REC_VRAM) rs.vram[idx] = (uint8_t)val;
                else if (type == REC_PAL) { rs.pal[idx & 31u] = (uint8_t)val; gv[idx & 31u] = raw ? (uint8_t)val : lut[val]; }
                else if (type == REC_OAM) rs.oam[idx & 255u] = (uint8_t)val;
            }
            ver++;
        }
        __syncwarp();
    }
    if (max_mode && first_row >= L.row_lo && first_row < L.row_hi) {
        uint8_t* row = fb + first_row * SCREEN_W;
        for (int xx = lane; xx < SCREEN_W; xx += 32) { uint8_t o = row[xx], st = stage[xx]; row[xx] = st > o ? st : o; }
    }
    __syncwarp();
}

// Area resize of output rows [dy_lo, dy_hi) from framebuffer rows starting at screen row row_lo (fb holds
// the rows the taps of those output rows read) into out (row dy at (dy - dy_lo) * 84). Warp-wide; lane owns
// columns lane, lane+32, lane+64.
__device__ void resize_band(const uint8_t* fb, int row_lo, int dy_lo, int dy_hi, uint8_t* out, int lane) {
    fb -= row_lo * SCREEN_W;
    // a column's taps are AREA_XTAPS consecutive source dots from xs0 (zero-weight padded; checked when the
    // table is built), so the lane's three columns fit in registers
    int32_t xs0[3];
    float xw[3][AREA_XTAPS];
#pragma unroll
    for (int q = 0; q < 3; q++) {
        int dx = lane + 32 * q;
        xs0[q] = dx < OBS ? c_area.xs[0][dx] : 0;
#pragma unroll
        for (int k = 0; k < AREA_XTAPS; k++) xw[q][k] = dx < OBS ? c_area.xw[k][dx] : 0.f;
    }
    // A source row's horizontal sums do not depend on the output row that reads them, so the row shared by
    // two consecutive output rows (240 / 84 is not whole) is summed once: the sums of the last row read are
    // kept and reused when the next output row's first tap is that row.
    int crow = -1;
    float cb[3] = {0.f, 0.f, 0.f};
    for (int dy = dy_lo; dy < dy_hi; dy++) {
        float sacc[3] = {0.f, 0.f, 0.f};
        for (int m = 0; m < 6; m++) {
            float wy = c_area.yw[m][dy];
            if (wy == 0.f) break;
            const int sr = c_area.ys[m][dy];
            if (sr != crow) {
                const uint8_t* row = fb + sr * SCREEN_W;
#pragma unroll
                for (int q = 0; q < 3; q++) {
                    float b = 0.f;
#pragma unroll
                    for (int k = 0; k < AREA_XTAPS; k++) {
                        if (xw[q][k] != 0.f) b = fadd(b, fmul((float)row[xs0[q] + k], xw[q][k]));
                    }
                    cb[q] = b;
                }
                crow = sr;
            }
#pragma unroll
            for (int q = 0; q < 3; q++) sacc[q] = fadd(sacc[q], fmul(wy, cb[q]));
        }
#pragma unroll
        for (int q = 0; q < 3; q++) {
            int dx = lane + 32 * q;
            if (dx < OBS) out[(dy - dy_lo) * OBS + dx] = sat_round(sacc[q]);
        }
    }
    __syncwarp();
}
// the whole 84x84 frame from the full framebuffer into RS_OBS
__device__ __forceinline__ void resize_fb(uint8_t* sm, int lane) { resize_band(sm + RS_FB, 0, 0, OBS, sm + RS_OBS, lane); }

// gray LUT (or identity) into shared memory before a render phase
__device__ __forceinline__ void load_lut(uint8_t* sm, const uint8_t* lut, int lane) {
    if (lane < 16) reinterpret_cast<uint4*>(sm + RS_LUT)[lane] = reinterpret_cast<const uint4*>(lut)[lane];
    __syncwarp();
}

// warp copy helpers (16-byte granules; all buffers here are 16-byte aligned and sized in 16-byte units)
__device__ __forceinline__ void wcopy16(uint8_t* dst, const uint8_t* src, int nbytes, int lane) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = lane; i < nbytes / 16; i += 32) d[i] = s[i];
}
__device__ __forceinline__ void wzero16(uint8_t* dst, int nbytes, int lane) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = lane; i < nbytes / 16; i += 32) d[i] = z;
}
// thread-private 16-byte copy
__device__ __forceinline__ void tcopy16(uint8_t* dst, const uint8_t* src, int nbytes) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = 0; i < nbytes / 16; i++) d[i] = s[i];
}
// forward move inside one buffer (dst < src); safe for overlapping ranges moved by >= 512 bytes
__device__ __forceinline__ void wmove16(uint8_t* dst, const uint8_t* src, int nbytes, int lane) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    const int n16 = nbytes / 16;
    for (int base = 0; base < n16; base += 32) {
        int i = base + lane;
        uint4 v;
        if (i < n16) v = s[i];
        __syncwarp();
        if (i < n16) d[i] = v;
    }
}

}  // namespace fme
