// fme.cu - kernels and the C ABI (include/fme.h) of libfme_cuda.so.
//
// The timed step (fme_step) is two kernels per env slice (up to four slices, each forked from the caller's
// stream onto a high-priority emulation stream and a low-priority render stream, joined back with events):
//   k_step<true>   emulation, one CTA = one warp = 32 envs: the group's RAM below a boundary in shared memory
//                  (48 KB, or 23 KB for large env counts; the rest of RAM, OAM and palette read through L1
//                  from the HBM slab), `skip` frames (+ busy-state frames) per env with
//                  per-frame PPU logs, rewards / dones / infos, auto-reset from the reset cache, and a render job
//                  word per env.
//   k_render       one warp per (env, band of 60 screen rows): the frame-stack shift of the band, replay of the
//                  PPU log(s) into the band's rows (max-pooled), the exact-order INTER_AREA resize and the store
//                  of the band's 21 rows of the new 84x84 frame (into final_obs when the episode ended).
// Construction and API helpers:
//   k_boot         boot each distinct level from power-on (the SMB boot protocol), snapshot + first obs.
//   k_step<false>  the reset-cache builder (no-op steps with the renderer fused, one CTA per 32 levels).
//   k_init         put every env at its level snapshot (the reference's Env::init state).
//   k_reset        random no-op starts from the reset cache + zero-padded stacks (fm_reset).
//   k_raw          one frame for n raw consoles (+ palette-value screens).
//   k_resize, k_ram_all, k_power   helpers.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>
#include <algorithm>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "fme_kernels.cuh"
#include "fme_ppo.cuh"
#include "fme_replay.cuh"
#include "../../include/fme.h"
#include "fme_tables.h"

using namespace fme;
using namespace fme::tables;

// ====================================================================== device kernels
namespace fme {

struct BootParams {
    Dev d;
    int n_levels;
    const int32_t* levels;  // n_levels x 3
    int boot_cap;
    uint8_t* level_img;
    int32_t* level_meta;    // n_levels x 2 (x_pos, time)
    uint8_t* obs0;
};

__global__ void __launch_bounds__(32) k_boot(BootParams P) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int lane = threadIdx.x, g = blockIdx.x, l = g * 32 + lane;
    const Dev& d = P.d;
    const bool active = l < P.n_levels;
    Core c;
    bind_core(c, d, sm, lane, l);
    uint8_t* slot = d.logs + slot_off(l, 0, d.log_cap);
    int phase = 0, frames = 0;
    int64_t tl = 0;
    bool running = active;
    if (active) {
        c.bad_ops = 0;
        c.power_on();
        begin_frame(c, slot, 8, d.log_cap);
    } else {
        uint32_t zw[S_CONSOLE_WORDS];
        for (int k = 0; k < S_CONSOLE_WORDS; k++) zw[k] = 0;
        c.load_scalars(zw);  // idle lanes still hold a defined (never executed) state
        c.bad_ops = 0; c.status = 0;
    }
    const int w = active ? P.levels[3 * l] : 1, s = active ? P.levels[3 * l + 1] : 1, ar = active ? P.levels[3 * l + 2] : 1;
    // Boot protocol of SuperMarioBrosEnv (fastmario.cpp:422-445), one frame per call of the state machine:
    // phase 0 fa(8), 1 fa(0), then loop A {2: fa(8); write level; 3: fa(0); $7A0=0} while time==0,
    // then loop B {4: fa(8), 5: fa(0)} while time >= tl.
    const Fast fst{c.ram, c.ramh, c.ram_end, d.prg, d.uop};
    Hot h;
    h.icount = 0;
    hot_in(h, c, fst);
    while (__any_sync(FULL, running)) {
        if (minpc_turn(running, h)) {
            if (!hot_step(h, c, fst)) {
                hot_out(h, c);
                c.end_frame();
                close_frame(c, slot);
                frames++;
                int next = -1;
                uint32_t btn = 0;
                if (phase == 0) { next = 1; btn = 0; }
                else if (phase == 1 || phase == 3) {
                    if (phase == 3) c.RAMW(0x7a0, 0);
                    if (smb_time(c) == 0) { next = 2; btn = 8; }
                    else { tl = smb_time(c); next = -2; }
                } else if (phase == 2) {
                    c.RAMW(0x75f, (uint32_t)(w - 1)); c.RAMW(0x75c, (uint32_t)(s - 1)); c.RAMW(0x760, (uint32_t)(ar - 1));
                    next = 3; btn = 0;
                } else if (phase == 4) { next = 5; btn = 0; }
                else if (phase == 5) { next = -2; }
                if (next == -2) {  // loop B test
                    if (smb_time(c) >= tl) { tl = smb_time(c); next = 4; btn = 8; }
                    else next = -1;
                }
                if (next >= 0 && frames >= P.boot_cap) { c.status |= ST_BOOT_CAP; next = -1; }
                if (next < 0) running = false;
                else { phase = next; begin_frame(c, slot, btn, d.log_cap); }
                hot_in(h, c, fst);
            }
        }
    }
    hot_out(h, c);
    if (active) {
        materialise_state(c);
        lane_to_image(c, P.level_img + (size_t)l * IMG_STRIDE);
        P.level_meta[2 * l] = smb_x_pos(c);
        P.level_meta[2 * l + 1] = (int32_t)smb_time(c);
        if (c.status) atomicOr(d.err, c.status);
    }
    __syncwarp();
    load_lut(sm, d.lut, lane);
    for (int j = 0; j < 32; j++) {
        int lj = g * 32 + j;
        if (lj >= P.n_levels) break;
        render_slot(d.logs + slot_off(lj, 0, d.log_cap), full_layout(sm), d, false, false, lane);
        resize_fb(sm, lane);
        wcopy16(P.obs0 + (size_t)lj * OBS_BYTES, sm + RS_OBS, OBS_BYTES, lane);
        __syncwarp();
    }
}

// load / store of the SoA scalar words of one env
__device__ __forceinline__ void load_words(const Dev& d, int e, uint32_t* w) {
#pragma unroll
    for (int k = 0; k < S_WORDS; k++) w[k] = d.scal[(size_t)k * d.n_pad + e];
}
__device__ __forceinline__ void store_words(const Dev& d, int e, const uint32_t* w) {
#pragma unroll
    for (int k = 0; k < S_WORDS; k++) d.scal[(size_t)k * d.n_pad + e] = w[k];
}

__device__ __forceinline__ AgentCfg agent_cfg(const StepParams& P) {
    AgentCfg g;
    g.mode = P.mode; g.skip = P.skip; g.max_steps = P.max_steps; g.noop_max = P.noop_max; g.maxpool = P.maxpool;
    g.sticky_on = P.sticky_on; g.hack_cap = P.hack_cap; g.cap = P.d.log_cap; g.sticky_thr = P.sticky_thr;
    g.simple = P.simple;
    return g;
}

// kStep: the timed step (MODE_STEP, frames drawn by k_render) — compiled without the reset-cache builder's
// branches and the fused renderer, which only MODE_NOOP (construction) uses.
template <bool kStep>
__global__ void __launch_bounds__(32, 1) k_step(StepParams P) {
    extern __shared__ __align__(16) uint8_t sm[];
    if (kStep) P.mode = MODE_STEP;
    const int lane = threadIdx.x, g = blockIdx.x + P.group_base, e = g * 32 + lane;
    const Dev& d = P.d;
    const bool active = e < d.n;
    const int cap = d.log_cap;
    const AgentCfg cfg = agent_cfg(P);
    uint8_t* const gslab = d.slab + (size_t)g * SLAB_BYTES;
    const int ram_sm = (int)P.ram_end * LANES;   // bytes of the slab's RAM held in shared memory
    copy_slab(sm, gslab, lane, ram_sm);
    __syncwarp();

    Core c;
    bind_core(c, d, sm, lane, e);
    c.ramh = gslab + SLAB_RAM_OFF + lane * 4;  // RAM from ram_end up, OAM and palette stay in HBM (L1-cached)
    c.ram_end = P.ram_end;
    c.oam = gslab + SLAB_OAM_OFF + lane * 4;
    c.pal = gslab + SLAB_PAL_OFF + lane * 4;
    uint32_t w[S_WORDS];
    for (int k = 0; k < S_WORDS; k++) w[k] = 0;
    if (active) load_words(d, e, w);
    c.load_scalars(w);
    c.bad_ops = w[S_BADOPS];
    c.status = w[S_STATUS];
    EnvVars ev;
    ev.load(w);
    const uint32_t draws0 = w[S_EPLEN];  // MODE_NOOP: the builder keeps its cumulative draw count here

    uint32_t act = 0;
    if (active && P.mode == MODE_STEP) {
        int64_t a64 = P.actions[e];
        if (a64 < 0 || a64 > 6) { c.status |= ST_BAD_ACTION; a64 = 0; }
        act = (uint32_t)a64;
    }
    Agent ag;
    bool running = active;
    if (active) ag.start(c, ev, cfg, act, d.logs + slot_off(e, 0, cap), d.logs + slot_off(e, 1, cap));
    // Two phases. (1) Every lane whose next instruction the datapath can run executes it, each lane its own
    // instruction (fme_dp.h): no vote, all lanes at once. (2) When no lane can, the warp votes for its
    // minimum key and those lanes take one step on the exact path (I/O, PPU catch-up and NMI, the idle-loop
    // fast-forward, the frame end), all lanes at that PC together. Lanes are independent, so the order in
    // which the warp serves them changes no result.
    const Fast fst{c.ram, c.ramh, c.ram_end, d.prg, d.uop};
    const uint32_t ip0 = __ldg(d.uop + UOP_WORDS), ip1 = __ldg(d.uop + UOP_WORDS + 1);
    Hot h;
    h.icount = 0;
    uint32_t emu_frames = 0;
    hot_in(h, c, fst);
    rf_pack(h);
    dfetch(h, d.dop);
    bool blocked = false;   // a computed address of the lane's next instruction is an I/O address
    int32_t lim = dp_limit(h);
    for (;;) {
        const bool ready = running && !blocked && dp_ready(h, lim);
        if (__any_sync(FULL, ready)) {
            const bool done = dp_exec(h, fst, d.dop, ready);   // all lanes run the code, ready ones commit
            blocked = blocked || (ready && !done);
            continue;
        }
        const uint32_t key = sched_key_pc(running, h, ip0, ip1);
        const uint32_t mn = __reduce_min_sync(FULL, key);
        if (mn == 0xffffffffu) break;
        if (key == mn) {
            rf_unpack(h);
            fetch(h, fst);   // the exact path's micro-op of pc
            if (!hot_step(h, c, fst)) {
                hot_out(h, c);
                c.end_frame();
                emu_frames++;
                running = ag.on_frame_end(c, ev, cfg);
                hot_in(h, c, fst);
            }
            rf_pack(h);
            dfetch(h, d.dop);
            lim = dp_limit(h);
            blocked = false;
        }
    }
    rf_unpack(h);
    hot_out(h, c);

    int reset_ci = 0;
    bool pooled = false, ended = false;
    int cur_slot = 0;
    if (active) {
        StepOut o = ag.finish(c, ev, cfg);
        pooled = o.pooled;
        cur_slot = o.cur_slot;
        if (P.mode == MODE_STEP) {
            ev.frames += o.re_frames;
            c.bad_ops += o.re_bad;
            P.rew[e] = (float)o.total;
            P.term[e] = o.term ? 1 : 0;
            P.trunc[e] = o.trunc ? 1 : 0;
            for (int k = 0; k < 10; k++) P.info[(size_t)e * 10 + k] = (int32_t)o.info[k];
            if (o.term || o.trunc) {
                ended = true;
                P.ep_ret[e] = ev.ep_ret;
                P.ep_len[e] = ev.ep_len;
                reset_ci = reset_from_cache(c, ev, P.cache, P.noop_max);
            }
        } else {
            // reset-cache builder: entry (level, noop_j) = state after noop_j no-op steps; a terminal step
            // restores the level snapshot (fastmario.cpp:394-397)
            uint64_t fr_entry = ev.frames + o.re_frames;
            uint32_t bad_entry = c.bad_ops + o.re_bad;
            uint32_t draws_total = draws0 + ag.draws;
            if (o.term) {
                uint32_t cw[S_CONSOLE_WORDS];
                image_to_lane(P.level_img + (size_t)ev.level * IMG_STRIDE, c, cw);
                c.load_scalars(cw);
                ev.x_last = P.level_meta[2 * ev.level]; ev.t_last = P.level_meta[2 * ev.level + 1]; ev.lives = -1;
                ended = true;
            }
            ev.prev = 0;
            int ci = ev.level * (P.noop_max + 1) + P.noop_j;
            lane_to_image(c, P.out_img + (size_t)ci * IMG_STRIDE);
            int32_t* meta = P.out_meta + (size_t)ci * META_WORDS;
            meta[META_X] = ev.x_last; meta[META_T] = ev.t_last; meta[META_LIVES] = ev.lives;
            meta[META_DRAWS] = (int32_t)draws_total;
            meta[META_FR_LO] = (int32_t)(uint32_t)fr_entry; meta[META_FR_HI] = (int32_t)(uint32_t)(fr_entry >> 32);
            meta[META_BAD] = (int32_t)bad_entry; meta[7] = 0;
            reset_ci = ci;
            ev.ep_len = (int32_t)draws_total;
            ev.t = 0; ev.ep_ret = 0.0;
        }
        c.store_scalars(w);
        ev.store(w);
        w[S_BADOPS] = c.bad_ops; w[S_STATUS] = c.status;
        // work counters: read back here rather than kept live across the emulation loop
        const uint64_t ic = ((uint64_t)d.scal[(size_t)S_INSTR_HI * d.n_pad + e] << 32 |
                             d.scal[(size_t)S_INSTR_LO * d.n_pad + e]) + h.icount;
        w[S_INSTR_LO] = (uint32_t)ic; w[S_INSTR_HI] = (uint32_t)(ic >> 32);
        w[S_EMU_FRAMES] = d.scal[(size_t)S_EMU_FRAMES * d.n_pad + e] + emu_frames;
        store_words(d, e, w);
        if (c.status) atomicOr(d.err, c.status);
    }
    __syncwarp();
    copy_slab(gslab, sm, lane, ram_sm);
    __syncwarp();

    const uint32_t summary = (active ? 1u : 0u) | (pooled ? 2u : 0u) | ((uint32_t)cur_slot << 2) | (ended ? 8u : 0u);
    const int K = P.frame_stack;
    if (kStep) {
        // ---- k_render draws the frame, shifts the stack and stages finished episodes (job word: summary bits,
        // reset-cache entry above them)
        if (active) P.jobs[e] = summary | ((uint32_t)reset_ci << 4);
        return;
    }

    // ---- render, resize, frame stack (warp-cooperative, one env at a time)
    load_lut(sm, d.lut, lane);
    for (int j = 0; j < 32; j++) {
        uint32_t sj = __shfl_sync(FULL, summary, j);
        int cij = __shfl_sync(FULL, reset_ci, j);
        if (!(sj & 1u)) continue;
        const int ej = g * 32 + j;
        const int cs = (int)((sj >> 2) & 1u);
        const bool pj = (sj & 2u) != 0, dj = (sj & 8u) != 0;
        if (P.mode == MODE_NOOP) {
            uint8_t* dst = P.out_obs + (size_t)cij * OBS_BYTES;
            if (dj) wcopy16(dst, P.level_obs0 + (size_t)(cij / (P.noop_max + 1)) * OBS_BYTES, OBS_BYTES, lane);
            else {
                render_slot(d.logs + slot_off(ej, cs, cap), full_layout(sm), d, false, false, lane);
                resize_fb(sm, lane);
                wcopy16(dst, sm + RS_OBS, OBS_BYTES, lane);
            }
            __syncwarp();
            continue;
        }
        if (pj) {
            render_slot(d.logs + slot_off(ej, cs ^ 1, cap), full_layout(sm), d, false, false, lane);
            render_slot(d.logs + slot_off(ej, cs, cap), full_layout(sm), d, false, true, lane);
        } else {
            render_slot(d.logs + slot_off(ej, cs, cap), full_layout(sm), d, false, false, lane);
        }
        resize_fb(sm, lane);
        uint8_t* o = P.obs + (size_t)ej * K * OBS_BYTES;
        if (K > 1) wmove16(o, o + OBS_BYTES, (K - 1) * OBS_BYTES, lane);
        __syncwarp();
        if (dj) {
            uint8_t* f = P.fin + (size_t)ej * K * OBS_BYTES;
            if (K > 1) wcopy16(f, o, (K - 1) * OBS_BYTES, lane);
            wcopy16(f + (size_t)(K - 1) * OBS_BYTES, sm + RS_OBS, OBS_BYTES, lane);
            __syncwarp();
            if (K > 1) wzero16(o, (K - 1) * OBS_BYTES, lane);
            wcopy16(o + (size_t)(K - 1) * OBS_BYTES, P.cache.obs + (size_t)cij * OBS_BYTES, OBS_BYTES, lane);
        } else {
            wcopy16(o + (size_t)(K - 1) * OBS_BYTES, sm + RS_OBS, OBS_BYTES, lane);
        }
        __syncwarp();
    }
}

// ---- k_render: the new frame of every env, one CTA (one warp) per (env, band of 60 screen rows).
// A band's 60 rows are exactly the source rows of 21 output rows (240/84 = 20/7), so each CTA replays the
// env's log(s) drawing only its rows, resizes them and writes its 21 rows of the stacked frame. The small
// shared-memory footprint (about 20 KB) lets 10 CTAs share an SM and hide each other's latencies.
constexpr int BAND_ROWS = 60, BAND_OUT = 21, NBANDS = SCREEN_H / BAND_ROWS;
constexpr int RB_FB = 0;
constexpr int RB_VRAM = RB_FB + BAND_ROWS * SCREEN_W;
constexpr int RB_PAL = RB_VRAM + VRAM_BYTES;
constexpr int RB_OAM = RB_PAL + PAL_BYTES;
constexpr int RB_STAGE = RB_OAM + OAM_BYTES;
constexpr int RB_OBS = RB_STAGE + SCREEN_W;
constexpr int RB_LUT = RB_OBS + (BAND_OUT * OBS + 15) / 16 * 16;
constexpr int RB_SPR = RB_LUT + 256;
constexpr int RB_GV = RB_SPR + 64;
constexpr int RB_BYTES = RB_GV + 32;
static_assert(NBANDS * BAND_OUT == OBS && BAND_ROWS * OBS == BAND_OUT * SCREEN_H, "bands must align with the taps");
static_assert(RB_VRAM % 16 == 0 && RB_OAM % 16 == 0 && RB_LUT % 16 == 0 && RB_OBS % 4 == 0, "alignment");

struct RenderParams {
    Dev d;
    const uint32_t* jobs;   // per env: 1 active | 2 max-pooled | 4 slot of the last frame | 8 ended | reset entry << 4
    uint8_t* obs; uint8_t* fin;
    const uint8_t* cache_obs;   // reset-cache observations (entry x 7056)
    int frame_stack;
    int env_base;   // first env of this launch
};

// The frame-stack update of one band (BAND_OUT rows of every 84x84 frame, 441 words at the same offset in
// each): frames 1..K-1 move down to 0..K-2 — into the final stack when the episode ended, whose live stack
// then restarts as K-1 zero frames and the reset observation. Frame K-1 (the new frame) is written by the
// caller. Each lane keeps its share of a frame in registers between the loads and the stores.
constexpr int BAND_WORDS = BAND_OUT * OBS / 4, FRAME_WORDS = OBS_BYTES / 4, BAND_PER_LANE = (BAND_WORDS + 31) / 32;
static_assert(BAND_OUT * OBS % 4 == 0, "bands are whole words");
__device__ __forceinline__ void stack_band(uint32_t* o, uint32_t* f, const uint32_t* reset_obs, int K, int lane) {
    uint32_t* dst = f ? f : o;
    for (int j = 0; j + 1 < K; j++) {
        uint32_t v[BAND_PER_LANE];
#pragma unroll
        for (int q = 0; q < BAND_PER_LANE; q++) {
            const int i = lane + 32 * q;
            if (i < BAND_WORDS) v[q] = o[(j + 1) * FRAME_WORDS + i];
        }
        __syncwarp();
#pragma unroll
        for (int q = 0; q < BAND_PER_LANE; q++) {
            const int i = lane + 32 * q;
            if (i < BAND_WORDS) dst[j * FRAME_WORDS + i] = v[q];
        }
    }
    if (f) {
        __syncwarp();
        for (int j = 0; j + 1 < K; j++)
            for (int i = lane; i < BAND_WORDS; i += 32) o[j * FRAME_WORDS + i] = 0u;
        for (int i = lane; i < BAND_WORDS; i += 32) o[(K - 1) * FRAME_WORDS + i] = reset_obs[i];
    }
    __syncwarp();
}
__global__ void __launch_bounds__(32) k_render(RenderParams P) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int lane = threadIdx.x;
    const int e = (int)(blockIdx.x / NBANDS) + P.env_base, band = (int)(blockIdx.x % NBANDS);
    const Dev& d = P.d;
    if (e >= d.n) return;
    const uint32_t job = P.jobs[e];
    if (!(job & 1u)) return;
    RLayout L;
    L.fb = sm + RB_FB; L.vram = sm + RB_VRAM; L.pal = sm + RB_PAL; L.oam = sm + RB_OAM; L.stage = sm + RB_STAGE;
    L.lut = sm + RB_LUT; L.spr = reinterpret_cast<uint32_t*>(sm + RB_SPR); L.gv = sm + RB_GV;
    L.bmask = reinterpret_cast<uint32_t*>(sm + RB_OBS);   // the resize output is written after the replays
    L.row_lo = band * BAND_ROWS; L.row_hi = L.row_lo + BAND_ROWS;
    if (lane < 16) reinterpret_cast<uint4*>(sm + RB_LUT)[lane] = reinterpret_cast<const uint4*>(d.lut)[lane];
    __syncwarp();
    const int K = P.frame_stack;
    const size_t band_off = (size_t)band * BAND_OUT * OBS;
    stack_band(reinterpret_cast<uint32_t*>(P.obs + (size_t)e * K * OBS_BYTES + band_off),
               (job & 8u) ? reinterpret_cast<uint32_t*>(P.fin + (size_t)e * K * OBS_BYTES + band_off) : nullptr,
               reinterpret_cast<const uint32_t*>(P.cache_obs + (size_t)(job >> 4) * OBS_BYTES + band_off), K, lane);
    const int cs = (int)((job >> 2) & 1u);
    const int cap = d.log_cap;
    if (job & 2u) {
        render_slot(d.logs + slot_off(e, cs ^ 1, cap), L, d, false, false, lane);
        render_slot(d.logs + slot_off(e, cs, cap), L, d, false, true, lane);
    } else {
        render_slot(d.logs + slot_off(e, cs, cap), L, d, false, false, lane);
    }
    resize_band(L.fb, L.row_lo, band * BAND_OUT, band * BAND_OUT + BAND_OUT, sm + RB_OBS, lane);
    uint8_t* dst = ((job & 8u) ? P.fin : P.obs) + ((size_t)e * K + (K - 1)) * OBS_BYTES + band_off;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(sm + RB_OBS);
    for (int i = lane; i < BAND_OUT * OBS / 4; i += 32) reinterpret_cast<uint32_t*>(dst)[i] = src[i];
}

// Every env at its level snapshot (Env::init -> restore_backup, fastmario.cpp:285-295), RNG from the host.
struct InitParams {
    Dev d;
    const uint8_t* level_img; const int32_t* level_meta;
    const int32_t* env_level;   // n
    const uint64_t* rng6;       // n x 6 (numpy words)
};
__global__ void __launch_bounds__(32) k_init(InitParams P) {
    const int lane = threadIdx.x, g = blockIdx.x, e = g * 32 + lane;
    const Dev& d = P.d;
    if (e >= d.n) return;
    uint8_t* slab = d.slab + (size_t)g * SLAB_BYTES;
    const int l = P.env_level[e];
    const uint8_t* img = P.level_img + (size_t)l * IMG_STRIDE;
    for (int w = 0; w < RAM_BYTES / 4; w++)
        reinterpret_cast<uint32_t*>(slab + SLAB_RAM_OFF)[w * 32 + lane] = reinterpret_cast<const uint32_t*>(img + IMG_RAM)[w];
    for (int w = 0; w < OAM_BYTES / 4; w++)
        reinterpret_cast<uint32_t*>(slab + SLAB_OAM_OFF)[w * 32 + lane] = reinterpret_cast<const uint32_t*>(img + IMG_OAM)[w];
    for (int w = 0; w < PAL_BYTES / 4; w++)
        reinterpret_cast<uint32_t*>(slab + SLAB_PAL_OFF)[w * 32 + lane] = reinterpret_cast<const uint32_t*>(img + IMG_PAL)[w];
    tcopy16(d.vram + (size_t)e * VRAM_BYTES, img + IMG_VRAM, VRAM_BYTES);
    uint32_t w[S_WORDS];
    for (int k = 0; k < S_WORDS; k++) w[k] = 0;
    for (int k = 0; k < S_CONSOLE_WORDS; k++) w[k] = reinterpret_cast<const uint32_t*>(img + IMG_SCAL)[k];
    w[S_XLAST] = (uint32_t)P.level_meta[2 * l]; w[S_TLAST] = (uint32_t)P.level_meta[2 * l + 1];
    w[S_PREV] = 0; w[S_LIVES] = (uint32_t)-1; w[S_T] = 0; w[S_EPLEN] = 0; w[S_EPRET_LO] = 0; w[S_EPRET_HI] = 0;
    const uint64_t* r = P.rng6 + (size_t)e * 6;
    w[S_RNG_S0] = (uint32_t)r[1]; w[S_RNG_S1] = (uint32_t)(r[1] >> 32);
    w[S_RNG_S2] = (uint32_t)r[0]; w[S_RNG_S3] = (uint32_t)(r[0] >> 32);
    w[S_RNG_I0] = (uint32_t)r[3]; w[S_RNG_I1] = (uint32_t)(r[3] >> 32);
    w[S_RNG_I2] = (uint32_t)r[2]; w[S_RNG_I3] = (uint32_t)(r[2] >> 32);
    w[S_RNG_HAS] = (uint32_t)r[4]; w[S_RNG_U32] = (uint32_t)r[5];
    w[S_LEVEL] = (uint32_t)l;
    store_words(d, e, w);
}

// fm_reset: every env draws k and takes cache entry (level, k); stacks become zeros + the reset frame.
__global__ void __launch_bounds__(32) k_reset(StepParams P) {
    const int lane = threadIdx.x, g = blockIdx.x, e = g * 32 + lane;
    const Dev& d = P.d;
    const bool active = e < d.n;
    int ci = 0;
    if (active) {
        uint32_t w[S_WORDS];
        load_words(d, e, w);
        Core c;
        uint8_t* slab = d.slab + (size_t)g * SLAB_BYTES;   // the lane-interleaved slab itself, in HBM
        c.ram = slab + SLAB_RAM_OFF + lane * 4; c.ramh = c.ram; c.ram_end = RAM_BYTES; c.oam = slab + SLAB_OAM_OFF + lane * 4;
        c.pal = slab + SLAB_PAL_OFF + lane * 4; c.vram = d.vram + (size_t)e * VRAM_BYTES;
        c.load_scalars(w);
        c.bad_ops = w[S_BADOPS]; c.status = w[S_STATUS];
        EnvVars ev;
        ev.load(w);
        ci = reset_from_cache(c, ev, P.cache, P.noop_max);
        c.store_scalars(w);
        ev.store(w);
        w[S_BADOPS] = c.bad_ops;
        store_words(d, e, w);
    }
    const int K = P.frame_stack;
    for (int j = 0; j < 32; j++) {
        int cij = __shfl_sync(FULL, ci, j);
        int ej = g * 32 + j;
        if (ej >= d.n) break;
        uint8_t* o = P.obs + (size_t)ej * K * OBS_BYTES;
        if (K > 1) wzero16(o, (K - 1) * OBS_BYTES, lane);
        wcopy16(o + (size_t)(K - 1) * OBS_BYTES, P.cache.obs + (size_t)cij * OBS_BYTES, OBS_BYTES, lane);
    }
}

// One NES frame for raw consoles (fm_raw_frame, fastmario.cpp:662-667).
struct RawParams {
    Dev d;
    const uint8_t* buttons;
    int render;
    uint8_t* screens;   // n x 240 x 256
};
__global__ void __launch_bounds__(32) k_raw(RawParams P) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int lane = threadIdx.x, g = blockIdx.x, e = g * 32 + lane;
    const Dev& d = P.d;
    const bool active = e < d.n;
    copy_slab(sm, d.slab + (size_t)g * SLAB_BYTES, lane);
    __syncwarp();
    Core c;
    bind_core(c, d, sm, lane, e);
    uint32_t w[S_WORDS];
    for (int k = 0; k < S_WORDS; k++) w[k] = 0;
    if (active) load_words(d, e, w);
    c.load_scalars(w);
    c.bad_ops = w[S_BADOPS];
    c.status = w[S_STATUS];
    uint8_t* slot = d.logs + slot_off(e, 0, d.log_cap);
    bool running = active;
    if (active) begin_frame(c, slot, P.buttons[e], d.log_cap);
    const Fast fst{c.ram, c.ramh, c.ram_end, d.prg, d.uop};
    Hot h;
    h.icount = 0;
    hot_in(h, c, fst);
    while (__any_sync(FULL, running)) {
        if (minpc_turn(running, h) && !hot_step(h, c, fst)) {
            hot_out(h, c);
            c.end_frame();
            close_frame(c, slot);
            running = false;
            hot_in(h, c, fst);
        }
    }
    hot_out(h, c);
    if (active) {
        materialise_state(c);
        c.store_scalars(w);
        w[S_BADOPS] = c.bad_ops; w[S_STATUS] = c.status;
        store_words(d, e, w);
        if (c.status) atomicOr(d.err, c.status);
    }
    __syncwarp();
    copy_slab(d.slab + (size_t)g * SLAB_BYTES, sm, lane);
    __syncwarp();
    if (!P.render) return;
    load_lut(sm, d.lut, lane);
    for (int j = 0; j < 32; j++) {
        int ej = g * 32 + j;
        if (ej >= d.n) break;
        render_slot(d.logs + slot_off(ej, 0, d.log_cap), full_layout(sm), d, true, false, lane);
        wcopy16(P.screens + (size_t)ej * SCREEN_W * SCREEN_H, sm + RS_FB, SCREEN_W * SCREEN_H, lane);
        __syncwarp();
    }
}

// PPU log slots for fme_raw_frame_static, reserved with the module rather than by cudaMalloc. Callers that
// drive a few consoles next to a process owning the rest of the device's memory (a trainer whose caching
// allocator has reserved HBM, where a cudaMalloc can fail or synchronise the device) step frames through it
// without any allocation. Slot layout as d.logs: two slots per console, k_raw writes slot 0.
constexpr size_t STATIC_SLOT_BYTES = (size_t)SLOT_HDR_BYTES + (size_t)FME_STATIC_LOG_CAPACITY * 16u;
static __device__ __align__(256) uint8_t g_raw_scratch[(size_t)FME_STATIC_MAX_CONSOLES * 2 * STATIC_SLOT_BYTES];

// Power-on state (Emulator(rom) + Reset, nes_core.hpp:128-147) for raw consoles.
__global__ void __launch_bounds__(32) k_power(Dev d) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int lane = threadIdx.x, g = blockIdx.x, e = g * 32 + lane;
    Core c;
    bind_core(c, d, sm, lane, e);
    if (e < d.n) {
        c.bad_ops = 0;
        c.power_on();
        uint32_t w[S_WORDS];
        for (int k = 0; k < S_WORDS; k++) w[k] = 0;
        c.store_scalars(w);
        store_words(d, e, w);
    }
    __syncwarp();
    copy_slab(d.slab + (size_t)g * SLAB_BYTES, sm, lane);
}

__global__ void __launch_bounds__(32) k_resize(const uint8_t* src, uint8_t* dst, int n) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int lane = threadIdx.x;
    for (int im = blockIdx.x; im < n; im += gridDim.x) {
        wcopy16(sm + RS_FB, src + (size_t)im * SCREEN_W * SCREEN_H, SCREEN_W * SCREEN_H, lane);
        __syncwarp();
        resize_fb(sm, lane);
        wcopy16(dst + (size_t)im * OBS_BYTES, sm + RS_OBS, OBS_BYTES, lane);
        __syncwarp();
    }
}

// (N, 2048) RAM rows from the lane-interleaved slabs
__global__ void k_ram_all(const uint8_t* slab, int n, uint8_t* out) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 32-bit word of one env
    size_t total = (size_t)n * (RAM_BYTES / 4);
    if (idx >= total) return;
    int e = (int)(idx / (RAM_BYTES / 4)), wd = (int)(idx % (RAM_BYTES / 4));
    const uint32_t* s = reinterpret_cast<const uint32_t*>(slab + (size_t)(e / 32) * SLAB_BYTES + SLAB_RAM_OFF);
    reinterpret_cast<uint32_t*>(out + (size_t)e * RAM_BYTES)[wd] = s[wd * 32 + (e % 32)];
}

}  // namespace fme

// ====================================================================== host side
namespace {

thread_local std::string g_err;
int fail(int code, const std::string& msg) { g_err = msg; return code; }
#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t _e = (call);                                                              \
        if (_e != cudaSuccess) return fail(FME_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(_e)); \
    } while (0)

// Per-device set-up (constant tables, the static scratch address) belongs to the device's CUDA context: a
// cudaDeviceReset destroys the primary context and with it both. The caches are therefore keyed by the unique
// id of the context current at the call (cuCtxGetId, through the runtime's driver entry points so that the
// library does not link libcuda), not by the device ordinal alone.
typedef int (*PfnCtxGetCurrent)(void**);
typedef int (*PfnCtxGetId)(void*, unsigned long long*);
int current_context_id(unsigned long long* id) {
    static PfnCtxGetCurrent get_current = nullptr;
    static PfnCtxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PfnCtxGetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PfnCtxGetId>(f);
    });
    if (!get_current || !get_id) return fail(FME_E_CUDA, "driver entry points cuCtxGetCurrent / cuCtxGetId unavailable");
    void* ctx = nullptr;
    if (get_current(&ctx) != 0 || !ctx) return fail(FME_E_CUDA, "no current CUDA context");
    if (get_id(ctx, id) != 0) return fail(FME_E_CUDA, "cuCtxGetId failed");
    return FME_OK;
}

std::mutex g_const_mu;
unsigned long long g_const_ctx[64];   // context id the constants were uploaded in (0 = none)

std::mutex g_scratch_mu;
void* g_scratch_addr[64];
unsigned long long g_scratch_ctx[64];

// Device address of g_raw_scratch on `device`, which must be current: looked up once per device and context.
int static_scratch(int device, uint8_t** out) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (device < 0 || device >= 64) return fail(FME_E_ARG, "device ordinal out of range");
    unsigned long long ctx = 0;
    int rc = current_context_id(&ctx);
    if (rc) return rc;
    if (!g_scratch_addr[device] || g_scratch_ctx[device] != ctx) {
        void* p = nullptr;
        CK(cudaGetSymbolAddress(&p, g_raw_scratch));
        g_scratch_addr[device] = p;
        g_scratch_ctx[device] = ctx;
    }
    *out = static_cast<uint8_t*>(g_scratch_addr[device]);
    return FME_OK;
}

int ensure_constants(int device) {
    std::lock_guard<std::mutex> lk(g_const_mu);
    if (device < 0 || device >= 64) return fail(FME_E_ARG, "device ordinal out of range");
    unsigned long long ctx = 0;
    int rc = current_context_id(&ctx);
    if (rc) return rc;
    if (g_const_ctx[device] == ctx) return FME_OK;
    uint32_t dt[256];
    build_dtab(dt);
    AreaTabs T;
    if (!build_area(T)) return fail(FME_E_ARG, "area table has more than 6 taps");
    for (int dx = 0; dx < OBS; dx++)  // resize_band keeps AREA_XTAPS consecutive column taps in registers
        for (int k = 1; k < 6; k++)
            if (T.xw[k][dx] != 0.f && (k >= AREA_XTAPS || T.xs[k][dx] != T.xs[0][dx] + k))
                return fail(FME_E_ARG, "area column taps are not consecutive");
    for (int dy = 0; dy < OBS; dy++)  // k_render: every tap of an output row lies in that row's band
        for (int m = 0; m < 6 && T.yw[m][dy] != 0.f; m++)
            if (T.ys[m][dy] / BAND_ROWS != dy / BAND_OUT) return fail(FME_E_ARG, "area taps cross a render band");
    CK(cudaMemcpyToSymbol(c_dtab, dt, sizeof(dt)));
    CK(cudaMemcpyToSymbol(c_area, &T, sizeof(T)));
    const int smem = SLAB_BYTES;
    CK(cudaFuncSetAttribute(k_step<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_step<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, STEP_SMEM));
    CK(cudaFuncSetAttribute(k_boot, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_raw, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_resize, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_power, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_render, cudaFuncAttributeMaxDynamicSharedMemorySize, RB_BYTES));
    g_const_ctx[device] = ctx;
    return FME_OK;
}

// iNES parse with the reference's acceptance rules (nes_core.hpp:67-87)
int parse_rom(const uint8_t* data, int64_t n, std::vector<uint8_t>& prg, std::vector<uint8_t>& chr, uint32_t nt[4]) {
    if (!data || n < 16 || memcmp(data, "NES\x1a", 4) != 0) return fail(FME_E_ROM, "not an iNES image");
    uint8_t mirroring = data[6] & 0xB;
    int mapper = ((data[6] >> 4) & 0xf) | (data[7] & 0xf0);
    int banks = data[4], vbanks = data[5];
    if (mapper != 0 || (data[6] & 0x2) || (data[6] & 0x4)) return fail(FME_E_ROM, "unsupported mapper / PRG-RAM / trainer");
    if (banks < 1 || banks > 2 || vbanks != 1) return fail(FME_E_ROM, "unsupported bank layout");
    if (n < 16 + 0x4000LL * banks + 0x2000) return fail(FME_E_ROM, "truncated image");
    prg.assign(0x8000, 0);
    memcpy(prg.data(), data + 16, 0x4000 * banks);
    if (banks == 1) memcpy(prg.data() + 0x4000, data + 16, 0x4000);
    chr.assign(data + 16 + 0x4000 * banks, data + 16 + 0x4000 * banks + 0x2000);
    if (mirroring == 0) { nt[0] = nt[1] = 0; nt[2] = nt[3] = 0x400; }
    else if (mirroring == 1) { nt[0] = nt[2] = 0; nt[1] = nt[3] = 0x400; }
    else { nt[0] = nt[1] = nt[2] = nt[3] = 0; }
    return FME_OK;
}

struct DevBufs {  // one set of per-env state buffers
    int n = 0, n_pad = 0, log_cap = 0;
    uint8_t* slab = nullptr;
    uint8_t* vram = nullptr;
    uint32_t* scal = nullptr;
    uint8_t* logs = nullptr;
    int alloc(int n_, int cap) {
        n = n_; n_pad = (n_ + 31) / 32 * 32; log_cap = cap;
        CK(cudaMalloc(&slab, (size_t)(n_pad / 32) * SLAB_BYTES));
        CK(cudaMalloc(&vram, (size_t)n_pad * VRAM_BYTES));
        CK(cudaMalloc(&scal, (size_t)S_WORDS * n_pad * 4));
        CK(cudaMalloc(&logs, (size_t)n_pad * 2 * slot_bytes(cap)));
        CK(cudaMemset(slab, 0, (size_t)(n_pad / 32) * SLAB_BYTES));
        CK(cudaMemset(vram, 0, (size_t)n_pad * VRAM_BYTES));
        CK(cudaMemset(scal, 0, (size_t)S_WORDS * n_pad * 4));
        return FME_OK;
    }
    void release() {
        cudaFree(slab); cudaFree(vram); cudaFree(scal); cudaFree(logs);
        slab = vram = logs = nullptr; scal = nullptr;
    }
    size_t bytes() const {
        return (size_t)(n_pad / 32) * SLAB_BYTES + (size_t)n_pad * VRAM_BYTES + (size_t)S_WORDS * n_pad * 4 +
               (size_t)n_pad * 2 * slot_bytes(log_cap);
    }
};

// The PRG image and its micro-op tables share one allocation: 32 KB of PRG, then 2 words per PRG address of
// exact micro-ops (+ the first two idle-loop PCs), then 2 words per PRG address of datapath micro-ops.
constexpr size_t PRG_UOP_OFF = 0x8000;
constexpr size_t PRG_DOP_OFF = PRG_UOP_OFF + (size_t)(UOP_WORDS + 2) * 4;
constexpr size_t PRG_ALLOC = PRG_DOP_OFF + (size_t)UOP_WORDS * 4;
static_assert(PRG_DOP_OFF % 8 == 0, "datapath micro-ops are read as 8-byte words");
cudaError_t upload_prg(uint8_t* d_prg, const std::vector<uint8_t>& prg) {
    uint32_t dt[256];
    build_dtab(dt);
    std::vector<uint32_t> uops(UOP_WORDS + 2), dops(UOP_WORDS);
    build_uops(prg.data(), dt, uops.data());
    build_dops(uops.data(), dops.data());
    uops[UOP_WORDS] = uops[UOP_WORDS + 1] = 0xffffffffu;  // no such pc
    for (uint32_t i = 0, k = 0; i < 0x8000u && k < 2; i++)
        if (uops[2 * i] & UOP_IDLE) uops[UOP_WORDS + k++] = 0x8000u + i;
    cudaError_t e = cudaMemcpy(d_prg, prg.data(), 0x8000, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d_prg + PRG_UOP_OFF, uops.data(), (size_t)(UOP_WORDS + 2) * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d_prg + PRG_DOP_OFF, dops.data(), (size_t)UOP_WORDS * 4, cudaMemcpyHostToDevice);
    return e;
}

Dev make_dev(const DevBufs& b, const uint8_t* prg, const uint8_t* chr, const uint32_t nt[4], const uint8_t* lut,
             uint32_t* err) {
    Dev d;
    d.n = b.n; d.n_pad = b.n_pad; d.slab = b.slab; d.vram = b.vram; d.scal = b.scal; d.logs = b.logs;
    d.log_cap = b.log_cap; d.prg = prg; d.chr = chr;
    d.uop = reinterpret_cast<const uint32_t*>(prg + PRG_UOP_OFF);
    d.dop = reinterpret_cast<const uint32_t*>(prg + PRG_DOP_OFF);
    for (int i = 0; i < 4; i++) d.nt[i] = nt[i];
    d.lut = lut; d.err = err;
    return d;
}

uint64_t sticky_threshold(double sticky) {
    if (!(sticky > 0.0)) return 0;  // also NaN: the reference draws but never repeats
    double s = sticky * 9007199254740992.0;  // exact scaling by 2^53
    if (s >= 9007199254740992.0) return 1ull << 53;
    return (uint64_t)std::ceil(s);
}

}  // namespace

constexpr int kChunks = 4;
constexpr int kTailParts = 4;   // fme_step_to_host renders the last slice in this many parts

// A few persistent host threads for the in-place stack shift of fme_step_to_host (memmove of frames 1..k-1
// to 0..k-2 in the caller's pinned buffer, as the reference's host engine shifts its stacks,
// csrc/fastmario.cpp:494-503). Runs inside a stream host function, so it makes no CUDA call.
class HostPool {
  public:
    explicit HostPool(int n) {
        for (int i = 0; i < n; i++) th_.emplace_back([this, i] { worker(i); });
    }
    ~HostPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : th_) t.join();
    }
    int size() const { return (int)th_.size() + 1; }
    // fn(part) for part in [0, size()), the calling thread taking the last part; returns when all are done
    void run(const std::function<void(int)>& fn) {
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_ = &fn;
            left_ = (int)th_.size();
            gen_++;
        }
        cv_.notify_all();
        fn((int)th_.size());
        std::unique_lock<std::mutex> lk(mu_);
        done_.wait(lk, [this] { return left_ == 0; });
        job_ = nullptr;
    }

  private:
    void worker(int i) {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(int)>* fn;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
                fn = job_;
            }
            (*fn)(i);
            std::lock_guard<std::mutex> lk(mu_);
            if (--left_ == 0) done_.notify_one();
        }
    }
    std::vector<std::thread> th_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::function<void(int)>* job_ = nullptr;
    int left_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

struct HostFix {  // arguments of the host functions of one fme_step_to_host call
    uint8_t* obs = nullptr;
    const uint8_t* term = nullptr;
    const uint8_t* trunc = nullptr;
    int n = 0, K = 0;
    int e0[kChunks + 1] = {};   // env range of each step slice (in-place shift)
    int shift_slice = 0;        // slice the next shift host function moves
    HostPool* pool = nullptr;
};

struct FmeEnv {
    FmeConfig cfg{};
    int n = 0, nl = 0, K = 4;
    uint32_t nt[4] = {0, 0, 0, 0};
    uint8_t* d_prg = nullptr;
    uint8_t* d_chr = nullptr;
    uint8_t* d_lut = nullptr;
    uint32_t* d_err = nullptr;
    DevBufs env;
    uint8_t* d_level_img = nullptr;
    int32_t* d_level_meta = nullptr;
    uint8_t* d_obs0 = nullptr;
    uint8_t* d_cache_img = nullptr;
    uint8_t* d_cache_obs = nullptr;
    int32_t* d_cache_meta = nullptr;
    uint32_t* d_jobs = nullptr;   // per-env render job of the last step (k_step -> k_render)
    // A step runs as kChunks slices of the env groups, each an emulation launch on a high-priority stream
    // followed by its render launch on a low-priority stream: the renders of finished slices fill the SMs
    // that the slower slices' last warps leave idle. Fork/join with events on the caller's stream.
    int nch = 0;
    uint32_t ram_end = RAM_END_DEEP;   // k_step's shared-memory RAM boundary for this env count (step_ram_end)
    cudaStream_t s_emu[kChunks] = {}, s_rnd[kChunks] = {};
    cudaEvent_t ev_in = nullptr, ev_emu[kChunks] = {}, ev_rnd[kChunks] = {};
    // fme_step_to_host: early copy of the old frames (s_copy, one event per slice) and the host-side fix-up
    cudaStream_t s_copy = nullptr;
    cudaEvent_t ev_pre[kChunks] = {}, ev_copy = nullptr, ev_part[kTailParts] = {};
    // one argument block per call still in flight (calls enqueued back to back may name other host buffers);
    // a block is reused only after the event recorded behind its call's last host function has completed
    static constexpr int kFixRing = 16;
    HostFix fix[kFixRing] = {};
    cudaEvent_t fix_done[kFixRing] = {};
    uint32_t fix_next = 0;
    HostPool* pool = nullptr;
    // host buffer the last fme_step_to_host wrote the stacks into; cleared by every other step or reset
    const uint8_t* host_obs_prev = nullptr;
    FmeBuffers buf{};
    bool bound = false;
    uint64_t sticky_thr = 0;
};

struct FmeRaw {
    int n = 0, device = 0;
    uint32_t nt[4] = {0, 0, 0, 0};
    uint8_t* d_prg = nullptr;
    uint8_t* d_chr = nullptr;
    uint8_t* d_lut = nullptr;
    uint32_t* d_err = nullptr;
    DevBufs st;
    uint8_t* d_screens = nullptr;
    uint8_t* d_bk_slab = nullptr;
    uint8_t* d_bk_vram = nullptr;
    uint32_t* d_bk_scal = nullptr;
};

static void free_env(FmeEnv* v) {
    if (!v) return;
    cudaFree(v->d_prg); cudaFree(v->d_chr); cudaFree(v->d_lut); cudaFree(v->d_err);
    v->env.release();
    cudaFree(v->d_level_img); cudaFree(v->d_level_meta); cudaFree(v->d_obs0);
    cudaFree(v->d_cache_img); cudaFree(v->d_cache_obs); cudaFree(v->d_cache_meta); cudaFree(v->d_jobs);
    for (int c = 0; c < kChunks; c++) {
        if (v->s_emu[c]) cudaStreamDestroy(v->s_emu[c]);
        if (v->s_rnd[c]) cudaStreamDestroy(v->s_rnd[c]);
        if (v->ev_emu[c]) cudaEventDestroy(v->ev_emu[c]);
        if (v->ev_rnd[c]) cudaEventDestroy(v->ev_rnd[c]);
    }
    if (v->ev_in) cudaEventDestroy(v->ev_in);
    if (v->s_copy) cudaStreamDestroy(v->s_copy);
    if (v->ev_copy) cudaEventDestroy(v->ev_copy);
    for (int c = 0; c < kChunks; c++)
        if (v->ev_pre[c]) cudaEventDestroy(v->ev_pre[c]);
    for (int q = 0; q < kTailParts; q++)
        if (v->ev_part[q]) cudaEventDestroy(v->ev_part[q]);
    for (int q = 0; q < FmeEnv::kFixRing; q++)
        if (v->fix_done[q]) cudaEventDestroy(v->fix_done[q]);
    delete v->pool;
    delete v;
}

// k_step's RAM boundary for a step of `groups` CTAs on `sms` SMs. While the deep layout (4 CTAs per SM)
// runs them in a few waves, the step is set by its slowest warps and the per-instruction latency of the
// shared-memory RAM wins; past about 4.5 waves it is throughput-bound and the wide layout's 8 CTAs per SM
// win (on a B200: deep ahead up to 65,536 envs, wide ahead from 98,304 envs, by 14 % at 262,144).
static uint32_t step_ram_end(int groups, int sms) {
    return (double)groups > 4.5 * 4.0 * (double)(sms > 0 ? sms : 1) ? RAM_END_WIDE : RAM_END_DEEP;
}

static StepParams base_params(FmeEnv* v, const Dev& d) {
    StepParams P;
    memset(&P, 0, sizeof(P));
    P.d = d;
    P.skip = v->cfg.skip; P.max_steps = v->cfg.max_steps; P.noop_max = v->cfg.noop_max;
    P.maxpool = v->cfg.maxpool ? 1 : 0; P.frame_stack = v->cfg.frame_stack;
    P.sticky_on = v->cfg.sticky != 0.0 ? 1 : 0;
    P.sticky_thr = v->sticky_thr;
    P.hack_cap = v->cfg.hack_cap;
    uint64_t simple = 0;
    for (int k = 0; k < 8; k++) simple |= (uint64_t)kSimple[k] << (8 * k);
    P.simple = simple;
    P.cache.img = v->d_cache_img; P.cache.obs = v->d_cache_obs; P.cache.meta = v->d_cache_meta;
    P.n_levels = v->nl;
    P.level_img = v->d_level_img; P.level_obs0 = v->d_obs0; P.level_meta = v->d_level_meta;
    P.ram_end = RAM_BYTES;   // the reset-cache builder holds the whole slab in shared memory
    return P;
}

static int create_impl(const FmeConfig* cfg, const uint8_t* rom, int64_t rom_len, const int32_t* levels,
                       const uint8_t* gray_lut, const uint64_t* rng, FmeEnv* v) {
    v->cfg = *cfg;
    FmeConfig& C = v->cfg;
    if (C.n_envs < 1) return fail(FME_E_ARG, "n_envs must be >= 1");
    if (C.skip < 1 || C.skip > 16) return fail(FME_E_ARG, "skip must be in 1..16");
    if (C.frame_stack < 1) return fail(FME_E_ARG, "frame_stack must be >= 1");
    if (C.noop_max < 0 || C.noop_max > 100000) return fail(FME_E_ARG, "noop_max out of range");
    if (!levels || !gray_lut || !rng) return fail(FME_E_ARG, "null levels / lut / rng");
    if (C.log_capacity <= 0) C.log_capacity = 2048;
    if (C.hack_cap <= 0) C.hack_cap = 20000;
    if (C.boot_cap <= 0) C.boot_cap = 20000;
    v->n = C.n_envs; v->K = C.frame_stack;
    v->sticky_thr = sticky_threshold(C.sticky);
    std::vector<uint8_t> prg, chr;
    int rc = parse_rom(rom, rom_len, prg, chr, v->nt);
    if (rc) return rc;
    CK(cudaSetDevice(C.device));
    rc = ensure_constants(C.device);
    if (rc) return rc;
    // distinct levels in order of first appearance
    std::vector<int32_t> uniq, env_level(v->n);
    for (int i = 0; i < v->n; i++) {
        int found = -1;
        for (size_t q = 0; q < uniq.size() / 3; q++)
            if (uniq[3 * q] == levels[3 * i] && uniq[3 * q + 1] == levels[3 * i + 1] && uniq[3 * q + 2] == levels[3 * i + 2])
                found = (int)q;
        if (found < 0) {
            found = (int)(uniq.size() / 3);
            uniq.push_back(levels[3 * i]); uniq.push_back(levels[3 * i + 1]); uniq.push_back(levels[3 * i + 2]);
        }
        env_level[i] = found;
    }
    const int nl = (int)(uniq.size() / 3);
    v->nl = nl;
    const int nk = C.noop_max + 1;
    CK(cudaMalloc(&v->d_prg, PRG_ALLOC));
    CK(cudaMalloc(&v->d_chr, 0x2000));
    CK(cudaMalloc(&v->d_lut, 256));
    CK(cudaMalloc(&v->d_err, 4));
    CK(cudaMalloc(&v->d_jobs, (size_t)(C.n_envs + 31) / 32 * 32 * 4));
    {
        int lo = 0, hi = 0;
        CK(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        const int groups = (C.n_envs + 31) / 32;
        v->nch = groups < kChunks ? groups : kChunks;
        int sms = 0;
        CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, C.device));
        v->ram_end = step_ram_end(groups, sms);
        CK(cudaEventCreateWithFlags(&v->ev_in, cudaEventDisableTiming));
        CK(cudaStreamCreateWithPriority(&v->s_copy, cudaStreamNonBlocking, lo));
        CK(cudaEventCreateWithFlags(&v->ev_copy, cudaEventDisableTiming));
        for (int c = 0; c < v->nch; c++) CK(cudaEventCreateWithFlags(&v->ev_pre[c], cudaEventDisableTiming));
        for (int q = 0; q < kTailParts; q++) CK(cudaEventCreateWithFlags(&v->ev_part[q], cudaEventDisableTiming));
        for (int q = 0; q < FmeEnv::kFixRing; q++) CK(cudaEventCreateWithFlags(&v->fix_done[q], cudaEventDisableTiming));
        for (int c = 0; c < v->nch; c++) {
            CK(cudaStreamCreateWithPriority(&v->s_emu[c], cudaStreamNonBlocking, hi));
            CK(cudaStreamCreateWithPriority(&v->s_rnd[c], cudaStreamNonBlocking, lo));
            CK(cudaEventCreateWithFlags(&v->ev_emu[c], cudaEventDisableTiming));
            CK(cudaEventCreateWithFlags(&v->ev_rnd[c], cudaEventDisableTiming));
        }
    }
    CK(upload_prg(v->d_prg, prg));
    CK(cudaMemcpy(v->d_chr, chr.data(), 0x2000, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(v->d_lut, gray_lut, 256, cudaMemcpyHostToDevice));
    CK(cudaMemset(v->d_err, 0, 4));
    CK(cudaMalloc(&v->d_level_img, (size_t)nl * IMG_STRIDE));
    CK(cudaMalloc(&v->d_level_meta, (size_t)nl * 2 * 4));
    CK(cudaMalloc(&v->d_obs0, (size_t)nl * OBS_BYTES));
    CK(cudaMalloc(&v->d_cache_img, (size_t)nl * nk * IMG_STRIDE));
    CK(cudaMalloc(&v->d_cache_obs, (size_t)nl * nk * OBS_BYTES));
    CK(cudaMalloc(&v->d_cache_meta, (size_t)nl * nk * META_WORDS * 4));
    int32_t* d_levels = nullptr;
    int32_t* d_env_level = nullptr;
    uint64_t* d_rng = nullptr;
    CK(cudaMalloc(&d_levels, uniq.size() * 4));
    CK(cudaMemcpy(d_levels, uniq.data(), uniq.size() * 4, cudaMemcpyHostToDevice));
    // ---- boot every level (k_boot) on a scratch state set
    {
        DevBufs bs;
        rc = bs.alloc(nl, C.log_capacity);
        if (rc) return rc;
        BootParams B;
        B.d = make_dev(bs, v->d_prg, v->d_chr, v->nt, v->d_lut, v->d_err);
        B.n_levels = nl; B.levels = d_levels; B.boot_cap = C.boot_cap;
        B.level_img = v->d_level_img; B.level_meta = v->d_level_meta; B.obs0 = v->d_obs0;
        k_boot<<<(nl + 31) / 32, 32, SLAB_BYTES>>>(B);
        CK(cudaGetLastError());
        CK(cudaDeviceSynchronize());
        bs.release();
    }
    uint32_t herr = 0;
    CK(cudaMemcpy(&herr, v->d_err, 4, cudaMemcpyDeviceToHost));
    if (herr & ST_BOOT_CAP) { cudaFree(d_levels); return fail(FME_E_DEVICE, "level boot exceeded boot_cap frames"); }
    // ---- reset cache: entry k = 0 is the boot snapshot; k >= 1 from a builder env per level
    {
        std::vector<int32_t> lm(2 * nl);
        CK(cudaMemcpy(lm.data(), v->d_level_meta, lm.size() * 4, cudaMemcpyDeviceToHost));
        std::vector<int32_t> meta0((size_t)nl * nk * META_WORDS, 0);
        for (int l = 0; l < nl; l++) {
            int32_t* m = &meta0[(size_t)(l * nk) * META_WORDS];
            m[META_X] = lm[2 * l]; m[META_T] = lm[2 * l + 1]; m[META_LIVES] = -1;
            CK(cudaMemcpy(v->d_cache_img + (size_t)(l * nk) * IMG_STRIDE, v->d_level_img + (size_t)l * IMG_STRIDE,
                          IMG_STRIDE, cudaMemcpyDeviceToDevice));
            CK(cudaMemcpy(v->d_cache_obs + (size_t)(l * nk) * OBS_BYTES, v->d_obs0 + (size_t)l * OBS_BYTES, OBS_BYTES,
                          cudaMemcpyDeviceToDevice));
        }
        CK(cudaMemcpy(v->d_cache_meta, meta0.data(), meta0.size() * 4, cudaMemcpyHostToDevice));
        if (C.noop_max > 0) {
            DevBufs bb;
            rc = bb.alloc(nl, C.log_capacity);
            if (rc) return rc;
            std::vector<int32_t> lidx(nl);
            std::vector<uint64_t> r6((size_t)nl * 6, 0);
            for (int l = 0; l < nl; l++) lidx[l] = l;
            CK(cudaMalloc(&d_env_level, (size_t)nl * 4));
            CK(cudaMalloc(&d_rng, r6.size() * 8));
            CK(cudaMemcpy(d_env_level, lidx.data(), lidx.size() * 4, cudaMemcpyHostToDevice));
            CK(cudaMemcpy(d_rng, r6.data(), r6.size() * 8, cudaMemcpyHostToDevice));
            InitParams I;
            I.d = make_dev(bb, v->d_prg, v->d_chr, v->nt, v->d_lut, v->d_err);
            I.level_img = v->d_level_img; I.level_meta = v->d_level_meta; I.env_level = d_env_level; I.rng6 = d_rng;
            k_init<<<(nl + 31) / 32, 32>>>(I);
            CK(cudaGetLastError());
            StepParams P = base_params(v, I.d);
            P.mode = MODE_NOOP;
            P.out_img = v->d_cache_img; P.out_obs = v->d_cache_obs; P.out_meta = v->d_cache_meta;
            for (int j = 1; j <= C.noop_max; j++) {
                P.noop_j = j;
                k_step<false><<<(nl + 31) / 32, 32, SLAB_BYTES>>>(P);
                CK(cudaGetLastError());
            }
            CK(cudaDeviceSynchronize());
            bb.release();
            cudaFree(d_env_level); d_env_level = nullptr;
            cudaFree(d_rng); d_rng = nullptr;
        }
    }
    cudaFree(d_levels);
    // ---- the envs themselves
    rc = v->env.alloc(v->n, C.log_capacity);
    if (rc) return rc;
    CK(cudaMalloc(&d_env_level, (size_t)v->n * 4));
    CK(cudaMalloc(&d_rng, (size_t)v->n * 6 * 8));
    CK(cudaMemcpy(d_env_level, env_level.data(), (size_t)v->n * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_rng, rng, (size_t)v->n * 6 * 8, cudaMemcpyHostToDevice));
    InitParams I;
    I.d = make_dev(v->env, v->d_prg, v->d_chr, v->nt, v->d_lut, v->d_err);
    I.level_img = v->d_level_img; I.level_meta = v->d_level_meta; I.env_level = d_env_level; I.rng6 = d_rng;
    k_init<<<(v->n + 31) / 32, 32>>>(I);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    cudaFree(d_env_level);
    cudaFree(d_rng);
    CK(cudaMemcpy(&herr, v->d_err, 4, cudaMemcpyDeviceToHost));
    if (herr & (ST_HACK_CAP | ST_LOG_OVERFLOW))
        return fail(FME_E_DEVICE, "reset-cache construction hit a device limit (status " + std::to_string(herr) + ")");
    return FME_OK;
}

extern "C" {

const char* fme_last_error(void) { return g_err.c_str(); }
const char* fme_version(void) { return "fme-b200 0.1 (sm_100a)"; }
int64_t fme_state_bytes(void) { return IMG_STRIDE; }
void fme_palette(uint32_t* out64) { if (out64) memcpy(out64, kPalette, sizeof(kPalette)); }

int fme_create(const FmeConfig* cfg, const uint8_t* rom, int64_t rom_len, const int32_t* levels,
               const uint8_t* gray_lut, const uint64_t* rng, FmeEnv** out) {
    if (!cfg || !out) return fail(FME_E_ARG, "null config / out");
    *out = nullptr;
    FmeEnv* v = new FmeEnv();
    int rc = create_impl(cfg, rom, rom_len, levels, gray_lut, rng, v);
    if (rc) { free_env(v); return rc; }
    *out = v;
    return FME_OK;
}

int fme_set_buffers(FmeEnv* v, const FmeBuffers* b) {
    if (!v || !b) return fail(FME_E_ARG, "null env / buffers");
    if (!b->obs || !b->final_obs || !b->rew || !b->term || !b->trunc || !b->info || !b->ep_ret || !b->ep_len)
        return fail(FME_E_ARG, "all output buffers are required");
    if (((uintptr_t)b->obs & 15) || ((uintptr_t)b->final_obs & 15))
        return fail(FME_E_ARG, "obs / final_obs must be 16-byte aligned");
    v->buf = *b;
    v->bound = true;
    return FME_OK;
}

// Per-env scalar outputs of envs [e0, e0 + ne) to the caller's pinned host buffers, on stream cs.
static cudaError_t copy_scalars(const StepParams& P, const FmeHostOut* host, int e0, size_t ne, cudaStream_t cs) {
    cudaError_t e = cudaMemcpyAsync(host->rew + e0, P.rew + e0, ne * 4, cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host->term + e0, P.term + e0, ne, cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host->trunc + e0, P.trunc + e0, ne, cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host->info + e0 * 10, P.info + e0 * 10, ne * 40, cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host->ep_ret + e0, P.ep_ret + e0, ne * 8, cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host->ep_len + e0, P.ep_len + e0, ne * 4, cudaMemcpyDeviceToHost, cs);
    return e;
}

// fme_step_to_host, after the last copy: an env whose episode ended restarts its stack as K-1 zero frames and
// the reset frame; the early copy (or the in-place shift) gave it the old frames, so they are cleared here (runs
// on a driver thread once the copies are done, before the caller's stream moves on).
static void CUDART_CB zero_restarted_stacks(void* arg) {
    const HostFix* f = static_cast<const HostFix*>(arg);
    const size_t ob = (size_t)f->K * OBS_BYTES;
    for (int e = 0; e < f->n; e++)
        if (f->term[e] | f->trunc[e]) memset(f->obs + (size_t)e * ob, 0, (size_t)(f->K - 1) * OBS_BYTES);
}

// In-place variant of the early copy: frames 1..K-1 of every stack of the next step slice move to 0..K-2 inside
// the host buffer, which holds the previous step's stacks. One call per slice, in slice order (stream order on
// the copy stream); the pool's threads split the slice's envs.
static void CUDART_CB shift_host_stacks(void* arg) {
    HostFix* f = static_cast<HostFix*>(arg);
    const int c = f->shift_slice++;
    const int a = f->e0[c], b = f->e0[c + 1];
    const size_t ob = (size_t)f->K * OBS_BYTES, mv = (size_t)(f->K - 1) * OBS_BYTES;
    uint8_t* obs = f->obs;
    const int parts = f->pool->size();
    f->pool->run([=](int q) {
        const int lo = a + (int)((int64_t)(b - a) * q / parts), hi = a + (int)((int64_t)(b - a) * (q + 1) / parts);
        for (int e = lo; e < hi; e++) memmove(obs + (size_t)e * ob, obs + (size_t)e * ob + OBS_BYTES, mv);
    });
}

static int launch_step_impl(FmeEnv* v, const int64_t* d_actions, void* stream, bool reset, void* mark,
                            const FmeHostOut* host);
static int launch_step_like(FmeEnv* v, const int64_t* d_actions, void* stream, bool reset, void* mark = nullptr,
                            const FmeHostOut* host = nullptr) {
    if (!v) return fail(FME_E_ARG, "null env");
    const int rc = launch_step_impl(v, d_actions, stream, reset, mark, host);
    // only a complete fme_step_to_host leaves the caller's buffer holding the stacks (for the next in-place call)
    v->host_obs_prev = (rc == FME_OK && host && !reset) ? host->obs : nullptr;
    return rc;
}
static int launch_step_impl(FmeEnv* v, const int64_t* d_actions, void* stream, bool reset, void* mark,
                            const FmeHostOut* host) {
    if (!v->bound) return fail(FME_E_STATE, "fme_set_buffers must be called first");
    if (!reset && !d_actions) return fail(FME_E_ARG, "null actions");
    CK(cudaSetDevice(v->cfg.device));
    Dev d = make_dev(v->env, v->d_prg, v->d_chr, v->nt, v->d_lut, v->d_err);
    StepParams P = base_params(v, d);
    P.mode = MODE_STEP;
    P.actions = d_actions;
    P.obs = v->buf.obs; P.fin = v->buf.final_obs; P.rew = v->buf.rew; P.term = v->buf.term;
    P.trunc = v->buf.trunc; P.info = v->buf.info; P.ep_ret = v->buf.ep_ret; P.ep_len = v->buf.ep_len;
    cudaStream_t s = (cudaStream_t)stream;
    const int groups = (v->n + 31) / 32;
    if (reset) {
        k_reset<<<groups, 32, 0, s>>>(P);
    } else {
        P.jobs = v->d_jobs;
        RenderParams R;
        R.d = d; R.jobs = v->d_jobs; R.obs = P.obs; R.fin = P.fin; R.cache_obs = P.cache.obs; R.frame_stack = P.frame_stack;
        CK(cudaEventRecord(v->ev_in, s));
        const int K = v->K;
        const size_t ob = (size_t)K * OBS_BYTES;
        // In place: the caller's buffer holds the stacks the previous call of this env wrote, unchanged.
        const bool in_place = host && K > 1 && (host->flags & FME_HOST_OBS_IN_PLACE) && v->host_obs_prev == host->obs;
        HostFix* fx = nullptr;
        cudaEvent_t fx_done = nullptr;
        if (host && K > 1) {
            const uint32_t slot = v->fix_next++ % FmeEnv::kFixRing;
            CK(cudaEventSynchronize(v->fix_done[slot]));   // that slot's earlier call has run its host functions
            fx = &v->fix[slot];
            fx_done = v->fix_done[slot];
            fx->obs = host->obs; fx->term = host->term; fx->trunc = host->trunc; fx->n = v->n; fx->K = K;
            fx->shift_slice = 0;
            for (int c = 0; c <= v->nch; c++) {
                const int gc = groups * c / v->nch;
                fx->e0[c] = gc * 32 < v->n ? gc * 32 : v->n;
            }
            if (in_place && !v->pool) {
                const unsigned hw = std::thread::hardware_concurrency();
                v->pool = new HostPool((int)std::min(7u, hw > 2 ? hw / 2 : 1u));
            }
            fx->pool = v->pool;
        }
        if (host && K > 1) {
            // Frames 1..K-1 of every stack are frames 0..K-2 of the new one. In place they move down inside the
            // host buffer; otherwise they are copied from the device (still untouched there) while the envs
            // emulate. Either way only each env's new frame is left for after its render.
            CK(cudaStreamWaitEvent(v->s_copy, v->ev_in, 0));
            for (int c = 0; c < v->nch; c++) {
                const int e0 = fx->e0[c], e1 = fx->e0[c + 1];
                if (in_place) {
                    CK(cudaLaunchHostFunc(v->s_copy, shift_host_stacks, fx));
                } else {
                    CK(cudaMemcpy2DAsync(host->obs + e0 * ob, ob, P.obs + e0 * ob + OBS_BYTES, ob,
                                         (size_t)(K - 1) * OBS_BYTES, (size_t)(e1 - e0), cudaMemcpyDeviceToHost,
                                         v->s_copy));
                }
                CK(cudaEventRecord(v->ev_pre[c], v->s_copy));
            }
        }
        for (int c = 0; c < v->nch; c++) {
            const int g0 = groups * c / v->nch, g1 = groups * (c + 1) / v->nch;
            const int e0 = g0 * 32, e1 = g1 * 32 < v->n ? g1 * 32 : v->n;
            CK(cudaStreamWaitEvent(v->s_emu[c], v->ev_in, 0));
            P.group_base = g0;
            P.ram_end = v->ram_end;
            k_step<true><<<g1 - g0, 32, (size_t)v->ram_end * LANES, v->s_emu[c]>>>(P);
            CK(cudaEventRecord(v->ev_emu[c], v->s_emu[c]));
            CK(cudaStreamWaitEvent(v->s_rnd[c], v->ev_emu[c], 0));
            // the device copy of the old frames must read them before the render moves them
            if (host && K > 1 && !in_place) CK(cudaStreamWaitEvent(v->s_rnd[c], v->ev_pre[c], 0));
            if (host && K > 1 && v->nch > 1 && c == v->nch - 1) {
                // the last slice's copies are the ones nothing hides: its scalars go as soon as it has emulated,
                // and it is rendered in parts, each part's new frames copied while the next part renders
                const size_t fo = (size_t)(K - 1) * OBS_BYTES;
                CK(cudaStreamWaitEvent(v->s_copy, v->ev_emu[c], 0));
                CK(copy_scalars(P, host, e0, (size_t)(e1 - e0), v->s_copy));
                for (int q = 0; q < kTailParts; q++) {
                    const int q0 = e0 + (e1 - e0) * q / kTailParts, q1 = e0 + (e1 - e0) * (q + 1) / kTailParts;
                    if (q1 <= q0) continue;
                    R.env_base = q0;
                    k_render<<<(unsigned)(q1 - q0) * NBANDS, 32, RB_BYTES, v->s_rnd[c]>>>(R);
                    CK(cudaEventRecord(v->ev_part[q], v->s_rnd[c]));
                    CK(cudaStreamWaitEvent(v->s_copy, v->ev_part[q], 0));
                    CK(cudaMemcpy2DAsync(host->obs + q0 * ob + fo, ob, P.obs + q0 * ob + fo, ob, OBS_BYTES,
                                         (size_t)(q1 - q0), cudaMemcpyDeviceToHost, v->s_copy));
                }
                CK(cudaEventRecord(v->ev_rnd[c], v->s_rnd[c]));
                continue;
            }
            R.env_base = e0;
            k_render<<<(unsigned)(e1 - e0) * NBANDS, 32, RB_BYTES, v->s_rnd[c]>>>(R);
            if (host) {  // this slice's outputs to the host while later slices still run
                const size_t ne = (size_t)(e1 - e0), fo = (size_t)(K - 1) * OBS_BYTES;
                cudaStream_t cs = v->s_rnd[c];
                // in place, the shift reads host frame K-1 before the new frame lands there
                if (in_place) CK(cudaStreamWaitEvent(cs, v->ev_pre[c], 0));
                CK(cudaMemcpy2DAsync(host->obs + e0 * ob + fo, ob, P.obs + e0 * ob + fo, ob, OBS_BYTES, ne,
                                     cudaMemcpyDeviceToHost, cs));
                CK(copy_scalars(P, host, e0, ne, cs));
            }
            CK(cudaEventRecord(v->ev_rnd[c], v->s_rnd[c]));
        }
        if (mark) {  // all emulation slices done (renders may already be running)
            for (int c = 1; c < v->nch; c++) CK(cudaStreamWaitEvent(v->s_emu[0], v->ev_emu[c], 0));
            CK(cudaEventRecord((cudaEvent_t)mark, v->s_emu[0]));
        }
        if (host && K > 1) {
            for (int c = 0; c < v->nch; c++) CK(cudaStreamWaitEvent(v->s_copy, v->ev_rnd[c], 0));
            CK(cudaLaunchHostFunc(v->s_copy, zero_restarted_stacks, fx));
            CK(cudaEventRecord(fx_done, v->s_copy));
            CK(cudaEventRecord(v->ev_copy, v->s_copy));
            CK(cudaStreamWaitEvent(s, v->ev_copy, 0));
        }
        for (int c = 0; c < v->nch; c++) CK(cudaStreamWaitEvent(s, v->ev_rnd[c], 0));
    }
    CK(cudaGetLastError());
    return FME_OK;
}

int fme_reset(FmeEnv* v, void* stream) { return launch_step_like(v, nullptr, stream, true); }
int fme_step(FmeEnv* v, const int64_t* d_actions, void* stream) { return launch_step_like(v, d_actions, stream, false); }
int fme_step_to_host(FmeEnv* v, const int64_t* d_actions, const FmeHostOut* out, void* stream) {
    if (!out || !out->obs || !out->rew || !out->term || !out->trunc || !out->info || !out->ep_ret || !out->ep_len)
        return fail(FME_E_ARG, "all host outputs are required");
    return launch_step_like(v, d_actions, stream, false, nullptr, out);
}
int fme_step_marked(FmeEnv* v, const int64_t* d_actions, void* stream, void* event) {
    if (!event) return fail(FME_E_ARG, "null event");
    return launch_step_like(v, d_actions, stream, false, event);
}

int fme_poll_error(FmeEnv* v, uint32_t* status) {
    if (!v || !status) return fail(FME_E_ARG, "null env / status");
    CK(cudaSetDevice(v->cfg.device));
    CK(cudaMemcpy(status, v->d_err, 4, cudaMemcpyDeviceToHost));
    return FME_OK;
}

int fme_env_ram(FmeEnv* v, int32_t i, uint8_t* host_out) {
    if (!v || !host_out || i < 0 || i >= v->n) return fail(FME_E_ARG, "bad env index");
    CK(cudaSetDevice(v->cfg.device));
    std::vector<uint32_t> words(RAM_BYTES / 4);
    const uint8_t* slab = v->env.slab + (size_t)(i / 32) * SLAB_BYTES + SLAB_RAM_OFF + (i % 32) * 4;
    CK(cudaMemcpy2D(words.data(), 4, slab, 128, 4, RAM_BYTES / 4, cudaMemcpyDeviceToHost));
    memcpy(host_out, words.data(), RAM_BYTES);
    return FME_OK;
}

int fme_ram_all(FmeEnv* v, uint8_t* d_out, void* stream) {
    if (!v || !d_out) return fail(FME_E_ARG, "null env / out");
    CK(cudaSetDevice(v->cfg.device));
    size_t total = (size_t)v->n * (RAM_BYTES / 4);
    k_ram_all<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(v->env.slab, v->n, d_out);
    CK(cudaGetLastError());
    return FME_OK;
}

static int sum_words(FmeEnv* v, int lo_word, int hi_word, int64_t* out) {
    CK(cudaSetDevice(v->cfg.device));
    std::vector<uint32_t> lo(v->n), hi(v->n, 0);
    CK(cudaMemcpy(lo.data(), v->env.scal + (size_t)lo_word * v->env.n_pad, (size_t)v->n * 4, cudaMemcpyDeviceToHost));
    if (hi_word >= 0)
        CK(cudaMemcpy(hi.data(), v->env.scal + (size_t)hi_word * v->env.n_pad, (size_t)v->n * 4, cudaMemcpyDeviceToHost));
    int64_t s = 0;
    for (int i = 0; i < v->n; i++) s += (int64_t)((uint64_t)lo[i] | ((uint64_t)hi[i] << 32));
    *out = s;
    return FME_OK;
}
int fme_frames(FmeEnv* v, int64_t* out) {
    if (!v || !out) return fail(FME_E_ARG, "null env / out");
    return sum_words(v, S_FRAMES_LO, S_FRAMES_HI, out);
}
int fme_bad_ops(FmeEnv* v, int64_t* out) {
    if (!v || !out) return fail(FME_E_ARG, "null env / out");
    return sum_words(v, S_BADOPS, -1, out);
}
int fme_work_counters(FmeEnv* v, int64_t* instructions, int64_t* frames) {
    if (!v || !instructions || !frames) return fail(FME_E_ARG, "null env / out");
    int rc = sum_words(v, S_INSTR_LO, S_INSTR_HI, instructions);
    return rc ? rc : sum_words(v, S_EMU_FRAMES, -1, frames);
}
int64_t fme_env_bytes(FmeEnv* v) {
    if (!v) return -1;
    return (int64_t)(v->env.bytes() / (size_t)v->n);
}
void fme_destroy(FmeEnv* v) {
    if (!v) return;
    cudaSetDevice(v->cfg.device);
    cudaDeviceSynchronize();
    free_env(v);
}

// ---------------------------------------------------------------- raw consoles
int fme_raw_create(const uint8_t* rom, int64_t rom_len, int32_t n, int32_t device, int32_t log_capacity, FmeRaw** out) {
    if (!out || n < 1) return fail(FME_E_ARG, "bad raw arguments");
    *out = nullptr;
    FmeRaw* r = new FmeRaw();
    r->n = n; r->device = device;
    std::vector<uint8_t> prg, chr;
    auto bail = [&](int code) { fme_raw_destroy(r); return code; };
    int rc = parse_rom(rom, rom_len, prg, chr, r->nt);
    if (rc) return bail(rc);
    if (cudaSetDevice(device) != cudaSuccess) return bail(fail(FME_E_CUDA, "cudaSetDevice failed"));
    rc = ensure_constants(device);
    if (rc) return bail(rc);
    if (log_capacity <= 0) log_capacity = 2048;
    rc = r->st.alloc(n, log_capacity);
    if (rc) return bail(rc);
    uint8_t ident[256];
    for (int i = 0; i < 256; i++) ident[i] = (uint8_t)i;
    if (cudaMalloc(&r->d_prg, PRG_ALLOC) || cudaMalloc(&r->d_chr, 0x2000) || cudaMalloc(&r->d_lut, 256) ||
        cudaMalloc(&r->d_err, 4) || cudaMalloc(&r->d_screens, (size_t)n * SCREEN_W * SCREEN_H) ||
        cudaMalloc(&r->d_bk_slab, (size_t)(r->st.n_pad / 32) * SLAB_BYTES) ||
        cudaMalloc(&r->d_bk_vram, (size_t)r->st.n_pad * VRAM_BYTES) ||
        cudaMalloc(&r->d_bk_scal, (size_t)S_WORDS * r->st.n_pad * 4))
        return bail(fail(FME_E_CUDA, "cudaMalloc failed"));
    if (upload_prg(r->d_prg, prg) != cudaSuccess) return bail(fail(FME_E_CUDA, "PRG upload failed"));
    cudaMemcpy(r->d_chr, chr.data(), 0x2000, cudaMemcpyHostToDevice);
    cudaMemcpy(r->d_lut, ident, 256, cudaMemcpyHostToDevice);
    cudaMemset(r->d_err, 0, 4);
    cudaMemset(r->d_screens, 0, (size_t)n * SCREEN_W * SCREEN_H);
    {
        Dev d = make_dev(r->st, r->d_prg, r->d_chr, r->nt, r->d_lut, r->d_err);
        k_power<<<(n + 31) / 32, 32, SLAB_BYTES>>>(d);
        if (cudaGetLastError() != cudaSuccess) return bail(fail(FME_E_CUDA, "power-on launch failed"));
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(fail(FME_E_CUDA, "raw init failed"));
    *out = r;
    return FME_OK;
}

int fme_raw_frame(FmeRaw* r, const uint8_t* d_buttons, int32_t render, void* stream) {
    if (!r || !d_buttons) return fail(FME_E_ARG, "null raw / buttons");
    CK(cudaSetDevice(r->device));
    RawParams P;
    P.d = make_dev(r->st, r->d_prg, r->d_chr, r->nt, r->d_lut, r->d_err);
    P.buttons = d_buttons; P.render = render ? 1 : 0; P.screens = r->d_screens;
    k_raw<<<(r->n + 31) / 32, 32, SLAB_BYTES, (cudaStream_t)stream>>>(P);
    CK(cudaGetLastError());
    return FME_OK;
}
int fme_raw_ram(FmeRaw* r, uint8_t* d_out, void* stream) {
    if (!r || !d_out) return fail(FME_E_ARG, "null raw / out");
    CK(cudaSetDevice(r->device));
    size_t total = (size_t)r->n * (RAM_BYTES / 4);
    k_ram_all<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(r->st.slab, r->n, d_out);
    CK(cudaGetLastError());
    return FME_OK;
}
int fme_raw_screen(FmeRaw* r, uint8_t* d_out, void* stream) {
    if (!r || !d_out) return fail(FME_E_ARG, "null raw / out");
    CK(cudaSetDevice(r->device));
    CK(cudaMemcpyAsync(d_out, r->d_screens, (size_t)r->n * SCREEN_W * SCREEN_H, cudaMemcpyDeviceToDevice,
                       (cudaStream_t)stream));
    return FME_OK;
}
int fme_raw_backup(FmeRaw* r, void* stream) {
    if (!r) return fail(FME_E_ARG, "null raw");
    CK(cudaSetDevice(r->device));
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemcpyAsync(r->d_bk_slab, r->st.slab, (size_t)(r->st.n_pad / 32) * SLAB_BYTES, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpyAsync(r->d_bk_vram, r->st.vram, (size_t)r->st.n_pad * VRAM_BYTES, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpyAsync(r->d_bk_scal, r->st.scal, (size_t)S_WORDS * r->st.n_pad * 4, cudaMemcpyDeviceToDevice, s));
    return FME_OK;
}
int fme_raw_restore(FmeRaw* r, void* stream) {
    if (!r) return fail(FME_E_ARG, "null raw");
    CK(cudaSetDevice(r->device));
    cudaStream_t s = (cudaStream_t)stream;
    // bad-op counters and status are not part of the console state (the first S_CONSOLE_WORDS rows are);
    // they survive a restore as in the reference (Nes::bad_ops is outside NesState)
    CK(cudaMemcpyAsync(r->st.slab, r->d_bk_slab, (size_t)(r->st.n_pad / 32) * SLAB_BYTES, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpyAsync(r->st.vram, r->d_bk_vram, (size_t)r->st.n_pad * VRAM_BYTES, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpyAsync(r->st.scal, r->d_bk_scal, (size_t)S_CONSOLE_WORDS * r->st.n_pad * 4, cudaMemcpyDeviceToDevice, s));
    return FME_OK;
}
int fme_raw_bad_ops(FmeRaw* r, int64_t* out) {
    if (!r || !out) return fail(FME_E_ARG, "null raw / out");
    CK(cudaSetDevice(r->device));
    std::vector<uint32_t> b(r->n);
    CK(cudaMemcpy(b.data(), r->st.scal + (size_t)S_BADOPS * r->st.n_pad, (size_t)r->n * 4, cudaMemcpyDeviceToHost));
    int64_t s = 0;
    for (uint32_t x : b) s += x;
    *out = s;
    return FME_OK;
}
int fme_raw_poll_error(FmeRaw* r, uint32_t* status) {
    if (!r || !status) return fail(FME_E_ARG, "null raw / status");
    CK(cudaSetDevice(r->device));
    CK(cudaMemcpy(status, r->d_err, 4, cudaMemcpyDeviceToHost));
    return FME_OK;
}
void fme_raw_destroy(FmeRaw* r) {
    if (!r) return;
    cudaSetDevice(r->device);
    cudaDeviceSynchronize();
    r->st.release();
    cudaFree(r->d_prg); cudaFree(r->d_chr); cudaFree(r->d_lut); cudaFree(r->d_err); cudaFree(r->d_screens);
    cudaFree(r->d_bk_slab); cudaFree(r->d_bk_vram); cudaFree(r->d_bk_scal);
    delete r;
}

int fme_raw_frame_static(FmeRaw* r, const uint8_t* d_buttons, uint8_t* d_screens, int32_t render, void* stream) {
    if (!r || !d_buttons) return fail(FME_E_ARG, "null raw / buttons");
    if (render && !d_screens) return fail(FME_E_ARG, "render needs a screen buffer");
    if (r->n > FME_STATIC_MAX_CONSOLES)
        return fail(FME_E_ARG, "fme_raw_frame_static takes at most " + std::to_string(FME_STATIC_MAX_CONSOLES) +
                                   " consoles, the handle has " + std::to_string(r->n));
    CK(cudaSetDevice(r->device));
    uint8_t* scratch = nullptr;
    int rc = static_scratch(r->device, &scratch);
    if (rc) return rc;
    RawParams P;
    P.d = make_dev(r->st, r->d_prg, r->d_chr, r->nt, r->d_lut, r->d_err);
    P.d.logs = scratch;
    P.d.log_cap = FME_STATIC_LOG_CAPACITY;
    P.buttons = d_buttons; P.render = render ? 1 : 0; P.screens = d_screens;
    k_raw<<<(r->n + 31) / 32, 32, SLAB_BYTES, (cudaStream_t)stream>>>(P);
    CK(cudaGetLastError());
    return FME_OK;
}

// ---------------------------------------------------------------- PPO data kernels
int fme_gae(const float* d_rew, const float* d_val, const float* d_done, const float* d_next_val,
            const float* d_next_done, int32_t T, int32_t N, float gamma, float gamma_lam, float* d_adv, float* d_ret,
            void* stream) {
    if (!d_rew || !d_val || !d_done || !d_next_val || !d_next_done || !d_adv || !d_ret || T < 1 || N < 1)
        return fail(FME_E_ARG, "bad GAE arguments");
    k_gae<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(d_rew, d_val, d_done, d_next_val, d_next_done, T, N,
                                                             gamma, gamma_lam, d_adv, d_ret);
    CK(cudaGetLastError());
    return FME_OK;
}
int fme_adv_norm(const float* d_in, float* d_out, int32_t n, void* stream) {
    if (!d_in || !d_out || n < 1) return fail(FME_E_ARG, "bad advantage-normalisation arguments");
    k_adv_norm<<<1, ADV_THREADS, 0, (cudaStream_t)stream>>>(d_in, d_out, n);
    CK(cudaGetLastError());
    return FME_OK;
}

// ---------------------------------------------------------------- frame-deduplicating replay buffer
static int replay_dev(const FmeReplayBufs* rb, ReplayDev* out) {
    if (!rb || !rb->frames || !rb->age || !rb->act || !rb->rew || !rb->flags || !rb->ptr || !rb->new_ep ||
        rb->n_envs < 1 || rb->capacity < 1)
        return fail(FME_E_ARG, "bad replay buffers");
    if ((uintptr_t)rb->frames & 15) return fail(FME_E_ARG, "replay frames must be 16-byte aligned");
    out->frames = rb->frames; out->age = rb->age; out->act = rb->act; out->rew = rb->rew; out->flags = rb->flags;
    out->ptr = rb->ptr; out->new_ep = rb->new_ep; out->E = rb->n_envs; out->C = rb->capacity;
    return FME_OK;
}
int fme_replay_add(const FmeReplayBufs* rb, const uint8_t* d_obs, const uint8_t* d_next_obs, int32_t k,
                   const int64_t* d_action, const float* d_reward, const uint8_t* d_done, const uint8_t* d_trunc,
                   void* stream) {
    ReplayDev R;
    int rc = replay_dev(rb, &R);
    if (rc) return rc;
    if (!d_obs || !d_next_obs || !d_action || !d_reward || !d_done || !d_trunc || k < 1)
        return fail(FME_E_ARG, "bad replay add arguments");
    if (((uintptr_t)d_obs & 15) || ((uintptr_t)d_next_obs & 15)) return fail(FME_E_ARG, "obs must be 16-byte aligned");
    k_replay_add<<<R.E, 32, 0, (cudaStream_t)stream>>>(R, d_obs, d_next_obs, d_action, d_reward, d_done, d_trunc, k);
    CK(cudaGetLastError());
    return FME_OK;
}
int fme_replay_gather(const FmeReplayBufs* rb, const int64_t* d_env, const int64_t* d_pos, int32_t B, int32_t k,
                      int32_t n_step, const float* d_gpow, const float* d_dpow, uint8_t* d_obs, uint8_t* d_next_obs,
                      int64_t* d_act, float* d_reward, float* d_discount, float* d_terminal, int64_t* d_steps,
                      void* stream) {
    ReplayDev R;
    int rc = replay_dev(rb, &R);
    if (rc) return rc;
    if (!d_env || !d_pos || !d_gpow || !d_dpow || !d_obs || !d_next_obs || !d_act || !d_reward || !d_discount ||
        !d_terminal || !d_steps || B < 0 || k < 1 || n_step < 1 || n_step > R.C)
        return fail(FME_E_ARG, "bad replay gather arguments");
    if (((uintptr_t)d_obs & 15) || ((uintptr_t)d_next_obs & 15)) return fail(FME_E_ARG, "obs must be 16-byte aligned");
    if (B == 0) return FME_OK;
    k_replay_gather<<<B, 32, 0, (cudaStream_t)stream>>>(R, d_env, d_pos, B, k, n_step, d_gpow, d_dpow, d_obs,
                                                        d_next_obs, d_act, d_reward, d_discount, d_terminal, d_steps);
    CK(cudaGetLastError());
    return FME_OK;
}

int fme_resize(const uint8_t* d_src, uint8_t* d_dst, int32_t n, void* stream) {
    if (!d_src || !d_dst || n < 0) return fail(FME_E_ARG, "bad resize arguments");
    int dev = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaSetDevice(dev));  // makes the device's primary context current (ensure_constants keys on it)
    int rc = ensure_constants(dev);
    if (rc) return rc;
    if (n == 0) return FME_OK;
    int grid = n < 4096 ? n : 4096;
    k_resize<<<grid, 32, SLAB_BYTES, (cudaStream_t)stream>>>(d_src, d_dst, n);
    CK(cudaGetLastError());
    return FME_OK;
}

}  // extern "C"

namespace fme {
uint32_t g_host_dtab[256];  // referenced by the host instantiation of Core::execute, never executed
}
