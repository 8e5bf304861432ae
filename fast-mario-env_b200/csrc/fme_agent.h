// fme_agent.h - the env wrapper chain around one console, per lane (host/device portable).
//
// Semantics are those of the reference Env (csrc/fastmario.cpp:268-412): per-NES-frame sticky actions from
// the env's numpy PCG64 stream (39-78, 344), frame skip with reward summing and early stop (336-353), the
// SMB reward/done/info of each frame-step (316-334), the busy-state / area skip hacks (304-314), life loss
// and flag as termination (367-372), time limit and episode bookkeeping (403-411), and the reset-cache
// form of the random no-op reset (389-401). What differs is the mechanics: every frame writes a PPU log
// into one of two slots so that the frames the observation needs (the last frame of the final frame-step
// group and of the one before it, which is exactly what the reference re-emulates on early termination,
// 354-365) can be rendered afterwards without snapshots or re-emulation.
#pragma once
#include "fme_core.h"

namespace fme {

// ---------------------------------------------------------------- numpy PCG64 (fastmario.cpp:39-78)
struct Pcg {
    uint64_t s_hi, s_lo, i_hi, i_lo;
    uint32_t has32, u32;
};
FME_HD uint64_t mulhi64(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
    return __umul64hi(a, b);
#else
    return (uint64_t)(((unsigned __int128)a * b) >> 64);
#endif
}
FME_HD uint64_t pcg_next64(Pcg& r) {
    const uint64_t M_HI = 0x2360ED051FC65DA4ull, M_LO = 0x4385DF649FCCF645ull;
    uint64_t lo = r.s_lo * M_LO;
    uint64_t hi = mulhi64(r.s_lo, M_LO) + r.s_lo * M_HI + r.s_hi * M_LO;
    uint64_t nlo = lo + r.i_lo;
    hi += r.i_hi + (nlo < lo ? 1ull : 0ull);
    r.s_lo = nlo; r.s_hi = hi;
    uint32_t rot = (uint32_t)(hi >> 58);
    uint64_t xv = hi ^ nlo;
    return (xv >> rot) | (xv << ((64u - rot) & 63u));
}
FME_HD uint32_t pcg_next32(Pcg& r) {
    if (r.has32) { r.has32 = 0; return r.u32; }
    uint64_t n = pcg_next64(r);
    r.has32 = 1;
    r.u32 = (uint32_t)(n >> 32);
    return (uint32_t)n;
}
// Generator.integers(0, high) for high <= 2^32 (Lemire with numpy's uint32 buffering)
FME_HD uint32_t pcg_integers(Pcg& r, uint32_t high) {
    uint32_t rng = high - 1u;
    if (rng == 0) return 0;
    if (rng == 0xFFFFFFFFu) return pcg_next32(r);
    uint32_t excl = rng + 1u;
    uint64_t m = (uint64_t)pcg_next32(r) * excl;
    uint32_t left = (uint32_t)m;
    if (left < excl) {
        uint32_t thr = (0xFFFFFFFFu - rng) % excl;
        while (left < thr) {
            m = (uint64_t)pcg_next32(r) * excl;
            left = (uint32_t)m;
        }
    }
    return (uint32_t)(m >> 32);
}

// ---------------------------------------------------------------- env bookkeeping (scalar words)
struct EnvVars {
    int32_t x_last, t_last;
    uint32_t prev;
    int32_t lives, t, ep_len;
    double ep_ret;
    Pcg rng;
    int32_t level;
    uint64_t frames;
    FME_HD void load(const uint32_t* w) {
        x_last = (int32_t)w[S_XLAST]; t_last = (int32_t)w[S_TLAST]; prev = w[S_PREV];
        lives = (int32_t)w[S_LIVES]; t = (int32_t)w[S_T]; ep_len = (int32_t)w[S_EPLEN];
        uint64_t eb = (uint64_t)w[S_EPRET_LO] | ((uint64_t)w[S_EPRET_HI] << 32);
        memcpy_d(&ep_ret, &eb);
        rng.s_lo = (uint64_t)w[S_RNG_S0] | ((uint64_t)w[S_RNG_S1] << 32);
        rng.s_hi = (uint64_t)w[S_RNG_S2] | ((uint64_t)w[S_RNG_S3] << 32);
        rng.i_lo = (uint64_t)w[S_RNG_I0] | ((uint64_t)w[S_RNG_I1] << 32);
        rng.i_hi = (uint64_t)w[S_RNG_I2] | ((uint64_t)w[S_RNG_I3] << 32);
        rng.has32 = w[S_RNG_HAS]; rng.u32 = w[S_RNG_U32];
        level = (int32_t)w[S_LEVEL];
        frames = (uint64_t)w[S_FRAMES_LO] | ((uint64_t)w[S_FRAMES_HI] << 32);
    }
    FME_HD void store(uint32_t* w) const {
        w[S_XLAST] = (uint32_t)x_last; w[S_TLAST] = (uint32_t)t_last; w[S_PREV] = prev;
        w[S_LIVES] = (uint32_t)lives; w[S_T] = (uint32_t)t; w[S_EPLEN] = (uint32_t)ep_len;
        uint64_t eb;
        memcpy_d(&eb, &ep_ret);
        w[S_EPRET_LO] = (uint32_t)eb; w[S_EPRET_HI] = (uint32_t)(eb >> 32);
        w[S_RNG_S0] = (uint32_t)rng.s_lo; w[S_RNG_S1] = (uint32_t)(rng.s_lo >> 32);
        w[S_RNG_S2] = (uint32_t)rng.s_hi; w[S_RNG_S3] = (uint32_t)(rng.s_hi >> 32);
        w[S_RNG_I0] = (uint32_t)rng.i_lo; w[S_RNG_I1] = (uint32_t)(rng.i_lo >> 32);
        w[S_RNG_I2] = (uint32_t)rng.i_hi; w[S_RNG_I3] = (uint32_t)(rng.i_hi >> 32);
        w[S_RNG_HAS] = rng.has32; w[S_RNG_U32] = rng.u32;
        w[S_LEVEL] = (uint32_t)level;
        w[S_FRAMES_LO] = (uint32_t)frames; w[S_FRAMES_HI] = (uint32_t)(frames >> 32);
    }
    template <class A, class B>
    FME_HD static void memcpy_d(A* dst, const B* src) {
        static_assert(sizeof(A) == sizeof(B), "size");
        const unsigned char* s = reinterpret_cast<const unsigned char*>(src);
        unsigned char* d = reinterpret_cast<unsigned char*>(dst);
        for (unsigned k = 0; k < sizeof(A); k++) d[k] = s[k];
    }
};

// ---------------------------------------------------------------- frame log slots
FME_HD void begin_frame(Core& c, uint8_t* slot, uint32_t buttons, int cap) {
    c.joy_buttons[0] = buttons;
    const uint4* src = reinterpret_cast<const uint4*>(c.vram);
    uint4* dst = reinterpret_cast<uint4*>(slot + SLOT_HDR_VRAM);
    for (int i = 0; i < VRAM_BYTES / 16; i++) dst[i] = src[i];
    uint32_t* pw = reinterpret_cast<uint32_t*>(slot + SLOT_HDR_PAL);
    for (int w = 0; w < PAL_BYTES / 4; w++) pw[w] = *reinterpret_cast<const uint32_t*>(c.pal + (w << 7));
    uint32_t* ow = reinterpret_cast<uint32_t*>(slot + SLOT_HDR_OAM);
    for (int w = 0; w < OAM_BYTES / 4; w++) ow[w] = *reinterpret_cast<const uint32_t*>(c.oam + (w << 7));
    uint32_t* lw = reinterpret_cast<uint32_t*>(slot + SLOT_HDR_LIST);
    lw[0] = c.nsl | ((c.ev_pend ? 1u : 0u) << 8) | (c.ev_y << 16);
    lw[1] = c.sl_lo; lw[2] = c.sl_hi; lw[3] = 0;
    c.rec = reinterpret_cast<uint4*>(slot + SLOT_HDR_BYTES);
    c.nrec = 0; c.cap = cap; c.seg_open = false; c.vram_burst = 0; c.vram_dirty = false;
}
FME_HD void close_frame(Core& c, uint8_t* slot) {
    reinterpret_cast<uint32_t*>(slot + SLOT_HDR_LIST)[3] = (uint32_t)c.nrec;
}
FME_HD void materialise_state(Core& c) {
    if (c.ev_pend) { c.eval_now(c.ev_y); c.ev_pend = false; }
}

// ---------------------------------------------------------------- console image <-> lane state
FME_HD void image_to_lane(const uint8_t* img, Core& c, uint32_t* scal_words) {
    for (int w = 0; w < RAM_BYTES / 4; w++)
        *reinterpret_cast<uint32_t*>(c.ram_at((uint32_t)w * 4)) = reinterpret_cast<const uint32_t*>(img + IMG_RAM)[w];
    for (int w = 0; w < OAM_BYTES / 4; w++)
        *reinterpret_cast<uint32_t*>(c.oam + (w << 7)) = reinterpret_cast<const uint32_t*>(img + IMG_OAM)[w];
    for (int w = 0; w < PAL_BYTES / 4; w++)
        *reinterpret_cast<uint32_t*>(c.pal + (w << 7)) = reinterpret_cast<const uint32_t*>(img + IMG_PAL)[w];
    const uint4* vs = reinterpret_cast<const uint4*>(img + IMG_VRAM);
    uint4* vd = reinterpret_cast<uint4*>(c.vram);
    for (int i = 0; i < VRAM_BYTES / 16; i++) vd[i] = vs[i];
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(img + IMG_SCAL);
    for (int w = 0; w < S_CONSOLE_WORDS; w++) scal_words[w] = sw[w];
}
FME_HD void lane_to_image(const Core& c, uint8_t* img) {
    for (int w = 0; w < RAM_BYTES / 4; w++)
        reinterpret_cast<uint32_t*>(img + IMG_RAM)[w] = *reinterpret_cast<const uint32_t*>(c.ram_at((uint32_t)w * 4));
    for (int w = 0; w < OAM_BYTES / 4; w++)
        reinterpret_cast<uint32_t*>(img + IMG_OAM)[w] = *reinterpret_cast<const uint32_t*>(c.oam + (w << 7));
    for (int w = 0; w < PAL_BYTES / 4; w++)
        reinterpret_cast<uint32_t*>(img + IMG_PAL)[w] = *reinterpret_cast<const uint32_t*>(c.pal + (w << 7));
    const uint4* vs = reinterpret_cast<const uint4*>(c.vram);
    uint4* vd = reinterpret_cast<uint4*>(img + IMG_VRAM);
    for (int i = 0; i < VRAM_BYTES / 16; i++) vd[i] = vs[i];
    uint32_t w[S_CONSOLE_WORDS];
    c.store_scalars(w);
    uint32_t* sw = reinterpret_cast<uint32_t*>(img + IMG_SCAL);
    for (int k = 0; k < S_CONSOLE_WORDS; k++) sw[k] = w[k];
}

// ---------------------------------------------------------------- reset cache
struct Cache {
    const uint8_t* img;     // entries x IMG_STRIDE console images (entry = level * (noop_max + 1) + k)
    const uint8_t* obs;     // entries x 7056
    const int32_t* meta;    // entries x 8
};
enum { META_X = 0, META_T, META_LIVES, META_DRAWS, META_FR_LO, META_FR_HI, META_BAD, META_WORDS = 8 };

// Env::reset through the cache: k = integers(noop_max + 1), then the state after k no-op agent steps of
// this level, with the RNG advanced by the random() draws those steps made. Returns the entry index.
FME_HD int reset_from_cache(Core& c, EnvVars& ev, const Cache& cache, int noop_max) {
    uint32_t k = noop_max ? pcg_integers(ev.rng, (uint32_t)noop_max + 1u) : 0u;
    int ci = ev.level * (noop_max + 1) + (int)k;
    const int32_t* meta = cache.meta + (size_t)ci * META_WORDS;
    for (int q = 0; q < meta[META_DRAWS]; q++) pcg_next64(ev.rng);
    uint32_t cw[S_CONSOLE_WORDS];
    image_to_lane(cache.img + (size_t)ci * IMG_STRIDE, c, cw);
    c.load_scalars(cw);
    ev.x_last = meta[META_X]; ev.t_last = meta[META_T]; ev.lives = meta[META_LIVES];
    ev.prev = 0; ev.t = 0; ev.ep_ret = 0.0; ev.ep_len = 0;
    ev.frames += (uint64_t)(uint32_t)meta[META_FR_LO] | ((uint64_t)(uint32_t)meta[META_FR_HI] << 32);
    c.bad_ops += (uint32_t)meta[META_BAD];
    return ci;
}

// ---------------------------------------------------------------- one agent step as a frame-level state machine
enum AgentMode : int { MODE_STEP = 0, MODE_NOOP = 1 };

struct AgentCfg {
    int mode, skip, max_steps, noop_max, maxpool, sticky_on, hack_cap, cap;
    uint64_t sticky_thr;   // a draw repeats the previous action when (next64 >> 11) < sticky_thr
    uint64_t simple;       // SIMPLE_MOVEMENT controller bytes, byte k = action k
};

struct StepOut {
    bool term, trunc, pooled, done_early;
    int32_t total;
    int64_t info[10];
    uint64_t re_frames;   // frames the reference re-emulates on early termination (counted, not run)
    uint32_t re_bad;
    int cur_slot;         // slot holding the final frame; the other holds the previous group's last frame
};

struct Agent {
    uint32_t act;
    int i, last, cur_slot, hacks_cur, hacks_prev;
    bool hack, done;
    int32_t total;
    int64_t info[10];
    uint32_t bad_group_start, bad_prev, draws;
    uint8_t* slot[2];

    FME_HD void begin_agent(Core& c, EnvVars& ev, const AgentCfg& g) {
        uint32_t ae = act;
        if (g.sticky_on) {
            if (g.mode == MODE_STEP) {
                uint64_t r = pcg_next64(ev.rng);
                if ((r >> 11) < g.sticky_thr) ae = ev.prev;
            } else {
                draws++;  // reset-cache builder: action 0 == previous 0, only the draw count matters
            }
        }
        ev.prev = ae;
        hacks_prev = hacks_cur; hacks_cur = 0;
        bad_prev = c.bad_ops - bad_group_start; bad_group_start = c.bad_ops;
        cur_slot ^= 1;
        hack = false;
        begin_frame(c, slot[cur_slot], (uint32_t)((g.simple >> (8 * ae)) & 0xffu), g.cap);
    }
    FME_HD void start(Core& c, EnvVars& ev, const AgentCfg& g, uint32_t action, uint8_t* s0, uint8_t* s1) {
        act = action; i = 0; last = 0; cur_slot = 1; hacks_cur = 0; hacks_prev = 0;
        hack = false; done = false; total = 0;
        for (int k = 0; k < 10; k++) info[k] = 0;
        bad_group_start = c.bad_ops; bad_prev = 0; draws = 0;
        slot[0] = s0; slot[1] = s1;
        begin_agent(c, ev, g);
    }
    // after Core::end_frame: bookkeeping of the finished frame; returns true if another frame was begun
    FME_HD bool on_frame_end(Core& c, EnvVars& ev, const AgentCfg& g) {
        close_frame(c, slot[cur_slot]);
        ev.frames++;
        if (!hack) {
            int32_t xp = smb_x_pos(c);
            int64_t xr = (int64_t)xp - ev.x_last; ev.x_last = xp;
            if (xr < -5 || xr > 5) xr = 0;
            int64_t tm = smb_time(c);
            int64_t tp = tm - ev.t_last; ev.t_last = (int32_t)tm;
            if (tp > 0) tp = 0;
            bool dying = smb_dying(c), dead = smb_dead(c);
            int64_t r = xr + tp + ((dying || dead) ? -25 : 0);
            if (r < -15) r = -15;
            if (r > 15) r = 15;
            total += (int32_t)r;
            smb_info(c, info);
            done = dying || dead || info[1] != 0;
            if (!done) {
                uint32_t cat = c.RAM(0x06de);
                if (cat > 1 && cat < 255) c.RAMW(0x06de, 1);
                if (smb_busy(c) || smb_world_over(c)) {
                    c.RAMW(0x07a0, 0);
                    hack = true;
                    begin_frame(c, slot[cur_slot], 0, g.cap);
                    return true;
                }
            }
        } else {
            hacks_cur++;
            if (hacks_cur >= g.hack_cap) {
                c.status |= ST_HACK_CAP;
            } else if (smb_busy(c) || smb_world_over(c)) {
                c.RAMW(0x07a0, 0);
                begin_frame(c, slot[cur_slot], 0, g.cap);
                return true;
            }
        }
        if (done) { last = i; return false; }
        if (++i < g.skip) { begin_agent(c, ev, g); return true; }
        last = g.skip - 1;
        return false;
    }
    // episode logic after the last frame (fastmario.cpp:353-373, 403-411)
    FME_HD StepOut finish(Core& c, EnvVars& ev, const AgentCfg& g) {
        StepOut o;
        materialise_state(c);
        o.pooled = g.maxpool && last >= 1;
        bool term_ = done;
        int life = (int)info[2];
        if (ev.lives >= 0 && life < ev.lives) term_ = true;
        ev.lives = life;
        if (info[1]) term_ = true;
        ev.t++;
        o.term = term_;
        o.trunc = ev.t >= g.max_steps;
        ev.ep_ret += (double)total;
        ev.ep_len++;
        o.done_early = done && last < g.skip - 1;
        uint32_t bad_last_group = c.bad_ops - bad_group_start;
        o.re_frames = 0; o.re_bad = 0;
        if (o.done_early) {
            o.re_frames = o.pooled ? (uint64_t)(2 + hacks_prev) : 1u;
            o.re_bad = (o.pooled ? bad_prev : 0u) + bad_last_group;
        }
        o.total = total;
        for (int k = 0; k < 10; k++) o.info[k] = info[k];
        o.cur_slot = cur_slot;
        return o;
    }
};

}  // namespace fme
