// Host build of the engine's emulation headers, used by the CPU test suite (tests/test_host_engine.py).
//
// Raw consoles are stepped one NES frame at a time with the code the GPU kernels run: Core (fme_core.h), the
// register-resident fast path and its per-PC micro-ops (fme_fast.h, fme_tables.h), the data-driven datapath
// and its micro-ops (fme_dp.h, lane_step: the per-lane meaning of the step kernel's two-phase warp loop) and
// the frame bookkeeping of fme_agent.h. Each console has a whole group slab to itself and uses lane 0 of it, so memory is laid out
// exactly as in the kernels. The per-frame flow follows k_raw: scalars in, begin_frame, hot_step until the
// frame end, end_frame / close_frame, scalars out. No pixels are drawn (the GPU renderer is warp code); the
// PPU log is produced and discarded, so its catch-up and logging paths still run.
#include <cstdint>
#include <cstring>
#include <vector>

#include "fme_core.h"
#include "fme_agent.h"
#include "fme_tables.h"
#include "fme_fast.h"
#include "fme_dp.h"

namespace fme { uint32_t g_host_dtab[256]; }
using namespace fme;

namespace {

constexpr int kLogCap = 4096;

struct HostRaw {
    int n = 0;
    std::vector<uint8_t> prg;      // 32 KB PRG, then the micro-op table (2 words per PRG address)
    std::vector<uint8_t> chr;      // 8 KB
    uint32_t nt[4] = {0, 0, 0, 0};
    std::vector<uint8_t> slab;     // n x SLAB_BYTES, lane 0 of each used
    std::vector<uint8_t> vram;     // n x VRAM_BYTES
    std::vector<uint32_t> words;   // n x S_WORDS
    std::vector<uint8_t> log;      // one log slot, reused by every console and frame
    std::vector<uint32_t> dops;    // datapath micro-ops (2 words per PRG address)
};

void bind(HostRaw* r, Core& c, int e) {
    uint8_t* s = r->slab.data() + (size_t)e * SLAB_BYTES;
    c.ram = s + SLAB_RAM_OFF;
    c.ramh = c.ram;
    c.ram_end = RAM_BYTES;
    c.oam = s + SLAB_OAM_OFF;
    c.pal = s + SLAB_PAL_OFF;
    c.vram = r->vram.data() + (size_t)e * VRAM_BYTES;
    c.cart.prg = r->prg.data();
    c.cart.chr = r->chr.data();
    for (int i = 0; i < 4; i++) c.cart.nt[i] = r->nt[i];
    c.rec = nullptr; c.nrec = 0; c.cap = 0; c.seg_open = false; c.seg_w0 = 0; c.seg_y1 = 0; c.status = 0;
    c.seg_idx = 0; c.seg_reads = 0; c.vram_burst = 0; c.vram_dirty = false;
}

}  // namespace

extern "C" {

// iNES mapper 0 (16 or 32 KB PRG, 8 KB CHR, H/V mirroring) -> n consoles at power-on; NULL for other images.
void* hr_create(const uint8_t* rom, int64_t len, int n) {
    if (!rom || len < 16 || n < 1 || memcmp(rom, "NES\x1a", 4) != 0) return nullptr;
    const int banks = rom[4], chr_banks = rom[5];
    const int mapper = (rom[6] >> 4) | (rom[7] & 0xF0);
    if (mapper != 0 || (banks != 1 && banks != 2) || chr_banks != 1) return nullptr;
    const size_t off = 16 + ((rom[6] & 4) ? 512 : 0);
    if ((size_t)len < off + (size_t)banks * 0x4000 + 0x2000) return nullptr;
    HostRaw* r = new HostRaw;
    r->n = n;
    r->prg.assign(0x8000 + (size_t)UOP_WORDS * 4, 0);
    for (int k = 0; k < 2; k++) memcpy(r->prg.data() + k * 0x4000, rom + off + (banks == 2 ? k : 0) * 0x4000, 0x4000);
    r->chr.assign(rom + off + (size_t)banks * 0x4000, rom + off + (size_t)banks * 0x4000 + 0x2000);
    if (rom[6] & 1) { r->nt[1] = r->nt[3] = 0x400; }   // vertical mirroring
    else { r->nt[2] = r->nt[3] = 0x400; }               // horizontal mirroring
    tables::build_dtab(g_host_dtab);
    tables::build_uops(r->prg.data(), g_host_dtab, reinterpret_cast<uint32_t*>(r->prg.data() + 0x8000));
    r->dops.assign((size_t)UOP_WORDS, 0);
    tables::build_dops(reinterpret_cast<const uint32_t*>(r->prg.data() + 0x8000), r->dops.data());
    r->slab.assign((size_t)n * SLAB_BYTES, 0);
    r->vram.assign((size_t)n * VRAM_BYTES, 0);
    r->words.assign((size_t)n * S_WORDS, 0);
    r->log.assign(slot_bytes(kLogCap), 0);
    for (int e = 0; e < n; e++) {  // k_power
        Core c;
        bind(r, c, e);
        c.bad_ops = 0;
        c.power_on();
        uint32_t* w = r->words.data() + (size_t)e * S_WORDS;
        c.store_scalars(w);
    }
    return r;
}

// One frame of every console with the given controller bytes (k_raw without the renderer).
void hr_frame(void* h, const uint8_t* buttons) {
    HostRaw* r = static_cast<HostRaw*>(h);
    for (int e = 0; e < r->n; e++) {
        Core c;
        bind(r, c, e);
        uint32_t* w = r->words.data() + (size_t)e * S_WORDS;
        c.load_scalars(w);
        c.bad_ops = w[S_BADOPS];
        c.status = w[S_STATUS];
        uint8_t* slot = r->log.data();
        begin_frame(c, slot, buttons[e], kLogCap);
        const Fast fst{c.ram, c.ramh, c.ram_end, r->prg.data(), reinterpret_cast<const uint32_t*>(r->prg.data() + 0x8000)};
        Hot hot{};
        hot_in(hot, c, fst);
        rf_pack(hot);
        dfetch(hot, r->dops.data());
        while (lane_step(hot, c, fst, r->dops.data())) {
        }
        rf_unpack(hot);
        hot_out(hot, c);
        c.end_frame();
        close_frame(c, slot);
        materialise_state(c);
        c.store_scalars(w);
        w[S_BADOPS] = c.bad_ops;
        w[S_STATUS] = c.status;
    }
}

void hr_ram(void* h, int e, uint8_t* out) {
    HostRaw* r = static_cast<HostRaw*>(h);
    Core c;
    bind(r, c, e);
    for (uint32_t a = 0; a < 0x800u; a++) out[a] = (uint8_t)c.RAM(a);
}

int64_t hr_bad_ops(void* h, int e) { return static_cast<HostRaw*>(h)->words[(size_t)e * S_WORDS + S_BADOPS]; }
int64_t hr_status(void* h, int e) { return static_cast<HostRaw*>(h)->words[(size_t)e * S_WORDS + S_STATUS]; }
void hr_destroy(void* h) { delete static_cast<HostRaw*>(h); }

// One instruction at a time, from random states: the datapath (dp_exec, the step kernel's bulk path) against
// the exact interpreter (Core::execute_op, which the lockstep tests pin to the reference). PRG is random
// bytes, so every PRG address starts an instruction with random operand bytes; registers, status byte and
// RAM are random. RAM is held whole in one buffer (ram_end 0x800) or split at `ram_end` across two buffers
// (the step kernel's shared-memory / HBM layout). Only instructions the datapath commits are compared: pc,
// A, X, Y, SP, P, the cycle count and all of RAM. Returns the number compared; *first_bad receives
// (opcode << 16 | pc & 0xffff) of the first mismatch, or -1; hist[opc] counts the comparisons per opcode.
int64_t hr_dp_check(uint64_t seed, int64_t trials, uint32_t ram_end, int32_t* first_bad, int64_t* hist) {
    uint64_t s = seed * 0x9E3779B97F4A7C15ull + 1u;
    auto rnd = [&]() -> uint32_t {  // xorshift64*
        s ^= s >> 12; s ^= s << 25; s ^= s >> 27;
        return (uint32_t)((s * 0x2545F4914F6CDD1Dull) >> 32);
    };
    std::vector<uint8_t> prg(0x8000 + (size_t)UOP_WORDS * 4, 0), chr(0x2000, 0), vram(VRAM_BYTES, 0);
    std::vector<uint32_t> dops((size_t)UOP_WORDS, 0);
    // exact side: one slab; datapath side: the RAM below ram_end in `lo`, the rest in `hi` (same layout)
    std::vector<uint8_t> slab(SLAB_BYTES, 0), lo(SLAB_BYTES, 0), hi(SLAB_BYTES, 0);
    tables::build_dtab(g_host_dtab);
    *first_bad = -1;
    int64_t compared = 0;
    for (int64_t t = 0; t < trials; t++) {
        if (t % 4096 == 0) {  // a new random PRG image every 4096 instructions
            for (uint32_t i = 0; i < 0x8000u; i++) prg[i] = (uint8_t)rnd();
            tables::build_uops(prg.data(), g_host_dtab, reinterpret_cast<uint32_t*>(prg.data() + 0x8000));
            tables::build_dops(reinterpret_cast<const uint32_t*>(prg.data() + 0x8000), dops.data());
        }
        const uint32_t pc = 0x8000u | (rnd() & 0x7fffu);
        const uint32_t a = rnd() & 0xffu, x = rnd() & 0xffu, y = rnd() & 0xffu, sp = rnd() & 0xffu, p = rnd() & 0xffu;
        for (uint32_t m = 0; m < (uint32_t)RAM_BYTES; m++) {
            const uint8_t v = (uint8_t)rnd();
            slab[il(m)] = v;
            (m < ram_end ? lo : hi)[il(m)] = v;
        }
        Hot h{};
        h.pc = pc; h.a = a; h.x = x; h.y = y; h.sp = sp; h.p = p; h.exec_at = 0; h.thresh = 1 << 30;
        rf_pack(h);
        dfetch(h, dops.data());
        if (!(h.ux & D_OK)) continue;
        const Fast f{lo.data(), hi.data(), ram_end, prg.data(), reinterpret_cast<const uint32_t*>(prg.data() + 0x8000)};
        if (!dp_exec(h, f, dops.data(), true)) continue;   // a computed I/O address: the exact path's case
        rf_unpack(h);
        Core c{};
        c.ram = c.ramh = slab.data(); c.ram_end = RAM_BYTES;
        c.oam = slab.data() + SLAB_OAM_OFF; c.pal = slab.data() + SLAB_PAL_OFF; c.vram = vram.data();
        c.cart.prg = prg.data(); c.cart.chr = chr.data();
        c.pc = pc; c.a = a; c.x = x; c.y = y; c.sp = sp; c.p = p;
        const uint32_t opc = prg[pc & 0x7fffu];
        const int32_t S = c.execute_op(opc);
        bool same = h.pc == c.pc && h.a == c.a && h.x == c.x && h.y == c.y && h.sp == c.sp && h.p == c.p &&
                    h.exec_at == (S >= 1 ? S : 1);
        for (uint32_t m = 0; same && m < (uint32_t)RAM_BYTES; m++)
            same = (m < ram_end ? lo : hi)[il(m)] == slab[il(m)];
        compared++;
        hist[opc]++;
        if (!same && *first_bad < 0) *first_bad = (int32_t)((opc << 16) | (pc & 0xffffu));
    }
    return compared;
}

}  // extern "C"
