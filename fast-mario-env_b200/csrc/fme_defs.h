// fme_defs.h - constants, data layouts and the opcode decode format shared by host and device code.
//
// Layouts (all chosen for the B200 kernels, not taken from the reference):
//  * Console memory that the 6502 touches every instruction (RAM, OAM, palette) is kept per warp-group
//    of 32 envs in a "lane-interleaved" slab: 32-bit word w of lane l lives at word (w * 32 + l). In
//    shared memory every lane therefore owns bank l, so any mix of addresses across the warp is
//    conflict-free; in HBM the slab is one contiguous 73 KB block that is streamed in and out whole.
//  * VRAM (2 KB) stays in HBM, contiguous per env: it is touched only by $2007 and the frame snapshot.
//  * Scalar state (CPU/PPU registers, timing, env bookkeeping) is SoA: word w of env e at w*n_pad + e.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define FME_HD __host__ __device__ __forceinline__
#define FME_NI __host__ __device__ __noinline__
#else
#define FME_HD inline
#define FME_NI inline
#include <vector_types.h>
#endif

namespace fme {

constexpr int RAM_BYTES = 0x800;
constexpr int VRAM_BYTES = 0x800;
constexpr int OAM_BYTES = 0x100;
constexpr int PAL_BYTES = 0x20;
constexpr int LANES = 32;
constexpr int SLAB_RAM_OFF = 0;                                  // bytes inside one group's slab
constexpr int SLAB_OAM_OFF = RAM_BYTES * LANES;                  // 65536
constexpr int SLAB_PAL_OFF = SLAB_OAM_OFF + OAM_BYTES * LANES;   // 73728
constexpr int SLAB_BYTES = SLAB_PAL_OFF + PAL_BYTES * LANES;     // 74752

// k_step's emulation keeps the RAM addresses below a boundary (ram_end) in shared memory and reaches the rest
// in the HBM slab itself (same lane-interleaved layout, through L1). Both parts are addressed through
// Core::RAM and Fast::R/W, which pick the base by address; the other kernels hold the whole RAM in shared
// memory (ram_end = 0x800). The step picks the boundary by how many CTAs it runs: latency first while they
// fill the SMs in a few waves, residency first beyond that.
//  * RAM_END_DEEP: 48 KB per CTA of 32 envs, so four fit an SM's 196 KB shared-memory configuration (three at
//    64 KB), leaving 60 KB of L1 for each env's top 512 bytes of RAM, OAM and palette;
//  * RAM_END_WIDE: 23 KB per CTA, eight per SM in the same configuration.
constexpr uint32_t RAM_END_DEEP = 0x600, RAM_END_WIDE = 0x2e0;
static_assert(RAM_END_DEEP % 4 == 0 && RAM_END_WIDE % 4 == 0 && RAM_END_WIDE >= 0x200 &&
              RAM_END_DEEP <= (uint32_t)RAM_BYTES, "boundaries are word aligned and keep zero page and stack in shared memory");

constexpr int FRAME_ITERS = 29781;           // CPU iterations per emulated frame (nes_core.hpp:53)
constexpr int FRAME_CALLS = 3 * FRAME_ITERS;  // PPU calls per emulated frame
constexpr int OBS = 84;
constexpr int OBS_BYTES = OBS * OBS;
constexpr int SCREEN_W = 256, SCREEN_H = 240;

// status flags (reversed bit order of nes-py's bitfield, N is bit 0; nes_core.hpp:36-38)
enum : uint32_t { F_N = 0x01, F_V = 0x02, F_ONE = 0x04, F_B = 0x08, F_D = 0x10, F_I = 0x20, F_Z = 0x40, F_C = 0x80 };
enum : uint32_t { PS_PRE = 0, PS_RENDER = 1, PS_POST = 2, PS_VBLANK = 3 };

// ---------------------------------------------------------------- opcode decode word
// bits 0-3 kind, 4-7 addressing mode, 8-12 operation, 13 page-cross penalty, 16-23 base cycles.
enum Kind : uint32_t {
    K_BAD = 0,      // unimplemented: bad_ops++, nothing else
    K_BAD_ZP = 1,   // decoded addressing (1 operand byte read) but no operation: bad_ops++
    K_BAD_ABS = 2,  // 2 operand bytes read, no operation
    K_BAD_ABSX = 3, // 2 operand bytes read, page-cross penalty with X, no operation
    K_IMPL = 4,
    K_BRANCH = 5,
    K_READ = 6,
    K_STORE = 7,
    K_RMW = 8,
    K_ACC = 9,
};
enum Mode : uint32_t { M_NONE = 0, M_IMM, M_ZP, M_ZPX, M_ZPY, M_ABS, M_ABSX, M_ABSY, M_INDX, M_INDY };
enum ReadOp : uint32_t { R_ORA = 0, R_AND, R_EOR, R_ADC, R_LDA, R_CMP, R_SBC, R_BIT, R_LDX, R_LDY, R_CPX, R_CPY };
enum StoreOp : uint32_t { W_STA = 0, W_STX, W_STY };
enum RmwOp : uint32_t { X_ASL = 0, X_ROL, X_LSR, X_ROR, X_DEC, X_INC };
enum ImplOp : uint32_t {
    I_BRK = 0, I_PHP, I_CLC, I_JSR, I_PLP, I_SEC, I_RTI, I_PHA, I_JMP, I_CLI, I_RTS, I_PLA, I_JMPI, I_SEI,
    I_DEY, I_TXA, I_TYA, I_TXS, I_TAY, I_TAX, I_CLV, I_TSX, I_INY, I_DEX, I_CLD, I_INX, I_NOP, I_SED
};
FME_HD uint32_t d_kind(uint32_t d) { return d & 15u; }
FME_HD uint32_t d_mode(uint32_t d) { return (d >> 4) & 15u; }
FME_HD uint32_t d_op(uint32_t d) { return (d >> 8) & 31u; }
FME_HD uint32_t d_pen(uint32_t d) { return (d >> 13) & 1u; }
FME_HD uint32_t d_cycles(uint32_t d) { return (d >> 16) & 255u; }

// ---------------------------------------------------------------- per-PC micro-op (fast path)
// word 0: handler | opcode<<8 | op<<16 | page-penalty<<21 | length<<22 | idle-loop<<24
// word 1: operand (immediate or ROM value, static address, pointer byte, branch target) | cycles<<16 | extra<<24
enum Hid : uint32_t {
    H_SLOW = 0,   // the exact path (I/O operands, code at $FFFE-$FFFF, unusual forms)
    H_RD_IMM, H_RD_ZP, H_RD_ZPX, H_RD_ZPY, H_RD_ABS, H_RD_ABSX, H_RD_ABSY, H_RD_INDX, H_RD_INDY,
    H_ST_ZP, H_ST_ZPX, H_ST_ZPY, H_ST_ABS, H_ST_ABSX, H_ST_ABSY, H_ST_INDX, H_ST_INDY, H_NOPW,
    H_RMW_ZP, H_RMW_ZPX, H_RMW_ABS, H_RMW_ABSX,
    H_ACC, H_BRANCH, H_IMPL, H_BAD, H_BAD_ABSX,
    H_JOY_RD, H_JOY_ST,  // abs read of $4016/$4017 (operand = port) / abs store to $4016: controller ports,
                         // run beside the exact path without the hand-over of the register state
    // specialised forms: the operation is part of the handler id, so one dispatch runs the instruction
    H_X_RD = 32,        // + op: operand value in the micro-op (immediate, ROM); + 16 + op: static RAM address
    H_X_ST = 64,        // + op: store to a static RAM address
    H_X_RMW = 72,       // + op: read-modify-write of a static RAM address
    H_X_ACC = 80,       // + op: accumulator shifts / rotates
    H_X_IMPL = 96,      // + op: implied, stack and jump instructions
    H_X_RDZX = 128,     // + op: read (zp,X)            the indexed reads below check the computed address
    H_X_RDAX = 144,     // + op: read abs,X             for I/O (exact path) and add the page-cross cycle
    H_X_RDAY = 160,     // + op: read abs,Y
    H_X_RDIY = 176,     // + op: read (zp),Y
    H_X_RDIX = 192,     // + op: read (zp,X)
};
constexpr uint32_t UOP_IDLE = 1u << 24;
constexpr int UOP_WORDS = 2 * 0x8000;

// ---------------------------------------------------------------- log records (16 B each)
enum RecType : uint32_t { REC_SEG = 0, REC_VRAM = 1, REC_PAL = 2, REC_OAM = 3, REC_DMA = 4, REC_LIST = 5, REC_VSNAP = 6 };
// VRAM writes logged one by one between two segments; past this many the next segment is preceded by a
// whole-VRAM snapshot instead (bulk nametable uploads), which bounds a burst at twice the snapshot size.
constexpr int VRAM_BURST_MAX = 128;
// SEG  w0: type | y0<<4 | x0<<12 | x1<<21     (dots [x0, 256) of line y0, all dots of the lines in between,
//      w3: y1                                   dots [0, x1) of line y1; [x0, x1) of y0 when y1 == y0)
//      w1: v at (y0, x0) (16 bits) | fine_x<<16 | render flags<<19
//      w2: pending-eval bit | eval_y<<1 | oam_addr<<9 | coarse x of t<<17 | nametable-x bit of t<<22
//      Nothing the CPU does changes a render input inside a segment, so the lines after y0 follow from the
//      first: v advances by the dot-257 fine-y increment and the dot-258 copy of t's x bits, and each line's
//      sprite list is the (pending) evaluation of the line before it.
// VRAM w0: type | index<<4 (11 bits) | value<<16       PAL/OAM the same with 5/8-bit index
// DMA  w0: type, followed by 16 records holding the whole OAM after the copy
// LIST w0: type | nsl<<4; w1: sl[0..3]; w2: sl[4..7]
// VSNAP w0: type, followed by 128 records holding the whole 2 KB VRAM
enum : uint32_t { TOUCH_ALL = 1, TOUCH_BG = 2, TOUCH_SPR = 4, TOUCH_VRAM = 8 };
enum : uint32_t { RF_SHOW_BG = 1, RF_SHOW_SPR = 2, RF_HIDE_BG = 4, RF_HIDE_SPR = 8, RF_LONG = 16,
                  RF_BG_PAGE = 32, RF_SPR_PAGE = 64 };

// v after L fine-y increments (the dot-257 step of nes_core.hpp:318-330 applied L times, closed form). Rows
// r = coarse_y*8 + fine_y count 0..239 and wrap with a nametable-y toggle; rows 240..255 (coarse y 30/31)
// run on to 255 and wrap to 0 without the toggle.
FME_HD uint32_t fine_y_add(uint32_t v, int L) {
    int r = (int)(((v >> 5) & 31u) * 8u + ((v >> 12) & 7u));
    uint32_t ny = (v >> 11) & 1u;
    if (r >= 240) {
        if (r + L < 256) { r += L; L = 0; }
        else { L -= 256 - r; r = 0; }
    }
    if (r < 240) {
        r += L;
        ny ^= (uint32_t)(r / 240) & 1u;
        r %= 240;
    }
    return (v & ~0x7be0u & 0xffffu) | ((uint32_t)(r & 7) << 12) | ((uint32_t)(r >> 3) << 5) | (ny << 11);
}

// A log slot: frame-start snapshot (VRAM, palette, OAM, sprite-list state) + record stream.
constexpr int SLOT_HDR_VRAM = 0;
constexpr int SLOT_HDR_PAL = 2048;
constexpr int SLOT_HDR_OAM = 2080;
constexpr int SLOT_HDR_LIST = 2336;   // 4 words: nsl | pend<<8 | eval_y<<16, sl[0..3], sl[4..7], nrec
constexpr int SLOT_HDR_BYTES = 2352;  // multiple of 16
FME_HD size_t slot_bytes(int cap) { return (size_t)SLOT_HDR_BYTES + (size_t)cap * 16u; }

// ---------------------------------------------------------------- scalar state words (SoA)
enum Scal : int {
    // console (part of the snapshot / reset image)
    S_CPU0 = 0,   // pc | a<<16 | x<<24
    S_CPU1,       // y | sp<<8 | p<<16 | zero_skip<<24
    S_ITER_LO, S_ITER_HI,  // CPU iteration at the frame boundary (nes-py cycle count)
    S_EXEC,       // exec_at - iter
    S_PPUC,       // ppu_calls - 3*iter
    S_THRESH,     // nmi_thresh - 3*iter
    S_JOY,        // strobe0 | strobe1<<1 | buttons0<<8 | buttons1<<16
    S_JOYB,       // bits0 | bits1<<8
    S_PPU0,       // pstate | scanline<<2 | pcyc<<12 | fine_x<<22 | first_write<<25 | vblank<<26 | s0hit<<27 | even<<28 | inc32<<29
    S_PPU1,       // v | t<<16
    S_PPU2,       // data_buffer | oam_addr<<8 | regflags<<16 | nsl<<24
    S_SL0, S_SL1, // sprite list sl[0..3], sl[4..7]
    S_CONSOLE_WORDS,
    // env bookkeeping
    S_XLAST = S_CONSOLE_WORDS, S_TLAST, S_PREV, S_LIVES, S_T, S_EPLEN, S_EPRET_LO, S_EPRET_HI,
    S_RNG_S0, S_RNG_S1, S_RNG_S2, S_RNG_S3,  // PCG64 state, least significant word first
    S_RNG_I0, S_RNG_I1, S_RNG_I2, S_RNG_I3,  // PCG64 increment
    S_RNG_HAS, S_RNG_U32,                    // numpy has_uint32 / uinteger
    S_LEVEL, S_FRAMES_LO, S_FRAMES_HI, S_BADOPS, S_STATUS,
    // emulated-work counters of the timed step kernel (not part of the env semantics): 6502 instructions
    // executed (the idle-loop fast-forward and the sprite-0 poll skip count none) and NES frames run
    S_INSTR_LO, S_INSTR_HI, S_EMU_FRAMES,
    S_WORDS
};
// register flag byte inside S_PPU2 (bits 16-23)
enum : uint32_t { PF_SHOW_BG = 1, PF_SHOW_SPR = 2, PF_HIDE_BG = 4, PF_HIDE_SPR = 8, PF_LONG = 16, PF_NMI = 32,
                  PF_BG_PAGE = 64, PF_SPR_PAGE = 128 };

// error / status bits (per env word S_STATUS and the global error word)
enum : uint32_t {
    ST_LOG_OVERFLOW = 1u,     // a frame produced more log records than the slot holds
    ST_HACK_CAP = 2u,         // the busy-state skip loop exceeded its frame cap
    ST_BOOT_CAP = 4u,         // level boot exceeded its frame cap
    ST_BAD_ACTION = 8u,       // action outside 0..6 (treated as 0)
    ST_FRAME_CAP = 16u,       // a frame exceeded its instruction cap
};

// Console image (contiguous, used for level boot snapshots, the reset cache and raw backups).
constexpr int IMG_RAM = 0, IMG_VRAM = 2048, IMG_OAM = 4096, IMG_PAL = 4352, IMG_SCAL = 4384;
constexpr int IMG_BYTES = IMG_SCAL + 4 * S_CONSOLE_WORDS + 8;  // + pad to 16
constexpr int IMG_STRIDE = (IMG_BYTES + 15) / 16 * 16;

}  // namespace fme
