/* fme.h - C ABI of libfme_cuda.so, the B200 batched NES / SMB-style environment engine.
 *
 * This is the boundary the Python host code (and any other FFI caller) binds. It replaces the reference's
 * GPU path, CudaVecEnv -> cujit.Module.launch -> cuLaunchKernel with a by-value StepArgs struct
 * (src/fast_mario_env/cuda/vec_env.py:197-231, 350-373; cuda/cujit.py:157-178), and mirrors the shape of the
 * reference's CPU C ABI (csrc/fastmario.cpp:562-674) so a caller of either finds the same concepts:
 * create -> set_buffers -> reset -> step, plus frames / bad_ops / per-env RAM and the raw console API.
 *
 * Conventions
 *  - Every function returns 0 on success or a negative FME_E* code; no C++ exception crosses the ABI.
 *    fme_last_error() gives a message for the last failure on the calling thread.
 *  - Device buffers passed in are owned by the caller (for example torch tensors) and must stay alive
 *    while the env uses them; the library never frees them.
 *  - fme_reset / fme_step only enqueue work on the given CUDA stream (cudaStream_t passed as void*;
 *    NULL = legacy default stream). They do not synchronise and do not allocate.
 *  - One env object must not be stepped from two threads or two streams at once.
 *  - Errors detected on the device (log overflow, frame caps, bad actions) are latched into a status word;
 *    read it with fme_poll_error after synchronising the stream.
 */
#ifndef FME_H
#define FME_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FME_OK 0
#define FME_E_ARG (-1)       /* invalid argument (sizes, skip outside 1..16, ...) */
#define FME_E_ROM (-2)       /* ROM rejected (not iNES, mapper != 0, PRG banks not 1..2, CHR banks != 1) */
#define FME_E_CUDA (-3)      /* a CUDA runtime call failed */
#define FME_E_DEVICE (-4)    /* a device-side status bit is set (see fme_poll_error) */
#define FME_E_STATE (-5)     /* call order violated (e.g. step before set_buffers) */

/* device status bits reported by fme_poll_error */
#define FME_ST_LOG_OVERFLOW 1u   /* a frame produced more PPU log records than log_capacity */
#define FME_ST_HACK_CAP 2u       /* the busy-state skip loop hit its frame cap (reference would spin) */
#define FME_ST_BOOT_CAP 4u       /* level boot hit its frame cap (reference would spin) */
#define FME_ST_BAD_ACTION 8u     /* an action outside 0..6 was given (treated as 0) */

typedef struct FmeEnv FmeEnv;
typedef struct FmeRaw FmeRaw;

/* Env configuration; field meanings follow FastVecEnv / CudaVecEnv (src/fast_mario_env/env.py:140-142,
 * cuda/vec_env.py:247-249) and fm_create (csrc/fastmario.cpp:566-568). */
typedef struct FmeConfig {
    int32_t n_envs;
    int32_t skip;          /* NES frames per agent step, 1..16 */
    int32_t max_steps;     /* time limit in agent steps */
    int32_t noop_max;      /* 0 disables random no-op starts */
    int32_t maxpool;       /* max over the gray frames of the last two frame-steps */
    int32_t frame_stack;   /* k >= 1 */
    double sticky;         /* probability of repeating the previous action, per NES frame */
    int32_t device;        /* CUDA device ordinal */
    int32_t log_capacity;  /* PPU log records per frame slot; 0 = default (2048) */
    int32_t hack_cap;      /* frame cap for one busy-state skip loop; 0 = default (20000) */
    int32_t boot_cap;      /* frame cap for booting one level; 0 = default (20000) */
} FmeConfig;

/* Output buffers (device pointers). Shapes as CudaVecEnv's (cuda/vec_env.py:316-328):
 * obs/final_obs uint8 (N, k, 84, 84); rew float32 (N,); term/trunc uint8 (N,); info int32 (N, 10) in the
 * order x_pos, flag_get, life, score, time, world, stage, coins, y_pos, status; ep_ret float64 (N,);
 * ep_len int32 (N,). final_obs / ep_ret / ep_len are written only for envs whose episode ended. */
typedef struct FmeBuffers {
    uint8_t* obs;
    uint8_t* final_obs;
    float* rew;
    uint8_t* term;
    uint8_t* trunc;
    int32_t* info;
    double* ep_ret;
    int32_t* ep_len;
} FmeBuffers;

/* Create N envs. Replaces fm_create (csrc/fastmario.cpp:566-601) and CudaVecEnv.__init__
 * (cuda/vec_env.py:247-347): validates the ROM (fm_create returns NULL on a bad ROM or skip), boots each
 * distinct level on the GPU and builds the per-(level, k) no-op reset cache.
 *   rom, rom_len   iNES image
 *   levels         N x 3 int32 (world, stage, area) as decode_level returns (rom.py:88-103)
 *   gray_lut       256 bytes, palette value -> gray (env.py:42-47)
 *   rng            N x 6 uint64: state_hi, state_lo, inc_hi, inc_lo, has_uint32, uinteger of
 *                  numpy default_rng(seed*1000 + env_offset + i) (env.py:50-55, 155-156)
 * Synchronises the device once at the end (boot and cache construction). */
int fme_create(const FmeConfig* cfg, const uint8_t* rom, int64_t rom_len, const int32_t* levels,
               const uint8_t* gray_lut, const uint64_t* rng, FmeEnv** out);

/* Bind caller-owned device output buffers. Replaces fm_set_buffers (csrc/fastmario.cpp:603-608). */
int fme_set_buffers(FmeEnv* env, const FmeBuffers* bufs);

/* Reset every env (random no-op start from the reset cache), write the zero-padded frame stacks.
 * Replaces fm_reset (csrc/fastmario.cpp:610) / CudaVecEnv.reset (cuda/vec_env.py:363-365). Async. */
int fme_reset(FmeEnv* env, void* stream);

/* One agent step for every env; d_actions is int64 (N,) on the device (0..6, SIMPLE_MOVEMENT index).
 * Replaces fm_step_async + fm_step_wait (csrc/fastmario.cpp:611-617) and CudaVecEnv.step
 * (cuda/vec_env.py:367-373): sticky actions, frame skip, max-pool, reward/done/info, busy-state skipping,
 * time limit, frame stack, final_obs and auto-reset. Async; enqueues only. */
int fme_step(FmeEnv* env, const int64_t* d_actions, void* stream);
/* fme_step that also records `event` (a cudaEvent_t as void*, created by the caller) on the stream between
 * the emulation kernel and the render kernel, so the two can be timed apart. No counterpart in the
 * reference (a profiling hook; the step itself is identical). */
int fme_step_marked(FmeEnv* env, const int64_t* d_actions, void* stream, void* event);

/* Pinned host destinations of fme_step_to_host (shapes as FmeBuffers; final_obs stays on the device). */
#define FME_HOST_OBS_IN_PLACE 1u   /* FmeHostOut.flags: obs holds this env's previous stacks (see below) */
typedef struct FmeHostOut {
    uint8_t* obs;
    float* rew;
    uint8_t* term;
    uint8_t* trunc;
    int32_t* info;
    double* ep_ret;
    int32_t* ep_len;
    uint32_t flags;   /* FME_HOST_OBS_IN_PLACE or 0 */
} FmeHostOut;
/* fme_step, and the step's outputs copied into pinned host memory while the step runs. Frames 1..k-1 of every
 * stack are frames 0..k-2 of the new one: with FME_HOST_OBS_IN_PLACE, when `obs` is the buffer this env's
 * previous fme_step_to_host filled (and the caller has not changed it since; no fme_step or fme_reset of the
 * env came in between), they move down inside that host buffer (host threads, as the reference's host engine
 * shifts its stacks in place, csrc/fastmario.cpp:494-503); otherwise they are copied from the device as soon
 * as the step starts. Then each slice's new frames and scalars go to the host once that slice's kernels are
 * done (the last slice rendered and copied in parts), and, last, a host function (cudaLaunchHostFunc) clears
 * frames 0..k-2 of the envs whose episode ended (their stack restarts as zeros + the reset frame). Replaces
 * fm_step_async + fm_step_wait's host-buffer outputs (csrc/fastmario.cpp:611-617) for callers that want host
 * arrays. Async: synchronise the stream before reading `out`. Up to 16 calls of one env may be in flight; a
 * 17th waits (on the host) until the oldest one's host functions have run. */
int fme_step_to_host(FmeEnv* env, const int64_t* d_actions, const FmeHostOut* out, void* stream);

/* OR of the device status bits of all envs since create (call after synchronising). */
int fme_poll_error(FmeEnv* env, uint32_t* status);

/* Copy env i's 2 KB RAM to host memory (synchronous). Replaces fm_env_ram (csrc/fastmario.cpp:630). */
int fme_env_ram(FmeEnv* env, int32_t i, uint8_t* host_out);
/* All envs' RAM as (N, 2048) uint8 into a device buffer, async. Replaces CudaVecEnv.ram (vec_env.py:375-378). */
int fme_ram_all(FmeEnv* env, uint8_t* d_out, void* stream);

/* Total emulated NES frames and unimplemented opcodes over all envs (synchronous).
 * Replace fm_frames / fm_bad_ops (csrc/fastmario.cpp:619-628). */
int fme_frames(FmeEnv* env, int64_t* out);
int fme_bad_ops(FmeEnv* env, int64_t* out);
/* Emulated work of the steps so far, summed over all envs (synchronous): 6502 instructions executed (the
 * idle-loop fast-forward and the sprite-0 poll skip execute none) and NES frames actually run by the step
 * kernel (unlike fme_frames, without the frames of no-op starts served from the reset cache or of the
 * early-termination frames the reference re-emulates). No counterpart in the reference; the reference quotes
 * emulated instructions per agent step in its documentation (README.md:261-262). */
int fme_work_counters(FmeEnv* env, int64_t* instructions, int64_t* frames);
/* Device bytes held per env (replaces fm_env_bytes, csrc/fastmario.cpp:632-635). */
int64_t fme_env_bytes(FmeEnv* env);

/* Destroy and free the library-owned device memory. Replaces fm_destroy (csrc/fastmario.cpp:618). */
void fme_destroy(FmeEnv* env);

/* ---- raw consoles (frame-level fidelity), replacing fm_raw_* (csrc/fastmario.cpp:651-673) ---- */
/* n independent consoles powered on from the same ROM. */
int fme_raw_create(const uint8_t* rom, int64_t rom_len, int32_t n, int32_t device, int32_t log_capacity,
                   FmeRaw** out);
/* One NES frame for every console: d_buttons uint8 (n,) device; render != 0 also writes the 240x256
 * palette-value screens (as fm_raw_frame with render=1 fills fm_raw_screen). Async. */
int fme_raw_frame(FmeRaw* raw, const uint8_t* d_buttons, int32_t render, void* stream);
/* RAM (n, 2048) and screens (n, 240, 256) into device buffers, async. */
int fme_raw_ram(FmeRaw* raw, uint8_t* d_out, void* stream);
int fme_raw_screen(FmeRaw* raw, uint8_t* d_out, void* stream);
/* Snapshot / restore every console (fm_raw_backup / fm_raw_restore). Async. */
int fme_raw_backup(FmeRaw* raw, void* stream);
int fme_raw_restore(FmeRaw* raw, void* stream);
int fme_raw_bad_ops(FmeRaw* raw, int64_t* out);
int fme_raw_poll_error(FmeRaw* raw, uint32_t* status);
void fme_raw_destroy(FmeRaw* raw);

/* One NES frame like fme_raw_frame, allocating nothing. No counterpart in the reference.
 * The per-frame PPU log (the scratch fme_raw_frame keeps in the handle) lives in a fixed device array
 * compiled into the library: FME_STATIC_MAX_CONSOLES consoles at FME_STATIC_LOG_CAPACITY records a frame
 * (about 4.3 MB). Handles with more consoles are rejected with FME_E_ARG; a frame with more records sets
 * FME_ST_LOG_OVERFLOW. render != 0 writes the 240x256 palette-value screens into d_screens ((n, 240, 256)
 * uint8, caller-owned; may be NULL when render == 0). Nothing in the array has to start at zero: every
 * frame rewrites its slot header before the records it reads back. The first call on a device looks the
 * array's address up (cudaGetSymbolAddress) with that device current; make it before any stream capture.
 * All calls on one device share the array, so calls that can overlap (other streams, other threads)
 * race and must be ordered by the caller. The screens go only to d_screens: the handle's own screen buffer
 * is not written, so fme_raw_screen keeps returning the screens of the last fme_raw_frame call. The array's
 * address is looked up again in a new CUDA context (after a cudaDeviceReset, for example). Async. */
#define FME_STATIC_MAX_CONSOLES 64
#define FME_STATIC_LOG_CAPACITY 2048
int fme_raw_frame_static(FmeRaw* raw, const uint8_t* d_buttons, uint8_t* d_screens, int32_t render,
                         void* stream);

/* ---- helpers ---- */
/* nes-py master palette, 64 x 0xRRGGBB (replaces fm_palette, csrc/fastmario.cpp:637). */
void fme_palette(uint32_t* out64);
/* 240x256 gray -> 84x84 INTER_AREA on the device, n images, async (replaces fm_resize_fast,
 * csrc/fastmario.cpp:643-649, with the same float operation order). */
int fme_resize(const uint8_t* d_src, uint8_t* d_dst, int32_t n, void* stream);
/* ---- PPO trainer data kernels (the network stays in torch) ---- */
/* GAE over a (T, N) rollout, replacing Learner._gae (src/fast_mario_env/ppo/train.py:148-160): fp32 rew, val,
 * done (1 = obs[t] starts a new episode) of shape (T, N), next_val / next_done (N,); writes adv and
 * ret = adv + val (T, N). gamma and gamma_lam = gamma*lam (computed in double, then rounded) as fp32 scalars.
 * Same fp32 operations in the same order as the reference. Async. */
int fme_gae(const float* d_rew, const float* d_val, const float* d_done, const float* d_next_val,
            const float* d_next_done, int32_t T, int32_t N, float gamma, float gamma_lam, float* d_adv, float* d_ret,
            void* stream);
/* Minibatch advantage normalisation of ppo_loss (src/fast_mario_env/ppo/model.py:61-62):
 * out = (in - mean) / (std + 1e-8), unbiased std, n values (in == out allowed). Async. */
int fme_adv_norm(const float* d_in, float* d_out, int32_t n, void* stream);

/* ---- frame-deduplicating replay buffer (replaces FrameReplay's add / sample gathers,
 *      src/fast_mario_env/replay.py:69-139); caller-owned device storage, a ring of `capacity` slots per env ---- */
typedef struct FmeReplayBufs {
    uint8_t* frames;   /* (n_envs, capacity, 84, 84), 16-byte aligned */
    uint8_t* age;      /* (n_envs, capacity) frames since the episode start, saturating at 255 */
    int16_t* act;      /* (n_envs, capacity) */
    float* rew;        /* (n_envs, capacity) */
    uint8_t* flags;    /* (n_envs, capacity) 1 valid start, 2 done, 4 terminal */
    int64_t* ptr;      /* (n_envs,) slots written per env */
    uint8_t* new_ep;   /* (n_envs,) 1 = the next add starts an episode (start at 1) */
    int32_t n_envs;
    int32_t capacity;
} FmeReplayBufs;
/* One transition per env (FrameReplay.add): obs / next_obs (n_envs, k, 84, 84) uint8 (frame k-1 is stored),
 * action int64, reward float32, done / trunc uint8 (n_envs,). Async. */
int fme_replay_add(const FmeReplayBufs* rb, const uint8_t* d_obs, const uint8_t* d_next_obs, int32_t k,
                   const int64_t* d_action, const float* d_reward, const uint8_t* d_done, const uint8_t* d_trunc,
                   void* stream);
/* The batch of FrameReplay.sample for sampled (env, pos) pairs: stacks at pos and pos+m with frames before the
 * episode start zeroed, action, n-step reward, discount gamma^m * (1 - terminal), terminal, m. gpow[i] = gamma^i
 * (i < n_step) and dpow[m] = gamma^m (m <= n_step) as float32 tables. Async. */
int fme_replay_gather(const FmeReplayBufs* rb, const int64_t* d_env, const int64_t* d_pos, int32_t B, int32_t k,
                      int32_t n_step, const float* d_gpow, const float* d_dpow, uint8_t* d_obs, uint8_t* d_next_obs,
                      int64_t* d_act, float* d_reward, float* d_discount, float* d_terminal, int64_t* d_steps,
                      void* stream);

/* Console state size in bytes of the reset-cache image (cf. fm_state_bytes, csrc/fastmario.cpp:631). */
int64_t fme_state_bytes(void);
const char* fme_last_error(void);
const char* fme_version(void);

#ifdef __cplusplus
}
#endif
#endif /* FME_H */
