// fme_replay.cuh - device side of the frame-deduplicating replay buffer: the per-step write of every env's
// newest frame(s) and the batched stack gather with n-step returns. Semantics of the reference FrameReplay
// (src/fast_mario_env/replay.py:69-139); the storage layout (E, C) ring per env is kept so batches are the same.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fme {

constexpr int RP_FRAME = 84 * 84;  // bytes per stored frame (16-byte multiple: 441 x 16)

struct ReplayDev {
    uint8_t* frames;   // (E, C, 84, 84)
    uint8_t* age;      // (E, C) frames since the episode start, saturating at 255
    int16_t* act;      // (E, C)
    float* rew;        // (E, C)
    uint8_t* flags;    // (E, C) 1 valid start, 2 done, 4 terminal
    int64_t* ptr;      // (E,) slots written per env (absolute)
    uint8_t* new_ep;   // (E,) the next add starts an episode
    int E, C;
};

__device__ __forceinline__ void rp_copy_frame(uint8_t* dst, const uint8_t* src, int lane) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = lane; i < RP_FRAME / 16; i += 32) d[i] = s[i];
}

// One warp per env (replay.py:86-104, add): a new episode first stores the newest frame of obs with age 0;
// then the transition's action, reward and flags go to the newest slot, and the newest frame of next_obs is
// stored with age + 1 (saturating); new_ep becomes done. obs / next_obs: (E, k, 84, 84), frame k-1 used.
__global__ void __launch_bounds__(32) k_replay_add(ReplayDev R, const uint8_t* __restrict__ obs,
                                                   const uint8_t* __restrict__ next_obs, const int64_t* __restrict__ action,
                                                   const float* __restrict__ reward, const uint8_t* __restrict__ done,
                                                   const uint8_t* __restrict__ trunc, int k) {
    const int e = blockIdx.x, lane = threadIdx.x;
    if (e >= R.E) return;
    int64_t p = R.ptr[e];
    const size_t row = (size_t)e * R.C;
    if (R.new_ep[e]) {
        const int s = (int)(p % R.C);
        rp_copy_frame(R.frames + (row + s) * RP_FRAME, obs + ((size_t)e * k + (k - 1)) * RP_FRAME, lane);
        if (lane == 0) { R.age[row + s] = 0; R.flags[row + s] = 0; }
        p++;
    }
    const int cur = (int)((p - 1) % R.C);
    const uint32_t d = done[e] ? 1u : 0u, tr = trunc[e] ? 1u : 0u;
    const int s2 = (int)(p % R.C);
    __syncwarp();
    uint32_t nage = 0;
    if (lane == 0) {
        nage = (uint32_t)R.age[row + cur] + 1u;   // lane 0 wrote the start slot's age itself
        R.act[row + cur] = (int16_t)action[e];
        R.rew[row + cur] = reward[e];
        R.flags[row + cur] = (uint8_t)(1u | (2u * d) | (4u * (d & (tr ^ 1u))));
    }
    rp_copy_frame(R.frames + (row + s2) * RP_FRAME, next_obs + ((size_t)e * k + (k - 1)) * RP_FRAME, lane);
    if (lane == 0) {
        R.age[row + s2] = (uint8_t)(nage > 255u ? 255u : nage);
        R.flags[row + s2] = 0;
        R.ptr[e] = p + 1;
        R.new_ep[e] = (uint8_t)d;
    }
}

// One warp per sampled transition (replay.py:112-139): the n-step discounted reward, step count and terminal
// flag walking the ring from slot p, then the stacks at p and p+m: the k most recent frames, those before the
// episode start (more frames back than the slot's age) zeroed. gpow[i] = gamma^i as the reference computes it
// for the reward (python float power) and dpow[m] = float(gamma^m in float64) for the discount.
__global__ void __launch_bounds__(32) k_replay_gather(ReplayDev R, const int64_t* __restrict__ env,
                                                      const int64_t* __restrict__ pos, int B, int k, int n_step,
                                                      const float* __restrict__ gpow, const float* __restrict__ dpow,
                                                      uint8_t* __restrict__ obs, uint8_t* __restrict__ next_obs,
                                                      int64_t* __restrict__ act, float* __restrict__ reward,
                                                      float* __restrict__ discount, float* __restrict__ terminal,
                                                      int64_t* __restrict__ steps) {
    const int b = blockIdx.x, lane = threadIdx.x;
    if (b >= B) return;
    const int64_t e = env[b], p = pos[b];
    const size_t row = (size_t)e * R.C;
    float Rs = 0.f, alive = 1.f, term = 0.f;
    int m = 0;
    for (int i = 0; i < n_step; i++) {
        const int s = (int)((p + i) % R.C);
        const uint32_t f = R.flags[row + s];
        Rs = __fadd_rn(Rs, __fmul_rn(__fmul_rn(alive, gpow[i]), R.rew[row + s]));
        m += alive != 0.f ? 1 : 0;
        const float tv = __fmul_rn(alive, (f & 4u) ? 1.f : 0.f);
        term = term > tv ? term : tv;
        alive = __fmul_rn(alive, (f & 2u) ? 0.f : 1.f);
    }
    if (lane == 0) {
        act[b] = (int64_t)R.act[row + (int)(p % R.C)];
        reward[b] = Rs;
        terminal[b] = term;
        discount[b] = __fmul_rn(dpow[m], __fsub_rn(1.f, term));
        steps[b] = m;
    }
    for (int which = 0; which < 2; which++) {
        const int64_t q = which == 0 ? p : p + m;
        const int age = (int)R.age[row + (int)(q % R.C)];
        uint8_t* out = (which == 0 ? obs : next_obs) + (size_t)b * k * RP_FRAME;
        for (int j = 0; j < k; j++) {                       // stack position j is (k-1-j) frames back
            const int back = k - 1 - j;
            uint4* d = reinterpret_cast<uint4*>(out + (size_t)j * RP_FRAME);
            if (back <= age) {
                const int s = (int)(((q - back) % R.C + R.C) % R.C);
                const uint4* src = reinterpret_cast<const uint4*>(R.frames + (row + s) * RP_FRAME);
                for (int i = lane; i < RP_FRAME / 16; i += 32) d[i] = src[i];
            } else {
                for (int i = lane; i < RP_FRAME / 16; i += 32) d[i] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
}

}  // namespace fme
