// fme_ppo.cuh - the two PPO data kernels of the trainer hot loop: GAE over a rollout and the per-minibatch
// advantage normalisation. The network itself (Nature-CNN forward/backward, Adam) stays in torch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fme {

// Generalised advantage estimation of the reference trainer (ppo/train.py:148-160, Learner._gae): for every
// env a backward pass over t = T-1..0 with
//   nnt = 1 - done[t+1] (next_done at T-1),  nv = val[t+1] (next_val at T-1)
//   delta = rew[t] + gamma*nv*nnt - val[t],  last = delta + (gamma*lam)*nnt*last,  adv[t] = last
// and ret = adv + val. Every fp32 operation is a separate rounding in the reference's order (the torch ops of
// the reference are elementwise kernels); the library is built with --fmad=false, and the intrinsics below
// make the order explicit. Layout (T, N) row-major; one thread per env, so each t is a coalesced row.
__global__ void k_gae(const float* __restrict__ rew, const float* __restrict__ val, const float* __restrict__ done,
                      const float* __restrict__ next_val, const float* __restrict__ next_done, int T, int N,
                      float gamma, float gl, float* __restrict__ adv, float* __restrict__ ret) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= N) return;
    float last = 0.f;
    for (int t = T - 1; t >= 0; t--) {
        const size_t i = (size_t)t * N + e;
        const bool tail = t == T - 1;
        const float nnt = __fsub_rn(1.0f, tail ? next_done[e] : done[i + N]);
        const float nv = tail ? next_val[e] : val[i + N];
        const float v = val[i];
        const float delta = __fsub_rn(__fadd_rn(rew[i], __fmul_rn(__fmul_rn(gamma, nv), nnt)), v);
        last = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nnt), last));
        adv[i] = last;
        ret[i] = __fadd_rn(last, v);
    }
}

// Per-minibatch advantage normalisation of the reference loss (ppo/model.py:61-62):
// out = (a - mean(a)) / (std(a) + 1e-8), std with Bessel's correction. One CTA; the sums are accumulated in
// fp64 and the mean and std rounded to fp32 before the fp32 elementwise step, as the reference applies fp32
// mean/std tensors.
constexpr int ADV_THREADS = 256;
__global__ void __launch_bounds__(ADV_THREADS) k_adv_norm(const float* __restrict__ in, float* __restrict__ out, int n) {
    __shared__ double red[ADV_THREADS / 32];
    __shared__ float stat[2];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    double s = 0.0;
    for (int i = tid; i < n; i += ADV_THREADS) s += (double)in[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[wid] = s;
    __syncthreads();
    if (tid == 0) {
        double t = 0.0;
        for (int k = 0; k < ADV_THREADS / 32; k++) t += red[k];
        stat[0] = (float)(t / (double)n);
    }
    __syncthreads();
    const double mean = (double)stat[0];
    double q = 0.0;
    for (int i = tid; i < n; i += ADV_THREADS) { const double d = (double)in[i] - mean; q += d * d; }
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    __syncthreads();
    if (lane == 0) red[wid] = q;
    __syncthreads();
    if (tid == 0) {
        double t = 0.0;
        for (int k = 0; k < ADV_THREADS / 32; k++) t += red[k];
        stat[1] = (float)sqrt(n > 1 ? t / (double)(n - 1) : 0.0);
    }
    __syncthreads();
    const float m = stat[0], den = __fadd_rn(stat[1], 1e-8f);
    for (int i = tid; i < n; i += ADV_THREADS) out[i] = __fdiv_rn(__fsub_rn(in[i], m), den);
}

}  // namespace fme
