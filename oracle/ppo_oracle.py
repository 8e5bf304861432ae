"""Test oracle for the PPO data kernels (used only by tests/ as the checker, never by the product path).

Plain numpy float32 restatements of the reference trainer's arithmetic:
  * gae          src/fast_mario_env/ppo/train.py:148-160 (Learner._gae): one backward pass over t with every
                 fp32 operation rounded separately, in the reference's order.
  * adv_norm     src/fast_mario_env/ppo/model.py:61-62: (a - mean) / (std + 1e-8), unbiased std.
Pinned by tests/test_ppo_oracle.py against tests/golden/ppo.npz, generated from the reference's own code by
tests/golden/make_ppo_golden.py.
"""
from __future__ import annotations

import numpy as np


def gae(rew, val, done, next_val, next_done, gamma, lam):
    f = np.float32
    rew, val, done = (np.asarray(x, f) for x in (rew, val, done))
    next_val, next_done = np.asarray(next_val, f), np.asarray(next_done, f)
    T = rew.shape[0]
    g, gl = f(gamma), f(gamma * lam)  # python-float scalars meet fp32 tensors as fp32
    adv = np.zeros_like(rew)
    last = np.zeros_like(next_val)
    for t in range(T - 1, -1, -1):
        if t == T - 1:
            nnt, nv = f(1.0) - next_done, next_val
        else:
            nnt, nv = f(1.0) - done[t + 1], val[t + 1]
        delta = (rew[t] + (g * nv) * nnt) - val[t]
        last = delta + (gl * nnt) * last
        adv[t] = last
    return adv, adv + val


def adv_norm(a):
    a = np.asarray(a, np.float32)
    m = np.float32(a.astype(np.float64).mean())
    s = np.float32(a.astype(np.float64).std(ddof=1))
    return (a - m) / (s + np.float32(1e-8))
