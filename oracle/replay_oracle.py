"""Test oracle for the replay-buffer kernels (used only by tests/ as the checker, never by the product path).

A numpy restatement of the reference FrameReplay's storage update and batch assembly
(src/fast_mario_env/replay.py:86-104 add, 106-139 stack / n-step return), fed with given (env, slot) pairs.
Pinned by tests/test_replay_oracle.py against tests/golden/replay.npz (made by the reference itself,
tests/golden/make_replay_golden.py).
"""
from __future__ import annotations

import numpy as np


class Ring:
    def __init__(self, C, E, k):
        self.C, self.E, self.k = C, E, k
        self.frames = np.zeros((E, C, 84, 84), np.uint8)
        self.age = np.zeros((E, C), np.uint8)
        self.act = np.zeros((E, C), np.int16)
        self.rew = np.zeros((E, C), np.float32)
        self.flags = np.zeros((E, C), np.uint8)
        self.ptr = np.zeros(E, np.int64)
        self.new_ep = np.ones(E, bool)

    def _put(self, e, frame, age):
        s = self.ptr[e] % self.C
        self.frames[e, s], self.age[e, s], self.flags[e, s] = frame, age, 0
        self.ptr[e] += 1

    def add(self, obs, next_obs, action, reward, done, trunc):
        for e in range(self.E):
            if self.new_ep[e]:
                self._put(e, obs[e, -1], 0)
            s = (self.ptr[e] - 1) % self.C
            self.act[e, s] = np.int16(action[e])
            self.rew[e, s] = np.float32(reward[e])
            d, t = bool(done[e]), bool(trunc[e])
            self.flags[e, s] = 1 | (2 * d) | (4 * (d and not t))
            age = min(int(self.age[e, s]) + 1, 255)
            self._put(e, next_obs[e, -1], age)
            self.new_ep[e] = d

    def stack(self, e, p):
        out = np.zeros((self.k, 84, 84), np.uint8)
        age = int(self.age[e, p % self.C])
        for j in range(self.k):
            back = self.k - 1 - j
            if back <= age:
                out[j] = self.frames[e, (p - back) % self.C]
        return out

    def gather(self, e, p, n_step, gamma):
        f32 = np.float32
        R, alive, term, m = f32(0), f32(1), f32(0), 0
        for i in range(n_step):
            s = (p + i) % self.C
            fl = int(self.flags[e, s])
            R = f32(R + f32(f32(alive * f32(gamma ** i)) * self.rew[e, s]))
            m += int(alive)
            term = max(term, f32(alive * f32(1.0 if fl & 4 else 0.0)))
            alive = f32(alive * f32(0.0 if fl & 2 else 1.0))
        disc = f32(np.float64(gamma) ** np.float64(m)) * f32(f32(1) - term)
        return dict(action=int(self.act[e, p % self.C]), reward=R, discount=f32(disc), terminal=term, steps=m,
                    obs=self.stack(e, p), next_obs=self.stack(e, p + m))
