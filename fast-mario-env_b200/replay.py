"""Frame-deduplicating replay buffer on the GPU (the reference's FrameReplay, src/fast_mario_env/replay.py:43-145).

Each env keeps a ring of `capacity_per_env` 84x84 frames plus per-slot age / action / reward / flags; stacks are
rebuilt at sample time from the k most recent slots with the frames before the episode start zeroed, exactly the
zero-padded reset stacks of the env. The two data-moving steps are library kernels (`fme_replay_add`: one
warp per env stores its newest frame(s); `fme_replay_gather`: one warp per sampled transition computes the
n-step return and writes both stacks); the rejection sampling of (env, slot) pairs keeps the reference's torch
calls, so with the same generator seed on the same device it draws the same batch.

    rb = FrameReplay(capacity_per_env, n_envs, k=4)
    rb.add(obs, next_obs, actions, rewards, dones, truncated)   # (N, k, 84, 84) uint8 CUDA tensors or arrays
    s = rb.sample(256, n_step=3, gamma=0.99)
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import numpy as np
import torch as th

from . import _native as N


class Batch(NamedTuple):
    obs: th.Tensor        # (B, k, H, W) uint8
    action: th.Tensor     # (B,) int64
    reward: th.Tensor     # (B,) float32, n-step discounted sum
    next_obs: th.Tensor   # (B, k, H, W) uint8 (state after m <= n steps)
    discount: th.Tensor   # (B,) float32 = gamma^m * (1 - terminal)
    terminal: th.Tensor   # (B,) float32
    steps: th.Tensor      # (B,) int64 m
    env: th.Tensor        # (B,) env index
    pos: th.Tensor        # (B,) absolute slot index


class FrameReplay:
    def __init__(self, capacity_per_env: int, n_envs: int, k: int = 4, hw=(84, 84), device="cuda", seed=None):
        if tuple(hw) != (84, 84):
            raise ValueError("FrameReplay stores 84x84 frames")
        self.C, self.E, self.k, self.hw = int(capacity_per_env), int(n_envs), int(k), tuple(hw)
        self.dev = th.device(device)
        if self.dev.type != "cuda":
            raise ValueError("FrameReplay runs on a CUDA device (there is no CPU path)")
        E, C, d = self.E, self.C, self.dev
        self.frames = th.zeros((E, C, *self.hw), dtype=th.uint8, device=d)
        self.age = th.zeros((E, C), dtype=th.uint8, device=d)
        self.act = th.zeros((E, C), dtype=th.int16, device=d)
        self.rew = th.zeros((E, C), dtype=th.float32, device=d)
        self.flags = th.zeros((E, C), dtype=th.uint8, device=d)
        self.ptr = th.zeros(E, dtype=th.int64, device=d)
        self.new_ep = th.ones(E, dtype=th.uint8, device=d)
        self.g = th.Generator(device=d)
        self.g.manual_seed(int(np.random.SeedSequence(seed).generate_state(1)[0]))
        self.n_transitions = 0
        self._rb = N.FmeReplayBufs(*[t.data_ptr() for t in (self.frames, self.age, self.act, self.rew, self.flags,
                                                             self.ptr, self.new_ep)], E, C)

    def _stream(self):
        return ctypes.c_void_p(th.cuda.current_stream(self.dev).cuda_stream)

    def _t(self, x, dtype):
        if isinstance(x, th.Tensor):
            return x.to(self.dev, dtype=dtype).contiguous()
        return th.as_tensor(np.ascontiguousarray(x), device=self.dev, dtype=dtype)

    def add(self, obs, next_obs, action, reward, done, truncated=None):
        """obs / next_obs: (N, k, H, W) stacks (next_obs = the terminal stack for done envs);
        done = terminated | truncated; truncated marks time-limit ends."""
        o = self._t(obs, th.uint8)
        no = self._t(next_obs, th.uint8)
        a = self._t(action, th.int64).reshape(-1)
        r = self._t(reward, th.float32).reshape(-1)
        dn = self._t(done, th.bool).reshape(-1).to(th.uint8)
        tr = th.zeros_like(dn) if truncated is None else self._t(truncated, th.bool).reshape(-1).to(th.uint8)
        N.check(N.lib().fme_replay_add(ctypes.byref(self._rb), N.ptr(o), N.ptr(no), self.k, N.ptr(a), N.ptr(r),
                                       N.ptr(dn), N.ptr(tr), self._stream()), "fme_replay_add")
        self.n_transitions += self.E

    def size(self):
        return int(min(self.n_transitions, self.E * self.C))

    def gather(self, e, p, n_step: int = 1, gamma: float = 0.99) -> Batch:
        """The batch for given (env, absolute slot) pairs (int64 CUDA tensors)."""
        B, k, d = int(e.numel()), self.k, self.dev
        gpow = th.tensor([gamma ** i for i in range(n_step)], dtype=th.float32, device=d)
        dpow = (th.tensor(gamma, dtype=th.float64) ** th.arange(n_step + 1, dtype=th.float64)).float().to(d)
        obs = th.empty((B, k, *self.hw), dtype=th.uint8, device=d)
        nobs = th.empty_like(obs)
        act = th.empty(B, dtype=th.int64, device=d)
        R, disc, term = (th.empty(B, dtype=th.float32, device=d) for _ in range(3))
        m = th.empty(B, dtype=th.int64, device=d)
        e, p = e.contiguous(), p.contiguous()
        N.check(N.lib().fme_replay_gather(ctypes.byref(self._rb), N.ptr(e), N.ptr(p), B, k, n_step, N.ptr(gpow),
                                          N.ptr(dpow), N.ptr(obs), N.ptr(nobs), N.ptr(act), N.ptr(R), N.ptr(disc),
                                          N.ptr(term), N.ptr(m), self._stream()), "fme_replay_gather")
        return Batch(obs, act, R, nobs, disc, term, m, e, p)

    def sample(self, batch: int, n_step: int = 1, gamma: float = 0.99) -> Batch:
        """Uniform over the stored transitions whose n-step window and stack lookback stay inside the live
        ring, by rejection of slots that do not start a transition (replay.py:112-127)."""
        B, C, k, d = batch, self.C, self.k, self.dev
        lo = th.clamp(self.ptr - C + k - 1, min=0)
        hi = self.ptr - 1 - n_step
        ok_env = th.nonzero(hi >= lo).flatten()
        if len(ok_env) == 0:
            raise ValueError("not enough data in buffer")
        e = th.empty(B, dtype=th.long, device=d)
        p = th.empty(B, dtype=th.long, device=d)
        todo = th.arange(B, device=d)
        for _ in range(64):
            n = len(todo)
            ee = ok_env[th.randint(len(ok_env), (n,), device=d, generator=self.g)]
            span = (hi[ee] - lo[ee] + 1).double()
            pp = lo[ee] + (th.rand(n, device=d, generator=self.g, dtype=th.float64) * span).long()
            good = (self.flags[ee, pp % C] & 1).bool()
            e[todo[good]], p[todo[good]] = ee[good], pp[good]
            todo = todo[~good]
            if len(todo) == 0:
                break
        else:
            raise RuntimeError("sampling failed")
        return self.gather(e, p, n_step, gamma)

    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in (self.frames, self.age, self.act, self.rew, self.flags))
