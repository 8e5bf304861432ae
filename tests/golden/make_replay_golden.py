"""Generate tests/golden/replay.npz from the reference's own FrameReplay (CPU).

    python tests/golden/make_replay_golden.py        # needs the reference installed in baseline/_ref

A ring of C=48 slots for E=4 envs, k=4, filled by ADDS transitions whose frames, actions, rewards and episode
ends come from numpy default_rng(INPUT_SEED) (inputs() regenerates them). Saved: the storage after the adds
(age, flags, actions, rewards, slot pointers, and a crc32 of every stored frame) and one sample(32, n_step=3,
gamma=0.99) with the generator seeded from SAMPLE_SEED: per sample env, pos, action, reward, discount, terminal,
steps and crc32s of both stacks.
"""
from __future__ import annotations

import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))

E, C, K, ADDS, INPUT_SEED, SAMPLE_SEED, B, NSTEP, GAMMA = 4, 48, 4, 120, 11, 123, 32, 3, 0.99


def crc(a) -> int:
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def inputs():
    """Per add: obs, next_obs (E, K, 84, 84) uint8, action, reward, done, truncated. A continuing env's obs is
    its previous next_obs; an env whose episode ended starts from a fresh stack (zeros + one frame)."""
    r = np.random.default_rng(INPUT_SEED)
    cur = np.zeros((E, K, 84, 84), np.uint8)
    cur[:, -1] = r.integers(0, 256, (E, 84, 84), dtype=np.uint8)
    out = []
    for _ in range(ADDS):
        nxt = np.concatenate([cur[:, 1:], r.integers(0, 256, (E, 1, 84, 84), dtype=np.uint8)], axis=1)
        act = r.integers(0, 7, E)
        rew = r.normal(0, 1, E).astype(np.float32)
        done = r.random(E) < 0.06
        trunc = done & (r.random(E) < 0.3)
        out.append((cur.copy(), nxt, act, rew, done, trunc))
        cur = nxt.copy()
        for i in np.flatnonzero(done):
            cur[i] = 0
            cur[i, -1] = r.integers(0, 256, (84, 84), dtype=np.uint8)
    return out


def main():
    import torch as th
    from fast_mario_env.replay import FrameReplay
    rb = FrameReplay(C, E, k=K, device="cpu", seed=SAMPLE_SEED)
    for obs, nxt, act, rew, done, trunc in inputs():
        rb.add(obs, nxt, act, rew, done, trunc)
    s = rb.sample(B, n_step=NSTEP, gamma=GAMMA)
    out = dict(age=rb.age.numpy(), flags=rb.flags.numpy(), act=rb.act.numpy(), rew=rb.rew.numpy(), ptr=rb.ptr.copy(),
               frame_crc=np.array([[crc(rb.frames[e, c].numpy()) for c in range(C)] for e in range(E)], np.int64),
               s_env=s.env.numpy(), s_pos=s.pos.numpy(), s_action=s.action.numpy(), s_reward=s.reward.numpy(),
               s_discount=s.discount.numpy(), s_terminal=s.terminal.numpy(), s_steps=s.steps.numpy(),
               s_obs_crc=np.array([crc(s.obs[b].numpy()) for b in range(B)], np.int64),
               s_next_crc=np.array([crc(s.next_obs[b].numpy()) for b in range(B)], np.int64))
    np.savez_compressed(os.path.join(HERE, "replay.npz"), **out)
    print("wrote replay.npz; terminal samples", int(s.terminal.sum()), "steps", np.bincount(s.steps.numpy()))


if __name__ == "__main__":
    main()
