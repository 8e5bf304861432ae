"""Generate the golden fixtures from the reference's own C++ core (oracle/_ref/libfastmario.so).

    make -C oracle ref && python tests/golden/make_golden.py

Fixtures (small .npz files committed next to this script):
  raw_seed0.npz   BASELINE config 0: 8 consoles on the synthetic NROM (seed 0), 1000 frames, uniform random joypad
                  bytes (numpy default_rng(2024)), render every frame. crc32 of the 2 KB RAM and of the 240x256
                  palette-value screen per console per frame, plus the full RAM and screen of the last frame.
  env_seed0.npz   the config 1 wrapper stack at small N: 16 envs over 4 levels, sticky 0.25, noop_max 30,
                  maxpool, max_steps 120, skip 4, frame_stack 4, 200 steps of uniform random actions
                  (default_rng(7)). Per step: crc32 of each env's stacked obs, rewards, term, trunc, info (int64),
                  and per episode end crc32 of final_obs, ep_ret, ep_len; the reset obs crc; total frames.
  resize.npz      cv2-verified INTER_AREA pairs: 8 random / blocky 240x256 images and their 84x84 resize.
"""
from __future__ import annotations

import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "fast-mario-env_b200"))

import ref  # noqa: E402
import synth_rom  # noqa: E402

RAW_N, RAW_FRAMES, RAW_SEED = 8, 1000, 2024
ENV_LEVELS = [(1, 1, 1), (4, 2, 3), (8, 4, 4), (2, 3, 4)]
ENV_N, ENV_STEPS, ENV_ACT_SEED = 16, 200, 7
ENV_KW = dict(seed=0, sticky=0.25, noop_max=30, maxpool=True, max_steps=120, skip=4, frame_stack=4)


def crc(a) -> int:
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def raw_buttons():
    return np.random.default_rng(RAW_SEED).integers(0, 256, (RAW_FRAMES, RAW_N)).astype(np.uint8)


def make_raw(rom: bytes):
    btn = raw_buttons()
    cons = [ref.RefRaw(rom) for _ in range(RAW_N)]
    ram_crc = np.zeros((RAW_FRAMES, RAW_N), np.uint32)
    scr_crc = np.zeros((RAW_FRAMES, RAW_N), np.uint32)
    for f in range(RAW_FRAMES):
        for i, c in enumerate(cons):
            c.frame(int(btn[f, i]), True)
            ram_crc[f, i] = crc(c.ram)
            scr_crc[f, i] = crc(c.screen)
    last_ram = np.stack([c.ram.copy() for c in cons])
    last_scr = np.stack([c.screen.copy() for c in cons])
    assert all(c.bad_ops() == 0 for c in cons)
    return dict(ram_crc=ram_crc, scr_crc=scr_crc, last_ram=last_ram, last_scr=last_scr)


def env_levels():
    return [ENV_LEVELS[i % len(ENV_LEVELS)] for i in range(ENV_N)]


def env_actions():
    return np.random.default_rng(ENV_ACT_SEED).integers(0, 7, (ENV_STEPS, ENV_N)).astype(np.int64)


def make_env(rom: bytes):
    e = ref.RefVecEnv(rom, env_levels(), ENV_N, **ENV_KW)
    obs0 = e.reset().copy()
    acts = env_actions()
    obs_crc = np.zeros((ENV_STEPS, ENV_N), np.uint32)
    rew = np.zeros((ENV_STEPS, ENV_N), np.float32)
    term = np.zeros((ENV_STEPS, ENV_N), bool)
    trunc = np.zeros((ENV_STEPS, ENV_N), bool)
    info = np.zeros((ENV_STEPS, ENV_N, 10), np.int64)
    fin_crc = np.zeros((ENV_STEPS, ENV_N), np.uint32)
    ep_ret = np.zeros((ENV_STEPS, ENV_N), np.float64)
    ep_len = np.zeros((ENV_STEPS, ENV_N), np.int64)
    for t in range(ENV_STEPS):
        o, r, te, tr, inf = e.step(acts[t])
        for i in range(ENV_N):
            obs_crc[t, i] = crc(o[i])
        rew[t], term[t], trunc[t], info[t] = r, te, tr, inf
        for i in np.flatnonzero(te | tr):
            fin_crc[t, i] = crc(e.fin[i])
            ep_ret[t, i] = e.ep_ret[i]
            ep_len[t, i] = e.ep_len[i]
    frames = e.frames
    assert e.bad_ops() == 0
    return dict(reset_crc=np.array([crc(obs0[i]) for i in range(ENV_N)], np.uint32), obs_crc=obs_crc, rew=rew,
                term=term, trunc=trunc, info=info, fin_crc=fin_crc, ep_ret=ep_ret, ep_len=ep_len,
                frames=np.array(frames, np.int64), last_obs=e.obs.copy())


def make_resize():
    import cv2
    rng = np.random.default_rng(11)
    lut = ref.gray_lut()
    imgs = []
    for t in range(8):
        if t % 2:
            img = rng.integers(0, 256, (240, 256), np.uint8)
        else:
            img = lut[rng.integers(0, 64, (30, 32))].repeat(8, 0).repeat(8, 1)
            img = np.roll(img, rng.integers(0, 8, 2), (0, 1)).copy()
        imgs.append(img)
    imgs = np.stack(imgs)
    outs = np.stack([cv2.resize(im, (84, 84), interpolation=cv2.INTER_AREA) for im in imgs])
    for im, o in zip(imgs, outs):
        assert np.array_equal(ref.resize_ref(im), o)
    return dict(src=imgs, dst=outs)


def main():
    rom = synth_rom.build_rom(0)
    np.savez_compressed(os.path.join(HERE, "raw_seed0.npz"), **make_raw(rom))
    np.savez_compressed(os.path.join(HERE, "env_seed0.npz"), **make_env(rom))
    np.savez_compressed(os.path.join(HERE, "resize.npz"), **make_resize())
    np.savez_compressed(os.path.join(HERE, "rom_seed0.npz"), crc=np.array(crc(np.frombuffer(rom, np.uint8)), np.uint32),
                        crc_div=np.array(crc(np.frombuffer(synth_rom.build_rom(0, divergence=True), np.uint8)), np.uint32))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
