"""GPU parity: the B200 engine against the reference's own C++ core (oracle/_ref) and the golden fixtures.

Everything is bit-exact: RAM and palette-value screens per frame (config 0), and per agent step the stacked
observations, rewards, terminated/truncated, infos, RAM, final_obs and episode statistics (config 1 at small N).
The comparison pattern is the reference's tests/test_cuda.py:22-59 (GPU vs CPU in lockstep)."""
import os
import zlib

import numpy as np
import pytest
from conftest import fme, scaled

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def crc(a):
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def test_raw_frames_config0_golden(rom):
    """8 consoles, 1000 frames, random joypad bytes, RAM and screen every frame."""
    import make_golden as mg
    g = np.load(os.path.join(GOLD, "raw_seed0.npz"))
    btn = mg.raw_buttons()
    b = fme.RawNESBatch(rom, mg.RAW_N)
    for f in range(mg.RAW_FRAMES):
        b.frame(btn[f], True)
        ram = b.ram().cpu().numpy()
        scr = b.screen().cpu().numpy()
        for i in range(mg.RAW_N):
            assert crc(ram[i]) == g["ram_crc"][f, i], f"RAM frame {f} console {i}"
            assert crc(scr[i]) == g["scr_crc"][f, i], f"screen frame {f} console {i}"
    assert np.array_equal(ram, g["last_ram"]) and np.array_equal(scr, g["last_scr"])
    b.check()
    assert b.bad_ops() == 0


def test_raw_frames_vs_oracle_with_backup_restore(oracle, rom_div):
    """Random render flags and random backup/restore on both sides (the reference's test_fidelity_raw pattern)."""
    n = 4
    b = fme.RawNESBatch(rom_div, n)
    refs = [oracle.RefRaw(rom_div) for _ in range(n)]
    rng = np.random.default_rng(1)
    have = False
    for f in range(scaled(600)):
        btn = rng.integers(0, 256, n).astype(np.uint8)
        render = bool(rng.random() < 0.5)
        u = rng.random()
        if u < 0.01:
            b.backup(); [r.backup() for r in refs]; have = True
        elif u < 0.02 and have:
            b.restore(); [r.restore() for r in refs]
        b.frame(btn, render)
        for r, x in zip(refs, btn):
            r.frame(int(x), render)
        ram = b.ram().cpu().numpy()
        for i, r in enumerate(refs):
            assert np.array_equal(ram[i], r.ram), (f, i)
        if render:
            scr = b.screen().cpu().numpy()
            for i, r in enumerate(refs):
                assert np.array_equal(scr[i], r.screen), (f, i)


def test_env_config1_golden(rom):
    import make_golden as mg
    g = np.load(os.path.join(GOLD, "env_seed0.npz"))
    kw = dict(mg.ENV_KW)
    levels = [f"{w}-{s}" for (w, s, a) in mg.env_levels()]
    e = fme.CudaVecEnv(levels, mg.ENV_N, rom=rom, **kw)
    o = e.reset().cpu().numpy()
    assert [crc(o[i]) for i in range(mg.ENV_N)] == list(g["reset_crc"])
    acts = mg.env_actions()
    import torch
    for t in range(mg.ENV_STEPS):
        o, r, te, tr, info = e.step(torch.from_numpy(acts[t]).cuda())
        o = o.cpu().numpy()
        assert [crc(o[i]) for i in range(mg.ENV_N)] == list(g["obs_crc"][t]), t
        assert np.array_equal(r.cpu().numpy(), g["rew"][t]), t
        assert np.array_equal(te.cpu().numpy(), g["term"][t]) and np.array_equal(tr.cpu().numpy(), g["trunc"][t]), t
        assert np.array_equal(e.info_t.cpu().numpy().astype(np.int64), g["info"][t]), t
        done = g["term"][t] | g["trunc"][t]
        if done.any():
            fin, epr, epl = e.final_obs.cpu().numpy(), e.ep_ret.cpu().numpy(), e.ep_len.cpu().numpy()
            for i in np.flatnonzero(done):
                assert crc(fin[i]) == g["fin_crc"][t, i] and epr[i] == g["ep_ret"][t, i] and epl[i] == g["ep_len"][t, i]
    assert np.array_equal(o, g["last_obs"])
    assert e.frames == int(g["frames"])
    e.check()


CONFIGS = {
    "default": dict(levels=["1-1"] * 8, n=8, kw=dict()),
    "config1": dict(levels=["1-1", "1-2", "4-1", "8-4"] * 4, n=16, kw=dict(sticky=0.25, noop_max=30, maxpool=True)),
    "short_timelimit": dict(levels=["2-3", "5-2"] * 8, n=16, kw=dict(sticky=0.25, noop_max=5, max_steps=40, maxpool=True)),
    "skip3_stack2": dict(levels=["3-4"] * 8, n=8, kw=dict(skip=3, frame_stack=2, noop_max=10)),
    "skip1_stack1_pool": dict(levels=["7-4"] * 8, n=8, kw=dict(skip=1, frame_stack=1, maxpool=True, sticky=0.5)),
    "skip6_divergent": dict(levels=["1-1", "6-3"] * 20, n=40, kw=dict(skip=6, sticky=0.25, noop_max=30, maxpool=True),
                            div=True),
    # 5 groups of 32 (the last ragged) in 4 step slices of uneven size
    "sliced_150": dict(levels=["1-1", "3-2", "5-4", "8-1", "2-2"] * 30, n=150,
                       kw=dict(sticky=0.25, noop_max=30, maxpool=True, max_steps=90)),
    # four `JMP *` loops, envs parked in different ones from frame to frame: the scheduler's vote knows only
    # the first two by address; which lanes it groups must not change any result
    "four_idle_loops": dict(levels=["1-1", "4-2", "6-3", "8-4"] * 16, n=64,
                            kw=dict(sticky=0.25, noop_max=30, maxpool=True), rom_kw=dict(idle_loops=4)),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_env_lockstep_vs_oracle(oracle, rom, rom_div, name):
    import torch
    c = CONFIGS[name]
    romb = rom_div if c.get("div") else rom
    if "rom_kw" in c:
        from fast_mario_env_b200.synth_rom import build_rom
        romb = build_rom(0, **c["rom_kw"])
    n, kw = c["n"], c["kw"]
    lv3 = [fme.decode_level(x) for x in c["levels"]]
    ref_env = oracle.RefVecEnv(romb, lv3, n, seed=7, **kw)
    new = fme.CudaVecEnv(c["levels"], n, seed=7, rom=romb, **kw)
    assert np.array_equal(ref_env.reset(), new.reset().cpu().numpy())
    rng = np.random.default_rng(130)
    eps = 0
    for t in range(scaled(250)):
        a = rng.choice(7, n, p=[.05, .2, .25, .15, .25, .05, .05])
        o1, r1, te1, tr1, i1 = ref_env.step(a)
        o2, r2, te2, tr2, _ = new.step(torch.from_numpy(a).cuda())
        assert np.array_equal(o1, o2.cpu().numpy()), t
        assert np.array_equal(r1, r2.cpu().numpy()), t
        assert np.array_equal(te1, te2.cpu().numpy()) and np.array_equal(tr1, tr2.cpu().numpy()), t
        assert np.array_equal(i1.astype(np.int32), new.info_t.cpu().numpy()), t
        ram = new.ram().cpu().numpy()
        for i in range(n):
            assert np.array_equal(ref_env.ram(i), ram[i]), (t, i)
        done = te1 | tr1
        if done.any():
            fin, epr, epl = new.final_obs.cpu().numpy(), new.ep_ret.cpu().numpy(), new.ep_len.cpu().numpy()
            for i in np.flatnonzero(done):
                eps += 1
                assert np.array_equal(ref_env.fin[i], fin[i]), (t, i)
                assert ref_env.ep_ret[i] == epr[i] and ref_env.ep_len[i] == epl[i], (t, i)
    assert new.frames == ref_env.frames
    assert new.bad_ops() == ref_env.bad_ops() == 0
    new.check()
    if name == "short_timelimit":
        assert eps > 0
