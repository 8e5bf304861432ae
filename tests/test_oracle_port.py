"""The plain-C restatement oracle (oracle/fme_oracle.c) is pinned against the golden fixtures and against the
reference's own build in lockstep (CPU only)."""
import os
import zlib

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def port():
    import port as p
    if not p.available():
        pytest.skip("oracle/_ref/libfme_oracle.so not built (make -C oracle port)")
    return p


def crc(a):
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def test_port_raw_matches_golden(port, rom):
    import make_golden as mg
    g = np.load(os.path.join(GOLD, "raw_seed0.npz"))
    btn = mg.raw_buttons()
    cons = [port.PortRaw(rom) for _ in range(mg.RAW_N)]
    for f in range(mg.RAW_FRAMES):
        for i, c in enumerate(cons):
            c.frame(int(btn[f, i]), True)
            assert crc(c.ram) == g["ram_crc"][f, i], (f, i)
            assert crc(c.screen) == g["scr_crc"][f, i], (f, i)
    assert all(c.bad_ops() == 0 for c in cons)


def test_port_raw_lockstep_with_backup_restore(port, oracle, rom_div):
    a, b = port.PortRaw(rom_div), oracle.RefRaw(rom_div)
    rng = np.random.default_rng(5)
    have = False
    for f in range(1500):
        btn, render, u = int(rng.integers(0, 256)), bool(rng.random() < 0.3), rng.random()
        if u < 0.005:
            a.backup(); b.backup(); have = True
        elif u < 0.01 and have:
            a.restore(); b.restore()
        a.frame(btn, render); b.frame(btn, render)
        assert np.array_equal(a.ram, b.ram), f
        if render:
            assert np.array_equal(a.screen, b.screen), f


def test_port_env_matches_golden(port, rom):
    import make_golden as mg
    g = np.load(os.path.join(GOLD, "env_seed0.npz"))
    e = port.PortVecEnv(rom, mg.env_levels(), mg.ENV_N, **mg.ENV_KW)
    o = e.reset()
    assert [crc(o[i]) for i in range(mg.ENV_N)] == list(g["reset_crc"])
    acts = mg.env_actions()
    for t in range(mg.ENV_STEPS):
        o, r, te, tr, inf = e.step(acts[t])
        assert [crc(o[i]) for i in range(mg.ENV_N)] == list(g["obs_crc"][t]), t
        assert np.array_equal(r, g["rew"][t]) and np.array_equal(te, g["term"][t]) and np.array_equal(tr, g["trunc"][t])
        assert np.array_equal(inf, g["info"][t]), t
        for i in np.flatnonzero(te | tr):
            assert crc(e.fin[i]) == g["fin_crc"][t, i] and e.ep_ret[i] == g["ep_ret"][t, i] and e.ep_len[i] == g["ep_len"][t, i]
    assert e.frames == int(g["frames"])


@pytest.mark.parametrize("kw", [dict(sticky=0.25, noop_max=30, maxpool=True, max_steps=300),
                                dict(skip=3, frame_stack=2, noop_max=4, max_steps=50)])
def test_port_env_lockstep_vs_reference(port, oracle, rom_div, kw):
    lv = [(1, 1, 1), (5, 2, 2), (7, 3, 4)] * 4
    a = port.PortVecEnv(rom_div, lv, 12, seed=9, **kw)
    b = oracle.RefVecEnv(rom_div, lv, 12, seed=9, **kw)
    assert np.array_equal(a.reset(), b.reset())
    rng = np.random.default_rng(2)
    for t in range(150):
        act = rng.integers(0, 7, 12)
        ra, rb = a.step(act), b.step(act)
        for x, y in zip(ra, rb):
            assert np.array_equal(x, y), t
        for i in range(12):
            assert np.array_equal(a.ram(i), b.ram(i)), (t, i)
    assert a.frames == b.frames


def test_port_resize_matches_cv2_golden(port):
    g = np.load(os.path.join(GOLD, "resize.npz"))
    for src, dst in zip(g["src"], g["dst"]):
        assert np.array_equal(port.resize(src), dst)
