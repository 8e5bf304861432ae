"""The test oracle (the reference's own C++ core, oracle/_ref) is pinned against the committed golden fixtures
and against OpenCV / numpy, before anything is compared with it (CPU only)."""
import os
import zlib

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def crc(a):
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def test_oracle_raw_frames_match_golden(oracle, rom):
    import make_golden as mg
    g = np.load(os.path.join(GOLD, "raw_seed0.npz"))
    btn = mg.raw_buttons()
    frames = 300  # a prefix keeps the CPU suite short; the GPU tests use all 1000 frames
    cons = [oracle.RefRaw(rom) for _ in range(mg.RAW_N)]
    for f in range(frames):
        for i, c in enumerate(cons):
            c.frame(int(btn[f, i]), True)
            assert crc(c.ram) == g["ram_crc"][f, i], (f, i)
            assert crc(c.screen) == g["scr_crc"][f, i], (f, i)


def test_oracle_env_matches_golden(oracle, rom):
    import make_golden as mg
    g = np.load(os.path.join(GOLD, "env_seed0.npz"))
    e = oracle.RefVecEnv(rom, mg.env_levels(), mg.ENV_N, **mg.ENV_KW)
    o = e.reset()
    assert [crc(o[i]) for i in range(mg.ENV_N)] == list(g["reset_crc"])
    acts = mg.env_actions()
    for t in range(mg.ENV_STEPS):
        o, r, te, tr, inf = e.step(acts[t])
        assert [crc(o[i]) for i in range(mg.ENV_N)] == list(g["obs_crc"][t]), t
        assert np.array_equal(r, g["rew"][t]) and np.array_equal(te, g["term"][t]) and np.array_equal(tr, g["trunc"][t])
        assert np.array_equal(inf, g["info"][t]), t
    assert e.frames == int(g["frames"])
    assert (g["term"] | g["trunc"]).sum() > 0, "the fixture must contain episode ends"


def test_oracle_gray_lut_matches_cv2(oracle):
    cv2 = pytest.importorskip("cv2")
    want = cv2.cvtColor(oracle.palette_rgb()[None], cv2.COLOR_RGB2GRAY)[0]
    assert np.array_equal(oracle.gray_lut()[:64], want)


def test_oracle_resize_matches_cv2_golden(oracle):
    g = np.load(os.path.join(GOLD, "resize.npz"))
    for src, dst in zip(g["src"], g["dst"]):
        assert np.array_equal(oracle.resize_ref(src), dst)


def test_rng_seeding_is_numpy_pcg64(oracle):
    # the 6 words passed to the engines reproduce numpy's generator state exactly
    for seed in (0, 1, 12345, 2**40 + 7):
        w = oracle.rng_state(seed)
        st = np.random.default_rng(seed).bit_generator.state
        assert (w[0] << 64 | w[1]) == st["state"]["state"] and (w[2] << 64 | w[3]) == st["state"]["inc"]
