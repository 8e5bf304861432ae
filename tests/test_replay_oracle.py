"""The replay oracle against the reference FrameReplay's own output (tests/golden/replay.npz)."""
import os
import zlib

import numpy as np

import make_replay_golden as mg
import replay_oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_oracle_storage_and_batch_match_reference():
    g = np.load(os.path.join(GOLD, "replay.npz"))
    r = replay_oracle.Ring(mg.C, mg.E, mg.K)
    for obs, nxt, act, rew, done, trunc in mg.inputs():
        r.add(obs, nxt, act, rew, done, trunc)
    for k in ("age", "flags", "act", "rew", "ptr"):
        assert np.array_equal(getattr(r, k), g[k]), k
    crcs = np.array([[zlib.crc32(r.frames[e, c].tobytes()) for c in range(mg.C)] for e in range(mg.E)])
    assert np.array_equal(crcs, g["frame_crc"])
    for b in range(mg.B):
        o = r.gather(int(g["s_env"][b]), int(g["s_pos"][b]), mg.NSTEP, mg.GAMMA)
        assert o["action"] == g["s_action"][b] and o["steps"] == g["s_steps"][b]
        assert o["reward"] == g["s_reward"][b] and o["discount"] == g["s_discount"][b]
        assert o["terminal"] == g["s_terminal"][b]
        assert zlib.crc32(o["obs"].tobytes()) == g["s_obs_crc"][b]
        assert zlib.crc32(o["next_obs"].tobytes()) == g["s_next_crc"][b]
