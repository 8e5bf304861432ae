"""The GPU FrameReplay (fme_replay_add / fme_replay_gather) against the reference FrameReplay's output
(tests/golden/replay.npz): storage after the same adds, and the batch for the same (env, slot) pairs, bit-exact."""
import os
import zlib

import numpy as np
import pytest
import torch

import make_replay_golden as mg

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _filled():
    from fast_mario_env_b200.replay import FrameReplay
    rb = FrameReplay(mg.C, mg.E, k=mg.K, seed=mg.SAMPLE_SEED)
    for obs, nxt, act, rew, done, trunc in mg.inputs():
        rb.add(torch.from_numpy(obs).cuda(), torch.from_numpy(nxt).cuda(), act, rew, done, trunc)
    return rb


def test_storage_matches_reference():
    g = np.load(os.path.join(GOLD, "replay.npz"))
    rb = _filled()
    for k in ("age", "flags", "act", "rew", "ptr"):
        assert np.array_equal(getattr(rb, k).cpu().numpy(), g[k]), k
    fr = rb.frames.cpu().numpy()
    crcs = np.array([[zlib.crc32(fr[e, c].tobytes()) for c in range(mg.C)] for e in range(mg.E)])
    assert np.array_equal(crcs, g["frame_crc"])
    assert rb.size() == min(mg.ADDS * mg.E, mg.E * mg.C)


def test_batch_matches_reference():
    g = np.load(os.path.join(GOLD, "replay.npz"))
    rb = _filled()
    e = torch.from_numpy(g["s_env"]).cuda()
    p = torch.from_numpy(g["s_pos"]).cuda()
    s = rb.gather(e, p, mg.NSTEP, mg.GAMMA)
    assert np.array_equal(s.action.cpu().numpy(), g["s_action"])
    assert np.array_equal(s.steps.cpu().numpy(), g["s_steps"])
    assert np.array_equal(s.reward.cpu().numpy(), g["s_reward"])
    assert np.array_equal(s.discount.cpu().numpy(), g["s_discount"])
    assert np.array_equal(s.terminal.cpu().numpy(), g["s_terminal"])
    ob, nb = s.obs.cpu().numpy(), s.next_obs.cpu().numpy()
    assert [zlib.crc32(ob[b].tobytes()) for b in range(mg.B)] == list(g["s_obs_crc"])
    assert [zlib.crc32(nb[b].tobytes()) for b in range(mg.B)] == list(g["s_next_crc"])


def test_sample_draws_valid_transitions():
    rb = _filled()
    s = rb.sample(256, n_step=3, gamma=0.99)
    flags = rb.flags.cpu().numpy()
    ptr = rb.ptr.cpu().numpy()
    e, p = s.env.cpu().numpy(), s.pos.cpu().numpy()
    assert np.all(flags[e, p % mg.C] & 1)
    assert np.all(p >= np.maximum(ptr[e] - mg.C + mg.K - 1, 0)) and np.all(p <= ptr[e] - 1 - 3)
    assert s.obs.shape == (256, mg.K, 84, 84) and s.next_obs.shape == (256, mg.K, 84, 84)
