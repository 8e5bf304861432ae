"""GPU API behaviour: shapes/dtypes, zero-padded stacks, determinism, env_offset sharding, the FastVecEnv
wrapper, the device resize, and device-side error reporting (the reference's tests/test_api.py pattern)."""
import os

import numpy as np
import pytest
from conftest import fme

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_shapes_and_infos(rom):
    v = fme.FastVecEnv("1-1", 3, seed=0, max_steps=20, rom=rom)
    obs = v.reset()
    assert obs.shape == (3, 4, 84, 84) and obs.dtype == np.uint8
    assert (obs[:, :3] == 0).all() and obs[:, 3].any()
    ended = 0
    for t in range(25):
        obs, r, te, tr, infos = v.step(np.full(3, 1))
        assert r.dtype == np.float32 and te.dtype == bool and tr.dtype == bool and len(infos) == 3
        assert set(fme.INFO_KEYS) <= set(infos[0])
        for i in np.flatnonzero(te | tr):
            ended += 1
            assert infos[i]["final_obs"].shape == (4, 84, 84)
            assert infos[i]["episode"]["l"] == 20 and infos[i]["TimeLimit.truncated"]
    assert ended == 3
    assert v.bad_ops() == 0 and v.frames > 0
    v.check()
    v.close()


def test_determinism(rom):
    import torch
    acts = torch.from_numpy(np.random.default_rng(0).integers(0, 7, (40, 64))).cuda()
    outs = []
    for _ in range(2):
        e = fme.CudaVecEnv(["1-1", "1-2", "4-1", "8-4"] * 16, 64, seed=5, sticky=0.25, noop_max=10, maxpool=True, rom=rom)
        o = [e.reset().clone()]
        for a in acts:
            o.append(e.step(a)[0].clone())
        outs.append(torch.stack(o))
        e.close()
    assert torch.equal(outs[0], outs[1])


def test_env_offset_matches_slice(rom):
    import torch
    acts = torch.from_numpy(np.random.default_rng(1).integers(0, 7, (30, 48))).cuda()
    a = fme.CudaVecEnv("1-1", 48, seed=2, sticky=0.25, noop_max=10, rom=rom)
    b = fme.CudaVecEnv("1-1", 16, seed=2, sticky=0.25, noop_max=10, env_offset=32, rom=rom)
    oa, ob = a.reset(), b.reset()
    assert torch.equal(oa[32:], ob)
    for x in acts:
        oa, ob = a.step(x)[0], b.step(x[32:].contiguous())[0]
        assert torch.equal(oa[32:], ob)


def test_fastvecenv_matches_cudavecenv(rom):
    import torch
    kw = dict(seed=3, sticky=0.25, noop_max=30, maxpool=True, max_steps=50, rom=rom)
    f = fme.FastVecEnv("1-1", 8, **kw)
    c = fme.CudaVecEnv("1-1", 8, **kw)
    assert np.array_equal(f.reset(), c.reset().cpu().numpy())
    rng = np.random.default_rng(4)
    for _ in range(60):
        a = rng.integers(0, 7, 8)
        o1, r1, te1, tr1, infos = f.step(a)
        o2, r2, te2, tr2, i2 = c.step(torch.from_numpy(a).cuda())
        assert np.array_equal(o1, o2.cpu().numpy()) and np.array_equal(r1, r2.cpu().numpy())
        assert np.array_equal(te1, te2.cpu().numpy()) and np.array_equal(tr1, tr2.cpu().numpy())
        for i in range(8):
            assert infos[i]["x_pos"] == int(i2["x_pos"][i])


def test_step_arrays_matches_step(rom):
    kw = dict(seed=5, sticky=0.25, noop_max=30, maxpool=True, max_steps=40, rom=rom)
    f = fme.FastVecEnv("1-1", 8, **kw)
    g = fme.FastVecEnv("1-1", 8, **kw)
    f.reset(); g.reset()
    rng = np.random.default_rng(6)
    ended = 0
    for _ in range(60):
        a = rng.integers(0, 7, 8)
        o1, r1, te1, tr1, infos = f.step(a)
        o2, r2, te2, tr2, inf2, fin = g.step_arrays(a)
        assert np.array_equal(o1, o2) and np.array_equal(r1, r2)
        assert np.array_equal(te1, te2) and np.array_equal(tr1, tr2)
        for i in range(8):
            assert infos[i]["x_pos"] == inf2[i, 0] and infos[i]["score"] == inf2[i, 3]
            if te1[i] or tr1[i]:
                assert np.array_equal(infos[i]["final_obs"], fin[i])
                ended += 1
        assert set(fin) == {i for i in range(8) if te1[i] or tr1[i]}
    assert ended > 0
    f.close(); g.close()


def test_host_outputs_match_device_outputs_across_slices(rom):
    """fme_step_to_host (early copy of the old frames, new frame after the render, stacks of restarted episodes
    cleared on the host) against the device buffers of fme_step: 150 envs = 4 step slices, short episodes."""
    import torch
    levels = ["1-1", "3-2", "5-4", "8-1", "2-2"] * 30
    kw = dict(seed=11, sticky=0.25, noop_max=30, maxpool=True, max_steps=25, rom=rom)
    f = fme.FastVecEnv(levels, 150, **kw)
    d = fme.CudaVecEnv(levels, 150, **kw)
    assert np.array_equal(f.reset(), d.reset().cpu().numpy())
    rng = np.random.default_rng(12)
    ended = 0
    for _ in range(60):
        a = rng.integers(0, 7, 150)
        o1, r1, te1, tr1, inf1, _ = f.step_arrays(a)
        o2, r2, te2, tr2, _ = d.step(torch.from_numpy(a).cuda())
        assert np.array_equal(o1, o2.cpu().numpy()) and np.array_equal(r1, r2.cpu().numpy())
        assert np.array_equal(te1, te2.cpu().numpy()) and np.array_equal(tr1, tr2.cpu().numpy())
        assert np.array_equal(inf1, d.info_t.cpu().numpy())
        ended += int((te1 | tr1).sum())
    assert ended > 50
    f.close(); d.close()


def test_step_to_host_back_to_back_with_two_buffer_sets(rom):
    """Two fme_step_to_host calls enqueued without a sync in between, into different pinned buffer sets: each
    set must hold its own step's outputs (the host fix-up of the first call must not use the second's)."""
    import ctypes
    import torch
    from fast_mario_env_b200 import _native as N
    levels = ["1-1", "3-2", "5-4", "8-1", "2-2"] * 30
    kw = dict(seed=21, sticky=0.25, noop_max=30, maxpool=True, max_steps=15, rom=rom)
    h = fme.CudaVecEnv(levels, 150, **kw)
    d = fme.CudaVecEnv(levels, 150, **kw)
    h.reset(); d.reset()
    pin = dict(pin_memory=True)

    def bufs():
        t = (torch.zeros(150, 4, 84, 84, dtype=torch.uint8, **pin), torch.zeros(150, dtype=torch.float32, **pin),
             torch.zeros(150, dtype=torch.bool, **pin), torch.zeros(150, dtype=torch.bool, **pin),
             torch.zeros(150, len(fme.INFO_FIELDS), dtype=torch.int32, **pin),
             torch.zeros(150, dtype=torch.float64, **pin), torch.zeros(150, dtype=torch.int32, **pin))
        return t, N.FmeHostOut(*[x.data_ptr() for x in t])

    (ta, oa), (tb, ob) = bufs(), bufs()
    rng = np.random.default_rng(22)
    ended = 0
    for _ in range(30):
        a1 = torch.from_numpy(rng.integers(0, 7, 150)).cuda()
        a2 = torch.from_numpy(rng.integers(0, 7, 150)).cuda()
        h.actions.copy_(a1)
        N.check(N.lib().fme_step_to_host(h.h, N.ptr(h.actions), ctypes.byref(oa), h._stream()), "step_to_host")
        h.actions.copy_(a2)
        N.check(N.lib().fme_step_to_host(h.h, N.ptr(h.actions), ctypes.byref(ob), h._stream()), "step_to_host")
        torch.cuda.synchronize()
        for act, (t, _) in ((a1, (ta, oa)), (a2, (tb, ob))):
            o, r, te, tr, _ = d.step(act)
            assert torch.equal(t[0], o.cpu()) and torch.equal(t[1], r.cpu())
            assert torch.equal(t[2].to(torch.uint8), te.cpu().to(torch.uint8))
            assert torch.equal(t[3].to(torch.uint8), tr.cpu().to(torch.uint8))
            ended += int((t[2] | t[3]).sum())
    assert ended > 50
    h.close(); d.close()


def test_step_to_host_in_place_shift_many_calls_in_flight(rom):
    """FME_HOST_OBS_IN_PLACE: 20 fme_step_to_host calls into one pinned buffer set, enqueued without a sync
    (more than the 16 argument blocks, so later calls wait for earlier ones' host functions); the host stacks
    are shifted in place by the library. Then calls alternating between two buffer sets with the flag set, which
    must fall back to copying the old frames from the device. Each is checked against fme_step's device buffers."""
    import ctypes
    import torch
    from fast_mario_env_b200 import _native as N
    levels = ["1-1", "3-2", "5-4", "8-1", "2-2"] * 30
    kw = dict(seed=31, sticky=0.25, noop_max=30, maxpool=True, max_steps=12, rom=rom)
    h = fme.CudaVecEnv(levels, 150, **kw)
    d = fme.CudaVecEnv(levels, 150, **kw)
    h.reset()
    d.reset()
    pin = dict(pin_memory=True)

    def bufs():
        t = (torch.zeros(150, 4, 84, 84, dtype=torch.uint8, **pin), torch.zeros(150, dtype=torch.float32, **pin),
             torch.zeros(150, dtype=torch.bool, **pin), torch.zeros(150, dtype=torch.bool, **pin),
             torch.zeros(150, len(fme.INFO_FIELDS), dtype=torch.int32, **pin),
             torch.zeros(150, dtype=torch.float64, **pin), torch.zeros(150, dtype=torch.int32, **pin))
        return t, N.FmeHostOut(*[x.data_ptr() for x in t], N.FME_HOST_OBS_IN_PLACE)

    (ta, oa), (tb, ob) = bufs(), bufs()
    ta[0].copy_(h.obs.cpu())   # the reset stacks (reset is device-only, so the first call copies anyway)
    rng = np.random.default_rng(32)
    acts = [torch.from_numpy(rng.integers(0, 7, 150)).cuda() for _ in range(20)]
    ended = 0
    for a in acts:
        h.actions.copy_(a)
        N.check(N.lib().fme_step_to_host(h.h, N.ptr(h.actions), ctypes.byref(oa), h._stream()), "step_to_host")
    torch.cuda.synchronize()
    for a in acts:
        o, r, te, tr, _ = d.step(a)
        ended += int((te | tr).sum())
    assert torch.equal(ta[0], o.cpu()) and torch.equal(ta[1], r.cpu())
    assert torch.equal(ta[4], d.info_t.cpu())
    assert ended > 50
    for k in range(6):   # alternating buffers: never the buffer the previous call wrote, so no in-place shift
        a = torch.from_numpy(rng.integers(0, 7, 150)).cuda()
        t, o_ = (tb, ob) if k % 2 == 0 else (ta, oa)
        h.actions.copy_(a)
        N.check(N.lib().fme_step_to_host(h.h, N.ptr(h.actions), ctypes.byref(o_), h._stream()), "step_to_host")
        torch.cuda.synchronize()
        o, r, te, tr, _ = d.step(a)
        assert torch.equal(t[0], o.cpu()) and torch.equal(t[1], r.cpu()), k
    h.close(); d.close()


def test_resize_matches_cv2_golden():
    g = np.load(os.path.join(GOLD, "resize.npz"))
    out = fme.resize_area(g["src"])
    assert np.array_equal(out, g["dst"])


def test_bad_action_is_reported(rom):
    import torch
    e = fme.CudaVecEnv("1-1", 4, rom=rom)
    e.reset()
    e.step(torch.tensor([0, 1, 9, 2], device="cuda"))
    with pytest.raises(Exception, match="action"):
        e.check()


def test_log_overflow_is_reported_not_silent(rom):
    # a capacity far below one frame's records: construction (which emulates the boot frames) must refuse with
    # the overflow status instead of producing wrong frames
    with pytest.raises(Exception, match="status 1|log"):
        fme.CudaVecEnv("1-1", 4, rom=rom, log_capacity=64)
