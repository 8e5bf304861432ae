"""Lockstep parity at the benchmark's own scale.

The reference checks its GPU engine against its CPU engine in lockstep (tests/test_cuda.py:22-59), and a slice
of a large run is the same as a small run started at that env offset (tests/test_api.py:89-98). Here one large
engine run is compared with the reference's C++ core (oracle/_ref) on slices of it:

* config 1 at its full size: 32,768 envs, the 32 level names cycled as in bench.py, seed 0, sticky 0.25,
  no-op starts up to 30, max-pool, max_steps 2000, frame stack 4; slices [0, 128), [16384, 16512) and
  [32640, 32768), i.e. the first, a middle and the last step slice of the engine (its 1,024 env groups run as
  four slices; the ragged tails of the device-to-host copies are covered by the API tests);
* config 2 (the divergence-stress image) at 4,096 envs, slices [0, 128) and [3968, 4096);
* config 3's size, 262,144 envs (8,192 env groups: the step kernel runs them with its wide shared-memory
  layout, 23 KB of RAM per CTA, where the two sizes above use the deep one), slices [0, 128),
  [131072, 131200) and [262016, 262144), 300 steps.

Every step compares, for every env of the slices: the stacked observation, reward, terminated, truncated and
the ten info fields; for envs whose episode ended also final_obs, episode return and length; every 50 steps
the 2 KB RAM. Uniform random actions over 7 from a host generator.

With the seed-0 image and uniform random actions an episode lasts about 220 agent steps and never past about
900: the "right" actions carry every env to the flag (x_pos 3072) long before the 2,000-step time limit. In
the config-1 run the odd envs therefore draw their actions from {NOOP, A, left} only ("stay-behind" envs:
they never reach the flag, so only the game's random deaths end their episodes and a few of them reach the
time limit), the even envs uniformly from all 7 as config 1 states. Envs still in their first episode after
1,500 steps join the comparison then: the oracle replays their 1,500 recorded actions, the engine's
observation and RAM of those envs must equal the oracle's at that point, and both are compared in lockstep
from there on, so every env of the run that reaches the 2,000-step truncation in its first episode is compared
at that step.

Length: 2,500 steps; FME_TEST_SCALE=4 gives the 10,000 steps of BASELINE config 1.
"""
import os

import numpy as np
import pytest
from conftest import fme, scaled

pytestmark = pytest.mark.gpu

JOIN_AT = 1500      # agent steps after reset at which first-episode survivors join the comparison
JOIN_MAX = 256      # at most this many of them (the first ones by env index)
RAM_EVERY = 50


def level_names(n):
    levels = [f"{w}-{s}" for w in range(1, 9) for s in range(1, 5)]
    return [levels[i % len(levels)] for i in range(n)]


class Mirror:
    """Envs `ids` of the engine's run, run by one reference engine seeded as those envs."""

    def __init__(self, oracle, rom, levels, ids, kw):
        self.ids = np.asarray(ids, np.int64)
        lv = [fme.decode_level(levels[i]) for i in self.ids]
        threads = min(len(self.ids), os.cpu_count() or 1)
        self.ref = oracle.RefVecEnv(rom, lv, len(self.ids), seed=0, env_ids=self.ids, n_threads=threads, **kw)

    def step(self, actions_all):
        return self.ref.step(actions_all[self.ids])


def _compare_step(t, m, got, ram=None):
    """got: this step's engine outputs for m's envs (host arrays)."""
    o1, r1, te1, tr1, i1 = m.ref.obs, m.ref.rew, m.ref.term.astype(bool), m.ref.trunc.astype(bool), m.ref.info
    assert np.array_equal(o1, got["obs"]), f"obs differ at step {t} (envs {m.ids[:4]}...)"
    assert np.array_equal(r1, got["rew"]), f"rewards differ at step {t}"
    assert np.array_equal(te1, got["term"]) and np.array_equal(tr1, got["trunc"]), f"dones differ at step {t}"
    assert np.array_equal(i1.astype(np.int32), got["info"]), f"infos differ at step {t}"
    done = te1 | tr1
    for k in np.flatnonzero(done):
        assert np.array_equal(m.ref.fin[k], got["fin"][k]), f"final_obs of env {m.ids[k]} differs at step {t}"
        assert m.ref.ep_ret[k] == got["ep_ret"][k] and m.ref.ep_len[k] == got["ep_len"][k], (t, int(m.ids[k]))
    if ram is not None:
        for k in range(len(m.ids)):
            assert np.array_equal(m.ref.ram(k), ram[k]), f"RAM of env {m.ids[k]} differs at step {t}"
    return int(done.sum()), int(tr1.sum())


def _gather(env, idx, with_ram):
    """The engine's outputs of envs idx (a device index tensor) on the host."""
    sel = lambda x: x.index_select(0, idx).cpu().numpy()  # noqa: E731
    got = dict(obs=sel(env.obs), rew=sel(env.rew), term=sel(env.term), trunc=sel(env.trunc), info=sel(env.info_t),
               fin=sel(env.final_obs), ep_ret=sel(env.ep_ret), ep_len=sel(env.ep_len))
    ram = sel(env.ram()) if with_ram else None
    return got, ram


STAY_BEHIND = np.array([0, 5, 6])   # NOOP, A, left: no action moves right


def _run(oracle, rom, n, slices, kw, steps, action_seed, stay_behind=False):
    import torch
    levels = level_names(n)
    env = fme.CudaVecEnv(levels, n, seed=0, rom=rom, **kw)
    dev = env.dev
    mirrors = [Mirror(oracle, rom, levels, np.arange(a, b), kw) for a, b in slices]
    obs0 = env.reset()
    for m in mirrors:
        ref_obs = m.ref.reset()
        assert np.array_equal(ref_obs, obs0.index_select(0, torch.from_numpy(m.ids).to(dev)).cpu().numpy())
    rng = np.random.default_rng(action_seed)
    history = np.zeros((JOIN_AT, n), np.uint8)
    first_ep = np.ones(n, bool)          # still in the episode that started at reset()
    late = None
    stats = dict(episodes=0, truncations=0, run_truncations=0, first_episode_truncations=0, joined=0)
    odd = np.arange(n) % 2 == 1
    for t in range(steps):
        a = rng.integers(0, 7, n)
        if stay_behind:
            a[odd] = STAY_BEHIND[a[odd] % 3]
        if t < JOIN_AT:
            history[t] = a
        env.step(torch.from_numpy(a).to(dev))
        for m in mirrors:            # the reference steps while the device runs
            m.step(a)
        term, trunc = env.term.cpu().numpy(), env.trunc.cpu().numpy()
        stats["run_truncations"] += int(trunc.sum())
        with_ram = (t + 1) % RAM_EVERY == 0
        for m in mirrors:
            got, ram = _gather(env, torch.from_numpy(m.ids).to(dev), with_ram)
            d, tr = _compare_step(t, m, got, ram)
            stats["episodes"] += d
            stats["truncations"] += tr
        stats["first_episode_truncations"] += int((first_ep & trunc).sum())
        first_ep &= ~(term | trunc)
        if t + 1 == JOIN_AT and steps > JOIN_AT:
            ids = np.flatnonzero(first_ep)[:JOIN_MAX]
            tracked = set(np.concatenate([m.ids for m in mirrors]).tolist())
            ids = np.array([i for i in ids if i not in tracked], np.int64)
            if len(ids):
                late = Mirror(oracle, rom, levels, ids, kw)
                late.ref.reset()
                for q in range(JOIN_AT):
                    late.step(history[q])
                got, ram = _gather(env, torch.from_numpy(late.ids).to(dev), True)
                assert np.array_equal(late.ref.obs, got["obs"]), "late-joined envs' obs differ at the join"
                for k in range(len(late.ids)):
                    assert np.array_equal(late.ref.ram(k), ram[k]), f"late-joined env {late.ids[k]}: RAM differs"
                mirrors.append(late)
                stats["joined"] = len(ids)
    env.check()
    assert env.bad_ops() == 0
    return stats


def test_config1_32768_envs_lockstep_slices(oracle, rom):
    kw = dict(sticky=0.25, noop_max=30, maxpool=True, max_steps=2000, skip=4, frame_stack=4)
    stats = _run(oracle, rom, 32768, [(0, 128), (16384, 16512), (32640, 32768)], kw, scaled(2500), action_seed=2500,
                 stay_behind=True)
    print("config1 32768 envs:", stats)
    assert stats["episodes"] > 0
    # the time limit: every env of the run that lasted 2,000 steps in its first episode joined the comparison
    # at step 1,500 and was compared when it truncated
    assert stats["first_episode_truncations"] > 0, "no env reached the 2,000-step time limit"
    assert stats["joined"] < JOIN_MAX
    assert stats["truncations"] >= stats["first_episode_truncations"]


def test_config2_divergent_4096_envs_lockstep_slices(oracle, rom_div):
    kw = dict(sticky=0.25, noop_max=30, maxpool=True, max_steps=2000, skip=4, frame_stack=4)
    stats = _run(oracle, rom_div, 4096, [(0, 128), (3968, 4096)], kw, scaled(2500), action_seed=4096)
    print("config2 4096 envs:", stats)
    assert stats["episodes"] > 0


def test_config3_262144_envs_wide_layout_lockstep_slices(oracle, rom):
    kw = dict(sticky=0.25, noop_max=30, maxpool=True, max_steps=2000, skip=4, frame_stack=4)
    stats = _run(oracle, rom, 262144, [(0, 128), (131072, 131200), (262016, 262144)], kw, scaled(300),
                 action_seed=262144)
    print("config3 262144 envs:", stats)
    assert stats["episodes"] > 0
