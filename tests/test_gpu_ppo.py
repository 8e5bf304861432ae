"""PPO trainer kernels and one update on the GPU against the reference trainer's fixture (tests/golden/ppo.npz).
Tolerance for the network (fp32, TF32 off): 1e-4 relative, the bar for PPO losses and gradients; GAE is
bit-exact (the same fp32 operations in the same order)."""
import os

import numpy as np
import pytest
import torch
from conftest import fme

import ppo_oracle

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLD, "ppo.npz"))


@pytest.fixture(autouse=True)
def no_tf32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _ppo():
    from fast_mario_env_b200 import ppo
    return ppo


def test_gae_kernel_matches_reference_bit_for_bit(g):
    ppo = _ppo()
    c = lambda k: torch.from_numpy(g[k]).cuda().contiguous()  # noqa: E731
    adv = torch.zeros_like(c("gae_rew")); ret = torch.zeros_like(adv)
    ppo.gae(c("gae_rew"), c("gae_val"), c("gae_done"), c("gae_next_val"), c("gae_next_done"), 0.99, 0.95, adv, ret)
    assert np.array_equal(adv.cpu().numpy(), g["gae_adv"]) and np.array_equal(ret.cpu().numpy(), g["gae_ret"])


def test_gae_kernel_large_rollout_matches_oracle():
    ppo = _ppo()
    r = np.random.default_rng(9)
    T, n = 128, 4096
    rew = r.normal(0, 1, (T, n)).astype(np.float32); val = r.normal(0, 3, (T, n)).astype(np.float32)
    done = (r.random((T, n)) < 0.02).astype(np.float32)
    nv = r.normal(0, 3, n).astype(np.float32); nd = (r.random(n) < 0.02).astype(np.float32)
    want_adv, want_ret = ppo_oracle.gae(rew, val, done, nv, nd, 0.99, 0.95)
    t = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
    adv = torch.zeros(T, n, device="cuda"); ret = torch.zeros_like(adv)
    ppo.gae(t(rew), t(val), t(done), t(nv), t(nd), 0.99, 0.95, adv, ret)
    assert np.array_equal(adv.cpu().numpy(), want_adv) and np.array_equal(ret.cpu().numpy(), want_ret)


def test_adv_norm_kernel(g):
    import make_ppo_golden as mg
    ppo = _ppo()
    adv = torch.from_numpy(mg.loss_inputs()[3]).cuda()
    np.testing.assert_allclose(ppo.adv_norm(adv).cpu().numpy(), g["adv_norm"], rtol=1e-5, atol=1e-6)
    x = torch.randn(1024, device="cuda") * 3 + 1
    np.testing.assert_allclose(ppo.adv_norm(x).cpu().numpy(), ((x - x.mean()) / (x.std() + 1e-8)).cpu().numpy(),
                               rtol=1e-5, atol=1e-6)


def test_loss_gradients_and_adam_step_match_reference(g):
    import make_ppo_golden as mg
    ppo = _ppo()
    torch.manual_seed(mg.NET_SEED)
    net = ppo.NatureAC(7)
    # same seed and init order as the reference; the orthogonal init's QR runs on the host CPU, whose LAPACK may
    # round differently from the machine that made the fixture, so the weights agree to about 1e-7
    np.testing.assert_allclose(np.array([p.detach().double().sum().item() for p in net.parameters()]), g["param_sums"],
                               rtol=1e-5, atol=1e-6)
    cfg = ppo.PPOConfig(n_envs=8, n_steps=8, batch=mg.B, epochs=1, graph=True)
    L = ppo.Learner(cfg, torch.device("cuda"), net=net)
    obs, act, old_logp, adv, ret, old_v = mg.loss_inputs()
    b = L.buf
    b.obs.view(-1, 4, 84, 84).copy_(torch.from_numpy(obs).cuda())
    b.act.view(-1).copy_(torch.from_numpy(act).cuda())
    b.logp.view(-1).copy_(torch.from_numpy(old_logp).cuda())
    b.val.view(-1).copy_(torch.from_numpy(old_v).cuda())
    L.adv.view(-1).copy_(torch.from_numpy(adv).cuda())
    L.ret.view(-1).copy_(torch.from_numpy(ret).cuda())
    before = [p.detach().clone() for p in L.params]
    # loss and gradients through the eager path first (same code the graph replays)
    L.mb_idx.copy_(torch.arange(mg.B, device="cuda"))
    st = L._forward_backward()
    np.testing.assert_allclose(st.cpu().numpy(), g["stats"], rtol=1e-4, atol=1e-6)
    norms = np.array([p.grad.double().norm().item() for p in L.params])
    np.testing.assert_allclose(norms, g["grad_norms"], rtol=1e-4)
    for k, p in enumerate(L.params):
        got = p.grad.reshape(-1)[torch.from_numpy(g["grad_idx"][k]).cuda()].double().cpu().numpy()
        np.testing.assert_allclose(got, g["grad_val"][k], rtol=1e-4, atol=1e-4 * float(g["grad_norms"][k]) / 50)
    # the captured minibatch step: clip + Adam from the restored state
    L.minibatch(torch.arange(mg.B, device="cuda"))
    torch.cuda.synchronize()
    for k, (p, q) in enumerate(zip(L.params, before)):
        d = (p.detach() - q).reshape(-1)[torch.from_numpy(g["grad_idx"][k]).cuda()].double().cpu().numpy()
        np.testing.assert_allclose(d, g["step_delta"][k], rtol=1e-3, atol=2e-7)


def test_trainer_iteration_on_the_gpu_env(rom):
    ppo = _ppo()
    env = fme.CudaVecEnv("1-1", 64, seed=0, sticky=0.25, noop_max=30, maxpool=True, rom=rom)
    cfg = ppo.PPOConfig(n_envs=64, n_steps=16, batch=256, epochs=2)
    tr = ppo.Trainer(env, cfg, torch.device("cuda"), seed=0)
    stats = tr.iterate().cpu().numpy()
    assert np.all(np.isfinite(stats)) and stats[-1] == 0
    assert tr.L.buf.obs.float().mean().item() > 0
    env.check()
    env.close()
