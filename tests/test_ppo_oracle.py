"""PPO trainer parity on the CPU: the numpy oracle and this package's network and loss against the fixture
generated from the reference trainer's own code (tests/golden/make_ppo_golden.py)."""
import os

import numpy as np
import pytest
import torch
from conftest import fme

import ppo_oracle
from fast_mario_env_b200 import ppo

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLD, "ppo.npz"))


def test_gae_oracle_matches_reference_bit_for_bit(g):
    adv, ret = ppo_oracle.gae(g["gae_rew"], g["gae_val"], g["gae_done"], g["gae_next_val"], g["gae_next_done"], 0.99, 0.95)
    assert np.array_equal(adv, g["gae_adv"]) and np.array_equal(ret, g["gae_ret"])


def test_adv_norm_oracle_matches_reference(g):
    import make_ppo_golden as mg
    adv = mg.loss_inputs()[3]
    np.testing.assert_allclose(ppo_oracle.adv_norm(adv), g["adv_norm"], rtol=1e-6, atol=1e-7)


def test_network_init_matches_reference(g):
    torch.manual_seed(0)
    net = ppo.NatureAC(7)
    sums = np.array([p.detach().double().sum().item() for p in net.parameters()])
    assert np.array_equal(sums, g["param_sums"])


def test_loss_and_gradients_match_reference_on_cpu(g):
    import make_ppo_golden as mg
    torch.manual_seed(0)
    net = ppo.NatureAC(7)
    obs, act, old_logp, adv, ret, _ = (torch.from_numpy(x) for x in mg.loss_inputs())
    adv_n = torch.from_numpy(ppo_oracle.adv_norm(adv.numpy()))
    loss, st = ppo.ppo_loss(net, obs, act, old_logp, adv_n, ret, 0.1, 0.01, 0.5)
    loss.backward()
    np.testing.assert_allclose(loss.item(), g["loss"][0], rtol=1e-5)
    np.testing.assert_allclose(st.numpy(), g["stats"], rtol=1e-5, atol=1e-7)
    norms = np.array([p.grad.double().norm().item() for p in net.parameters()])
    np.testing.assert_allclose(norms, g["grad_norms"], rtol=1e-4)


def test_gradient_average_over_two_gloo_ranks():
    import torch.multiprocessing as mp
    mp.spawn(_avg_worker, args=(2,), nprocs=2, join=True)


def _avg_worker(rank, world):
    import datetime
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29561")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ps = [torch.nn.Parameter(torch.zeros(3, 2)), torch.nn.Parameter(torch.zeros(5)),
              torch.nn.Parameter(torch.zeros(2, 3, 2, 2).to(memory_format=torch.channels_last))]
        ps[0].grad = torch.full((3, 2), float(rank + 1))
        ps[1].grad = torch.arange(5, dtype=torch.float32) * (rank + 1)
        g2 = torch.arange(24, dtype=torch.float32).view(2, 3, 2, 2) * (rank + 1)
        ps[2].grad = g2.contiguous(memory_format=torch.channels_last)
        flat = torch.zeros(35)
        ppo.average_grads(ps, flat, world)
        assert torch.allclose(ps[0].grad, torch.full((3, 2), 1.5))
        assert torch.allclose(ps[1].grad, torch.arange(5, dtype=torch.float32) * 1.5)
        assert torch.allclose(ps[2].grad, torch.arange(24, dtype=torch.float32).view(2, 3, 2, 2) * 1.5)
    finally:
        dist.destroy_process_group()
