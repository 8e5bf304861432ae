"""Generate tests/golden/ppo.npz from the reference trainer's own code (CPU, fp32).

    python tests/golden/make_ppo_golden.py        # needs the reference installed in baseline/_ref

Contents:
  gae_*      a (T=16, N=32) rollout (rewards, values, done flags with episode starts, bootstrap values) and the
             advantages / returns of the reference's Learner._gae (ppo/train.py:148-160), called unbound on a
             stand-in object that carries exactly the attributes it reads.
  loss_*     one minibatch (B=64, inputs regenerated from LOSS_SEED) through the reference NatureAC built after
             torch.manual_seed(NET_SEED) and its ppo_loss (model.py:55-74, clip 0.1, ent 0.01, vf 0.5): the loss,
             the stats, per-parameter sums of the initial weights, per-parameter gradient norms and sampled
             gradient entries.
  step_*     the same minibatch after clip_grad_norm_(0.5) and one Adam step (lr 2.5e-4, eps 1e-5): sampled
             parameter deltas.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))

T, NE, GAMMA, LAM = 16, 32, 0.99, 0.95
B, NET_SEED, LOSS_SEED, SAMPLES = 64, 0, 5, 48


def gae_inputs():
    r = np.random.default_rng(3)
    rew = r.normal(0, 1, (T, NE)).astype(np.float32)
    val = r.normal(0, 2, (T, NE)).astype(np.float32)
    done = (r.random((T, NE)) < 0.1).astype(np.float32)
    next_val = r.normal(0, 2, NE).astype(np.float32)
    next_done = (r.random(NE) < 0.1).astype(np.float32)
    return rew, val, done, next_val, next_done


def loss_inputs():
    r = np.random.default_rng(LOSS_SEED)
    obs = r.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8)
    act = r.integers(0, 7, B).astype(np.int64)
    old_logp = (-r.random(B) * 2.5).astype(np.float32)
    adv = r.normal(0, 1.5, B).astype(np.float32)
    ret = r.normal(0, 1, B).astype(np.float32)
    old_v = r.normal(0, 1, B).astype(np.float32)
    return obs, act, old_logp, adv, ret, old_v


def sample_index(numel, k, salt):
    return np.random.default_rng(1000 + salt).integers(0, numel, k)


def main():
    from fast_mario_env.ppo.model import NatureAC, ppo_loss
    from fast_mario_env.ppo.train import Learner
    torch.use_deterministic_algorithms(True)
    out = {}
    # ---- GAE through the reference method
    rew, val, done, nv, nd = gae_inputs()
    tt = torch.from_numpy
    fake = types.SimpleNamespace(a=types.SimpleNamespace(n_steps=T, gamma=GAMMA, lam=LAM),
                                 buf=types.SimpleNamespace(rew=tt(rew), val=tt(val), done=tt(done), next_val=tt(nv),
                                                           next_done=tt(nd)),
                                 adv=torch.zeros(T, NE), ret=torch.zeros(T, NE))
    Learner._gae(fake)
    out.update(gae_rew=rew, gae_val=val, gae_done=done, gae_next_val=nv, gae_next_done=nd,
               gae_adv=fake.adv.numpy().copy(), gae_ret=fake.ret.numpy().copy())
    # ---- one minibatch: loss, stats, gradients
    torch.manual_seed(NET_SEED)
    net = NatureAC(7)
    params = list(net.parameters())
    out["param_sums"] = np.array([p.detach().double().sum().item() for p in params])
    obs, act, old_logp, adv, ret, old_v = loss_inputs()
    loss, st = ppo_loss(net, tt(obs), tt(act), tt(old_logp), tt(adv), tt(ret), tt(old_v), 0.1, 0.01, 0.5)
    loss.backward()
    out["loss"] = np.array([loss.item()])
    out["stats"] = st.numpy().astype(np.float64)
    out["adv_norm"] = ((tt(adv) - tt(adv).mean()) / (tt(adv).std() + 1e-8)).numpy()
    out["grad_norms"] = np.array([p.grad.double().norm().item() for p in params])
    gidx, gval = [], []
    for k, p in enumerate(params):
        ix = sample_index(p.numel(), SAMPLES, k)
        gidx.append(ix); gval.append(p.grad.view(-1)[torch.from_numpy(ix)].numpy().astype(np.float64))
    out["grad_idx"] = np.stack(gidx); out["grad_val"] = np.stack(gval)
    # ---- clip + one Adam step
    before = [p.detach().clone() for p in params]
    torch.nn.utils.clip_grad_norm_(params, 0.5)
    opt = torch.optim.Adam(params, lr=2.5e-4, eps=1e-5)
    opt.step()
    dval = []
    for k, (p, q) in enumerate(zip(params, before)):
        dval.append((p.detach() - q).view(-1)[torch.from_numpy(gidx[k])].numpy().astype(np.float64))
    out["step_delta"] = np.stack(dval)
    np.savez_compressed(os.path.join(HERE, "ppo.npz"), **out)
    print("wrote", os.path.join(HERE, "ppo.npz"), "loss", loss.item())


if __name__ == "__main__":
    main()
