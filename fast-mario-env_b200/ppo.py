"""PPO trainer hot loop on the B200 engine: rollout on the GPU env, GAE and per-minibatch advantage
normalisation in the library's kernels (`fme_gae`, `fme_adv_norm`), Nature-CNN forward/backward and Adam in
torch, minibatch step captured in a CUDA graph, gradients averaged over ranks with NCCL.

Mirrors the reference trainer (src/fast_mario_env/ppo/train.py:112-247, model.py:13-74): the same network,
initialisation, sampling, loss, gradient clipping, non-finite-minibatch skip and Adam settings, so one update
from identical weights and rollouts matches it to fp32 accuracy. Defaults are BASELINE config 4 (4096 envs per
GPU x 128 steps, gamma 0.99, lambda 0.95, clip 0.1, vf 0.5, ent 0.01, 4 epochs, minibatch 1024, Adam 2.5e-4,
eps 1e-5, max grad norm 0.5).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as N

STAT_NAMES = ("policy_gradient_loss", "value_loss", "entropy", "clip_fraction", "approx_kl", "nonfinite_skips")


@dataclass
class PPOConfig:
    n_envs: int = 4096
    n_steps: int = 128
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.1
    vf: float = 0.5
    ent: float = 0.01
    epochs: int = 4
    batch: int = 1024
    lr: float = 2.5e-4
    adam_eps: float = 1e-5
    max_grad_norm: float = 0.5
    graph: bool = True
    channels_last: bool = True   # NHWC activations and weights for the convolutions (the reference's default)
    trunc_budget: int = 64       # time-limit truncations bootstrapped per rollout step without a host sync


class NatureAC(nn.Module):
    """Nature-CNN actor-critic (model.py:13-30): conv 32@8x8/4, 64@4x4/2, 64@3x3/1, FC 512, policy and value
    heads; orthogonal init with gains sqrt(2) (trunk), 0.01 (policy), 1 (value), zero biases, in the
    reference's module order so the same torch seed gives the same weights."""

    def __init__(self, n_actions: int = 7, in_ch: int = 4):
        super().__init__()
        self.cnn = nn.Sequential(nn.Conv2d(in_ch, 32, 8, 4), nn.ReLU(), nn.Conv2d(32, 64, 4, 2), nn.ReLU(),
                                 nn.Conv2d(64, 64, 3, 1), nn.ReLU(), nn.Flatten())
        self.fc = nn.Linear(3136, 512)
        self.pi = nn.Linear(512, n_actions)
        self.vf = nn.Linear(512, 1)
        for m in [mod for mod in self.cnn if isinstance(mod, nn.Conv2d)] + [self.fc]:
            nn.init.orthogonal_(m.weight, math.sqrt(2.0))
            nn.init.zeros_(m.bias)
        nn.init.orthogonal_(self.pi.weight, 0.01)
        nn.init.zeros_(self.pi.bias)
        nn.init.orthogonal_(self.vf.weight, 1.0)
        nn.init.zeros_(self.vf.bias)

    def forward(self, obs_u8, channels_last: bool = False):
        x = obs_u8.float().mul_(1.0 / 255.0)
        if channels_last:
            x = x.contiguous(memory_format=torch.channels_last)
        h = F.relu(self.fc(self.cnn(x)))
        return self.pi(h), self.vf(h).squeeze(-1)

    @torch.no_grad()
    def act(self, obs_u8, channels_last: bool = False):
        """Gumbel-max sample of the policy (graph-capturable): action int64, its log-prob, value."""
        logits, v = self(obs_u8, channels_last)
        logp_all = F.log_softmax(logits, -1)
        u = torch.rand_like(logits).clamp_(1e-20, 1.0)
        a = (logp_all - torch.log(-torch.log(u))).argmax(-1)
        return a, logp_all.gather(-1, a[:, None]).squeeze(-1), v


def _stream_ptr(dev=None):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def gae(rew, val, done, next_val, next_done, gamma, lam, adv, ret):
    """fme_gae on the current stream: (T, N) fp32 contiguous CUDA tensors; writes adv and ret in place."""
    T, n = rew.shape
    for t in (rew, val, done, adv, ret):
        assert t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.shape == (T, n)
    N.check(N.lib().fme_gae(N.ptr(rew), N.ptr(val), N.ptr(done), N.ptr(next_val), N.ptr(next_done), T, n,
                            ctypes.c_float(gamma), ctypes.c_float(gamma * lam), N.ptr(adv), N.ptr(ret),
                            _stream_ptr(rew.device)), "fme_gae")


def adv_norm(x, out=None):
    """fme_adv_norm on the current stream: (x - mean) / (std + 1e-8) of a contiguous fp32 CUDA vector."""
    out = torch.empty_like(x) if out is None else out
    N.check(N.lib().fme_adv_norm(N.ptr(x), N.ptr(out), x.numel(), _stream_ptr(x.device)), "fme_adv_norm")
    return out


def ppo_loss(net, obs, act, old_logp, adv_n, ret, clip, ent_coef, vf_coef, channels_last=False):
    """The reference loss (model.py:55-74) with the advantages already normalised by `adv_norm`: clipped
    surrogate, unclipped MSE value loss, -mean(entropy); stats as the reference (pg, vf, entropy, clip
    fraction, approx kl)."""
    logits, v = net(obs, channels_last)
    logp_all = F.log_softmax(logits, -1)
    logp = logp_all.gather(-1, act[:, None]).squeeze(-1)
    ent = -(logp_all.exp() * logp_all).sum(-1)
    lr_ = (logp - old_logp).clamp(-20.0, 20.0)
    ratio = torch.exp(lr_)
    pg = -torch.min(adv_n * ratio, adv_n * ratio.clamp(1 - clip, 1 + clip)).mean()
    vl = F.mse_loss(ret, v)
    el = -ent.mean()
    loss = pg + ent_coef * el + vf_coef * vl
    with torch.no_grad():
        stats = torch.stack([pg, vl, -el, ((ratio - 1).abs() > clip).float().mean(), ((torch.exp(lr_) - 1) - lr_).mean()])
    return loss, stats


def average_grads(params, flat, world):
    """Data-parallel gradient mean: pack every gradient into one flat buffer, one all-reduce (sum) over the
    default process group, divide by the world size, unpack."""
    off = 0
    for p in params:  # reshape / view_as keep the logical order whatever the memory format (channels-last)
        flat[off:off + p.numel()].copy_(p.grad.reshape(-1))
        off += p.numel()
    torch.distributed.all_reduce(flat)
    flat.div_(world)
    off = 0
    for p in params:
        p.grad.copy_(flat[off:off + p.numel()].view(p.grad.shape))
        off += p.numel()


class Storage:
    """Rollout buffers on the device; done[t] = 1 when obs[t] starts a new episode (train.py:96-107)."""

    def __init__(self, T, n, dev):
        z = lambda *s, dt=torch.float32: torch.zeros(s, dtype=dt, device=dev)  # noqa: E731
        self.obs = z(T, n, 4, 84, 84, dt=torch.uint8)
        self.act = z(T, n, dt=torch.int64)
        self.logp, self.val, self.rew, self.done = z(T, n), z(T, n), z(T, n), z(T, n)
        self.next_val, self.next_done = z(n), z(n)


class Learner:
    """GAE + epochs x shuffled minibatches (train.py:112-247). With a process group of world size > 1 the
    gradients are averaged over ranks (NCCL all-reduce of one flat buffer) before clipping, inside the captured
    minibatch graph."""

    def __init__(self, cfg: PPOConfig, dev, net: NatureAC | None = None):
        self.cfg, self.dev = cfg, dev
        T, n = cfg.n_steps, cfg.n_envs
        self.net = (net if net is not None else NatureAC(7)).to(dev)
        if cfg.channels_last:
            self.net = self.net.to(memory_format=torch.channels_last)
        self.params = list(self.net.parameters())
        self.world = torch.distributed.get_world_size() if torch.distributed.is_initialized() else 1
        self.opt = torch.optim.Adam(self.params, lr=torch.tensor(cfg.lr, device=dev) if cfg.graph else cfg.lr,
                                    eps=cfg.adam_eps, fused=True, capturable=bool(cfg.graph))
        self.buf = Storage(T, n, dev)
        self.adv = torch.zeros(T, n, device=dev)
        self.ret = torch.zeros(T, n, device=dev)
        self.adv_mb = torch.zeros(cfg.batch, device=dev)
        self.stats = torch.zeros(len(STAT_NAMES), device=dev)
        self.mb_idx = torch.zeros(cfg.batch, dtype=torch.int64, device=dev)
        self.flat = torch.zeros(sum(p.numel() for p in self.params), device=dev) if self.world > 1 else None
        self.graph = None
        if cfg.graph:
            self._capture()

    def _gae(self):
        b, c = self.buf, self.cfg
        gae(b.rew, b.val, b.done, b.next_val, b.next_done, c.gamma, c.lam, self.adv, self.ret)

    def _forward_backward(self):
        c, b, i = self.cfg, self.buf, self.mb_idx
        obs = b.obs.view(-1, 4, 84, 84)[i]
        adv_norm(self.adv.view(-1)[i], self.adv_mb)
        loss, st = ppo_loss(self.net, obs, b.act.view(-1)[i], b.logp.view(-1)[i], self.adv_mb, self.ret.view(-1)[i],
                            c.clip, c.ent, c.vf, channels_last=c.channels_last)
        self.opt.zero_grad(set_to_none=not c.graph)
        loss.backward()
        return st

    def _allreduce(self):
        if self.world > 1:
            average_grads(self.params, self.flat, self.world)

    def _apply(self, st):
        c = self.cfg
        gn = torch.nn.utils.clip_grad_norm_(self.params, c.max_grad_norm, foreach=True)
        ok = torch.isfinite(gn)
        for p in self.params:  # a non-finite minibatch is skipped (zero step) instead of poisoning the weights
            p.grad.copy_(torch.where(ok, p.grad, torch.zeros_like(p.grad)))
        self.opt.step()
        self.stats[:-1].add_(st)
        self.stats[-1].add_((~ok).float())

    def _mb_step(self):
        st = self._forward_backward()
        self._allreduce()
        self._apply(st)

    def _capture(self):
        """One graph for the minibatch step, captured on dummy indices; parameters and Adam state are restored
        afterwards. With several ranks the NCCL all-reduce of the gradients is part of the graph (every rank
        captures, and later replays, the same collective in the same order); the eager warm-up steps before
        the capture set up the communicator."""
        snap = [p.detach().clone() for p in self.params]
        self.mb_idx.copy_(torch.randint(0, self.cfg.n_steps * self.cfg.n_envs, (self.cfg.batch,), device=self.dev))
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(3):
                self._mb_step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.opt.zero_grad(set_to_none=False)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self._mb_step()
        with torch.no_grad():
            for p, q in zip(self.params, snap):
                p.copy_(q)
            for st in self.opt.state.values():
                for k in ("exp_avg", "exp_avg_sq", "step"):
                    st[k].zero_()
        self.stats.zero_()
        torch.cuda.synchronize(self.dev)

    def minibatch(self, idx):
        """One minibatch step on the given flat sample indices (int64 CUDA tensor of size batch)."""
        self.mb_idx.copy_(idx)
        self.graph.replay() if self.graph is not None else self._mb_step()

    def update(self, perms=None):
        """GAE, then epochs x shuffled minibatches. perms: optional list of per-epoch permutations (for
        reproducing a given shuffle). Returns the mean stats tensor (no sync)."""
        c = self.cfg
        self._gae()
        TN = c.n_steps * c.n_envs
        nmb = TN // c.batch
        self.stats.zero_()
        for ep in range(c.epochs):
            perm = perms[ep] if perms is not None else torch.randperm(TN, device=self.dev)
            for k in range(nmb):
                self.minibatch(perm[k * c.batch:(k + 1) * c.batch])
        return self.stats / (c.epochs * nmb)


class Trainer:
    """Rollouts on the GPU env (zero-copy: the policy reads the env's obs buffer) + Learner updates."""

    def __init__(self, env, cfg: PPOConfig, dev, seed: int = 0):
        torch.manual_seed(seed)
        self.env, self.cfg, self.dev = env, cfg, dev
        self.L = Learner(cfg, dev)
        self.obs = env.reset()
        self.inp = torch.zeros((cfg.n_envs, 4, 84, 84), dtype=torch.uint8, device=dev)
        self.a = torch.zeros(cfg.n_envs, dtype=torch.int64, device=dev)
        self.lp, self.v = torch.zeros(cfg.n_envs, device=dev), torch.zeros(cfg.n_envs, device=dev)
        # set on the device when a rollout step had more truncations than cfg.trunc_budget (checked per iteration)
        self.trunc_overflow = torch.zeros((), dtype=torch.bool, device=dev)
        self.pgraph = None
        if cfg.graph:
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(3):
                    self._policy()
            torch.cuda.current_stream(dev).wait_stream(s)
            self.pgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.pgraph, stream=s):
                self._policy()

    def _policy(self):
        a, lp, v = self.L.net.act(self.inp, self.cfg.channels_last)
        self.a.copy_(a); self.lp.copy_(lp); self.v.copy_(v)

    def collect(self):
        """One rollout of n_steps (train.py:393-435, device backend): obs, actions, log-probs, values, rewards,
        done flags; time-limit truncations add gamma * V(final obs) to the reward."""
        c, b, e = self.cfg, self.L.buf, self.env
        self.inp.copy_(self.obs)
        for t in range(c.n_steps):
            b.obs[t].copy_(self.inp)
            self.pgraph.replay() if self.pgraph is not None else self._policy()
            b.act[t].copy_(self.a); b.logp[t].copy_(self.lp); b.val[t].copy_(self.v)
            obs, rew, term, trunc, info = e.step(self.a)
            self.inp.copy_(obs)
            b.rew[t].copy_(rew)
            d = (term | trunc).float()
            (b.done[t + 1] if t + 1 < c.n_steps else b.next_done).copy_(d)
            self._bootstrap_truncations(t, trunc & ~term, info["final_obs"])
        self.obs = self.inp
        with torch.no_grad():
            _, nv = self.L.net(self.inp, c.channels_last)
        b.next_val.copy_(nv)

    def _bootstrap_truncations(self, t, tmask, final_obs):
        """SB3's time-limit bootstrap (train.py:416-421): r[t, i] += gamma * V(final_obs[i]) for the envs cut off
        by the time limit, without a host sync. A fixed number (trunc_budget) of such envs is gathered each step
        (torch.nonzero_static, padded with an out-of-range index whose contribution is masked to zero); a step
        with more sets trunc_overflow, which iterate() turns into an error rather than a silently missing
        bootstrap."""
        c, b = self.cfg, self.L.buf
        n = c.n_envs
        ti = torch.nonzero_static(tmask, size=c.trunc_budget, fill_value=n).squeeze(-1)
        valid = ti < n
        ti = ti.clamp(max=n - 1)
        with torch.no_grad():
            _, v = self.L.net(final_obs.index_select(0, ti), c.channels_last)
        b.rew[t].index_add_(0, ti, torch.where(valid, c.gamma * v, torch.zeros_like(v)))
        self.trunc_overflow |= tmask.sum() > c.trunc_budget

    def iterate(self):
        self.collect()
        stats = self.L.update()
        if bool(self.trunc_overflow):
            raise RuntimeError(f"a rollout step had more than trunc_budget={self.cfg.trunc_budget} time-limit "
                               "truncations; raise PPOConfig.trunc_budget")
        return stats
