"""Data-parallel PPO minibatch step with the NCCL gradient all-reduce captured inside the CUDA graph (two GPUs,
one process each; skipped with fewer devices).

* Both ranks given the same minibatch: the averaged gradient is each rank's own gradient ((g + g) / 2 == g in
  fp32), so the captured two-rank step must equal a single-rank captured step from the same weights, bit for bit.
* Ranks given different minibatches: the parameters after the step must be identical on both ranks (the
  collective ran inside the graph) and differ from the same-data result.
The reference trainer captures its own update step the same way (src/fast_mario_env/ppo/train.py:169-196).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp
from conftest import PKG_DIR, PKG_NAME

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _load():
    import importlib.util
    import sys
    if PKG_NAME not in sys.modules:
        spec = importlib.util.spec_from_file_location(PKG_NAME, os.path.join(PKG_DIR, "__init__.py"),
                                                      submodule_search_locations=[PKG_DIR])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[PKG_NAME] = mod
        spec.loader.exec_module(mod)
    from fast_mario_env_b200 import ppo
    return ppo


def _fill(L, seed):
    g = torch.Generator(device=L.dev)
    g.manual_seed(seed)
    b = L.buf
    b.obs.copy_(torch.randint(0, 256, b.obs.shape, generator=g, device=L.dev, dtype=torch.int64).to(torch.uint8))
    b.act.copy_(torch.randint(0, 7, b.act.shape, generator=g, device=L.dev))
    b.logp.copy_(-torch.rand(b.logp.shape, generator=g, device=L.dev) * 2.0)
    L.adv.copy_(torch.randn(L.adv.shape, generator=g, device=L.dev))
    L.ret.copy_(torch.randn(L.ret.shape, generator=g, device=L.dev))


def _params(L):
    return torch.cat([p.detach().reshape(-1) for p in L.params]).cpu().numpy()


def _worker(rank, world, port, q):
    import torch.distributed as dist
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.deterministic = True   # bit-exact comparisons need deterministic convolution gradients
    torch.backends.cudnn.benchmark = False
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ppo = _load()
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    out = {}
    try:
        cfg = ppo.PPOConfig(n_envs=64, n_steps=16, batch=256, epochs=1, graph=True)
        idx = torch.arange(256, device=dev) * 3 % (cfg.n_envs * cfg.n_steps)
        for name, data_seed in (("same", 5), ("diff", 100 + rank)):
            torch.manual_seed(0)
            L = ppo.Learner(cfg, dev, net=ppo.NatureAC(7))
            assert L.world == world and L.graph is not None
            _fill(L, data_seed)
            L.minibatch(idx)
            torch.cuda.synchronize(dev)
            out[name] = _params(L)
            L.graph = None   # a graph holding NCCL calls is released before the process group goes
            del L
        torch.cuda.synchronize(dev)
        dist.barrier()
    finally:
        dist.destroy_process_group()
    if rank == 0:   # the same step on one rank (world 1), same weights and data as "same"
        torch.manual_seed(0)
        cfg = ppo.PPOConfig(n_envs=64, n_steps=16, batch=256, epochs=1, graph=True)
        L = ppo.Learner(cfg, dev, net=ppo.NatureAC(7))
        assert L.world == 1
        _fill(L, 5)
        L.minibatch(torch.arange(256, device=dev) * 3 % (cfg.n_envs * cfg.n_steps))
        torch.cuda.synchronize(dev)
        out["single"] = _params(L)
    q.put((rank, out))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_captured_data_parallel_step_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(res[0]["same"], res[1]["same"])
    assert np.array_equal(res[0]["same"], res[0]["single"]), "two-rank step with equal data differs from one rank"
    assert np.array_equal(res[0]["diff"], res[1]["diff"]), "ranks out of sync after the captured step"
    assert not np.array_equal(res[0]["diff"], res[0]["same"])
