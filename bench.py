"""Benchmark of the B200 env step (BASELINE.json metric: agent env-steps/s, skip 4, 84x84x4 obs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--envs E] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one process per GPU, env_offset = rank * E)

Workload = BASELINE config 1: E = 32768 envs per GPU on the synthetic NROM (seed 0), the 32 level names cycled,
skip 4, sticky 0.25, noop_max 30, maxpool, max_steps 2000, frame_stack 4, uniform random actions over 7.
`value` is device-timed (CUDA events on the stepping stream, barrier + synchronize on both sides, max over ranks)
with the actions already in HBM; `e2e` is the same steps through the FastVecEnv host API (pinned host actions
in, full stacked obs / rewards / dones / infos out, every step). The per-step working set (console slabs, VRAM,
PPU logs, frame stacks) is several GB, far above the 126 MB L2, so no L2 flush is inserted between steps.

--impl reference times the reference's own CPU engine (oracle/_ref/libfastmario.so, built from the reference's
csrc by oracle/Makefile) with all host threads on the same config; rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "fast-mario-env_b200")
METRIC = "agent env-steps/sec (skip 4, 84x84x4 obs)"
UNIT = "env-steps/s"
# algorithmic HBM bytes per env-step of each kernel of the step:
#   k_step   console state in and out (RAM+OAM+palette 2336 B and VRAM 2048 B each way, 37 scalar words each
#            way), actions and outputs (58 B) and the render job word (4 B)
#   k_render the frame-stack shift (frames 1..3 read and written to 0..2, 3 x 7056 B each way), the new 84x84
#            frame (7056 B) and the job word (the PPU logs it replays are the emulation kernel's intermediate
#            output, not counted)
ALGO_BYTES = {"k_step": 2 * (2336 + 2048) + 2 * 37 * 4 + 58 + 4, "k_render": 2 * 3 * 7056 + 7056 + 4}


def load_package():
    name = "fast_mario_env_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def workload(args):
    name = "config2 (divergence-stress image)" if getattr(args, "divergent", False) else "config1"
    return dict(workload=f"{name}: synthetic NROM seed 0, 32 levels cycled, skip 4, sticky 0.25, noop_max 30, "
                         "maxpool, max_steps 2000, frame_stack 4, uniform random actions",
                n_envs_per_gpu=args.envs, skip=4, frame_stack=4, maxpool=True, sticky=0.25, noop_max=30,
                max_steps=2000, l2="working set per step >> 126 MB L2 (no flush needed)")


def level_names(n):
    levels = [f"{w}-{s}" for w in range(1, 9) for s in range(1, 5)]
    return [levels[i % len(levels)] for i in range(n)]


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def profile_figure(kernel, key):
    """A per-env-step figure of `kernel` from its committed ncu summary (profiles/<kernel>_full_config1_4096.md,
    lines `key = value`): DRAM bytes (read + write) and thread-instructions of a small-case capture, per env-step,
    which grow in proportion to the envs."""
    p = os.path.join(ROOT, "profiles", f"{kernel}_full_config1_4096.md")
    if os.path.exists(p):
        for line in open(p):
            if line.startswith(key + " "):
                return float(line.split("=")[1])
    return None


def committed_traffic(kernel):
    return profile_figure(kernel, "traffic_per_env_step_bytes")


def issue_roofline(per_gpu_value, clk, sm_count):
    """The roof that binds this branchy integer interpreter: useful-lane issue slots. achieved = the step's
    thread-instructions per env-step (both kernels, from the committed ncu captures) x env-steps/s of one GPU;
    peak = SMs x 4 schedulers x 32 lanes x the median SM clock sampled during the timed region."""
    f_mhz = (clk or {}).get("sm_mhz") or 0.0
    if not f_mhz:
        return None
    per = {k: profile_figure(k, "thread_inst_per_env_step") for k in ("k_step", "k_render")}
    lanes = {k: profile_figure(k, "lanes_per_inst") for k in ("k_step", "k_render")}
    if any(v is None for v in per.values()):
        return None
    peak = sm_count * 4 * 32 * f_mhz * 1e6
    achieved = sum(per.values()) * per_gpu_value
    return {"bound": "issue", "unit": "thread-inst/s", "achieved": achieved, "peak": peak, "frac": achieved / peak,
            "per_kernel_frac": {k: v * per_gpu_value / peak for k, v in per.items()},
            "thread_inst_per_env_step": per,
            "warp_exec_efficiency": {k: (v / 32.0 if v else None) for k, v in lanes.items()},
            "sm_count": sm_count, "sm_mhz": f_mhz,
            "source": "thread-instructions per env-step and lanes per instruction from the committed ncu captures "
                      "(profiles/*_full_config1_4096.md); env-steps/s and clock from this run"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        loaded = [s for s in sm] or [0.0]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(rom, args, seconds=12.0):
    """The reference FastVecEnv engine (oracle/_ref) with all host threads, bounded sample."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref
    if not ref.available():
        return None
    cores = os.cpu_count() or 1
    n = 64 * cores
    levels = [(lambda w, s: (w, s, s + 1 if (w in (1, 2, 4, 7) and s >= 2) else s))(w, s)
              for w in range(1, 9) for s in range(1, 5)]
    lv = [levels[i % 32] for i in range(n)]
    e = ref.RefVecEnv(rom, lv, n, seed=0, sticky=0.25, noop_max=30, maxpool=True, max_steps=2000, n_threads=cores)
    e.reset()
    rng = np.random.default_rng(1)
    for _ in range(5):
        e.step(rng.integers(0, 7, n))
    steps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        e.step(rng.integers(0, 7, n))
        steps += 1
    dt = time.perf_counter() - t0
    e.close()
    return {"value": n * steps / dt, "unit": UNIT, "cores": cores, "kind": "reference",
            "sample": f"{steps} steps x {n} envs ({dt:.1f} s) of the reference FastVecEnv C++ thread pool "
                      f"(oracle/_ref/libfastmario.so, {cores} threads), same config"}


def reference_cuda(rom, E, steps, warmup, dev):
    """The reference's own GPU engine (CudaVecEnv, one thread per env, NVRTC-compiled from baseline/_ref) and
    this engine, both at maxpool=False (the only setting the reference's GPU path supports), same levels,
    seeds and actions otherwise. Device-timed steps with the actions already on the device."""
    import torch
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "fast_mario_env")):
        return {"unavailable": "baseline/_ref not installed"}
    sys.path.insert(0, ref_dir)
    try:
        from fast_mario_env.cuda.vec_env import CudaVecEnv as RefCuda
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference CudaVecEnv import failed: {e}"}
    fme = load_package()
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    acts = torch.randint(0, 7, (warmup + steps, E), dtype=torch.int64, device=dev, generator=g)
    out = {"config": "the workload above with maxpool=False", "n_envs": E, "steps": steps}
    with tempfile.NamedTemporaryFile(suffix=".nes", delete=False) as f:
        f.write(rom)
        rom_path = f.name
    try:
        for name, make in (("reference_cudavecenv", lambda: RefCuda(level_names(E), E, seed=0, sticky=0.25, noop_max=30,
                                                                     max_steps=2000, skip=4, device=dev, rom_path=rom_path)),
                           ("ours", lambda: fme.CudaVecEnv(level_names(E), E, seed=0, sticky=0.25, noop_max=30,
                                                           max_steps=2000, skip=4, frame_stack=4, maxpool=False,
                                                           device=dev, rom=rom))):
            env = make()
            env.reset()
            for t in range(warmup):
                env.step(acts[t])
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for t in range(warmup, warmup + steps):
                env.step(acts[t])
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1) / steps
            out[name] = {"value": E / (ms / 1000.0), "ms_per_step": ms, "unit": UNIT}
            if hasattr(env, "close"):
                env.close()
            del env
            torch.cuda.empty_cache()
    finally:
        os.unlink(rom_path)
    return out


def run_ppo(args, rank, world, dev, dist):
    """PPO samples/s — rollouts on this engine (4096 envs per GPU x 128 steps) and the update
    (GAE kernel, 4 epochs of minibatch 1024 with advantage normalisation kernel, Nature-CNN fwd/bwd, Adam, CUDA
    graph; gradients averaged over ranks with NCCL). Device-timed with CUDA events, max over ranks."""
    import torch
    fme = load_package()
    from fast_mario_env_b200 import ppo, shard
    from fast_mario_env_b200.synth_rom import build_rom
    E = args.ppo_envs
    torch.backends.cudnn.benchmark = True   # as the reference trainer (train.py main)
    rom = build_rom(0)
    env = fme.CudaVecEnv(level_names(E), E, seed=0, sticky=0.25, noop_max=30, max_steps=2000, skip=4, frame_stack=4,
                         maxpool=True, device=dev, rom=rom, env_offset=shard.env_offset(rank, E))
    cfg = ppo.PPOConfig(n_envs=E, n_steps=128, batch=1024, epochs=4)
    tr = ppo.Trainer(env, cfg, dev, seed=rank)
    iters = max(1, args.steps // 5)
    for _ in range(1):
        tr.iterate()  # warm-up (cudnn autotune, graph pools)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    clocks = ClockSampler(torch.cuda.current_device())
    e0, e1, em = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    coll = 0.0
    e0.record()
    for _ in range(iters):
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(); tr.collect(); c1.record()
        tr.L.update()
        c1.synchronize()
        coll += c0.elapsed_time(c1)
    e1.record()
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    if bool(tr.trunc_overflow):
        raise RuntimeError("time-limit truncations exceeded PPOConfig.trunc_budget in a rollout step")
    ms = e0.elapsed_time(e1)
    ms_max = shard.max_over_ranks(ms, device=dev)
    samples = world * E * cfg.n_steps * iters
    if rank == 0:
        print(json.dumps({"metric": "PPO samples/sec (config 4)", "value": samples / (ms_max / 1000.0), "unit": "samples/s",
                          "n_gpus": world, "iterations": iters, "ms_per_iteration": ms_max / iters,
                          "rollout_ms_per_iteration": coll / iters, "clocks": clk, "higher_is_better": True,
                          "scaling": "weak",
                          "dtype": "fp32", "data": "synthetic",
                          "config": {"workload": "config4: Nature-CNN PPO on config-1 envs", "n_envs_per_gpu": E,
                                     "n_steps": 128, "epochs": 4, "minibatch": 1024, "gamma": 0.99, "lam": 0.95,
                                     "parallelism": f"dp{world} (NCCL gradient all-reduce inside the captured "
                                                    "minibatch graph)" if world > 1 else "dp1"}}))
    tr.L.graph = None   # graphs holding NCCL calls are released before the process group is destroyed
    tr.pgraph = None
    del tr
    torch.cuda.synchronize(dev)
    env.close()


def run_reference_ppo(args):
    """The reference trainer itself (baseline/_ref, `python -m fast_mario_env.ppo.train`, unmodified) in its
    throughput mode on its CUDA env backend with the config-4 hyper-parameters and this synthetic ROM; its
    reported fps (env steps = samples per second) is the line's value."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "fast_mario_env")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}))
        return
    load_package()
    from fast_mario_env_b200.synth_rom import build_rom
    with tempfile.NamedTemporaryFile(suffix=".nes", delete=False) as f:
        f.write(build_rom(0))
        rom_path = f.name
    cmd = [sys.executable, "-m", "fast_mario_env.ppo.train", "--env-backend", "cuda", "--n-envs", str(args.ppo_envs),
           "--groups", "1", "--n-steps", "128", "--batch", "1024", "--epochs", "4", "--gamma", "0.99", "--lam", "0.95",
           "--bench", str(max(10, 4 * args.steps)), "--eval-every", "1e12", "--no-tb", "--rom", rom_path]
    env = dict(os.environ, PYTHONPATH=ref_dir + os.pathsep + os.environ.get("PYTHONPATH", ""))
    try:
        r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=1200)
    finally:
        os.unlink(rom_path)
    done = [l for l in r.stdout.splitlines() if l.startswith("DONE ")]
    if r.returncode != 0 or not done:
        print(json.dumps({"impl": "reference", "unavailable": f"reference trainer failed (rc {r.returncode}): "
                                                              f"{(r.stderr or r.stdout).strip().splitlines()[-1:]}"}))
        return
    res = json.loads(done[-1][5:])
    print(json.dumps({"impl": "reference", "metric": "PPO samples/sec (config 4)", "value": float(res["fps"]),
                      "unit": "samples/s", "n_gpus": 1, "higher_is_better": True, "scaling": "weak", "dtype": "fp32",
                      "data": "synthetic", "config": {"workload": "config4 via the reference trainer (cuda env backend, "
                                                                  "maxpool off: the only setting it supports)",
                                                      "n_envs_per_gpu": args.ppo_envs, "n_steps": 128, "epochs": 4,
                                                      "minibatch": 1024},
                      "e2e": {"value": float(res["fps"]), "unit": "samples/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}))


def run_reference(args, rank):
    if rank != 0:
        return
    if args.ppo:
        run_reference_ppo(args)
        return
    load_package()
    from fast_mario_env_b200.synth_rom import build_rom
    rom = build_rom(0)
    cb = cpu_baseline(rom, args, seconds=max(5.0, 2.0 * args.steps))
    if cb is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libfastmario.so not built"}))
        return
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": workload(args),
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--envs", type=int, default=32768)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ppo", action="store_true", help="config 4: PPO samples/s instead of env-steps/s")
    ap.add_argument("--ppo-envs", type=int, default=4096)
    ap.add_argument("--divergent", action="store_true",
                    help="config 2: the divergence-stress image (controller/LFSR-dependent control flow and sprites)")
    ap.add_argument("--ref-gpu", action="store_true",
                    help="time the reference's CudaVecEnv (baseline/_ref) against this engine at maxpool=False "
                         "(on by default at one GPU; kept for compatibility)")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip the reference CudaVecEnv arm that the default 1-GPU run times beside this engine")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    fme = load_package()
    from fast_mario_env_b200.synth_rom import build_rom
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from fast_mario_env_b200 import shard
    if args.ppo:
        run_ppo(args, rank, world, dev, dist)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    rom = build_rom(0, divergence=args.divergent)
    E = args.envs
    off = shard.env_offset(rank, E)
    env = fme.CudaVecEnv(level_names(E), E, seed=0, sticky=0.25, noop_max=30, max_steps=2000, skip=4, frame_stack=4,
                         maxpool=True, device=dev, rom=rom, env_offset=off)
    total = args.warmup + args.steps
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    acts = torch.randint(0, 7, (total, E), dtype=torch.int64, device=dev, generator=g)
    stream = torch.cuda.current_stream(dev)
    env.reset()
    for t in range(args.warmup):
        env.step(acts[t])
    torch.cuda.synchronize(dev)
    env.check()
    instr0, emu0 = env.work_counters()
    frames0 = env.frames
    if dist:
        dist.barrier()
    # per step: an event before it and one between its two kernels (fme_step_marked), for the per-kernel times
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for e_ in starts + mids:
        e_.record(stream)  # creates the events outside the timed region
    clocks = ClockSampler(local)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i, t in enumerate(range(args.warmup, total)):
        starts[i].record(stream)
        env.step(acts[t], mark=mids[i])
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    emu_ms = sum(starts[i].elapsed_time(mids[i]) for i in range(args.steps)) / args.steps
    rend_ms = sum(mids[i].elapsed_time(starts[i + 1] if i + 1 < args.steps else ev1) for i in range(args.steps)) / args.steps
    env.check()
    instr1, emu1 = env.work_counters()
    frames1 = env.frames
    env_steps = E * args.steps
    work = {"instructions_per_env_step": (instr1 - instr0) / env_steps,
            "emulated_frames_per_env_step": (emu1 - emu0) / env_steps,
            "reference_frames_per_env_step": (frames1 - frames0) / env_steps,
            "note": "device counters over the timed steps: 6502 instructions executed (idle-loop fast-forward and "
                    "sprite-0 poll skip excluded) and NES frames run by the step kernel; reference_frames also "
                    "counts the no-op-start frames served from the reset cache and re-emulated frames, as fm_frames"}
    if dist:
        dist.barrier()
    ms_max = shard.max_over_ranks(ms, device=dev)
    value = shard.job_throughput(world, E, args.steps, ms_max)
    ms_step = ms_max / args.steps
    kernel_ms = {"k_step": emu_ms, "k_render": rend_ms}

    # ---- end to end through the C ABI with host buffers (FastVecEnv.step_arrays = fme_step between a
    # pinned-host action upload and pinned-host copies of every output; final_obs rows of ended envs)
    e2e = None
    if not args.no_e2e:
        fenv = fme.FastVecEnv(level_names(E), E, seed=0, sticky=0.25, noop_max=30, max_steps=2000, maxpool=True,
                              rom=rom, env_offset=off, device=dev)
        fenv.reset()
        hacts = np.random.default_rng(99 + rank).integers(0, 7, (total, E))
        for t in range(args.warmup):
            fenv.step_arrays(hacts[t])
        if dist:
            dist.barrier()
        n_final = 0
        t0 = time.perf_counter()
        for t in range(args.warmup, total):
            n_final += len(fenv.step_arrays(hacts[t])[5])
        dt = time.perf_counter() - t0
        fenv.check()
        dt_max = shard.max_over_ranks(dt, device=dev)
        h2d = E * 8
        # FastVecEnv reuses one pinned obs buffer and passes FME_HOST_OBS_IN_PLACE: frames 1..3 of every stack
        # move down inside it on the host, so each step copies one new 84x84 frame per env, the scalars, and
        # the full stacks of the ended envs' final_obs rows
        d2h = E * (84 * 84 + 4 + 1 + 1 + 4 * 10 + 8 + 4) + (n_final * 4 * 84 * 84) // args.steps
        e2e = {"value": shard.job_throughput(world, E, args.steps, dt_max * 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "api": "FastVecEnv.step_arrays: fme_step_to_host with pinned host actions in and every output "
                      "(stacked obs, rew, term, trunc, info, episode stats, final_obs rows) in pinned host "
                      "memory; the stacks shift in place on the host, so only each env's new frame crosses"}
        fenv.close()

    peak, peak_kind = read_peaks()
    top = max(kernel_ms, key=kernel_ms.get)  # the dominant kernel of the step
    achieved = ALGO_BYTES[top] * E / (kernel_ms[top] / 1000.0) / 1e9
    traffic_per_step = committed_traffic(top)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic_per_step * E if traffic_per_step else None,
                "kernel": top, "kernel_ms": kernel_ms,
                "kernel_ms_note": "spans per step, not single-launch durations: k_step = the step's start until "
                                  "the last of its 4 concurrent emulation slices ends (earlier slices' renders "
                                  "overlap it); k_render = the rest of the step (the last slice's render)",
                "algorithmic_bytes_per_env_step": ALGO_BYTES[top],
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
                "note": "the env step is an issue-bound integer interpreter: the HBM fraction is reported as the "
                        "contract asks, the binding roof is roofline.issue"}
    work["emulated_instructions_per_s"] = work["instructions_per_env_step"] * value
    issue = issue_roofline(value / world, clk, torch.cuda.get_device_properties(dev).multi_processor_count)
    if issue is not None:
        roofline["issue"] = issue
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(rom, args)
    ref_cuda = None
    if rank == 0 and world == 1 and not args.no_ref_gpu:
        ref_cuda = reference_cuda(rom, E, args.steps, args.warmup, dev)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": workload(args),
                "parallelism": f"env shards by env_offset x{world}, no collective",
                # per step and GPU: an emulation and a render launch for each of the library's step slices
                # (4, or one per 32-env group below 128 envs)
                "gpu_launches": 2 * min((E + 31) // 32, 4) * args.steps,
                "roofline": roofline, "cpu_baseline": cb, "e2e": e2e, "clocks": clk, "work": work}
        if ref_cuda is not None:
            line["reference_cuda"] = ref_cuda
        print(json.dumps(line))
    env.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
