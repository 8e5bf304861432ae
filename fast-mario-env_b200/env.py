"""Python API of the B200 engine, mirroring the reference's env classes on top of the C ABI (include/fme.h).

* `CudaVecEnv` - device-tensor API of the reference's CudaVecEnv (src/fast_mario_env/cuda/vec_env.py:238-393):
  reset() -> obs (N, k, 84, 84) uint8 CUDA tensor; step(actions int64 CUDA tensor) -> obs, rew f32, term bool,
  trunc bool, info (dict of int32 (N,) tensors + ep_ret f64, ep_len i32, final_obs). Tensors are the env's own
  buffers, overwritten by the next call. Unlike the reference it also supports maxpool=True and any
  frame_stack.
* `FastVecEnv` - numpy API of the reference's FastVecEnv (src/fast_mario_env/env.py:113-266): step_async /
  step_wait with host arrays and per-env info dicts (episode, final_obs, TimeLimit.truncated). It runs the
  same GPU engine: actions go host->device, outputs device->host through pinned buffers.
* `RawNES` / `RawNESBatch` - raw consoles (env.py:58-90) for frame-level fidelity checks.

Seeding follows the reference: env i uses numpy's PCG64 stream default_rng(seed*1000 + env_offset + i)
(env.py:50-55, 155-156), so a run here is step-for-step identical to the reference on the same ROM.
"""
from __future__ import annotations

import ctypes
import json
import os
import time

import numpy as np

from . import _native as N
from .rom import check_rom, decode_level, load_rom

OBS_HW = 84
N_ACTIONS = 7
SIMPLE_MOVEMENT = [["NOOP"], ["right"], ["right", "A"], ["right", "B"], ["right", "A", "B"], ["A"], ["left"]]
INFO_FIELDS = ("x_pos", "flag_get", "life", "score", "time", "world", "stage", "coins", "y_pos", "status")
INFO_KEYS = ("x_pos", "flag_get", "life", "score", "time", "world", "stage")


def palette_rgb() -> np.ndarray:
    """nes-py master palette as (64, 3) uint8 RGB."""
    p = np.zeros(64, np.uint32)
    N.lib().fme_palette(N.ptr(p))
    return np.stack([(p >> 16) & 255, (p >> 8) & 255, p & 255], -1).astype(np.uint8)


def gray_lut() -> np.ndarray:
    """palette value (0-255, taken & 63) -> gray, cv2.cvtColor(RGB2GRAY) fixed point (14-bit BT.601 weights,
    round half up), as the reference computes it (env.py:42-47)."""
    rgb = palette_rgb().astype(np.int64)
    g = (rgb[:, 0] * 4899 + rgb[:, 1] * 9617 + rgb[:, 2] * 1868 + (1 << 13)) >> 14
    return np.ascontiguousarray(g[np.arange(256) & 63], np.uint8)


def rng_state(seed: int) -> list[int]:
    """numpy PCG64 state of default_rng(seed) as (state_hi, state_lo, inc_hi, inc_lo, has_uint32, uinteger)."""
    st = np.random.default_rng(seed).bit_generator.state
    s, inc = st["state"]["state"], st["state"]["inc"]
    m = (1 << 64) - 1
    return [s >> 64, s & m, inc >> 64, inc & m, st["has_uint32"], st["uinteger"]]


def _torch():
    import torch
    return torch


def _rom_bytes(rom, rom_path) -> bytes:
    if rom is None:
        return load_rom(rom_path)
    data = bytes(rom)
    check_rom(data)
    return data


class CudaVecEnv:
    """N envs stepped by the B200 engine; device-tensor API (see module docstring).

    Args follow the reference CudaVecEnv / FastVecEnv: level ('w-s' or a list of N levels), n_envs, seed, sticky,
    noop_max, max_steps, skip, frame_stack, maxpool, env_offset, device; plus rom (iNES bytes) or rom_path, and
    log_capacity (PPU log records per frame, default 2048).
    """

    def __init__(self, level="1-1", n_envs=1024, seed=0, sticky=0.0, noop_max=0, max_steps=2000, skip=4,
                 frame_stack=4, maxpool=False, device="cuda", rom=None, rom_path=None, env_offset=0,
                 log_capacity=0, hack_cap=0, boot_cap=0):
        torch = _torch()
        if not 1 <= skip <= 16:
            raise ValueError("skip must be in 1..16")
        if frame_stack < 1:
            raise ValueError("frame_stack must be >= 1")
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise ValueError("CudaVecEnv needs a CUDA device (there is no CPU path)")
        di = self.dev.index if self.dev.index is not None else torch.cuda.current_device()
        self.dev = torch.device("cuda", di)
        self.n = n = int(n_envs)
        self.num_envs = n
        self.k = frame_stack
        levels = [level] * n if isinstance(level, (str, tuple)) else list(level)
        if len(levels) != n:
            raise ValueError(f"got {len(levels)} levels for {n} envs")
        self.levels = levels
        self._rom = np.frombuffer(_rom_bytes(rom, rom_path), np.uint8).copy()
        lv = np.array([decode_level(x) for x in levels], np.int32).reshape(-1)
        self._rng = np.array([rng_state(seed * 1000 + env_offset + i) for i in range(n)], np.uint64).reshape(-1)
        self._lut = gray_lut()
        cfg = N.FmeConfig(n_envs=n, skip=skip, max_steps=max_steps, noop_max=int(noop_max), maxpool=int(bool(maxpool)),
                          frame_stack=frame_stack, sticky=float(sticky), device=di, log_capacity=int(log_capacity),
                          hack_cap=int(hack_cap), boot_cap=int(boot_cap))
        L = N.lib()
        with torch.cuda.device(di):
            torch.zeros(1, device=self.dev)  # make torch's primary context current before the library runs
            h = ctypes.c_void_p()
            N.check(L.fme_create(ctypes.byref(cfg), N.ptr(self._rom), len(self._rom), N.ptr(lv), N.ptr(self._lut),
                                 N.ptr(self._rng), ctypes.byref(h)), "fme_create")
        self.h = h
        z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=self.dev)  # noqa: E731
        self.obs = z(n, frame_stack, OBS_HW, OBS_HW, dt=torch.uint8)
        self.final_obs = z(n, frame_stack, OBS_HW, OBS_HW, dt=torch.uint8)
        self.rew = z(n, dt=torch.float32)
        self.term = z(n, dt=torch.bool)
        self.trunc = z(n, dt=torch.bool)
        self.info_t = z(n, len(INFO_FIELDS), dt=torch.int32)
        self.ep_ret = z(n, dt=torch.float64)
        self.ep_len = z(n, dt=torch.int32)
        self.actions = z(n, dt=torch.int64)
        bufs = N.FmeBuffers(*[t.data_ptr() for t in (self.obs, self.final_obs, self.rew, self.term, self.trunc,
                                                        self.info_t, self.ep_ret, self.ep_len)])
        N.check(L.fme_set_buffers(self.h, ctypes.byref(bufs)), "fme_set_buffers")
        self.info = {k: self.info_t[:, i] for i, k in enumerate(INFO_FIELDS)}
        self.info["ep_ret"] = self.ep_ret
        self.info["ep_len"] = self.ep_len
        self.info["final_obs"] = self.final_obs

    def _stream(self):
        return ctypes.c_void_p(_torch().cuda.current_stream(self.dev).cuda_stream)

    def reset(self):
        N.check(N.lib().fme_reset(self.h, self._stream()), "fme_reset")
        return self.obs

    def step(self, actions, mark=None):
        """mark: optional torch.cuda.Event, recorded between the emulation and the render kernel."""
        torch = _torch()
        if not isinstance(actions, torch.Tensor):
            actions = torch.as_tensor(np.asarray(actions), dtype=torch.int64)
        if actions.dtype != torch.int64 or actions.device != self.dev or not actions.is_contiguous():
            actions = actions.to(self.dev, torch.int64).contiguous()
        if actions.numel() != self.n:
            raise ValueError(f"expected {self.n} actions, got {actions.numel()}")
        if actions.data_ptr() != self.actions.data_ptr():
            self.actions.copy_(actions.view(-1))
        if mark is None:
            N.check(N.lib().fme_step(self.h, N.ptr(self.actions), self._stream()), "fme_step")
        else:
            N.check(N.lib().fme_step_marked(self.h, N.ptr(self.actions), self._stream(), ctypes.c_void_p(mark.cuda_event)),
                    "fme_step_marked")
        return self.obs, self.rew, self.term, self.trunc, self.info

    def ram(self):
        """(N, 2048) uint8 RAM of every env (a copy)."""
        torch = _torch()
        out = torch.empty(self.n, 0x800, dtype=torch.uint8, device=self.dev)
        N.check(N.lib().fme_ram_all(self.h, N.ptr(out), self._stream()), "fme_ram_all")
        return out

    def check(self):
        """Synchronise and raise if a device-side status bit is set (log overflow, frame caps, bad actions)."""
        _torch().cuda.synchronize(self.dev)
        st = ctypes.c_uint32()
        N.check(N.lib().fme_poll_error(self.h, ctypes.byref(st)), "fme_poll_error")
        if st.value:
            raise N.FmeError(f"device status {st.value:#x}: {N.status_text(st.value)}")
        return 0

    @property
    def frames(self) -> int:
        _torch().cuda.synchronize(self.dev)
        v = ctypes.c_int64()
        N.check(N.lib().fme_frames(self.h, ctypes.byref(v)), "fme_frames")
        return int(v.value)

    def bad_ops(self) -> int:
        _torch().cuda.synchronize(self.dev)
        v = ctypes.c_int64()
        N.check(N.lib().fme_bad_ops(self.h, ctypes.byref(v)), "fme_bad_ops")
        return int(v.value)

    def work_counters(self) -> tuple[int, int]:
        """(6502 instructions executed, NES frames run) by all envs' steps so far (fme_work_counters)."""
        _torch().cuda.synchronize(self.dev)
        i, f = ctypes.c_int64(), ctypes.c_int64()
        N.check(N.lib().fme_work_counters(self.h, ctypes.byref(i), ctypes.byref(f)), "fme_work_counters")
        return int(i.value), int(f.value)

    def bytes_per_env(self) -> float:
        own = int(N.lib().fme_env_bytes(self.h))
        outs = sum(t.numel() * t.element_size() for t in (self.obs, self.final_obs, self.rew, self.term, self.trunc,
                                                          self.info_t, self.ep_ret, self.ep_len, self.actions))
        return own + outs / self.n

    def close(self):
        h, self.h = getattr(self, "h", None), None
        if h:
            N.lib().fme_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _monitor_file(path: str) -> str:
    """Where a monitor writes: an existing directory gets monitor.monitor.csv inside it, any other path gains the
    .monitor.csv suffix unless it already ends with it (the file name SB3's load_results looks for)."""
    suffix = ".monitor.csv"
    if path.endswith(suffix):
        return path
    return os.path.join(path, "monitor" + suffix) if os.path.isdir(path) else path + suffix


class MonitorCSV:
    """Episode log in SB3's VecMonitor CSV format, written as the reference FastVecEnv writes it
    (src/fast_mario_env/env.py:93-110): a '#'-prefixed JSON line (t_start, env_id), the header
    r,l,t,x_pos,flag_get, then one row per finished episode, flushed at once so a crash loses nothing."""

    COLUMNS = ("r", "l", "t", "x_pos", "flag_get")

    def __init__(self, path: str):
        target = _monitor_file(path)
        os.makedirs(os.path.dirname(os.path.abspath(target)), exist_ok=True)
        self.f = open(target, "w")
        self._emit("#" + json.dumps({"t_start": time.time(), "env_id": "None"}))
        self._emit(",".join(self.COLUMNS))

    def _emit(self, line: str) -> None:
        self.f.write(line + "\n")
        self.f.flush()

    def write(self, episode: dict) -> None:
        self._emit(",".join(str(episode[c]) for c in self.COLUMNS))

    def close(self) -> None:
        self.f.close()


class FastVecEnv:
    """The reference FastVecEnv API (numpy in / numpy out, info dicts) served by the GPU engine.

    step_async() copies the actions to the device and enqueues the step; step_wait() waits for it and copies
    obs / rewards / dones / infos back through pinned host buffers. n_threads is accepted for compatibility
    and ignored.
    """

    def __init__(self, level="1-1", n_envs=8, seed=0, frame_stack=4, sticky=0.0, noop_max=0, max_steps=2000,
                 maxpool=False, skip=4, n_threads=None, copy_obs=True, rom=None, rom_path=None, monitor_path=None,
                 env_offset=0, device="cuda", log_capacity=0):
        torch = _torch()
        self.env = CudaVecEnv(level, n_envs, seed=seed, sticky=sticky, noop_max=noop_max, max_steps=max_steps,
                              skip=skip, frame_stack=frame_stack, maxpool=maxpool, device=device, rom=rom,
                              rom_path=rom_path, env_offset=env_offset, log_capacity=log_capacity)
        self.n = self.num_envs = n_envs
        self.k = frame_stack
        self.copy_obs = copy_obs
        self.n_threads = n_threads
        pin = dict(pin_memory=True)
        self._act = torch.zeros(n_envs, dtype=torch.int64, **pin)
        self._obs = torch.zeros(n_envs, frame_stack, OBS_HW, OBS_HW, dtype=torch.uint8, **pin)
        self._rew = torch.zeros(n_envs, dtype=torch.float32, **pin)
        self._term = torch.zeros(n_envs, dtype=torch.bool, **pin)
        self._trunc = torch.zeros(n_envs, dtype=torch.bool, **pin)
        self._info = torch.zeros(n_envs, len(INFO_FIELDS), dtype=torch.int32, **pin)
        self._epr = torch.zeros(n_envs, dtype=torch.float64, **pin)
        self._epl = torch.zeros(n_envs, dtype=torch.int32, **pin)
        self._event = torch.cuda.Event()
        # the pinned obs buffer always holds the stacks of the last step, so the library shifts it in place
        self._hout = N.FmeHostOut(*[t.data_ptr() for t in (self._obs, self._rew, self._term, self._trunc, self._info,
                                                            self._epr, self._epl)], N.FME_HOST_OBS_IN_PLACE)
        self.monitor = MonitorCSV(monitor_path) if monitor_path else None
        self.t0 = time.time()
        self._pending = False

    @property
    def frames(self) -> int:
        return self.env.frames

    def bad_ops(self) -> int:
        return self.env.bad_ops()

    def bytes_per_env(self) -> float:
        return self.env.bytes_per_env()

    def _out(self):
        o = self._obs.numpy()
        return o.copy() if self.copy_obs else o

    def reset(self):
        self.env.reset()
        self._obs.copy_(self.env.obs, non_blocking=True)
        self._event.record()
        self._event.synchronize()
        return self._out()

    def step_async(self, actions):
        a = np.ascontiguousarray(np.asarray(actions).reshape(-1), np.int64)
        if a.shape[0] != self.n:
            raise ValueError(f"expected {self.n} actions, got {a.shape[0]}")
        self._act.numpy()[:] = a
        e = self.env
        e.actions.copy_(self._act, non_blocking=True)
        # the step, with each env slice's outputs copied to the pinned host arrays as soon as it is done
        N.check(N.lib().fme_step_to_host(e.h, N.ptr(e.actions), ctypes.byref(self._hout), e._stream()),
                "fme_step_to_host")
        self._event.record()
        self._pending = True

    def step_wait(self):
        if self._pending:
            self._event.synchronize()
            self._pending = False
        term = self._term.numpy().copy()
        trunc = self._trunc.numpy().copy()
        inf = self._info.numpy().tolist()
        ended = np.flatnonzero(term | trunc)
        fin = {}
        if len(ended):  # final_obs only for the envs whose episode ended (usually a small fraction)
            idx = _torch().from_numpy(ended).to(self.env.dev)
            rows = self.env.final_obs.index_select(0, idx).cpu().numpy()
            fin = {int(i): rows[k] for k, i in enumerate(ended)}
        epr, epl = self._epr.numpy(), self._epl.numpy()
        infos = []
        for i in range(self.n):
            r = inf[i]
            info = {"x_pos": r[0], "flag_get": bool(r[1]), "life": r[2], "score": r[3], "time": r[4],
                    "world": r[5], "stage": r[6]}
            if term[i] or trunc[i]:
                info["final_obs"] = fin[i]
                info["TimeLimit.truncated"] = bool(trunc[i] and not term[i])
                ep = dict(r=round(float(epr[i]), 6), l=int(epl[i]), t=round(time.time() - self.t0, 6),
                          x_pos=info["x_pos"], flag_get=info["flag_get"])
                info["episode"] = ep
                if self.monitor:
                    self.monitor.write(ep)
            infos.append(info)
        return self._out(), self._rew.numpy().copy(), term, trunc, infos

    def step(self, actions):
        self.step_async(actions)
        return self.step_wait()

    def step_arrays(self, actions):
        """One step with host buffers and no per-env Python objects, at the level of the reference's
        fm_step_async + fm_step_wait (fastmario.cpp:599-617): actions in, then (obs, rew, term, trunc, info,
        final_obs) where obs/rew/info are views of the pinned host buffers (valid until the next step),
        info is (N, len(INFO_FIELDS)) int32 and final_obs maps env index -> its final stacked frame
        for the envs whose episode ended."""
        self.step_async(actions)
        self._event.synchronize()
        self._pending = False
        term = self._term.numpy()
        trunc = self._trunc.numpy()
        ended = np.flatnonzero(term | trunc)
        fin = {}
        if len(ended):
            idx = _torch().from_numpy(ended).to(self.env.dev)
            rows = self.env.final_obs.index_select(0, idx).cpu().numpy()
            fin = {int(i): rows[k] for k, i in enumerate(ended)}
        return self._obs.numpy(), self._rew.numpy(), term, trunc, self._info.numpy(), fin

    def ram(self, i: int) -> np.ndarray:
        out = np.zeros(0x800, np.uint8)
        _torch().cuda.synchronize(self.env.dev)
        N.check(N.lib().fme_env_ram(self.env.h, int(i), N.ptr(out)), "fme_env_ram")
        return out

    def check(self):
        return self.env.check()

    def close(self):
        self.env.close()
        if self.monitor:
            self.monitor.close()
            self.monitor = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class RawNESBatch:
    """n raw consoles on the GPU (the batched form of the reference's RawNES, env.py:58-90)."""

    def __init__(self, rom_bytes: bytes, n: int = 1, device="cuda", log_capacity=0):
        torch = _torch()
        check_rom(bytes(rom_bytes))
        self.dev = torch.device(device)
        di = self.dev.index if self.dev.index is not None else torch.cuda.current_device()
        self.dev = torch.device("cuda", di)
        self.n = n
        self._rom = np.frombuffer(bytes(rom_bytes), np.uint8).copy()
        with torch.cuda.device(di):
            torch.zeros(1, device=self.dev)
            h = ctypes.c_void_p()
            N.check(N.lib().fme_raw_create(N.ptr(self._rom), len(self._rom), n, di, int(log_capacity), ctypes.byref(h)),
                    "fme_raw_create")
        self.h = h
        self._btn = torch.zeros(n, dtype=torch.uint8, device=self.dev)
        self._ram = torch.zeros(n, 0x800, dtype=torch.uint8, device=self.dev)
        self._scr = torch.zeros(n, 240, 256, dtype=torch.uint8, device=self.dev)

    def _stream(self):
        return ctypes.c_void_p(_torch().cuda.current_stream(self.dev).cuda_stream)

    def frame(self, buttons, render: bool = True):
        torch = _torch()
        b = torch.as_tensor(np.asarray(buttons, dtype=np.uint8).reshape(-1)) if not isinstance(buttons, torch.Tensor) else buttons
        self._btn.copy_(b.to(self.dev, torch.uint8).view(-1))
        N.check(N.lib().fme_raw_frame(self.h, N.ptr(self._btn), int(bool(render)), self._stream()), "fme_raw_frame")

    def ram(self):
        N.check(N.lib().fme_raw_ram(self.h, N.ptr(self._ram), self._stream()), "fme_raw_ram")
        return self._ram

    def screen(self):
        N.check(N.lib().fme_raw_screen(self.h, N.ptr(self._scr), self._stream()), "fme_raw_screen")
        return self._scr

    def backup(self):
        N.check(N.lib().fme_raw_backup(self.h, self._stream()), "fme_raw_backup")

    def restore(self):
        N.check(N.lib().fme_raw_restore(self.h, self._stream()), "fme_raw_restore")

    def bad_ops(self) -> int:
        _torch().cuda.synchronize(self.dev)
        v = ctypes.c_int64()
        N.check(N.lib().fme_raw_bad_ops(self.h, ctypes.byref(v)), "fme_raw_bad_ops")
        return int(v.value)

    def check(self):
        _torch().cuda.synchronize(self.dev)
        st = ctypes.c_uint32()
        N.check(N.lib().fme_raw_poll_error(self.h, ctypes.byref(st)), "fme_raw_poll_error")
        if st.value:
            raise N.FmeError(f"device status {st.value:#x}: {N.status_text(st.value)}")

    def close(self):
        h, self.h = getattr(self, "h", None), None
        if h:
            N.lib().fme_raw_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RawNES:
    """One raw console with the reference RawNES interface: frame(buttons, render), .ram, .screen (numpy
    copies refreshed after every frame), backup(), restore(), bad_ops()."""

    def __init__(self, rom_bytes: bytes, device="cuda"):
        self.b = RawNESBatch(rom_bytes, 1, device)
        self.ram = np.zeros(0x800, np.uint8)
        self.screen = np.zeros((240, 256), np.uint8)

    def frame(self, buttons: int, render: bool = True):
        self.b.frame([buttons], render)
        self.ram[:] = self.b.ram()[0].cpu().numpy()
        if render:
            self.screen[:] = self.b.screen()[0].cpu().numpy()

    def backup(self):
        self.b.backup()

    def restore(self):
        self.b.restore()
        self.ram[:] = self.b.ram()[0].cpu().numpy()

    def bad_ops(self) -> int:
        return self.b.bad_ops()


def resize_area(gray) -> np.ndarray:
    """240x256 uint8 -> 84x84, OpenCV INTER_AREA float order, computed on the GPU (one image or a batch)."""
    torch = _torch()
    g = np.ascontiguousarray(gray, np.uint8)
    single = g.ndim == 2
    if single:
        g = g[None]
    if g.shape[1:] != (240, 256):
        raise ValueError("expected (240, 256) uint8 image(s)")
    src = torch.from_numpy(g).cuda()
    dst = torch.empty(g.shape[0], OBS_HW, OBS_HW, dtype=torch.uint8, device=src.device)
    N.check(N.lib().fme_resize(N.ptr(src), N.ptr(dst), g.shape[0],
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "fme_resize")
    out = dst.cpu().numpy()
    return out[0] if single else out


__all__ = ["CudaVecEnv", "FastVecEnv", "RawNES", "RawNESBatch", "MonitorCSV", "palette_rgb", "gray_lut", "rng_state",
           "resize_area", "OBS_HW", "N_ACTIONS", "SIMPLE_MOVEMENT", "INFO_FIELDS", "INFO_KEYS"]
