"""The emulation headers compiled for the host CPU (tests/host_raw.cpp) in lockstep with the reference build.

The GPU kernels run Core, the register-resident fast path with its per-PC micro-ops, and the frame
bookkeeping from portable headers. Built with g++ they step raw consoles here, without a GPU, so the CPU suite
checks that very code frame by frame against the reference's own emulator (oracle/_ref): the RAM of every
console after every frame, bit for bit, on the default, divergent and four-idle-loop synthetic images.
"""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import fme  # noqa: F401  (puts the package on sys.path)

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "fast-mario-env_b200", "csrc")


def _cuda_include():
    cands = [os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"]
    nvcc = shutil.which("nvcc")
    if nvcc:
        cands.insert(0, os.path.dirname(os.path.dirname(os.path.realpath(nvcc))))
    for c in cands:
        if c and os.path.exists(os.path.join(c, "include", "vector_types.h")):
            return os.path.join(c, "include")
    return None


@pytest.fixture(scope="module")
def host(tmp_path_factory):
    gxx, inc = shutil.which("g++"), _cuda_include()
    if not gxx or not inc:
        pytest.skip("needs g++ and the CUDA headers (vector_types.h)")
    out = str(tmp_path_factory.mktemp("host_engine") / "libhost_raw.so")
    subprocess.run([gxx, "-std=c++17", "-O2", "-shared", "-fPIC", "-I", CSRC, "-I", inc,
                    os.path.join(HERE, "host_raw.cpp"), "-o", out], check=True, capture_output=True)
    H = ctypes.CDLL(out)
    P = ctypes.c_void_p
    H.hr_create.restype = P
    H.hr_create.argtypes = [P, ctypes.c_int64, ctypes.c_int]
    H.hr_frame.argtypes = [P, P]
    H.hr_ram.argtypes = [P, ctypes.c_int, P]
    for f in (H.hr_bad_ops, H.hr_status):
        f.restype = ctypes.c_int64
        f.argtypes = [P, ctypes.c_int]
    H.hr_destroy.argtypes = [P]
    H.hr_dp_check.restype = ctypes.c_int64
    H.hr_dp_check.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_uint32, P, P]
    return H


@pytest.mark.parametrize("image", [dict(), dict(divergence=True), dict(idle_loops=4)],
                         ids=["default", "divergent", "four_idle_loops"])
def test_host_build_of_the_engine_matches_reference(host, oracle, image):
    from fast_mario_env_b200.synth_rom import build_rom
    rom = build_rom(0, **image)
    n, frames = 4, 500
    rb = np.frombuffer(rom, np.uint8).copy()
    h = host.hr_create(rb.ctypes.data, len(rb), n)
    assert h
    try:
        refs = [oracle.RefRaw(rom) for _ in range(n)]
        rng = np.random.default_rng(3)
        ram = np.zeros(0x800, np.uint8)
        for f in range(frames):
            b = rng.integers(0, 256, n).astype(np.uint8)
            host.hr_frame(h, b.ctypes.data)
            for i, r in enumerate(refs):
                r.frame(int(b[i]), False)
                host.hr_ram(h, i, ram.ctypes.data)
                assert np.array_equal(ram, r.ram), (f, i, np.flatnonzero(ram != r.ram)[:8].tolist())
        for i, r in enumerate(refs):
            assert host.hr_bad_ops(h, i) == r.bad_ops() == 0
            assert host.hr_status(h, i) == 0
    finally:
        host.hr_destroy(h)


# the datapath runs every official opcode whose memory accesses are RAM or PRG only, i.e. all of them except
# BRK ($00), RTI ($40) and JMP (ind) ($6C), which stay on the exact path
_EXACT_ONLY = {0x00, 0x40, 0x6C}


@pytest.mark.parametrize("ram_end", [0x800, 0x600, 0x2E0], ids=["whole_ram", "split_0600", "split_02e0"])
def test_datapath_matches_exact_interpreter_per_instruction(host, ram_end):
    """dp_exec against Core::execute_op on random PRG bytes, registers, status bytes and RAM: pc, registers,
    status, cycles and RAM after each committed instruction, with RAM whole or split across two buffers."""
    bad = ctypes.c_int32(0)
    hist = np.zeros(256, np.int64)
    n = host.hr_dp_check(11 + ram_end, 400_000, ram_end, ctypes.byref(bad), hist.ctypes.data)
    assert bad.value == -1, f"opcode ${bad.value >> 16:02X} at ${bad.value & 0xffff:04X} differs"
    assert n > 100_000
    from fast_mario_env_b200 import asm6502
    official = set(asm6502.OPCODES.values())
    covered = {opc for opc in range(256) if hist[opc] > 0}
    assert official - _EXACT_ONLY <= covered, sorted(official - _EXACT_ONLY - covered)
    assert not covered & _EXACT_ONLY
