"""fme_raw_frame_static (the allocation-free frame call, PPU log in a fixed device array) against
fme_raw_frame on the same consoles. Collected last so that it also runs after every other GPU test."""
import ctypes

import numpy as np
import pytest
from conftest import fme

from fast_mario_env_b200 import _native as N

pytestmark = pytest.mark.gpu

N_CONSOLES = 40        # two warps, the second one ragged
LEAD_FRAMES = 150      # past the boot so that the compared screens have content


def _stream(b):
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream(b.dev).cuda_stream)


def test_static_frame_matches_raw_frame_on_two_calls_in_a_row(rom_div):
    import torch
    a = fme.RawNESBatch(rom_div, N_CONSOLES)
    b = fme.RawNESBatch(rom_div, N_CONSOLES)
    rng = np.random.default_rng(11)
    for _ in range(LEAD_FRAMES):
        btn = rng.integers(0, 256, N_CONSOLES).astype(np.uint8)
        a.frame(btn, False)
        b.frame(btn, False)
    L = N.lib()
    scr = torch.full((N_CONSOLES, 240, 256), 0xEE, dtype=torch.uint8, device=b.dev)
    for call in range(2):
        btn = torch.as_tensor(rng.integers(0, 256, N_CONSOLES).astype(np.uint8)).to(b.dev)
        a.frame(btn, True)
        N.check(L.fme_raw_frame_static(b.h, N.ptr(btn), N.ptr(scr), 1, _stream(b)), "fme_raw_frame_static")
        want_scr = a.screen().cpu().numpy()
        got_scr = scr.cpu().numpy()
        assert np.unique(want_scr).size > 2, "compared screens are blank"
        assert np.array_equal(got_scr, want_scr), f"screens differ on call {call}"
        assert np.array_equal(b.ram().cpu().numpy(), a.ram().cpu().numpy()), f"RAM differs on call {call}"
    a.check()
    b.check()
    a.close()
    b.close()


def test_static_frame_with_the_full_array_and_untouched_handle_screens(rom_div):
    """64 consoles, every slot of the array, rendering on two calls in a row; the handle's own screen buffer
    keeps the screens of its last fme_raw_frame."""
    import torch
    n = N.FME_STATIC_MAX_CONSOLES
    a = fme.RawNESBatch(rom_div, n)
    b = fme.RawNESBatch(rom_div, n)
    rng = np.random.default_rng(64)
    for f in range(LEAD_FRAMES):
        btn = rng.integers(0, 256, n).astype(np.uint8)
        a.frame(btn, f == LEAD_FRAMES - 1)
        b.frame(btn, f == LEAD_FRAMES - 1)
    before = b.screen().cpu().numpy()
    scr = torch.zeros((n, 240, 256), dtype=torch.uint8, device=b.dev)
    for call in range(2):
        btn = torch.as_tensor(rng.integers(0, 256, n).astype(np.uint8)).to(b.dev)
        a.frame(btn, True)
        N.check(N.lib().fme_raw_frame_static(b.h, N.ptr(btn), N.ptr(scr), 1, _stream(b)), "fme_raw_frame_static")
        want = a.screen().cpu().numpy()
        assert not np.array_equal(want, before), "the compared frames did not change the screens"
        assert np.array_equal(scr.cpu().numpy(), want), f"screens differ on call {call}"
        assert np.array_equal(b.ram().cpu().numpy(), a.ram().cpu().numpy()), f"RAM differs on call {call}"
    assert np.array_equal(b.screen().cpu().numpy(), before), "fme_raw_screen changed after static calls"
    a.check()
    b.check()
    a.close()
    b.close()


def test_static_frame_without_render_takes_no_screen_buffer(rom):
    import torch
    a = fme.RawNESBatch(rom, 3)
    b = fme.RawNESBatch(rom, 3)
    btn = torch.zeros(3, dtype=torch.uint8, device=b.dev)
    for _ in range(2):
        a.frame(btn, False)
        N.check(N.lib().fme_raw_frame_static(b.h, N.ptr(btn), None, 0, _stream(b)), "fme_raw_frame_static")
    assert np.array_equal(b.ram().cpu().numpy(), a.ram().cpu().numpy())
    b.check()
    a.close()
    b.close()


def test_static_frame_rejects_more_consoles_than_the_array_holds(rom):
    import torch
    n = 65
    b = fme.RawNESBatch(rom, n)
    btn = torch.zeros(n, dtype=torch.uint8, device=b.dev)
    scr = torch.zeros((n, 240, 256), dtype=torch.uint8, device=b.dev)
    rc = N.lib().fme_raw_frame_static(b.h, N.ptr(btn), N.ptr(scr), 1, _stream(b))
    assert rc == -1 and "at most 64" in N.last_error()
    rc = N.lib().fme_raw_frame_static(b.h, N.ptr(btn), None, 1, _stream(b))
    assert rc == -1
    b.close()
