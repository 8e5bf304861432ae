"""Shared test setup.

* Registers the `gpu` marker (tests that need a B200 / CUDA device).
* Loads the package directory `fast-mario-env_b200/` as the module `fast_mario_env_b200` (its directory name has
  hyphens, so it cannot be imported by name).
* Exposes the test oracle (oracle/ref.py: the reference's own C++ core built by oracle/Makefile).
FME_TEST_SCALE multiplies the lengths of the lockstep tests, as the reference's conftest does (conftest.py:10-15).
"""
from __future__ import annotations

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "fast-mario-env_b200")
PKG_NAME = "fast_mario_env_b200"
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))

SCALE = max(1, int(os.environ.get("FME_TEST_SCALE", "1")))


def scaled(n: int) -> int:
    return n * SCALE


def load_package():
    if PKG_NAME in sys.modules:
        return sys.modules[PKG_NAME]
    spec = importlib.util.spec_from_file_location(PKG_NAME, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[PKG_NAME] = mod
    spec.loader.exec_module(mod)
    return mod


fme = load_package()


def _have_cuda() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAVE_CUDA = _have_cuda()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    if HAVE_CUDA:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def oracle(request):
    """The reference's own C++ core (oracle/_ref/libfastmario.so). A GPU parity test without it fails: a parity
    suite that turned into skips would pass while checking nothing. CPU-only tests skip instead."""
    import ref
    if not ref.available():
        msg = "reference oracle not built (make -C oracle REF=<reference checkout>)"
        if request.node.get_closest_marker("gpu") is not None:
            pytest.fail(msg)
        pytest.skip(msg)
    return ref


@pytest.fixture(scope="session")
def rom():
    from fast_mario_env_b200.synth_rom import build_rom
    return build_rom(0)


@pytest.fixture(scope="session")
def rom_div():
    from fast_mario_env_b200.synth_rom import build_rom
    return build_rom(0, divergence=True)
