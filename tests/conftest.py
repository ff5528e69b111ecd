"""Test set-up: the `gpu` marker, the package (its directory name has a
hyphen, so it is loaded by path) and the CPU oracle."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "ppocr-native_b200"


def load_package():
    name = "ppocr_native_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _build_library():
    """Compile libppocr_cuda.so when a source is newer than it (a no-op on a
    GPU box that received the prebuilt library)."""
    spec = importlib.util.spec_from_file_location("_ppocr_build", PKG_DIR / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    try:
        mod.build()
    except RuntimeError:
        if not mod.LIB.exists():
            raise


_build_library()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libppocr_cuda.so")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_mod():
    """The binding with its library built; GPU tests only."""
    from ppocr_native_b200 import cuda

    if cuda.device_count() < 1:
        pytest.fail("a gpu-marked test ran without a CUDA device")
    return cuda
