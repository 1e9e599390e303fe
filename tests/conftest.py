"""Shared test setup: the `gpu` marker, the package loader and checkpoints."""

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "irodori-tts-burn_b200"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_pkg():
    """Import the package directory `irodori-tts-burn_b200/` as `irodori_b200`."""
    if "irodori_b200" in sys.modules:
        return sys.modules["irodori_b200"]
    spec = importlib.util.spec_from_file_location("irodori_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["irodori_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def synth(pkg):
    import irodori_b200.synth as s
    return s


@pytest.fixture(scope="session")
def oracle():
    from oracle import irodori_oracle
    return irodori_oracle


@pytest.fixture(scope="session")
def ckpt_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("ckpt")
