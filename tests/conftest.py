"""Shared test setup: the `gpu` marker, repo imports and library loading."""
import importlib.util
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
PKG_DIR = os.path.join(REPO, "rocket-userspace_b200")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def load_pkg():
    """Import the package directory (its name is not a Python identifier)."""
    if "rocket_userspace_b200" in sys.modules:
        return sys.modules["rocket_userspace_b200"]
    spec = importlib.util.spec_from_file_location(
        "rocket_userspace_b200", os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["rocket_userspace_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def rkb():
    if not os.path.exists(os.path.join(PKG_DIR, "librocketnpu.so")):
        import subprocess
        subprocess.run(["make", "-C", PKG_DIR, "-j8"], check=True, capture_output=True)
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def dev(rkb):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    d = rkb.Device()
    yield d
    d.close()
