"""Shared test setup: the `gpu` marker, and the product package (directory `xtier-go_b200/`) importable as
`xtier_go_b200`."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_product():
    if "xtier_go_b200" in sys.modules:
        return sys.modules["xtier_go_b200"]
    pkg = os.path.join(ROOT, "xtier-go_b200")
    spec = importlib.util.spec_from_file_location("xtier_go_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xtier_go_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and runs the CUDA library")


@pytest.fixture(scope="session")
def xtg():
    return load_product()


@pytest.fixture(scope="session")
def cuda(xtg):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a GPU")
    return xtg.lib()
