"""Shared pytest setup.

- registers the ``gpu`` marker (tests that need a B200);
- puts the repo root and ``oracle/`` on sys.path;
- loads the product package from the ``nyion.rs_b200`` directory under the
  import name ``nyion_rs_b200`` (the directory name carries a dot).
"""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
ORACLE_DIR = os.path.join(ROOT, "oracle")
if ORACLE_DIR not in sys.path:
    sys.path.insert(0, ORACLE_DIR)


def load_package():
    if "nyion_rs_b200" in sys.modules:
        return sys.modules["nyion_rs_b200"]
    pkg_dir = os.path.join(ROOT, "nyion.rs_b200")
    spec = importlib.util.spec_from_file_location(
        "nyion_rs_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["nyion_rs_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
