"""Shared test setup.

- The `gpu` marker: tests that need a CUDA device (a B200 on the GPU box).
- `pkg`: the package (its directory name contains '-', so it is imported
  with importlib).
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

PKG_NAME = "distributed-llm-inference_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu on a B200)")


def golden_module():
    """tests/golden/make_golden.py as a module (input generators, digests)."""
    import importlib.util
    name = "pdb_make_golden"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, REPO / "tests" / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def import_pkg():
    return importlib.import_module(PKG_NAME)


def import_module(name: str):
    return importlib.import_module(f"{PKG_NAME}.{name}")


@pytest.fixture(scope="session")
def pkg():
    return import_pkg()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    # The library must be present: there is no fallback.
    import_pkg().load_library()
    return torch.device("cuda:0")
