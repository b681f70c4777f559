"""Shared test setup: the `gpu` marker, the package loader and input generators."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_package():
    """The package directory is `xn-ptts_b200`; register it as `xn_ptts_b200`."""
    if "xn_ptts_b200" in sys.modules:
        return sys.modules["xn_ptts_b200"]
    path = os.path.join(ROOT, "xn-ptts_b200", "__init__.py")
    spec = importlib.util.spec_from_file_location("xn_ptts_b200", path,
                                                  submodule_search_locations=[os.path.dirname(path)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xn_ptts_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def ptts():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def cuda(ptts):
    """A CUDA device with the built library; the library itself must load (no fallback)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ptts.lib()
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def elementwise(got: np.ndarray, want: np.ndarray, floor: float = 1e-2) -> float:
    """max_i |got_i - want_i| / max(|want_i|, floor * ||want||_inf): the element-wise relative
    error, with an absolute floor at `floor` of the largest magnitude (elements near zero are
    measured against the floor, not against themselves). Reported beside the normwise gate:
    after a bf16 store (unit roundoff 2^-8) no element-wise bound below 2e-3 can hold without
    such a floor."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    top = np.abs(want).max()
    den = np.maximum(np.abs(want), floor * (top if top > 0 else 1.0))
    return float((np.abs(got - want) / den).max())


def normwise(got: np.ndarray, want: np.ndarray) -> float:
    """||got - want||_inf / ||want||_inf, the parity metric of every test here."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.abs(want).max()
    return float(np.abs(got - want).max() / (den if den > 0 else 1.0))
