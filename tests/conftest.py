"""Shared test setup.

Markers: ``gpu`` -- needs a B200 (the parity tests proper, through the C ABI).
The CPU suite (``-m "not gpu"``) checks the oracle against the golden
vectors, the host logic, and that the C-ABI library loads and exports its
symbols, without touching a GPU.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA kernels")


@pytest.fixture(scope="session")
def kf_lib():
    from kernelfoundry_b200 import build

    build.build()
    from kernelfoundry_b200._lib import lib

    return lib()


@pytest.fixture(scope="session")
def c_oracle():
    import oracle

    return oracle.load_c_oracle()


@pytest.fixture(scope="session")
def sdpa_golden():
    return np.load(os.path.join(GOLDEN, "sdpa_golden.npz"))


@pytest.fixture(scope="session")
def legacy_golden():
    return np.load(os.path.join(GOLDEN, "legacy18_golden.npz"))


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU test run without a GPU"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"needs sm_100, got sm_{major}{minor}"
    from kernelfoundry_b200 import build

    build.build()
    return torch.device("cuda:0")


def golden_case(g, name):
    B, Hq, Hkv, Sq, Skv, D, seed = (int(x) for x in g[f"{name}/shape"])
    Q = g[f"{name}/Q"].view(np.float16)
    K = g[f"{name}/K"].view(np.float16)
    V = g[f"{name}/V"].view(np.float16)
    return (B, Hq, Hkv, Sq, Skv, D, seed), Q, K, V


def golden_names(g):
    return sorted({k.split("/")[0] for k in g.files if not k.startswith("smoke")})
