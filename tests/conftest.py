"""Shared pytest setup: import paths, the `gpu` marker, golden fixtures."""
from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent
PKG = REPO / "qwen2-7b-triton_engine_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden" / "awq_golden.npz"
SILU_GOLDEN = REPO / "tests" / "golden" / "silu_golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden():
    data = np.load(GOLDEN, allow_pickle=False)
    cases = {}
    for name in data["cases"]:
        name = str(name)
        p = name + "/"
        case = {k[len(p):]: data[k] for k in data.files if k.startswith(p)}
        case["group_size"] = int(case["group_size"])
        cases[name] = case
    return cases


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("needs an sm_100 device")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def silu_golden():
    """Cases of tests/golden/make_golden_silu.py: name -> {array name: array}."""
    data = np.load(SILU_GOLDEN, allow_pickle=False)
    cases = {}
    for key in data.files:
        name, field = key.split("/", 1)
        cases.setdefault(name, {})[field] = data[key]
    return cases
