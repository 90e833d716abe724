"""Test configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs here without a GPU (oracle vs golden fixtures, host logic,
library load/exports, gloo multi-rank host logic).  `-m gpu` runs the parity tests
proper on a B200 through the C ABI.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_golden(name: str):
    """(arrays dict, meta dict) of a committed fixture."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    arrays = {k: z[k] for k in z.files if k != "meta_json"}
    meta = json.loads(bytes(z["meta_json"]).decode())
    return arrays, meta


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip("needs an sm_100 device")
    from easyinfra_b200 import build
    build.build()
    return torch.device("cuda", torch.cuda.current_device())
