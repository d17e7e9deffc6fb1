"""Shared fixtures: golden fixture loader, the CPU oracle, GPU gating.

Tests marked ``gpu`` need a CUDA device and the built library; everything
else runs on CPU.  The oracle (oracle/hv_oracle.py) is the checker only.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running parity sweep")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle():
    import hv_oracle
    hv_oracle.build()
    return hv_oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from heatvit_b200 import _lib
    _lib.lib()  # fails loudly when the library is missing
    return torch


def golden_ckpt(g, prefix):
    """Decode a packed golden result into {key: [rows][192]} plus logits."""
    keys = [str(k) for k in g[f"{prefix}_ckpt_keys"]]
    data, off = g[f"{prefix}_ckpt"], g[f"{prefix}_ckpt_off"]
    ck = {k: data[off[i]:off[i + 1]].astype(np.int8) for i, k in enumerate(keys)}
    return ck, g[f"{prefix}_logits"].astype(np.int32), g[f"{prefix}_summary"]


def slot_of(key):
    if key == "patch":
        return 0
    if key == "final_ln":
        return 25
    kind, num = key.split("_")
    return int(num) + (12 if kind == "selector" else 0)
