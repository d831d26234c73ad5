"""Shared test setup: import paths, the `gpu` marker, golden-vector loaders.

CPU tests (-m "not gpu") check the oracle against the reference's golden vectors, the
host-side logic of the library (validation, allocator, table format) and that
libbgtq.so loads and exports its C ABI.  GPU tests (-m gpu) drive the CUDA kernels
through the C ABI and compare them with the oracle.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT / "block-gqt-webgpu_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libbgtq.so")


def mixed_cases():
    return sorted(p.stem for p in (GOLDEN / "mixed").glob("*.npz"))


def attention_cases():
    return sorted(p.stem for p in (GOLDEN / "attention").glob("*.npz"))


def load_mixed(name):
    return np.load(GOLDEN / "mixed" / f"{name}.npz")


def load_attention(name):
    return np.load(GOLDEN / "attention" / f"{name}.npz")


def load_config(name):
    return np.load(GOLDEN / f"{name}.npz")


def allocator_cases():
    return json.loads((GOLDEN / "allocator.json").read_text())["cases"]


def params_tables(z):
    from bgtq.layout import BlockGTQParameters, tables
    p = BlockGTQParameters.from_arrays(z)
    return p, *tables(p)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test requires CUDA")
    torch.cuda.init()
    return torch.device("cuda:0")
