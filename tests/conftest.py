"""Shared test setup: the gpu marker, import paths, and oracle fixtures.

`-m "not gpu"` runs on a CPU-only machine (oracle vs golden vectors, host
logic, C-ABI loading). `-m gpu` tests are the parity tests on a B200: they
call the CUDA library through its C ABI and compare with the CPU oracle.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mlxfast-qwen38-125b-a6b-engine_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "mlx_cpu_golden.npz")

# Tolerances. The north star asks layer outputs within 1e-2 relative L2 of the
# reference path (bf16 outputs, fp32 accumulation); products are additionally
# held to a max-abs bound of a few bf16 ulps of the output scale.
REL_L2 = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C ABI")


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def b2q_mod():
    import b2q

    return b2q


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    torch.cuda.init()
    return torch.device("cuda:0")
