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


def moe_layer_reference_products(ref, orc, x, idx, wts, layer, k, group_size=64):
    """One MoE layer whose every product is the reference's own MLX CPU kernel
    over fp32 operands (fp32 products and running sum, backend/cpu/quantized.cpp:155,
    :341), composed the way the Runner's decode operators compose them: gate and
    up rounded to bf16, SwiGLU with the Runner's bf16 rounding points
    (TrackFastKernels2.swift:22-31), the down product rounded to bf16, times the
    routing weight, folded in the mlx_colsum_small_f32 order
    (TrackFastKernels2.swift:36-47), rounded to bf16. x bf16 bits [T, H];
    idx / wts [T, k]; returns bf16 bits [T, H]."""
    from oracle.oracle import bf16_to_f32, f32_to_bf16

    T = x.shape[0]
    H = x.shape[1]
    out = np.zeros((T, H), np.uint16)
    for t in range(T):
        prods = []
        for j in range(k):
            e = int(idx[t, j])
            g = ref.qmm_f32(x[t:t + 1], layer["wg"][e], layer["sg"][e], layer["bg"][e], group_size)
            u = ref.qmm_f32(x[t:t + 1], layer["wu"][e], layer["su"][e], layer["bu"][e], group_size)
            act = orc.swiglu(f32_to_bf16(g), f32_to_bf16(u)).reshape(1, -1)
            y = ref.qmm_f32(act, layer["wd"][e], layer["sd"][e], layer["bd"][e], group_size)
            prods.append(bf16_to_f32(f32_to_bf16(y[0])) * np.float32(wts[t, j]))
        P = np.stack(prods).astype(np.float32)  # [k, H]
        out[t] = f32_to_bf16(np.array([orc.colsum_small(P[:, h]) for h in range(H)], np.float32))
    return out
