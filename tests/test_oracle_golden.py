"""Pins the CPU oracle to the reference's own MLX CPU code (golden vectors).

The fixtures in tests/golden/mlx_cpu_golden.npz were produced by the
reference's backend/cpu/quantized.cpp compiled from the reference tree
(tests/golden/make_golden.py). The oracle's restatements must match them
bit for bit; when the compiled reference library is present the same holds
live on fresh random inputs.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import REL_L2, rel_l2
from oracle.oracle import MlxRef, bf16_to_f32, f32_to_bf16


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_matches_mlx_golden(oracle, golden, gs):
    w = golden[f"quantize_gs{gs}_w"]
    wq, s, b = oracle.quantize(w, gs, 4)
    assert np.array_equal(wq, golden[f"quantize_gs{gs}_wq"])
    assert np.array_equal(s, golden[f"quantize_gs{gs}_s"])
    assert np.array_equal(b, golden[f"quantize_gs{gs}_b"])


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_mlx_cpu_qmm_restatement_matches_golden(oracle, golden, gs):
    x = golden[f"qmm_gs{gs}_x"]
    y = oracle.qmm_mlx_cpu(x, golden[f"quantize_gs{gs}_wq"], golden[f"quantize_gs{gs}_s"],
                           golden[f"quantize_gs{gs}_b"], gs, 4)
    assert np.array_equal(y, golden[f"qmm_gs{gs}_y"])


def test_c0_slice_golden(oracle, golden):
    y = oracle.qmm_mlx_cpu(golden["c0_x"], golden["c0_wq"], golden["c0_s"], golden["c0_b"], 64, 4)
    assert np.array_equal(y, golden["c0_y"])
    # the fp32 restatements agree with each other to well inside the parity bound,
    # while the bf16-accumulating MLX CPU path sits further away (informational)
    ym = bf16_to_f32(oracle.qmv_metal(golden["c0_x"], golden["c0_wq"], golden["c0_s"], golden["c0_b"]))
    yt = oracle.qmm_tile_f32(golden["c0_x"], golden["c0_wq"], golden["c0_s"], golden["c0_b"])
    assert rel_l2(ym, yt) < 5e-3
    assert rel_l2(bf16_to_f32(golden["c0_y"]), yt) < 0.2


def test_dequantize_variants(oracle, golden):
    w, s, b = golden["quantize_gs64_wq"], golden["quantize_gs64_s"], golden["quantize_gs64_b"]
    dm = oracle.dequantize(w, s, b, 64, 4, "metal")
    dc = oracle.dequantize(w, s, b, 64, 4, "cpu")
    # independent numpy statement of both rounding variants
    q = ((w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF).reshape(w.shape[0], -1).astype(np.float32)
    sf = np.repeat(bf16_to_f32(s), 64, axis=1)
    bfv = np.repeat(bf16_to_f32(b), 64, axis=1)
    assert np.array_equal(dm, f32_to_bf16(sf * q + bfv))
    assert np.array_equal(dc, f32_to_bf16(bf16_to_f32(f32_to_bf16(q * sf)) + bfv))


def test_quantize_roundtrip_error_bound(oracle):
    # |w - dequant(quant(w))| <= scale per group (test_quantized.py:23-53 method)
    rng = np.random.default_rng(5)
    w = f32_to_bf16(rng.standard_normal((16, 256)).astype(np.float32))
    wq, s, b = oracle.quantize(w, 64, 4)
    wh = bf16_to_f32(oracle.dequantize(wq, s, b, 64, 4, "metal"))
    wf = bf16_to_f32(w).reshape(16, 4, 64)
    err = np.abs(wh.reshape(16, 4, 64) - wf).max(-1)
    # one scale step, plus the bf16 rounding of the stored scale and of the
    # dequantized value (one bf16 ulp of the group's largest magnitude)
    ulp = 2.0 ** (np.floor(np.log2(np.abs(wf).max(-1))) - 7)
    assert np.all(err <= np.abs(bf16_to_f32(s)) * 1.01 + ulp)


@pytest.mark.skipif(not MlxRef.available(), reason="reference MLX CPU library not built here")
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_live_against_reference_build(oracle, gs):
    ref = MlxRef()
    rng = np.random.default_rng(gs)
    w = f32_to_bf16(rng.standard_normal((24, 1024)).astype(np.float32) * 0.02)
    a = oracle.quantize(w, gs, 4)
    r = ref.quantize(w, gs, 4)
    for u, v in zip(a, r):
        assert np.array_equal(u, v)
    x = f32_to_bf16(rng.standard_normal((2, 1024)).astype(np.float32))
    assert np.array_equal(oracle.qmm_mlx_cpu(x, *a, gs, 4), ref.qmm(x, *a, gs, 4))


def test_metal_association_vs_tile_product(oracle):
    rng = np.random.default_rng(7)
    for K in (512, 1536, 640, 256):
        wq = rng.integers(0, 2**32, size=(32, K // 8), dtype=np.uint64).astype(np.uint32)
        s = f32_to_bf16(rng.uniform(0.002, 0.02, (32, K // 32)).astype(np.float32))
        b = f32_to_bf16(-8 * bf16_to_f32(s) + rng.normal(0, 1e-3, s.shape).astype(np.float32))
        x = f32_to_bf16(rng.standard_normal((2, K)).astype(np.float32))
        ym = oracle.qmv_metal_f32(x, wq, s, b, 32, 4)
        yt = oracle.qmm_tile_f32(x, wq, s, b, 32, 4)
        assert rel_l2(ym, yt) < REL_L2 / 2
