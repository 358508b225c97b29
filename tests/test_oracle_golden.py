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

from conftest import REL_L2, moe_layer_reference_products, rel_l2
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


def _rand_layer(rng, E, H, F, gs):
    def packed(rows, K):
        wq = rng.integers(0, 2**32, size=(E, rows, K // 8), dtype=np.uint64).astype(np.uint32)
        s = f32_to_bf16(rng.uniform(0.002, 0.02, (E, rows, K // gs)).astype(np.float32))
        b = f32_to_bf16(-8.0 * bf16_to_f32(s) + rng.normal(0, 1e-3, s.shape).astype(np.float32))
        return wq, s, b

    L = {}
    for n, (rows, K) in (("g", (F, H)), ("u", (F, H)), ("d", (H, F))):
        L["w" + n], L["s" + n], L["b" + n] = packed(rows, K)
    return L


@pytest.mark.skipif(not MlxRef.available(), reason="reference MLX CPU library not built here")
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_fp32_restatements_against_reference_fp32_kernel(oracle, gs):
    """The reference's own CPU kernel over fp32 operands (fp32 accumulation, the
    north star's arithmetic) pins the oracle's fp32 restatement of the Metal qmv
    association to fp32 rounding of the sum order; the tile-loader restatement
    rounds every dequantized weight to bf16 first (the operand the tensor-core
    path feeds), which moves it about 1.5e-3 from exact."""
    ref = MlxRef()
    if not ref.has_f32:
        pytest.skip("reference library built without the fp32 entry points")
    rng = np.random.default_rng(100 + gs)
    for K, N in ((1024, 48), (4096, 64), (1536, 32)):
        if K % (gs * 8):
            continue
        wq = rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32)
        s = f32_to_bf16(rng.uniform(0.002, 0.02, (N, K // gs)).astype(np.float32))
        b = f32_to_bf16(-8.0 * bf16_to_f32(s) + rng.normal(0, 1e-3, s.shape).astype(np.float32))
        x = f32_to_bf16(rng.standard_normal((3, K)).astype(np.float32))
        yr = ref.qmm_f32(x, wq, s, b, gs)
        assert rel_l2(oracle.qmv_metal_f32(x, wq, s, b, gs, 4), yr) < 1e-5
        assert rel_l2(oracle.qmm_tile_f32(x, wq, s, b, gs, 4), yr) < 3e-3
        # and the bf16 outputs of the restatement sit within a bf16 rounding of it
        assert rel_l2(bf16_to_f32(oracle.qmv_metal(x, wq, s, b, gs, 4)), yr) < 3e-3


@pytest.mark.skipif(not MlxRef.available(), reason="reference MLX CPU library not built here")
def test_gather_loop_of_the_reference(oracle):
    """The reference's gather over (lhs, rhs) pairs equals per-pair products."""
    ref = MlxRef()
    if not ref.has_f32:
        pytest.skip("reference library built without the fp32 entry points")
    rng = np.random.default_rng(3)
    n_x, n_w, M, N, K, gs = 3, 5, 2, 32, 512, 64
    L = _rand_layer(rng, n_w, K, N, gs)
    x = f32_to_bf16(rng.standard_normal((n_x, M, K)).astype(np.float32))
    lhs = np.array([2, 0, 1, 1, 2, 0], np.uint32)
    rhs = np.array([4, 4, 0, 3, 1, 2], np.uint32)
    y = ref.gather_qmm(x, L["wg"], L["sg"], L["bg"], lhs, rhs, gs)
    for i in range(len(lhs)):
        yi = ref.qmm_f32(x[lhs[i]], L["wg"][rhs[i]], L["sg"][rhs[i]], L["bg"][rhs[i]], gs)
        assert np.array_equal(y[i], yi)
        yo = oracle.qmv_metal_f32(x[lhs[i]], L["wg"][rhs[i]], L["sg"][rhs[i]], L["bg"][rhs[i]], gs, 4)
        assert rel_l2(yo, yi) < 1e-5
    yb = ref.gather_qmm(x, L["wg"], L["sg"], L["bg"], lhs, rhs, gs, fp32=False)
    assert np.array_equal(yb[1], ref.qmm(x[0], L["wg"][4], L["sg"][4], L["bg"][4], gs))


@pytest.mark.skipif(not MlxRef.available(), reason="reference MLX CPU library not built here")
def test_moe_restatement_against_reference_products(oracle):
    """The oracle's MoE decode layer (Metal qdot association for every product)
    against the same layer built from the reference's own fp32 CPU products."""
    ref = MlxRef()
    if not ref.has_f32:
        pytest.skip("reference library built without the fp32 entry points")
    rng = np.random.default_rng(11)
    E, H, F, k, gs = 12, 512, 256, 4, 64
    L = _rand_layer(rng, E, H, F, gs)
    x = f32_to_bf16(rng.standard_normal((2, H)).astype(np.float32))
    wr = f32_to_bf16(rng.normal(0, 0.02, (E, H)).astype(np.float32))
    idx, w = oracle.route(oracle.router_logits(x, wr), k)
    a = oracle.moe_experts_decode(x, idx, w, L, k, gs)
    r = moe_layer_reference_products(ref, oracle, x, idx, w, L, k, gs)
    assert rel_l2(bf16_to_f32(a), bf16_to_f32(r)) < 2e-3
