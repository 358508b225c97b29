"""Parity of the packing and product kernels with the CPU oracle (B200).

Method of the reference's own tests (python/tests/test_quantized.py:23-53,
:600-626, :1162-1300 of the vendored MLX): dequantized weights bit-exact;
products compared with the reference arithmetic (the oracle's Metal qmv
association) within the parity bound, across group sizes, token counts,
ragged row counts and gathered experts.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import REL_L2, rel_l2

pytestmark = pytest.mark.gpu

TIGHT = 3e-3  # observed rounding-only differences sit well below this


def _np(t):
    from b2q.synth import to_numpy_bits

    return to_numpy_bits(t)


def _bf(a):
    from oracle.oracle import bf16_to_f32

    return bf16_to_f32(a)


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_dequantize_bit_exact(cuda, b2q_mod, oracle, gs):
    from b2q import synth

    w, s, b = synth.packed_weights((40,), 1024, gs, seed=gs)
    out = b2q_mod.dequantize(w, s, b, gs, 4)
    ref = oracle.dequantize(_np(w), _np(s), _np(b), gs, 4, "metal")
    assert np.array_equal(_np(out), ref)


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_bit_exact(cuda, b2q_mod, oracle, golden, gs):
    from b2q.synth import from_numpy_bits

    w = from_numpy_bits(golden[f"quantize_gs{gs}_w"])
    wq, s, b = b2q_mod.quantize(w, gs, 4)
    assert np.array_equal(_np(wq), golden[f"quantize_gs{gs}_wq"])
    assert np.array_equal(_np(s), golden[f"quantize_gs{gs}_s"])
    assert np.array_equal(_np(b), golden[f"quantize_gs{gs}_b"])


@pytest.mark.parametrize("M", [1, 2, 3, 8])
@pytest.mark.parametrize("gs", [64, 32, 128])
def test_qmv_streaming(cuda, b2q_mod, oracle, M, gs):
    from b2q import synth

    N, K = 272, 2048  # 17 row blocks: a ragged per-CTA split
    w, s, b = synth.packed_weights((N,), K, gs, seed=3)
    x = synth.activations((M, K), seed=4)
    y = b2q_mod.quantized_matmul(x, w, s, b, True, gs, 4)
    ref = oracle.qmv_metal(_np(x), _np(w), _np(s), _np(b), gs, 4)
    assert rel_l2(_bf(_np(y)), _bf(ref)) < TIGHT


def _top_mantissa_x(M, K, gs, seed):
    """Activations whose every group has its max |x| at +-(2 - 2^-7): the
    largest fixed-point value of the integer split (positive: the edge of the
    int8 pieces' range)."""
    import torch

    from b2q import synth

    x = synth.activations((M, K), seed=seed).float() * 0.25
    g = torch.arange(K // gs, device=x.device)
    pos = g * gs + (g * 7) % gs
    sign = torch.where(g % 3 == 2, -1.0, 1.0).to(x.device)
    x[:, pos] = sign * 1.9921875
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_qmv_group_max_at_top_mantissa(cuda, b2q_mod, oracle, gs):
    from b2q import synth

    N, K = 272, 2048
    w, s, b = synth.packed_weights((N,), K, gs, seed=5)
    x = _top_mantissa_x(1, K, gs, seed=6)
    y = b2q_mod.quantized_matmul(x, w, s, b, True, gs, 4)
    ref = oracle.qmv_metal(_np(x), _np(w), _np(s), _np(b), gs, 4)
    assert rel_l2(_bf(_np(y)), _bf(ref)) < TIGHT


def test_qmv_c0_full_size(cuda, b2q_mod, oracle):
    """Config 0: x [1, 4096], W [4096, 4096] g64."""
    from b2q import synth

    w, s, b = synth.packed_weights((4096,), 4096, 64, seed=0)
    x = synth.activations((1, 4096), seed=1)
    y = b2q_mod.quantized_matmul(x, w, s, b)
    ref = oracle.qmv_metal(_np(x), _np(w), _np(s), _np(b), 64, 4)
    assert rel_l2(_bf(_np(y)), _bf(ref)) < TIGHT
    assert rel_l2(_bf(_np(y)), _bf(ref)) < REL_L2
    # repeated calls are deterministic
    y2 = b2q_mod.quantized_matmul(x, w, s, b)
    assert np.array_equal(_np(y), _np(y2))


def test_qmv_golden_c0_slice(cuda, b2q_mod, golden):
    """Against the reference's own MLX CPU output (bf16 running sum): informational bound."""
    from b2q.synth import from_numpy_bits

    x, wq, s, b = (from_numpy_bits(golden[k]) for k in ("c0_x", "c0_wq", "c0_s", "c0_b"))
    y = b2q_mod.quantized_matmul(x, wq, s, b)
    assert rel_l2(_bf(_np(y)), _bf(golden["c0_y"])) < 0.2


@pytest.mark.parametrize("K,N,gs", [(640, 40, 32), (200 * 8, 24, 64), (96, 8, 32)])
def test_qmv_shape_general_path(cuda, b2q_mod, oracle, K, N, gs):
    """Shapes outside the streaming fast path (K not a multiple of 8 groups)."""
    from b2q import synth

    if K % gs:
        pytest.skip("K must be a multiple of the group size")
    w, s, b = synth.packed_weights((N,), K, gs, seed=5)
    x = synth.activations((3, K), seed=6)
    y = b2q_mod.quantized_matmul(x, w, s, b, True, gs, 4)
    ref = oracle.qmv_metal(_np(x), _np(w), _np(s), _np(b), gs, 4)
    assert rel_l2(_bf(_np(y)), _bf(ref)) < TIGHT


def test_gather_qmv(cuda, b2q_mod, oracle):
    import torch

    from b2q import synth

    E, N, K, M = 6, 64, 1024, 2
    w, s, b = synth.packed_weights((E, N), K, 64, seed=7)
    x = synth.activations((3, M, K), seed=8)
    lhs = torch.tensor([0, 2, 1, 2, 0], dtype=torch.int32, device="cuda").view(torch.uint32)
    rhs = torch.tensor([5, 0, 3, 3, 1], dtype=torch.int32, device="cuda").view(torch.uint32)
    y = b2q_mod.gather_qmm(x, w, s, b, lhs, rhs)
    assert tuple(y.shape) == (5, M, N)
    xs, ws_, ss, bs = _np(x), _np(w), _np(s), _np(b)
    for i, (l, r) in enumerate(zip([0, 2, 1, 2, 0], [5, 0, 3, 3, 1])):
        ref = oracle.qmv_metal(xs[l], ws_[r], ss[r], bs[r], 64, 4)
        assert rel_l2(_bf(_np(y[i])), _bf(ref)) < TIGHT


def test_gather_out_of_range_items_are_zero(cuda, b2q_mod):
    import torch

    from b2q import synth

    E, N, K = 2, 32, 512
    w, s, b = synth.packed_weights((E, N), K, 64, seed=9)
    x = synth.activations((1, 1, K), seed=10)
    lhs = torch.tensor([0, 0, 7], dtype=torch.int32, device="cuda").view(torch.uint32)
    rhs = torch.tensor([1, 9, 0], dtype=torch.int32, device="cuda").view(torch.uint32)
    y = b2q_mod.gather_qmm(x, w, s, b, lhs, rhs)
    yy = _np(y)
    assert np.all(yy[1] == 0) and np.all(yy[2] == 0)
    assert np.any(yy[0] != 0)


# ---- many rows per weight matrix (M > 8): the tcgen05 grouped GEMM ----------
# The tensor-core path rounds the dequantized weight to bf16 before the product
# (the reference's tile loader, quantized.h:485-530), so it is compared with the
# oracle's tile-loader arithmetic.

@pytest.mark.parametrize("M,N,K,gs", [(64, 256, 1024, 64), (200, 128, 2048, 32), (33, 384, 1024, 128)])
def test_qmm_tensor_core(cuda, b2q_mod, oracle, M, N, K, gs):
    from b2q import synth

    w, s, b = synth.packed_weights((N,), K, gs, seed=11)
    x = synth.activations((M, K), seed=12)
    y = b2q_mod.quantized_matmul(x, w, s, b, True, gs, 4)
    ref = oracle.qmm_tile_f32(_np(x), _np(w), _np(s), _np(b), gs, 4)
    assert rel_l2(_bf(_np(y)), ref) < TIGHT


def test_gather_qmm_tensor_core(cuda, b2q_mod, oracle):
    """Unsorted items, repeated experts, an out-of-range expert and an
    out-of-range x index (both give zeros)."""
    import torch

    from b2q import synth

    E, N, K, M = 5, 256, 1024, 24
    w, s, b = synth.packed_weights((E, N), K, 64, seed=13)
    x = synth.activations((4, M, K), seed=14)
    lhs_l = [3, 0, 2, 1, 0, 9, 2]
    rhs_l = [4, 0, 4, 2, 7, 1, 0]
    lhs = torch.tensor(lhs_l, dtype=torch.int32, device="cuda").view(torch.uint32)
    rhs = torch.tensor(rhs_l, dtype=torch.int32, device="cuda").view(torch.uint32)
    y = b2q_mod.gather_qmm(x, w, s, b, lhs, rhs)
    assert tuple(y.shape) == (7, M, N)
    xs, ws_, ss, bs = _np(x), _np(w), _np(s), _np(b)
    yy = _np(y)
    for i, (l, r) in enumerate(zip(lhs_l, rhs_l)):
        if l >= 4 or r >= E:
            assert np.all(yy[i] == 0), i
            continue
        ref = oracle.qmm_tile_f32(xs[l], ws_[r], ss[r], bs[r], 64, 4)
        assert rel_l2(_bf(yy[i]), ref) < TIGHT, i


def test_ws_forms_match_allocating_forms(cuda, b2q_mod):
    """b2q_qmm_ws / b2q_gather_qmm_ws run the same kernels as b2q_qmm /
    b2q_gather_qmm on the caller's workspace: identical bits, two calls in a
    row on one uncleared workspace, M on both sides of the tensor-core switch."""
    import torch

    from b2q import synth

    E, N, K = 5, 256, 1024
    w, s, b = synth.packed_weights((E, N), K, 64, seed=31)
    lhs = torch.tensor([3, 0, 2, 1, 0, 2], dtype=torch.int32, device="cuda").view(torch.uint32)
    rhs = torch.tensor([4, 0, 4, 2, 1, 0], dtype=torch.int32, device="cuda").view(torch.uint32)
    for M in (1, 5, 24, 130):
        x = synth.activations((4, M, K), seed=32 + M)
        need = b2q_mod.gather_qmm_workspace_size(6, M, N, K, E)
        ws = torch.full((need,), 0xA5, dtype=torch.uint8, device="cuda")  # garbage: nothing is read before written
        ref = b2q_mod.gather_qmm(x, w, s, b, lhs, rhs)
        for _ in range(2):
            y = b2q_mod.gather_qmm(x, w, s, b, lhs, rhs, workspace=ws)
            assert torch.equal(y, ref), M
        x1 = synth.activations((M, K), seed=40 + M)
        need1 = b2q_mod.gather_qmm_workspace_size(1, M, N, K, 1)
        ws1 = torch.full((need1,), 0x5A, dtype=torch.uint8, device="cuda")
        ref1 = b2q_mod.quantized_matmul(x1, w[1], s[1], b[1])
        for _ in range(2):
            assert torch.equal(b2q_mod.quantized_matmul(x1, w[1], s[1], b[1], workspace=ws1), ref1), M
