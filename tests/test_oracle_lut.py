"""The metadata pair index restatement (CPU, no device): the literal host loop
of TrackAffineLUT.build (Runner/FastModel/TrackAffineLUT.swift:64-83) against
the vectorised oracle, the table order rule (first occurrence below 2^20
groups, ascending pair value from 2^20: :63, :88-103), the fail-closed limit,
and the C ABI's host-side refusals."""
from __future__ import annotations

import ctypes

import numpy as np

from oracle import oracle as orc


def _pairs_tensor(rng, shape, n_scales, n_noise):
    """bf16 bit patterns with few distinct (scale, bias) pairs, as in a real
    checkpoint: scales from a small set, biases -8*scale plus a small set of
    offsets."""
    sv = orc.f32_to_bf16(rng.uniform(0.002, 0.02, n_scales).astype(np.float32))
    si = rng.integers(0, n_scales, shape)
    s = sv[si]
    off = rng.integers(0, n_noise, shape).astype(np.float32) * 1e-4
    b = orc.f32_to_bf16((-8.0 * orc.bf16_to_f32(s) + off).astype(np.float32))
    return s, b


def test_hand_case_first_occurrence():
    s = np.array([[3, 1], [3, 2]], np.uint16)
    b = np.array([[0, 0], [0, 7]], np.uint16)
    idx, table = orc.affine_lut_build(s, b)
    assert table.tolist() == [3, 1, 2 | (7 << 16)]
    assert idx.tolist() == [[0, 1], [0, 2]]


def test_loop_and_vectorised_agree():
    rng = np.random.default_rng(5)
    s, b = _pairs_tensor(rng, (64, 96), 40, 7)
    a = orc.affine_lut_build_loop(s, b)
    v = orc.affine_lut_build(s, b)
    assert np.array_equal(a[0], v[0]) and np.array_equal(a[1], v[1])
    assert np.array_equal(v[1][v[0].astype(np.int64)], orc.affine_lut_pairs(s, b))


def test_value_order_from_2p20_groups():
    rng = np.random.default_rng(6)
    s, b = _pairs_tensor(rng, (1 << 14, 64), 50, 9)  # exactly 2^20 groups
    idx, table = orc.affine_lut_build(s, b)
    assert np.all(np.diff(table.astype(np.int64)) > 0)  # ascending, distinct
    assert np.array_equal(table[idx.astype(np.int64)], orc.affine_lut_pairs(s, b))
    # one group fewer: the host loop's first-occurrence order
    s2, b2 = s.reshape(-1)[:-1], b.reshape(-1)[:-1]
    idx2, table2 = orc.affine_lut_build(s2, b2)
    assert idx2[0] == 0 and table2[0] == orc.affine_lut_pairs(s2[:1], b2[:1])[0]


def test_limit_fails_closed():
    rng = np.random.default_rng(7)
    s, b = _pairs_tensor(rng, (32, 64), 30, 5)
    n = np.unique(orc.affine_lut_pairs(s, b)).size
    assert orc.affine_lut_build(s, b, max_entries=n) is not None
    assert orc.affine_lut_build(s, b, max_entries=n - 1) is None
    assert orc.affine_lut_build_loop(s, b, max_entries=n - 1) is None


def test_config_distribution_fits_the_reference_limit():
    """The configs' own metadata (scale ~ U(0.002, 0.02) in bf16, bias =
    -8 scale + N(0, 1e-3) in bf16) has far fewer distinct pairs than groups:
    the index applies to the benchmark tensors."""
    rng = np.random.default_rng(0)
    s = orc.f32_to_bf16(rng.uniform(0.002, 0.02, (4096, 64)).astype(np.float32))
    b = orc.f32_to_bf16((-8.0 * orc.bf16_to_f32(s) + rng.normal(0, 1e-3, s.shape)).astype(np.float32))
    res = orc.affine_lut_build(s, b)
    assert res is not None and res[1].size < 16384


def test_abi_refusals(b2q_mod):
    lib = b2q_mod.lib()
    cnt = ctypes.c_int(7)
    fake = 1 << 20
    # null count_out, bad max_entries (not a multiple of 4 / too large), null workspace
    assert lib.b2q_affine_lut_build(fake, fake, 16, fake, fake, 32768, None, fake, 1 << 30, None) == -1
    assert lib.b2q_affine_lut_build(fake, fake, 16, fake, fake, 30, ctypes.addressof(cnt), fake, 1 << 30, None) == -1
    assert cnt.value == -1
    assert lib.b2q_affine_lut_build(fake, fake, 16, fake, fake, 1 << 17, ctypes.addressof(cnt), fake, 1 << 30,
                                    None) == -1
    assert lib.b2q_affine_lut_build(fake, fake, 16, fake, fake, 32768, ctypes.addressof(cnt), None, 0, None) == -1
    need = lib.b2q_affine_lut_workspace_size(32768)
    assert need >= 32768 * 4 * 8  # a hash set of 4x the limit (8-byte slots)
    assert lib.b2q_affine_lut_build(fake, fake, 16, fake, fake, 32768, ctypes.addressof(cnt), fake, need - 1,
                                    None) == -1
    # qmv through the table: only 4-bit; bad shapes
    assert lib.b2q_qmv_lut(fake, fake, fake, fake, 100, fake, 4096, 4096, 64, 8, None) == -2
    assert lib.b2q_qmv_lut(fake, fake, fake, fake, 0, fake, 4096, 4096, 64, 4, None) == -1
