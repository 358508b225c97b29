"""The metadata pair index on the GPU (TrackAffineLUT,
Runner/FastModel/TrackAffineLUT.swift:58-110) and the one-row product through
it (TrackLUTGemv, :114-368).

* The device build gives the reference's index and table bit for bit: first
  occurrence order for a config-0 weight's metadata (262,144 groups), ascending
  pair value for a config-1 expert stack (12,582,912 groups).
* The expansion gives back the loaded scales / biases bit for bit.
* The product through the table is bit-identical to the plain product on the
  same metadata (the same bf16 bits reach the same arithmetic), which is itself
  pinned to the reference's fp32 kernel.
* Tensors that do not qualify are reported as not indexed (fail closed); tables
  larger than the kernel's shared-memory copy fall back to the plain product.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _np(t):
    from b2q.synth import to_numpy_bits

    return to_numpy_bits(t)


@pytest.mark.parametrize("rows_shape,K", [((4096,), 4096), ((128, 1536), 4096)])
def test_build_matches_reference_order(cuda, b2q_mod, rows_shape, K):
    from b2q import lut, synth

    _, s, b = synth.packed_weights(rows_shape, K, 64, seed=21)
    meta = lut.AffineLUT.build(s, b)
    assert meta is not None
    ref_idx, ref_table = orc.affine_lut_build(_np(s), _np(b))
    assert meta.count == ref_table.size
    assert np.array_equal(_np(meta.table)[: meta.count], ref_table)
    assert np.all(_np(meta.table)[meta.count: (meta.count + 3) // 4 * 4] == 0)
    assert np.array_equal(_np(meta.index).view(np.uint16), ref_idx)
    import torch

    assert torch.equal(meta.lazy_scales(), s) and torch.equal(meta.lazy_biases(), b)


def test_not_indexed_past_the_limit(cuda, b2q_mod):
    from b2q import lut, synth

    _, s, b = synth.packed_weights((64,), 4096, 64, seed=22)
    n = np.unique(orc.affine_lut_pairs(_np(s), _np(b))).size
    assert lut.AffineLUT.build(s, b, max_entries=(n + 3) // 4 * 4) is not None
    assert lut.AffineLUT.build(s, b, max_entries=(n - 4) // 4 * 4) is None
    # twice in a row on the same sizes: no state carried between builds
    assert lut.AffineLUT.build(s, b, max_entries=(n - 4) // 4 * 4) is None
    assert lut.AffineLUT.build(s, b, max_entries=(n + 3) // 4 * 4).count == n


@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("N", [4096, 1040])
def test_qmv_lut_bit_identical(cuda, b2q_mod, gs, N):
    import torch

    from b2q import lut, synth

    K = 4096
    w, s, b = synth.packed_weights((N,), K, gs, seed=23 + gs)
    meta = lut.AffineLUT.build(s, b)
    assert meta is not None
    for seed in (24, 25):  # two calls in a row
        x = synth.activations((1, K), seed=seed)
        y = lut.qmv_lut(x, w, meta, gs)
        assert y is not None
        ref = b2q_mod.quantized_matmul(x, w, s, b, True, gs)
        assert torch.equal(y, ref)


def test_quantized_linear_with_pair_index(cuda, b2q_mod):
    import torch

    from b2q import synth

    w, s, b = synth.packed_weights((2048,), 4096, 64, seed=26)
    plain = b2q_mod.QuantizedLinear(w, s, b, 64)
    indexed = plain.with_pair_index()
    assert indexed.meta is not None and indexed is not plain
    x1 = synth.activations((1, 4096), seed=27)
    assert torch.equal(indexed(x1), plain(x1))
    x3 = synth.activations((3, 4096), seed=28)  # not one row: the plain product
    assert torch.equal(indexed(x3), plain(x3))


def test_large_table_falls_back(cuda, b2q_mod):
    """20,000 distinct pairs: indexed (under the reference's 32,768), but past
    the kernel's 16,384-entry shared-memory copy, so the one-row product
    declines and the caller takes the plain product."""
    import torch

    from b2q import lut, synth

    N, K = 1024, 4096
    w, _, _ = synth.packed_weights((N,), K, 64, seed=29)
    G = N * (K // 64)
    g = np.arange(G)
    sbits = (0x3B00 + (g % 200)).astype(np.uint16)          # 200 scales in [2^-9, 2^-7)
    bbits = (0xBC00 + (g // 200) % 100).astype(np.uint16)   # 100 biases near -2^-7
    s = synth.from_numpy_bits(sbits.reshape(N, K // 64))
    b = synth.from_numpy_bits(bbits.reshape(N, K // 64))
    meta = lut.AffineLUT.build(s, b)
    assert meta is not None and meta.count == 20000
    x = synth.activations((1, K), seed=30)
    assert lut.qmv_lut(x, w, meta, 64) is None
    lin = b2q_mod.QuantizedLinear(w, s, b, 64, meta=meta)
    assert torch.equal(lin(x), b2q_mod.quantized_matmul(x, w, s, b))
