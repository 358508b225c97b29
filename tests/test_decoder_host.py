"""Host-side arithmetic of the decoder around the path (no GPU): its shape
rules and the bytes one decode step reads (the roofline basis of the
full-decoder benchmark leg)."""
from __future__ import annotations

import pytest


def test_decode_bytes_of_the_config3_model():
    from b2q.model import DecoderConfig

    c = DecoderConfig()
    H = 4096
    attn = (c.qkv_rows + H) * (H // 2 + 4 * (H // 64))
    assert attn == 21_233_664  # q|k|v [5120, 4096] + o [4096, 4096], 4-bit g64
    expert = 3 * 1536 * (H // 2 + 4 * (H // 64))
    assert expert == 10_616_832
    lm_head = 151936 * (H // 2 + 4 * (H // 64))
    kv = 2 * 4 * 128 * 2 * 1025
    total = 48 * (attn + 128 * H * 2 + 8 * expert + kv) + lm_head
    assert c.decode_bytes_per_token(1024) == total
    assert 5.4e9 < total < 5.7e9


def test_config_rules():
    from b2q.model import DecoderConfig

    with pytest.raises(ValueError):
        DecoderConfig(n_heads=30, n_kv_heads=4).validate()
    with pytest.raises(ValueError):
        DecoderConfig(top_k=200).validate()
    assert DecoderConfig(n_layers=2).validate().qkv_rows == (32 + 8) * 128


def test_decoder_kernels_refuse_bad_shapes(b2q_mod):
    lib = b2q_mod.lib()
    assert lib.b2q_rms_norm(None, None, None, 2, 1001, 1e-6, None) == -1
    assert lib.b2q_rms_norm(None, None, None, 0, 1024, 1e-6, None) == 0
    assert lib.b2q_rope(None, 1, 4, 127, None, 0, 1e6, None) == -1
    assert lib.b2q_embed_gather(None, None, None, None, None, 1, 10, 1024, 48, 4, None, None) == -2
    assert lib.b2q_embed_gather(None, None, None, None, None, 0, 10, 1024, 64, 4, None, None) == 0
    assert lib.b2q_gqa_decode_workspace_size(1, 32, 4, 128, 1280) == 4 * 4 * 10 * 8 * 130  # 128-key chunks
    assert lib.b2q_gqa_decode(None, 4096, None, None, None, None, 1, 30, 4, 128, 64, None, None, 0, None) == -1
    assert lib.b2q_rope_kv(None, 0, 8, 2, 128, None, 1e6, None, None, 64, None, None) == 0
    assert lib.b2q_add_rms_norm(None, None, None, None, None, 1, 1001, 1e-6, None) == -1


def test_moe_decode_norm_refuses_host_tensors():
    """MoE.decode_norm hands raw pointers to a kernel: host tensors, other
    dtypes and wrong sizes are refused before the library is called."""
    import pytest
    import torch

    from b2q.nn import MoE

    m = MoE.__new__(MoE)  # the refusals need only the hidden size (no device here)
    m._H, m._ws1 = 16, None
    h = torch.zeros((1, 16), dtype=torch.bfloat16)
    nw = torch.ones(16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="h: expected"):
        m.decode_norm(h, None, nw, 1e-6, None)
    with pytest.raises(ValueError, match="expected"):
        m.decode_norm(h.float(), None, nw, 1e-6, None)


def test_qmv_lut_refuses_host_tensors():
    """b2q.lut.qmv_lut hands raw pointers to a kernel: a host x or w of the
    one-row shape is refused before the library is called."""
    import pytest
    import torch

    from b2q.lut import AffineLUT, qmv_lut

    meta = AffineLUT(torch.zeros((32, 8), dtype=torch.int16), torch.zeros(4, dtype=torch.int32), 1)
    x = torch.zeros((1, 512), dtype=torch.bfloat16)
    w = torch.zeros((32, 64), dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA device"):
        qmv_lut(x, w, meta)
    # not the one-row product: left to the plain path
    assert qmv_lut(torch.zeros((2, 512), dtype=torch.bfloat16), w, meta) is None
