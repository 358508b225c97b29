"""The bench's algorithmic work figures (the roofline numerators) and CPU-baseline
extrapolations, checked on the CPU against the configuration's stated sizes."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_algorithmic_bytes_and_flops():
    # config 1: 8 experts x 10,616,832 B + router 1,048,576 B + 65,536 B of activations
    assert bench.EXPERT_BYTES == 10_616_832
    assert bench.DECODE_BYTES == 86_049_344
    # config 0: packed 8,388,608 + metadata 1,048,576 + x + y
    assert bench.C0_BYTES == 9_453_568
    # config 2: 16384 assignments x (gate|up + down) + the router GEMM
    assert bench.PREFILL_FLOP == 620_622_774_272


def test_row_equivalents():
    # gate + up: 2 x 1536 rows of K 4096; down 4096 rows of K 1536 = 1536 K-4096 rows
    assert bench.prefill_rows_per_assignment() == 4608
    assert bench.decode_rows_per_token() == 8 * 4608
    # config 3: 48 x (q|k|v 5120 + o 4096 + 36864) + lm_head 151936
    assert bench.decoder_rows_per_token() == 48 * (5120 + 4096 + 36864) + 151936


def test_decoder_rows_follow_the_model_config():
    from b2q.model import DecoderConfig

    cfg = DecoderConfig()
    assert bench.DEC_LAYERS == cfg.n_layers
    assert bench.DEC_QKV_ROWS == cfg.qkv_rows
    assert bench.DEC_ATTN_DIM == cfg.n_heads * cfg.head_dim
    assert bench.DEC_VOCAB == cfg.vocab
    # the weights a token reads are the row-equivalents' packed bytes (K = 4096, g64:
    # 2048 + 256 bytes per row) plus the bf16 router, up to the KV cache
    weights = bench.decoder_rows_per_token() * (4096 // 2 + 4 * 4096 // 64) + cfg.n_layers * cfg.n_experts * 4096 * 2
    kv = cfg.decode_bytes_per_token(1024) - weights
    assert 0 <= kv < 0.05 * weights


def test_cpu_baseline_extrapolations():
    t_row = 20e-6
    dec = bench.decoder_cpu_baseline(t_row, "reference")
    assert dec["value"] == pytest.approx(1.0 / (bench.decoder_rows_per_token() * t_row))
    assert dec["cores"] == 1 and "lower bound" in dec["sample"] and "quantized share only" in dec["sample"]
    pre = bench.prefill_cpu_baseline(t_row, "port")
    rows = bench.PREFILL_T * bench.TOPK * 4608 + bench.PREFILL_T * bench.E
    assert pre["value"] == pytest.approx(bench.PREFILL_T / (rows * t_row))
    assert pre["kind"] == "port" and "extrapolated" in pre["sample"]
