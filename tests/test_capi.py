"""The C-ABI library loads, exports every declared entry point, and its host
side rejects bad arguments before touching the device (CPU-only checks)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "b2q.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^B2Q_API\s+[\w\s\*]+?\b(b2q_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_surface():
    syms = declared_symbols()
    for must in ("b2q_qmm", "b2q_gather_qmm", "b2q_dequantize", "b2q_quantize", "b2q_moe_route",
                 "b2q_moe_gate_up_act", "b2q_moe_down_combine", "b2q_moe_decode", "b2q_moe_prefill",
                 "b2q_moe_sort", "b2q_last_error"):
        assert must in syms


def test_library_exports_every_declared_symbol(b2q_mod):
    from b2q._lib import LIB_PATH, SIGNATURES

    lib = ctypes.CDLL(LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in SIGNATURES, f"{name} missing from the Python binding"


def test_host_side_argument_errors(b2q_mod):
    lib = b2q_mod.lib()
    # unsupported bit width / group size: refused before any CUDA call
    assert lib.b2q_qmm(None, None, None, None, None, 1, 16, 512, 64, 3, 1, None) == -2
    assert b"bits=3" in lib.b2q_last_error()
    assert lib.b2q_qmm(None, None, None, None, None, 1, 16, 512, 48, 4, 1, None) == -2
    # transpose=false is not implemented for the path
    assert lib.b2q_gather_qmm(None, None, None, None, None, None, None, 1, 1, 16, 512, 1, 1, 64, 4, 0, 0,
                              None) == -2
    # bad shapes
    assert lib.b2q_dequantize(None, None, None, None, 4, 100, 64, 4, None) == -1
    assert lib.b2q_moe_route(None, None, None, 1, 16, 40, None) == -1
    assert lib.b2q_moe_decode(*([None] * 15), 1, 4096, 128, 1536, 9, 64, 4, None, 0, None) == -2
    # empty work is a no-op success
    assert lib.b2q_qmm(None, None, None, None, None, 0, 16, 512, 64, 4, 1, None) == 0
    # a null workspace is refused
    assert lib.b2q_workspace_status(None, 0, None) == -1


def test_workspace_sizes(b2q_mod):
    lib = b2q_mod.lib()
    d = lib.b2q_moe_decode_workspace_size(1, 4096, 128, 1536, 8)
    assert d >= 256 + 8 * 1536 * 2 + 128 * 4
    p = lib.b2q_moe_prefill_workspace_size(2048, 4096, 128, 1536, 8)
    assert p >= 16384 * (3 * 1536 * 2 + 4096 * 2)
    assert lib.b2q_moe_decode_workspace_size(0, 4096, 128, 1536, 8) == 0
    # the allocation-free product forms: the sorted copy of x dominates
    q = lib.b2q_gather_qmm_workspace_size(64, 32, 4096, 4096, 16)
    assert q >= 64 * 32 * 4096 * 2
    assert lib.b2q_gather_qmm_workspace_size(1, 8, 4096, 4096, 1) > 0


def test_ws_products_refuse_small_or_null_workspace(b2q_mod):
    """Checked on the host before any device call: fake 16-byte aligned
    addresses are never dereferenced."""
    lib = b2q_mod.lib()
    fake = 1 << 20  # aligned, never touched
    M, N, K = 64, 256, 1024
    need = lib.b2q_gather_qmm_workspace_size(1, M, N, K, 1)
    assert lib.b2q_qmm_ws(fake, fake, fake, fake, fake, M, N, K, 64, 4, 1, None, 0, None) == -1
    assert b"null workspace" in lib.b2q_last_error()
    assert lib.b2q_qmm_ws(fake, fake, fake, fake, fake, M, N, K, 64, 4, 1, fake, need - 256, None) == -1
    assert b"workspace" in lib.b2q_last_error()
    assert lib.b2q_gather_qmm_ws(fake, fake, fake, fake, None, None, fake, 2, M, N, K, 2, 2, 64, 4, 1, 0,
                                 fake + 16, 1 << 30, None) == -1  # not 256-byte aligned


def test_python_ops_validate_inputs(b2q_mod):
    import torch

    x = torch.zeros(1, 512, dtype=torch.bfloat16)
    w = torch.zeros(16, 64, dtype=torch.int32)
    s = torch.zeros(16, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA device"):
        b2q_mod.quantized_matmul(x, w, s, s)
    with pytest.raises(ValueError):
        b2q_mod.ops._check_quant(w, s, s[:, :4], 64, 4)
    with pytest.raises(ValueError, match="only 4-bit"):
        b2q_mod.ops._check_quant(w, s, s, 64, 8)


def test_new_entry_points_refuse_bad_arguments(b2q_mod):
    """Host-side refusals of the fused-norm products, the one-launch decode
    attention and the peer exchange set-up, checked before any device call
    (fake aligned addresses are never dereferenced)."""
    import ctypes

    lib = b2q_mod.lib()
    fake = 1 << 20
    # fused norm: h_out aliasing h, missing h_out with delta, unsupported bits
    assert lib.b2q_qmv_norm(fake, fake + 4096, fake, 1e-6, fake, fake, fake, fake, fake, 4096, 4096, 64, 4,
                            None) == -1
    assert b"alias" in lib.b2q_last_error()
    assert lib.b2q_qmv_norm(fake, fake, fake, 1e-6, None, fake, fake, fake, fake, 4096, 4096, 64, 4, None) == -1
    assert lib.b2q_qmv_norm(fake, None, fake, 1e-6, None, fake, fake, fake, fake, 4096, 4096, 64, 8, None) == -2
    assert lib.b2q_moe_decode_norm(fake, fake + 4096, fake, 1e-6, fake, *([fake] * 10), fake, None, None, None,
                                   4096, 128, 1536, 8, 64, 4, None, 0, None) == -1
    # attention: too many window rows, head_dim not a multiple of 16, q_ld too short, null workspace
    assert lib.b2q_attn_decode(fake, 5120, fake, fake, fake, fake, 9, 32, 4, 128, 1e6, 1280, None, fake, 1 << 30,
                               None) == -1
    assert lib.b2q_attn_decode(fake, 5120, fake, fake, fake, fake, 1, 32, 4, 120, 1e6, 1280, None, fake, 1 << 30,
                               None) == -1
    assert lib.b2q_attn_decode(fake, 100, fake, fake, fake, fake, 1, 32, 4, 128, 1e6, 1280, None, fake, 1 << 30,
                               None) == -1
    assert lib.b2q_attn_decode(fake, 5120, fake, fake, fake, fake, 1, 32, 4, 128, 1e6, 1280, None, None, 0,
                               None) == -1
    assert lib.b2q_attn_decode_workspace_size(9, 32, 4, 128, 1280) == 0
    assert lib.b2q_attn_decode_workspace_size(8, 32, 4, 128, 1280) >= 8 * 4 * 4
    # the native host loop: no steps, or null buffers
    w9 = (ctypes.c_void_p * 9)(*([fake] * 9))
    wr = (ctypes.c_void_p * 1)(fake)
    assert lib.b2q_moe_decode_host_loop(fake, 1, fake, wr, w9, 1, 4096, 128, 1536, 8, 64, 4, fake, fake, fake,
                                        1 << 20, 1, 0, None, ctypes.byref(ctypes.c_float())) == -1
    assert lib.b2q_moe_decode_host_loop(fake, 1, fake, wr, w9, 1, 4096, 128, 1536, 8, 64, 4, None, fake, fake,
                                        1 << 20, 1, 4, None, ctypes.byref(ctypes.c_float())) == -1
    # peer exchange: no communicator, short handle buffer, open before set-up
    h = (ctypes.c_char * 64)()
    assert lib.b2q_ep_peer_setup(None, 4096, ctypes.cast(h, ctypes.c_void_p), 64) == -1
    assert lib.b2q_ep_peer_open(None, ctypes.cast(h, ctypes.c_void_p), 64) == -1
    # a one-rank communicator (no NCCL needed) has nothing to exchange and no buffer to open
    comm = ctypes.c_void_p()
    assert lib.b2q_ep_comm_init(ctypes.byref(comm), 1, 0, None, 0) == 0
    try:
        assert lib.b2q_ep_peer_setup(comm, 4096, ctypes.cast(h, ctypes.c_void_p), 64) == -1
        assert b"one rank" in lib.b2q_last_error()
        assert lib.b2q_ep_peer_open(comm, ctypes.cast(h, ctypes.c_void_p), 64) == -1
        assert b"setup first" in lib.b2q_last_error()
    finally:
        assert lib.b2q_ep_comm_destroy(comm) == 0
    assert lib.b2q_ep_peer_buffer_bytes(4096) >= 2 * 8 * 4096 * 4
    assert lib.b2q_ep_peer_buffer_bytes(0) == 0
