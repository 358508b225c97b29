"""ctypes binding of libb2q.so (the C ABI declared in include/b2q.h).

The library is the product: if it is missing this module raises at import
time -- there is no Python or CPU fallback for any operator.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("B2Q_LIB", os.path.join(PKG_DIR, "lib", "libb2q.so"))

B2Q_OK = 0
B2Q_EINVAL = -1
B2Q_EUNSUPPORTED = -2
B2Q_ECUDA = -3
B2Q_ETIMEOUT = -4
B2Q_ENCCL = -5

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_LL = ctypes.c_longlong

# name -> (restype, argtypes); mirrors include/b2q.h one to one
SIGNATURES = {
    "b2q_last_error": (ctypes.c_char_p, []),
    "b2q_version": (_I, []),
    "b2q_device_sm_count": (_I, []),
    "b2q_dequantize": (_I, [_P, _P, _P, _P, _I64, _I, _I, _I, _P]),
    "b2q_quantize": (_I, [_P, _P, _P, _P, _I64, _I, _I, _I, _P]),
    "b2q_qmm": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "b2q_gather_qmm": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P]),
    "b2q_gather_qmm_workspace_size": (_SZ, [_I] * 5),
    "b2q_qmm_ws": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "b2q_gather_qmm_ws": (_I, [_P] * 7 + [_I] * 10 + [_P, _SZ, _P]),
    "b2q_affine_lut_workspace_size": (_SZ, [_I]),
    "b2q_affine_lut_build": (_I, [_P, _P, _I64, _P, _P, _I, _P, _P, _SZ, _P]),
    "b2q_affine_lut_expand": (_I, [_P, _P, _I64, _P, _P, _P]),
    "b2q_qmv_lut": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "b2q_moe_router_logits": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "b2q_moe_route": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "b2q_moe_gate_up_act": (_I, [_P] * 10 + [_I] * 7 + [_P]),
    "b2q_moe_down_combine": (_I, [_P] * 7 + [_I] * 7 + [_P]),
    "b2q_moe_decode_workspace_size": (_SZ, [_I] * 5),
    "b2q_moe_decode": (_I, [_P] * 15 + [_I] * 7 + [_P, _SZ, _P]),
    "b2q_moe_decode_noalloc": (_I, [_P] * 15 + [_I] * 6 + [_P, _P]),
    "b2q_moe_decode_host_loop": (_I, [_P, _I, _P, _P, _P, _I] + [_I] * 6 + [_P, _P, _P, _SZ, _I, _I, _P, _P]),
    "b2q_moe_prefill_workspace_size": (_SZ, [_I] * 5),
    "b2q_moe_prefill": (_I, [_P] * 14 + [_I] * 7 + [_P, _SZ, _P]),
    "b2q_swiglu": (_I, [_P, _P, _P, _I64, _P]),
    "b2q_moe_sorted_combine": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "b2q_sort_workspace_size": (_SZ, [_I, _I]),
    "b2q_moe_sort": (_I, [_P] * 5 + [_I] * 3 + [_P, _SZ, _P]),
    "b2q_ep_unique_id": (_I, [_P, _SZ]),
    "b2q_ep_comm_init": (_I, [_P, _I, _I, _P, _SZ]),
    "b2q_ep_comm_destroy": (_I, [_P]),
    "b2q_ep_peer_buffer_bytes": (_SZ, [_I]),
    "b2q_ep_peer_setup": (_I, [_P, _I, _P, _SZ]),
    "b2q_ep_peer_open": (_I, [_P, _P, _SZ]),
    "b2q_ep_moe_decode_workspace_size": (_SZ, [_I] * 5),
    "b2q_ep_moe_decode": (_I, [_P] * 16 + [_I] * 9 + [_P, _SZ, _P]),
    "b2q_ep_moe_prefill_workspace_size": (_SZ, [_I] * 5),
    "b2q_ep_moe_prefill": (_I, [_P] * 16 + [_I] * 9 + [_P, _SZ, _P]),
    "b2q_ep_expert_range": (_I, [_I, _I, _I, _P, _P]),
    "b2q_ep_a2a_dispatch_workspace_size": (_SZ, [_I] * 5),
    "b2q_ep_a2a_dispatch": (_I, [_P] * 8 + [_I] * 5 + [_P, _SZ, _P]),
    "b2q_ep_a2a_experts_workspace_size": (_SZ, [_I] * 5),
    "b2q_ep_a2a_experts": (_I, [_P] * 12 + [_I] * 9 + [_P, _SZ, _P]),
    "b2q_ep_a2a_combine": (_I, [_P] * 3 + [_I] * 3 + [_P]),
    "b2q_ep_moe_prefill_a2a_workspace_size": (_SZ, [_I] * 6),
    "b2q_ep_moe_prefill_a2a": (_I, [_P] * 15 + [_I] * 8 + [_P, _SZ, _P]),
    "b2q_embed_gather": (_I, [_P] * 5 + [_I] * 5 + [_P, _P]),
    "b2q_rms_norm": (_I, [_P] * 3 + [_I, _I, ctypes.c_float, _P]),
    "b2q_rope": (_I, [_P, _I, _I, _I, _P, _I, ctypes.c_float, _P]),
    "b2q_add_rms_norm": (_I, [_P] * 5 + [_I, _I, ctypes.c_float, _P]),
    "b2q_rope_kv": (_I, [_P, _I, _I, _I, _I, _P, ctypes.c_float, _P, _P, _I, _P, _P]),
    "b2q_gqa_decode_workspace_size": (_SZ, [_I] * 5),
    "b2q_gqa_decode": (_I, [_P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "b2q_qmv_norm": (_I, [_P, _P, _P, ctypes.c_float] + [_P] * 5 + [_I] * 4 + [_P]),
    "b2q_moe_decode_norm": (_I, [_P, _P, _P, ctypes.c_float] + [_P] * 15 + [_I] * 6 + [_P, _SZ, _P]),
    "b2q_attn_decode_workspace_size": (_SZ, [_I] * 5),
    "b2q_attn_decode": (_I, [_P, _I, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _SZ, _P]),
    "b2q_st_open": (_I, [ctypes.c_char_p, _P]),
    "b2q_st_close": (_I, [_P]),
    "b2q_st_count": (_I, [_P]),
    "b2q_st_name": (_I, [_P, _I, ctypes.c_char_p, _SZ]),
    "b2q_st_info": (_I, [_P, ctypes.c_char_p, ctypes.c_char_p, _SZ, _P, _I, _P, _P]),
    "b2q_st_read": (_I, [_P, ctypes.c_char_p, _P, _SZ, _I, _P]),
    "b2q_workspace_reset": (_I, [_P, _SZ, _P]),
    "b2q_workspace_status": (_I, [_P, _SZ, _P]),
    "b2q_selftest_wait_timeout": (_I, [_P, _SZ, _LL, _P]),
}


class B2QError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"b2q error {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"libb2q.so not found at {path}; build it with "
            "`python mlxfast-qwen38-125b-a6b-engine_b200/build.py` (no fallback exists)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


def check(rc: int) -> None:
    if rc != B2Q_OK:
        msg = lib().b2q_last_error()
        raise B2QError(rc, msg.decode() if msg else "")
