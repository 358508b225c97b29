"""b2q -- B200 affine 4-bit weight products (host-side mirror of the reference surface).

The compute lives in lib/libb2q.so (C ABI, include/b2q.h); this package binds
it with ctypes and uses PyTorch tensors for device memory and streams.
"""
from ._lib import B2QError, lib  # noqa: F401
from . import ep, loader, lut, ops, nn  # noqa: F401
from .lut import AffineLUT  # noqa: F401
from .ops import (  # noqa: F401
    dequantize, down_combine, gate_up_act, gather_qmm, gather_qmm_workspace_size, moe_decode, moe_prefill, moe_sort, quantize,
    quantized_matmul, route, router_logits, sorted_combine, swiglu, Workspace,
)
from .nn import MoE, QuantizedLinear, SwitchGLU, SwitchLinear  # noqa: F401

__version__ = "0.1.0"
