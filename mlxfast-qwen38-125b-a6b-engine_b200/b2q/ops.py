"""Tensor-level operators over the C ABI (PyTorch tensors for device memory).

Names, argument meaning and error behaviour follow MLX's quantized operator
surface as the reference engine calls it:

* ``quantize`` / ``dequantize``   -- mlx_quantize / mlx_dequantize
  (Vendor/mlx-swift/Source/Cmlx/mlx-c/mlx/c/ops.h:801, :359)
* ``quantized_matmul``            -- mlx_quantized_matmul (ops.h:809)
* ``gather_qmm``                  -- mlx_gather_qmm (ops.h:475)
* ``router_logits`` / ``route`` / ``gate_up_act`` / ``down_combine`` --
  TrackFastMoEKernels.routerGemv / route / gateUpAct / downCombine
  (Runner/FastModel/TrackFastMoE.swift:2300, :894, :1371, :1554)

Shape or dtype errors raise ``ValueError`` (MLX raises std::invalid_argument);
device-side failures raise ``B2QError``. Every call enqueues on the current
torch CUDA stream.
"""
from __future__ import annotations

import torch

from ._lib import B2QError, check, lib

__all__ = [
    "quantize", "dequantize", "quantized_matmul", "gather_qmm", "gather_qmm_workspace_size", "router_logits", "route",
    "gate_up_act", "down_combine", "swiglu", "sorted_combine", "moe_decode", "moe_prefill", "moe_sort", "Workspace", "B2QError",
]


try:  # the raw handle without building a torch.cuda.Stream object (a per-call cost)
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream(device=None):
    if _raw_stream is not None:
        idx = device.index if device is not None and device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def _dev(t: torch.Tensor, name: str, dtypes) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name}: tensor must live on a CUDA device (got {t.device})")
    if t.dtype not in dtypes:
        raise ValueError(f"{name}: dtype {t.dtype} not in {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: tensor must be contiguous")
    return t


_BF16 = (torch.bfloat16,)
_PACK = (torch.uint32, torch.int32)
_IDX = (torch.uint32, torch.int32)
_F32 = (torch.float32,)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _check_quant(w, scales, biases, group_size, bits):
    if bits != 4:
        raise ValueError(f"bits={bits}: only 4-bit affine weights are implemented")
    if group_size not in (32, 64, 128):
        raise ValueError("Quantization group size must be 32, 64 or 128.")
    K = w.shape[-1] * 32 // bits
    if scales.shape != biases.shape or scales.shape[:-1] != w.shape[:-1] or scales.shape[-1] * group_size != K:
        raise ValueError(
            "[quantized] Shape of scales and biases does not match the matrix given the quantization parameters")
    return K


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """bf16 [..., K] -> (packed uint32 [..., K/8], scales bf16 [..., K/gs], biases bf16 [..., K/gs])."""
    _dev(w, "w", _BF16)
    K = w.shape[-1]
    if K % group_size:
        raise ValueError("[quantize] The last dimension must be divisible by the group size")
    rows = w.numel() // K
    wq = torch.empty(w.shape[:-1] + (K * bits // 32,), dtype=torch.uint32, device=w.device)
    s = torch.empty(w.shape[:-1] + (K // group_size,), dtype=torch.bfloat16, device=w.device)
    b = torch.empty_like(s)
    check(lib().b2q_quantize(w.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(), rows, K, group_size, bits,
                             _stream()))
    return wq, s, b


def dequantize(w, scales, biases, group_size: int = 64, bits: int = 4) -> torch.Tensor:
    _dev(w, "w", _PACK), _dev(scales, "scales", _BF16), _dev(biases, "biases", _BF16)
    K = _check_quant(w, scales, biases, group_size, bits)
    rows = w.numel() // w.shape[-1]
    out = torch.empty(w.shape[:-1] + (K,), dtype=torch.bfloat16, device=w.device)
    check(lib().b2q_dequantize(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), out.data_ptr(), rows, K,
                               group_size, bits, _stream()))
    return out


def gather_qmm_workspace_size(batch: int, M: int, N: int, K: int, n_w: int) -> int:
    """Bytes of caller workspace the allocation-free product forms need."""
    return int(lib().b2q_gather_qmm_workspace_size(batch, M, N, K, n_w))


def quantized_matmul(x, w, scales, biases, transpose: bool = True, group_size: int = 64, bits: int = 4,
                     workspace=None):
    """x [..., M, K] bf16, w [N, K/8] -> [..., M, N] (x . dequant(w)^T).

    ``workspace`` (a uint8 device tensor of at least
    ``gather_qmm_workspace_size(1, M, N, K, 1)`` bytes) selects the form that
    allocates nothing (``b2q_qmm_ws``)."""
    _dev(x, "x", _BF16), _dev(w, "w", _PACK), _dev(scales, "scales", _BF16), _dev(biases, "biases", _BF16)
    if w.dim() != 2:
        raise ValueError("[quantized_matmul] w must be 2-D (use gather_qmm for stacked experts)")
    K = _check_quant(w, scales, biases, group_size, bits)
    if x.shape[-1] != K:
        raise ValueError(f"[quantized_matmul] inner dimensions do not match: x {tuple(x.shape)} vs K={K}")
    N = w.shape[0]
    M = x.numel() // K
    y = torch.empty(x.shape[:-1] + (N,), dtype=torch.bfloat16, device=x.device)
    if workspace is not None:
        check(lib().b2q_qmm_ws(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), y.data_ptr(), M, N,
                               K, group_size, bits, 1 if transpose else 0, workspace.data_ptr(),
                               workspace.numel() * workspace.element_size(), _stream()))
        return y
    check(lib().b2q_qmm(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), y.data_ptr(), M, N, K,
                        group_size, bits, 1 if transpose else 0, _stream()))
    return y


def gather_qmm(x, w, scales, biases, lhs_indices=None, rhs_indices=None, transpose: bool = True,
               group_size: int = 64, bits: int = 4, sorted_indices: bool = False, workspace=None):
    """MLX gather_qmm: out[i] = x[lhs[i]] . dequant(w[rhs[i]])^T.

    x [..., M, K] (leading dims flattened into n_x matrices), w [E, N, K/8];
    indices of the same shape (broadcasting to a common shape is the caller's
    job, as in the reference's Runner); output lhs.shape + [M, N].
    ``workspace`` selects the allocation-free form (``b2q_gather_qmm_ws``).
    """
    _dev(x, "x", _BF16), _dev(w, "w", _PACK), _dev(scales, "scales", _BF16), _dev(biases, "biases", _BF16)
    if w.dim() != 3:
        raise ValueError("[gather_qmm] w must be [E, N, K/8]")
    K = _check_quant(w, scales, biases, group_size, bits)
    if x.shape[-1] != K:
        raise ValueError("[gather_qmm] inner dimensions do not match")
    M = x.shape[-2] if x.dim() >= 2 else 1
    n_x = x.numel() // (M * K)
    E, N = w.shape[0], w.shape[1]
    lhs = rhs = None
    if lhs_indices is not None:
        lhs = _dev(lhs_indices, "lhs_indices", _IDX)
    if rhs_indices is not None:
        rhs = _dev(rhs_indices, "rhs_indices", _IDX)
    shape = (lhs if lhs is not None else rhs).shape if (lhs is not None or rhs is not None) else (n_x,)
    if lhs is not None and rhs is not None and lhs.shape != rhs.shape:
        raise ValueError("[gather_qmm] lhs and rhs indices must have the same shape")
    batch = 1
    for d in shape:
        batch *= d
    if lhs is None and batch > n_x:
        raise ValueError("[gather_qmm] without lhs indices the batch cannot exceed x's matrices")
    y = torch.empty(tuple(shape) + (M, N), dtype=torch.bfloat16, device=x.device)
    if workspace is not None:
        check(lib().b2q_gather_qmm_ws(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), _ptr(lhs),
                                      _ptr(rhs), y.data_ptr(), batch, M, N, K, n_x, E, group_size, bits,
                                      1 if transpose else 0, 1 if sorted_indices else 0, workspace.data_ptr(),
                                      workspace.numel() * workspace.element_size(), _stream()))
        return y
    check(lib().b2q_gather_qmm(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), _ptr(lhs), _ptr(rhs),
                               y.data_ptr(), batch, M, N, K, n_x, E, group_size, bits, 1 if transpose else 0,
                               1 if sorted_indices else 0, _stream()))
    return y


def router_logits(x, wr):
    """f32(x [T, H]) . f32(wr [E, H])^T -> f32 [T, E]."""
    _dev(x, "x", _BF16), _dev(wr, "wr", _BF16)
    H = x.shape[-1]
    T = x.numel() // H
    E = wr.shape[0]
    out = torch.empty(x.shape[:-1] + (E,), dtype=torch.float32, device=x.device)
    check(lib().b2q_moe_router_logits(x.data_ptr(), wr.data_ptr(), out.data_ptr(), T, E, H, _stream()))
    return out


def route(logits, k: int):
    """Top-k (ties to the lower index) + softmax over the selected: (idx uint32, w f32)."""
    _dev(logits, "logits", _F32)
    E = logits.shape[-1]
    T = logits.numel() // E
    idx = torch.empty(logits.shape[:-1] + (k,), dtype=torch.uint32, device=logits.device)
    w = torch.empty(logits.shape[:-1] + (k,), dtype=torch.float32, device=logits.device)
    check(lib().b2q_moe_route(logits.data_ptr(), idx.data_ptr(), w.data_ptr(), T, E, k, _stream()))
    return idx, w


def gate_up_act(x, wg, sg, bg, wu, su, bu, idx, xrow=None, group_size: int = 64, bits: int = 4):
    """act[z] = silu(bf16 gate) * bf16 up for routed slot z (expert idx[z], token xrow[z])."""
    for n, t, d in (("x", x, _BF16), ("wg", wg, _PACK), ("wu", wu, _PACK), ("idx", idx, _IDX)):
        _dev(t, n, d)
    S, H = x.shape[-2], x.shape[-1]
    E, F = wg.shape[0], wg.shape[1]
    n_slots = idx.numel()
    act = torch.empty((n_slots, F), dtype=torch.bfloat16, device=x.device)
    if xrow is not None:
        _dev(xrow, "xrow", _IDX)
    check(lib().b2q_moe_gate_up_act(x.data_ptr(), wg.data_ptr(), sg.data_ptr(), bg.data_ptr(), wu.data_ptr(),
                                    su.data_ptr(), bu.data_ptr(), idx.data_ptr(), _ptr(xrow), act.data_ptr(), n_slots,
                                    S, H, E, F, group_size, bits, _stream()))
    return act


def down_combine(act, wd, sd, bd, idx, w, group_size: int = 64, bits: int = 4):
    """out[t] = bf16(colsum_j f32(bf16(qmv(wd[idx[t,j]], act[t*k+j]))) * w[t, j])."""
    _dev(act, "act", _BF16), _dev(wd, "wd", _PACK), _dev(idx, "idx", _IDX), _dev(w, "w", _F32)
    S, k = idx.shape[0], idx.shape[1]
    E, H = wd.shape[0], wd.shape[1]
    F = act.shape[-1]
    out = torch.empty((S, H), dtype=torch.bfloat16, device=act.device)
    check(lib().b2q_moe_down_combine(act.data_ptr(), wd.data_ptr(), sd.data_ptr(), bd.data_ptr(), idx.data_ptr(),
                                     w.data_ptr(), out.data_ptr(), S, H, E, F, k, group_size, bits, _stream()))
    return out


def swiglu(g, u):
    """silu(g) * u elementwise in bf16 (TrackFastKernels.swiglu2)."""
    _dev(g, "g", _BF16), _dev(u, "u", _BF16)
    if g.shape != u.shape:
        raise ValueError("swiglu: gate and up shapes differ")
    act = torch.empty_like(g)
    check(lib().b2q_swiglu(g.data_ptr(), u.data_ptr(), act.data_ptr(), g.numel(), _stream()))
    return act


def sorted_combine(y, inverse, w):
    """out[t] = bf16(colsum_j f32(y[inverse[t*k+j]]) * w[t, j]); y [T*k, H] sorted rows."""
    _dev(y, "y", _BF16), _dev(inverse, "inverse", _IDX), _dev(w, "w", _F32)
    T, k = w.shape
    H = y.shape[-1]
    out = torch.empty((T, H), dtype=torch.bfloat16, device=y.device)
    check(lib().b2q_moe_sorted_combine(y.data_ptr(), inverse.data_ptr(), w.data_ptr(), out.data_ptr(), T, H, k,
                                       _stream()))
    return out


class Workspace:
    """Caller-owned scratch for the layer-level entry points (zeroed once)."""

    def __init__(self, nbytes: int, device=None):
        self.nbytes = int(nbytes)
        self.buf = torch.zeros(max(256, self.nbytes), dtype=torch.uint8, device=device or "cuda")

    def ptr(self):
        return self.buf.data_ptr()

    def status(self) -> int:
        return lib().b2q_workspace_status(self.ptr(), self.buf.numel(), _stream())

    def reset(self):
        check(lib().b2q_workspace_reset(self.ptr(), self.buf.numel(), _stream()))


_ws_cache: dict = {}


def _workspace(kind, size, device):
    key = (kind, device)
    ws = _ws_cache.get(key)
    if ws is None or ws.nbytes < size:
        ws = Workspace(size, device)
        _ws_cache[key] = ws
    return ws


def moe_decode(x, wr, layer: dict, k: int, group_size: int = 64, bits: int = 4, workspace: Workspace | None = None,
               return_routing: bool = False):
    """One decode MoE layer (S <= 8 tokens). layer: wg/sg/bg, wu/su/bu, wd/sd/bd."""
    _dev(x, "x", _BF16), _dev(wr, "wr", _BF16)
    S, H = x.shape
    E = wr.shape[0]
    F = layer["wg"].shape[1]
    size = lib().b2q_moe_decode_workspace_size(S, H, E, F, k)
    ws = workspace or _workspace("decode", size, x.device)
    out = torch.empty((S, H), dtype=torch.bfloat16, device=x.device)
    idx = torch.empty((S, k), dtype=torch.uint32, device=x.device) if return_routing else None
    w = torch.empty((S, k), dtype=torch.float32, device=x.device) if return_routing else None
    logits = torch.empty((S, E), dtype=torch.float32, device=x.device) if return_routing else None
    L = layer
    check(lib().b2q_moe_decode(x.data_ptr(), wr.data_ptr(), L["wg"].data_ptr(), L["sg"].data_ptr(), L["bg"].data_ptr(),
                               L["wu"].data_ptr(), L["su"].data_ptr(), L["bu"].data_ptr(), L["wd"].data_ptr(),
                               L["sd"].data_ptr(), L["bd"].data_ptr(), out.data_ptr(), _ptr(idx), _ptr(w),
                               _ptr(logits), S, H, E, F, k, group_size, bits, ws.ptr(), ws.buf.numel(), _stream()))
    if return_routing:
        return out, idx, w, logits
    return out


def moe_prefill(x, wr, layer: dict, k: int, group_size: int = 64, bits: int = 4, workspace: Workspace | None = None,
                return_routing: bool = False):
    """One prefill MoE layer over T tokens (sorted expert products + combine)."""
    _dev(x, "x", _BF16), _dev(wr, "wr", _BF16)
    T, H = x.shape
    E = wr.shape[0]
    F = layer["wg"].shape[1]
    size = lib().b2q_moe_prefill_workspace_size(T, H, E, F, k)
    ws = workspace or _workspace("prefill", size, x.device)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    idx = torch.empty((T, k), dtype=torch.uint32, device=x.device) if return_routing else None
    w = torch.empty((T, k), dtype=torch.float32, device=x.device) if return_routing else None
    L = layer
    check(lib().b2q_moe_prefill(x.data_ptr(), wr.data_ptr(), L["wg"].data_ptr(), L["sg"].data_ptr(),
                                L["bg"].data_ptr(), L["wu"].data_ptr(), L["su"].data_ptr(), L["bu"].data_ptr(),
                                L["wd"].data_ptr(), L["sd"].data_ptr(), L["bd"].data_ptr(), out.data_ptr(), _ptr(idx),
                                _ptr(w), T, H, E, F, k, group_size, bits, ws.ptr(), ws.buf.numel(), _stream()))
    if return_routing:
        return out, idx, w
    return out


def moe_sort(ids, E: int, k: int):
    """Stable sort of the flat routed ids: (sorted_ids, token_rows, inverse, offsets)."""
    _dev(ids, "ids", _IDX)
    R = ids.numel()
    dev = ids.device
    sorted_ids = torch.empty(R, dtype=torch.uint32, device=dev)
    token_rows = torch.empty(R, dtype=torch.uint32, device=dev)
    inverse = torch.empty(R, dtype=torch.uint32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.uint32, device=dev)
    ws = _workspace("sort", 256, dev)
    check(lib().b2q_moe_sort(ids.data_ptr(), sorted_ids.data_ptr(), token_rows.data_ptr(), inverse.data_ptr(),
                             offsets.data_ptr(), R, E, k, ws.ptr(), ws.buf.numel(), _stream()))
    return sorted_ids, token_rows, inverse, offsets
