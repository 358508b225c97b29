"""Module-level call sites of the path, mirroring the reference's surface.

* ``QuantizedLinear``  -- MLXNN QuantizedLinear.callAsFunction
  (Vendor/mlx-swift/Source/MLXNN/Quantized.swift:238-350) and the Runner's
  TrackQuantWeight.apply (Runner/FastModel/TrackFastWeights.swift:43-53).
* ``SwitchLinear`` / ``SwitchGLU`` -- mlx-swift-lm's stacked-expert layers
  (behaviour per docs/qwen38-125b-a6b-port-notes.md:628-735 and
  Runner/FastModel/TrackP12Prefill.swift:198-237): gate/up/down projections of
  E experts, ``act = silu(gate) * up``, computed through gather_qmm.
* ``MoE``              -- the Runner's TrackMoE bundle and moeForwardShared
  (Runner/FastModel/TrackFastModel.swift:225-248, :867-1009) without the
  shared expert: router logits, top-k routing, experts, weighted combine;
  decode windows (<= 8 tokens) take the fused decode operator, larger windows
  the sorted prefill operator.
"""
from __future__ import annotations

import torch

from . import lut, ops


class QuantizedLinear:
    def __init__(self, weight, scales, biases, group_size: int = 64, bits: int = 4, bias=None, meta=None):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits = group_size, bits
        self.bias = bias
        # load-time metadata pair index (TrackQuantWeight.meta,
        # Runner/FastModel/TrackFastWeights.swift:15-17); None when absent
        self.meta = meta

    def with_pair_index(self, max_entries: int = lut.MAX_ENTRIES) -> "QuantizedLinear":
        """The same layer with its metadata pair index built (load time only),
        as TrackQuantWeight.withPairIndex (TrackFastWeights.swift:29-35); the
        layer itself when the tensor does not qualify."""
        if self.meta is not None or self.bits != 4:
            return self
        built = lut.AffineLUT.build(self.scales, self.biases, max_entries)
        if built is None:
            return self
        return QuantizedLinear(self.weight, self.scales, self.biases, self.group_size, self.bits, self.bias, built)

    @property
    def rows(self) -> int:
        return self.weight.shape[0]

    @classmethod
    def from_linear(cls, w_bf16: torch.Tensor, group_size: int = 64, bits: int = 4):
        wq, s, b = ops.quantize(w_bf16.contiguous(), group_size, bits)
        return cls(wq, s, b, group_size, bits)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        # one-row windows read the metadata through the pair index when there is
        # one (TrackQuantWeight.apply, TrackFastWeights.swift:41-53)
        y = lut.qmv_lut(x, self.weight, self.meta, self.group_size, self.bits) if self.meta is not None else None
        if y is None:
            y = ops.quantized_matmul(x.contiguous(), self.weight, self.scales, self.biases, True, self.group_size,
                                     self.bits)
        if self.bias is not None:
            y = y + self.bias
        return y


class SwitchLinear:
    """Stacked expert projection: weight [E, N, K/8], scales/biases [E, N, K/gs]."""

    def __init__(self, weight, scales, biases, group_size: int = 64, bits: int = 4):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits = group_size, bits

    def __call__(self, x, indices, sorted_indices: bool = False):
        # x [..., 1, K] per index (expanded), indices of x's leading shape
        return ops.gather_qmm(x, self.weight, self.scales, self.biases, None, indices.contiguous(), True,
                              self.group_size, self.bits, sorted_indices)


class SwitchGLU:
    def __init__(self, gate_proj: SwitchLinear, up_proj: SwitchLinear, down_proj: SwitchLinear):
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """x [T, H], indices [T, k] -> [T, k, H] (per-expert outputs, not combined)."""
        T, H = x.shape
        k = indices.shape[-1]
        E = self.gate_proj.weight.shape[0]
        sorted_ids, token_rows, inverse, _ = ops.moe_sort(indices.contiguous().view(-1), E, k)
        x3 = x.contiguous().view(T, 1, H)
        lhs = token_rows.view(-1)
        g = ops.gather_qmm(x3, self.gate_proj.weight, self.gate_proj.scales, self.gate_proj.biases, lhs, sorted_ids,
                           True, self.gate_proj.group_size, self.gate_proj.bits, True)
        u = ops.gather_qmm(x3, self.up_proj.weight, self.up_proj.scales, self.up_proj.biases, lhs, sorted_ids,
                           True, self.up_proj.group_size, self.up_proj.bits, True)
        act = ops.swiglu(g, u)
        y = ops.gather_qmm(act, self.down_proj.weight, self.down_proj.scales, self.down_proj.biases, None, sorted_ids,
                           True, self.down_proj.group_size, self.down_proj.bits, True)
        # unsort: row p of y belongs to flat slot order[p]; inverse[slot] = p
        return y.view(T * k, -1)[inverse.long()].view(T, k, -1)


class MoE:
    """Router + routed experts + weighted combine (no shared expert)."""

    def __init__(self, router_weight: torch.Tensor, experts: dict, top_k: int, group_size: int = 64, bits: int = 4):
        self.router_weight = router_weight  # bf16 [E, H]
        self.experts = experts  # wg/sg/bg, wu/su/bu, wd/sd/bd
        self.top_k = top_k
        self.group_size, self.bits = group_size, bits
        # The one-token call is host-latency bound: its weight pointers and
        # shape arguments are fixed per layer, so they are prepared once.
        ops._dev(router_weight, "router_weight", ops._BF16)
        for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd"):
            ops._dev(experts[n], n, ops._PACK if n.startswith("w") else ops._BF16)
        self._E, self._H = router_weight.shape
        self._F = experts["wg"].shape[1]
        self._wptrs = (router_weight.data_ptr(),) + tuple(
            experts[n].data_ptr() for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd"))
        self._ws1 = None

    @property
    def num_experts(self) -> int:
        return self.router_weight.shape[0]

    def _decode_one(self, x2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One token through the fused decode operator with the prepared
        arguments; ``out`` (CUDA bf16, H elements, contiguous) is written in place
        of a new tensor, so a caller's decode loop allocates nothing."""
        if x2.dtype != torch.bfloat16 or x2.device.type != "cuda" or x2.shape[1] != self._H:
            raise ValueError("x: expected a CUDA bf16 tensor [1, H] matching the router weight")
        if self._ws1 is None or self._ws1.buf.device != x2.device:
            size = ops.lib().b2q_moe_decode_workspace_size(1, self._H, self._E, self._F, self.top_k)
            self._ws1 = ops.Workspace(size, x2.device)
        if out is None:
            out = torch.empty((1, self._H), dtype=torch.bfloat16, device=x2.device)
        elif (out.dtype != torch.bfloat16 or out.device != x2.device or out.numel() != self._H
              or not out.is_contiguous()):
            raise ValueError("out: expected a contiguous CUDA bf16 tensor of H elements on x's device")
        ops.check(ops.lib().b2q_moe_decode(x2.data_ptr(), *self._wptrs, out.data_ptr(), None, None, None, 1, self._H,
                                           self._E, self._F, self.top_k, self.group_size, self.bits, self._ws1.ptr(),
                                           self._ws1.buf.numel(), ops._stream(x2.device)))
        return out

    def decode_norm(self, h: torch.Tensor, delta, norm_weight: torch.Tensor, eps: float, h_out,
                    out: torch.Tensor | None = None):
        """One token with the residual add + RMSNorm of its input fused into the
        decode kernel: h_out = h + delta (skipped when delta is None), the layer
        applied to rms_norm(h_out) * norm_weight. Returns the layer output, or
        None when the shape is outside the fused kernel (the caller then takes
        the separate norm and the plain call)."""
        for name, t in (("h", h), ("norm_weight", norm_weight), ("delta", delta), ("h_out", h_out), ("out", out)):
            if t is None and name in ("delta", "h_out", "out"):
                continue
            # the kernel dereferences these pointers on the device: refuse host or mis-shaped tensors here
            if (not isinstance(t, torch.Tensor) or t.dtype != torch.bfloat16 or t.device.type != "cuda"
                    or t.device != h.device or t.numel() != self._H or not t.is_contiguous()):
                raise ValueError(f"{name}: expected a contiguous CUDA bf16 tensor of H={self._H} elements on h's "
                                 "device")
        if self._ws1 is None or self._ws1.buf.device != h.device:
            size = ops.lib().b2q_moe_decode_workspace_size(1, self._H, self._E, self._F, self.top_k)
            self._ws1 = ops.Workspace(size, h.device)
        if out is None:
            out = torch.empty((1, self._H), dtype=torch.bfloat16, device=h.device)
        rc = ops.lib().b2q_moe_decode_norm(h.data_ptr(), None if delta is None else delta.data_ptr(),
                                           norm_weight.data_ptr(), eps, None if h_out is None else h_out.data_ptr(),
                                           *self._wptrs, out.data_ptr(), None, None, None, self._H, self._E, self._F,
                                           self.top_k, self.group_size, self.bits, self._ws1.ptr(),
                                           self._ws1.buf.numel(), ops._stream(h.device))
        if rc == -2:  # B2Q_EUNSUPPORTED
            return None
        ops.check(rc)
        return out

    def __call__(self, x: torch.Tensor, return_routing: bool = False, out: torch.Tensor | None = None):
        """``out`` (one-token calls only): a persistent output buffer the call writes."""
        x2 = x.contiguous().view(-1, x.shape[-1])
        if x2.shape[0] == 1 and not return_routing:
            return self._decode_one(x2, out).view(x.shape)
        if out is not None:
            raise ValueError("out: only for one-token calls without routing outputs")
        if x2.shape[0] <= 8:
            r = ops.moe_decode(x2, self.router_weight, self.experts, self.top_k, self.group_size, self.bits,
                               return_routing=return_routing)
        else:
            r = ops.moe_prefill(x2, self.router_weight, self.experts, self.top_k, self.group_size, self.bits,
                                return_routing=return_routing)
        if return_routing:
            return (r[0].view(x.shape),) + tuple(r[1:])
        return r.view(x.shape)
