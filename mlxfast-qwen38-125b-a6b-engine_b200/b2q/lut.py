"""Load-time pair index of a 4-bit tensor's affine metadata.

Mirror of the reference's ``TrackAffineLUT`` (Runner/FastModel/TrackAffineLUT.swift:21-110)
and ``TrackLUTGemv.apply`` (:330-368) over ``b2q_affine_lut_*`` / ``b2q_qmv_lut``:

* ``AffineLUT.build(scales, biases)`` -> an ``AffineLUT`` (u16 ``index`` in
  the scales' shape, u32 ``table`` of ``scale_bits | bias_bits << 16``,
  ``count``), or ``None`` when the tensor does not qualify (more distinct
  pairs than ``max_entries``, or a group that does not reconstruct its exact
  bits), as the reference returns nil;
* ``lazy_scales()`` / ``lazy_biases()`` -> the bf16 arrays the index encodes;
* ``qmv_lut(x, w, meta, group_size)`` -> the one-row product with the metadata
  read through the table, or ``None`` when the shape is not the one-row
  product the kernel serves (the caller then takes the plain product).
"""
from __future__ import annotations

import torch

from ._lib import B2QError, check, lib
from .ops import _BF16, _PACK, _dev, _stream

MAX_ENTRIES = 32768  # the reference's table limit (TrackAffineLUT.swift:57)


class AffineLUT:
    def __init__(self, index: torch.Tensor, table: torch.Tensor, count: int):
        self.index, self.table, self.count = index, table, count

    @classmethod
    def build(cls, scales: torch.Tensor, biases: torch.Tensor, max_entries: int = MAX_ENTRIES):
        if biases is None or scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
            return None
        if scales.shape != biases.shape or scales.numel() == 0 or not scales.is_cuda:
            return None
        s, b = scales.contiguous(), biases.contiguous()
        G = s.numel()
        cap = (max_entries + 3) // 4 * 4
        index = torch.empty(s.shape, dtype=torch.int16, device=s.device).view(torch.uint16)
        table = torch.zeros(cap, dtype=torch.int32, device=s.device).view(torch.uint32)
        ws = torch.empty(int(lib().b2q_affine_lut_workspace_size(cap)), dtype=torch.uint8, device=s.device)
        import ctypes

        count = ctypes.c_int(-1)
        check(lib().b2q_affine_lut_build(s.data_ptr(), b.data_ptr(), G, index.data_ptr(), table.data_ptr(), cap,
                                         ctypes.addressof(count), ws.data_ptr(), ws.numel(), _stream()))
        if count.value < 0:
            return None
        return cls(index, table, count.value)

    def _expand(self):
        s = torch.empty(self.index.shape, dtype=torch.bfloat16, device=self.index.device)
        b = torch.empty_like(s)
        check(lib().b2q_affine_lut_expand(self.index.data_ptr(), self.table.data_ptr(), self.index.numel(),
                                          s.data_ptr(), b.data_ptr(), _stream()))
        return s, b

    def lazy_scales(self) -> torch.Tensor:
        return self._expand()[0]

    def lazy_biases(self) -> torch.Tensor:
        return self._expand()[1]


def qmv_lut(x: torch.Tensor, w: torch.Tensor, meta: AffineLUT, group_size: int = 64, bits: int = 4):
    """x [..., 1, K] (one row) -> [..., 1, N], or None outside the kernel's shapes."""
    if bits != 4 or x.dim() < 2 or x.shape[-2] != 1 or x.dtype != torch.bfloat16 or w.dim() != 2:
        return None
    K, N = x.shape[-1], w.shape[0]
    if K != w.shape[1] * 8 or K % group_size or x.numel() != K:
        return None
    x = _dev(x.contiguous(), "x", _BF16)
    _dev(w, "w", _PACK)  # the kernel reads these pointers on the device
    if x.device != w.device or meta.index.device != w.device:
        raise ValueError("qmv_lut: x, w and the pair index must be on one CUDA device")
    y = torch.empty(x.shape[:-1] + (N,), dtype=torch.bfloat16, device=x.device)
    rc = lib().b2q_qmv_lut(x.data_ptr(), w.data_ptr(), meta.index.data_ptr(), meta.table.data_ptr(), meta.count,
                           y.data_ptr(), N, K, group_size, bits, _stream())
    if rc == -2:  # B2Q_EUNSUPPORTED: not the one-row product the kernel serves
        return None
    check(rc)
    return y


__all__ = ["AffineLUT", "MAX_ENTRIES", "qmv_lut", "B2QError"]
