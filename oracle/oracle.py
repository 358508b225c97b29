"""ctypes front end of the CPU checker libraries (TEST INFRASTRUCTURE ONLY).

Only tests/, bench.py's CPU-baseline legs and ``__graft_entry__.smoke()`` may
import this module, and only to check or to time the CPU baseline; the product
path never does.

* ``Oracle``   -- liboracle.so, the C restatement in b2q_oracle.c.
* ``MlxRef``   -- _ref/libmlxref.so, the reference's own MLX CPU quantized
                 kernels (backend/cpu/quantized.cpp:155-419, :701-747,
                 :1158-1236) compiled from the reference tree: the bf16 kernel,
                 the same kernel over fp32 operands (fp32 accumulation) and the
                 gather loop over index pairs.
* ``affine_lut_*`` -- the metadata pair index, restated from the Runner's
                 Swift source (TrackAffineLUT.swift). No Swift toolchain is
                 here and the reference holds no test vectors for it, so this
                 part is parity unpinned: it is checked by its own exact round
                 trip (table[index] reproduces every group's bits) and by the
                 two build orders agreeing with the literal loop.

bf16 arrays are numpy ``uint16`` bit patterns; packed weights are ``uint32``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmlxref.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_P)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def build(reference: str | None = None) -> None:
    """Run oracle/Makefile (the C restatement; the MLX kernels when the reference tree exists)."""
    cmd = ["make", "-s", "-C", HERE]
    if reference:
        cmd.append(f"REFERENCE={reference}")
    subprocess.run(cmd, check=True)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even, NaN -> 0x7FC0 (MLX types/bf16.h:39-58)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + ((u >> 16) & 1) + 0x7FFF) >> 16).astype(np.uint16)
    r[np.isnan(a)] = 0x7FC0
    return r


def ep_owner(e: int, E: int, nranks: int) -> int:
    """Rank holding expert e when E experts are split into contiguous blocks over
    nranks ranks, the first E % nranks ranks one expert more."""
    base, extra = divmod(E, nranks)
    split = extra * (base + 1)
    return e // (base + 1) if e < split else extra + (e - split) // base


def ep_a2a_plan(idx: np.ndarray, E: int, nranks: int):
    """Dispatch plan of the expert-parallel all-to-all prefill, restated in plain
    Python. The reference has no expert parallelism (its experts share one GPU),
    so this pins the build's own rule: token t goes to rank d once if d holds
    any of its k experts; pos[t, d] = number of earlier tokens sent to d, or -1;
    counts[d] = tokens sent to d."""
    T = idx.shape[0]
    pos = np.full((T, nranks), -1, np.int32)
    counts = np.zeros(nranks, np.int32)
    for t in range(T):
        for d in sorted({ep_owner(int(e), E, nranks) for e in idx[t]}):
            pos[t, d] = counts[d]
            counts[d] += 1
    return pos, counts


AFFINE_LUT_MAX = 32768          # TrackAffineLUT.maxEntries (TrackAffineLUT.swift:57)
AFFINE_LUT_DEVICE_FROM = 1 << 20  # groups from which the reference builds on the device (:63)


def affine_lut_pairs(scales: np.ndarray, biases: np.ndarray) -> np.ndarray:
    """scale_bits | bias_bits << 16 per group (TrackAffineLUT.swift:62)."""
    return scales.astype(np.uint32) | (biases.astype(np.uint32) << 16)


def affine_lut_build_loop(scales: np.ndarray, biases: np.ndarray, max_entries: int = AFFINE_LUT_MAX):
    """The reference's host loop, restated literally in Python (small tensors
    only): TrackAffineLUT.build, Runner/FastModel/TrackAffineLUT.swift:64-83.
    Entries in first-occurrence order; None past max_entries."""
    pairs = affine_lut_pairs(scales, biases).reshape(-1)
    seen: dict[int, int] = {}
    table: list[int] = []
    index = np.zeros(pairs.size, np.uint16)
    for i, p in enumerate(pairs.tolist()):
        j = seen.get(p)
        if j is None:
            if len(table) >= max_entries:
                return None
            j = len(table)
            seen[p] = j
            table.append(p)
        index[i] = j
    return index.reshape(scales.shape), np.array(table, np.uint32)


def affine_lut_build(scales: np.ndarray, biases: np.ndarray, max_entries: int = AFFINE_LUT_MAX):
    """(index u16 in the scales' shape, table u32) as the reference builds them,
    or None when the tensor does not qualify. Below 2^20 groups the host loop's
    first-occurrence order (TrackAffineLUT.swift:64-83), otherwise the device
    build's ascending pair value (argSort, run starts, cumsum ranks: :88-103);
    both verified by the round trip (:106-110). Vectorised with numpy."""
    pairs = affine_lut_pairs(scales, biases).reshape(-1)
    uniq, first, inv = np.unique(pairs, return_index=True, return_inverse=True)
    if uniq.size > max_entries:
        return None
    if pairs.size < AFFINE_LUT_DEVICE_FROM:
        order = np.argsort(first, kind="stable")  # entry j = j-th pair to appear
        rank = np.empty(uniq.size, np.int64)
        rank[order] = np.arange(uniq.size)
        table, index = uniq[order], rank[inv.reshape(-1)]
    else:
        table, index = uniq, inv.reshape(-1)
    index = index.astype(np.uint16)
    if not np.array_equal(table[index], pairs):
        return None
    return index.reshape(scales.shape), table.astype(np.uint32)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        self.L = L
        L.orc_quantize.argtypes = [_P, _I64, _I, _I, _P, _P, _P]
        for fn in (L.orc_dequantize_metal, L.orc_dequantize_cpu):
            fn.argtypes = [_P, _P, _P, _P, _I64, _I, _I, _I]
        for fn in (L.orc_qmv_metal, L.orc_qmv_metal_f32, L.orc_qmm_mlx_cpu, L.orc_qmm_tile):
            fn.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I]
        L.orc_router_logits.argtypes = [_P, _P, _P, _I, _I, _I]
        L.orc_route.argtypes = [_P, _P, _P, _I, _I, _I]
        L.orc_sigmoid_bf16.argtypes = [ctypes.c_uint16]
        L.orc_sigmoid_bf16.restype = ctypes.c_uint16
        L.orc_silu_bf16.argtypes = [ctypes.c_uint16]
        L.orc_silu_bf16.restype = ctypes.c_uint16
        L.orc_swiglu_bf16.argtypes = [ctypes.c_uint16, ctypes.c_uint16]
        L.orc_swiglu_bf16.restype = ctypes.c_uint16
        L.orc_colsum_small.argtypes = [_P, _I]
        L.orc_colsum_small.restype = ctypes.c_float
        L.orc_moe_decode.argtypes = [_P] * 11 + [_I] * 6 + [_P] * 5
        L.orc_moe_experts_decode.argtypes = [_P] * 12 + [_I] * 5 + [_P, _I, _P]
        L.orc_moe_experts_prefill.argtypes = [_P] * 12 + [_I] * 5 + [_P, _I, _P]
        L.orc_sort_by_expert.argtypes = [_P, _I, _I, _I, _P, _P, _P, _P]

    @staticmethod
    def _check(rc, what):
        if rc != 0:
            raise ValueError(f"oracle {what} failed with status {rc}")

    def quantize(self, w_bf16, group_size=64, bits=4):
        w = _c(w_bf16, np.uint16)
        K = w.shape[-1]
        rows = w.size // K
        wq = np.zeros(rows * K * bits // 32, np.uint32)
        s = np.zeros(rows * K // group_size, np.uint16)
        b = np.zeros_like(s)
        self._check(self.L.orc_quantize(_ptr(w), w.size, group_size, bits, _ptr(wq), _ptr(s), _ptr(b)), "quantize")
        lead = w.shape[:-1]
        return (wq.reshape(lead + (K * bits // 32,)), s.reshape(lead + (K // group_size,)),
                b.reshape(lead + (K // group_size,)))

    def dequantize(self, w, s, b, group_size=64, bits=4, variant="metal"):
        w, s, b = _c(w, np.uint32), _c(s, np.uint16), _c(b, np.uint16)
        K = w.shape[-1] * 32 // bits
        rows = w.size // w.shape[-1]
        out = np.zeros(w.shape[:-1] + (K,), np.uint16)
        fn = self.L.orc_dequantize_metal if variant == "metal" else self.L.orc_dequantize_cpu
        self._check(fn(_ptr(w), _ptr(s), _ptr(b), _ptr(out), rows, K, group_size, bits), "dequantize")
        return out

    def _mm(self, fn, x, w, s, b, group_size, bits, out_dtype):
        x, w, s, b = _c(x, np.uint16), _c(w, np.uint32), _c(s, np.uint16), _c(b, np.uint16)
        K = x.shape[-1]
        M = x.size // K
        N = w.shape[-2]
        y = np.zeros((M, N), out_dtype)
        self._check(fn(_ptr(x), _ptr(w), _ptr(s), _ptr(b), _ptr(y), M, N, K, group_size, bits), "matmul")
        return y.reshape(x.shape[:-1] + (N,))

    def qmv_metal(self, x, w, s, b, group_size=64, bits=4):
        return self._mm(self.L.orc_qmv_metal, x, w, s, b, group_size, bits, np.uint16)

    def qmv_metal_f32(self, x, w, s, b, group_size=64, bits=4):
        return self._mm(self.L.orc_qmv_metal_f32, x, w, s, b, group_size, bits, np.float32)

    def qmm_mlx_cpu(self, x, w, s, b, group_size=64, bits=4):
        return self._mm(self.L.orc_qmm_mlx_cpu, x, w, s, b, group_size, bits, np.uint16)

    def qmm_tile_f32(self, x, w, s, b, group_size=64, bits=4):
        return self._mm(self.L.orc_qmm_tile, x, w, s, b, group_size, bits, np.float32)

    def router_logits(self, x, wr):
        x, wr = _c(x, np.uint16), _c(wr, np.uint16)
        H = x.shape[-1]
        T = x.size // H
        E = wr.shape[0]
        out = np.zeros((T, E), np.float32)
        self._check(self.L.orc_router_logits(_ptr(x), _ptr(wr), _ptr(out), T, E, H), "router")
        return out

    def route(self, logits, k):
        lg = _c(logits, np.float32)
        E = lg.shape[-1]
        T = lg.size // E
        idx = np.zeros((T, k), np.uint32)
        w = np.zeros((T, k), np.float32)
        self._check(self.L.orc_route(_ptr(lg), _ptr(idx), _ptr(w), T, E, k), "route")
        return idx, w

    def swiglu(self, g, u):
        g = np.asarray(g, np.uint16).ravel()
        u = np.asarray(u, np.uint16).ravel()
        return np.array([self.L.orc_swiglu_bf16(int(a), int(c)) for a, c in zip(g, u)], np.uint16)

    def sigmoid(self, x):
        return np.array([self.L.orc_sigmoid_bf16(int(v)) for v in np.asarray(x, np.uint16).ravel()], np.uint16)

    def colsum_small(self, r):
        r = _c(r, np.float32)
        return float(self.L.orc_colsum_small(_ptr(r), r.size))

    def moe_decode(self, x, wr, layer, k, group_size=64):
        """Full decode MoE (router included). layer = dict of gate/up/down w, s, b."""
        x = _c(x, np.uint16)
        S, H = x.shape
        E = wr.shape[0]
        F = layer["wg"].shape[1]
        logits = np.zeros((S, E), np.float32)
        idx = np.zeros((S, k), np.uint32)
        wts = np.zeros((S, k), np.float32)
        act = np.zeros((S * k, F), np.uint16)
        out = np.zeros((S, H), np.uint16)
        a = [_c(layer[n], np.uint32 if n[0] == "w" else np.uint16)
             for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")]
        self._check(self.L.orc_moe_decode(_ptr(x), _ptr(_c(wr, np.uint16)), *[_ptr(t) for t in a],
                                          S, H, E, F, k, group_size,
                                          _ptr(logits), _ptr(idx), _ptr(wts), _ptr(act), _ptr(out)),
                    "moe_decode")
        return dict(logits=logits, idx=idx, w=wts, act=act, out=out)

    def _experts(self, fn, x, idx, wts, layer, k, group_size, rows):
        x = _c(x, np.uint16)
        T, H = x.shape
        E = layer["wg"].shape[0]
        F = layer["wg"].shape[1]
        rows_a = None if rows is None else _c(rows, np.int32)
        n = T if rows is None else rows_a.size
        out = np.zeros((n, H), np.uint16)
        a = [_c(layer[nm], np.uint32 if nm[0] == "w" else np.uint16)
             for nm in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")]
        self._check(fn(_ptr(x), _ptr(_c(idx, np.uint32)), _ptr(_c(wts, np.float32)), *[_ptr(t) for t in a],
                       H, E, F, k, group_size, _ptr(rows_a), n, _ptr(out)), "moe experts")
        return out

    def moe_experts_decode(self, x, idx, wts, layer, k, group_size=64, rows=None):
        return self._experts(self.L.orc_moe_experts_decode, x, idx, wts, layer, k, group_size, rows)

    def moe_experts_prefill(self, x, idx, wts, layer, k, group_size=64, rows=None):
        return self._experts(self.L.orc_moe_experts_prefill, x, idx, wts, layer, k, group_size, rows)

    def sort_by_expert(self, ids, E, k):
        ids = _c(ids, np.uint32).ravel()
        R = ids.size
        sorted_ids = np.zeros(R, np.uint32)
        token_rows = np.zeros(R, np.uint32)
        inverse = np.zeros(R, np.uint32)
        offsets = np.zeros(E + 1, np.uint32)
        self._check(self.L.orc_sort_by_expert(_ptr(ids), R, E, k, _ptr(sorted_ids), _ptr(token_rows),
                                              _ptr(inverse), _ptr(offsets)), "sort")
        return sorted_ids, token_rows, inverse, offsets


class MlxRef:
    """The reference's own MLX CPU kernels (built from the reference tree)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        self.L = L
        L.mlxref_qmm_bf16.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        L.mlxref_quantize_bf16.argtypes = [_P, _P, _P, _P, _I, _I, ctypes.c_longlong]
        self.has_f32 = hasattr(L, "mlxref_qmm_f32")
        if self.has_f32:
            L.mlxref_qmm_f32.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I]
            for fn in (L.mlxref_gather_qmm_bf16, L.mlxref_gather_qmm_f32):
                fn.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I]

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def qmm(self, x, w, s, b, group_size=64, bits=4, out=None):
        x, w, s, b = _c(x, np.uint16), _c(w, np.uint32), _c(s, np.uint16), _c(b, np.uint16)
        K = x.shape[-1]
        M = x.size // K
        N = w.shape[-2]
        y = np.zeros((M, N), np.uint16) if out is None else out
        rc = self.L.mlxref_qmm_bf16(_ptr(y), _ptr(x), _ptr(w), _ptr(s), _ptr(b), M, N, K, group_size, bits, 1)
        if rc:
            raise ValueError("mlx reference qmm failed")
        return y

    def qmm_f32(self, x, w, s, b, group_size=64, bits=4):
        """The reference kernel over fp32 operands (fp32 products and running sum):
        x, s, b are bf16 bit patterns, widened exactly to fp32; returns fp32 [M, N]."""
        xf, sf, bf = (_c(bf16_to_f32(a), np.float32) for a in (x, s, b))
        w = _c(w, np.uint32)
        K = xf.shape[-1]
        M = xf.size // K
        N = w.shape[-2]
        y = np.zeros((M, N), np.float32)
        rc = self.L.mlxref_qmm_f32(_ptr(y), _ptr(xf), _ptr(w), _ptr(sf), _ptr(bf), M, N, K, group_size, bits, 1)
        if rc:
            raise ValueError("mlx reference qmm (fp32) failed")
        return y

    def gather_qmm(self, x, w, s, b, lhs, rhs, group_size=64, bits=4, fp32=True):
        """gather_qmm as the reference's CPU loop: y[i] = x[lhs[i]] . dequant(w[rhs[i]])^T.
        x [n_x, M, K], w [n_w, N, K/8], s/b [n_w, N, K/gs]; lhs/rhs uint32 [pairs] or None
        (identity modulo n_x / n_w). fp32=True widens x, s, b exactly and returns fp32
        [pairs, M, N]; otherwise the bf16 kernel's bf16 bits."""
        w = _c(w, np.uint32)
        n_w, N = w.shape[0], w.shape[1]
        x = np.asarray(x)
        n_x, M, K = x.shape
        lhs_a = None if lhs is None else _c(lhs, np.uint32)
        rhs_a = None if rhs is None else _c(rhs, np.uint32)
        pairs = len(lhs_a) if lhs_a is not None else len(rhs_a)
        if fp32:
            xf, sf, bf = (_c(bf16_to_f32(a), np.float32) for a in (x, s, b))
            y = np.zeros((pairs, M, N), np.float32)
            fn = self.L.mlxref_gather_qmm_f32
        else:
            xf, sf, bf = _c(x, np.uint16), _c(s, np.uint16), _c(b, np.uint16)
            y = np.zeros((pairs, M, N), np.uint16)
            fn = self.L.mlxref_gather_qmm_bf16
        rc = fn(_ptr(y), _ptr(xf), _ptr(w), _ptr(sf), _ptr(bf), _ptr(lhs_a), _ptr(rhs_a), pairs, M, N, K, n_x, n_w,
                group_size, bits)
        if rc:
            raise ValueError(f"mlx reference gather_qmm failed ({rc})")
        return y

    def quantize(self, w_bf16, group_size=64, bits=4):
        w = _c(w_bf16, np.uint16)
        K = w.shape[-1]
        wq = np.zeros(w.size * bits // 32, np.uint32)
        s = np.zeros(w.size // group_size, np.uint16)
        b = np.zeros_like(s)
        rc = self.L.mlxref_quantize_bf16(_ptr(w), _ptr(wq), _ptr(s), _ptr(b), bits, group_size, w.size)
        if rc:
            raise ValueError("mlx reference quantize failed")
        lead = w.shape[:-1]
        return (wq.reshape(lead + (K * bits // 32,)), s.reshape(lead + (K // group_size,)),
                b.reshape(lead + (K // group_size,)))
