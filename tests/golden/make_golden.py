"""Regenerate tests/golden/mlx_cpu_golden.npz from the reference's own code.

Runs the reference's MLX CPU quantized kernels (oracle/_ref/libmlxref.so,
built by `make -C oracle` from backend/cpu/quantized.cpp of the reference
tree) on seeded inputs and stores inputs + outputs:

* quantize_gs{32,64,128}: w bf16 [8, 512] (incl. zero, constant, one-signed
  rows) -> packed w, scales, biases   (quantized.cpp:1158-1236)
* qmm_gs{32,64,128}: x bf16 [3, 512] . dequant^T -> y bf16, the scalar bf16
  running-sum path the x86 build takes (quantized.cpp:155-210, :341-419)
* c0_slice: x [1, 4096] against 16 rows of a C0-distributed matrix -> y bf16

Usage (in a checkout that has the reference tree):
    make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.oracle import MlxRef, f32_to_bf16, bf16_to_f32  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mlx_cpu_golden.npz")


def quant_input(rng, gs):
    w = rng.standard_normal((8, 512)).astype(np.float32) * 0.05
    w[1] = 0.0                       # all-zero groups (bias 0, q0 == 0 branch)
    w[2] = 0.25                      # constant groups
    w[3] = np.abs(w[3])              # one-signed (max edge)
    w[4] = -np.abs(w[4])             # one-signed (min edge)
    w[5, ::7] = 3.0                  # outliers
    return f32_to_bf16(w)


def main():
    ref = MlxRef()
    rng = np.random.default_rng(1234)
    out = {}
    for gs in (32, 64, 128):
        w = quant_input(rng, gs)
        wq, s, b = ref.quantize(w, gs, 4)
        out[f"quantize_gs{gs}_w"] = w
        out[f"quantize_gs{gs}_wq"] = wq
        out[f"quantize_gs{gs}_s"] = s
        out[f"quantize_gs{gs}_b"] = b
        x = f32_to_bf16(rng.standard_normal((3, 512)).astype(np.float32))
        out[f"qmm_gs{gs}_x"] = x
        out[f"qmm_gs{gs}_y"] = ref.qmm(x, wq, s, b, gs, 4)
    # C0-distributed slice
    K, N = 4096, 16
    wq = rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32)
    s = f32_to_bf16(rng.uniform(0.002, 0.02, (N, K // 64)).astype(np.float32))
    b = f32_to_bf16(-8.0 * bf16_to_f32(s) + rng.normal(0, 1e-3, (N, K // 64)).astype(np.float32))
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    out.update(c0_x=x, c0_wq=wq, c0_s=s, c0_b=b, c0_y=ref.qmm(x, wq, s, b, 64, 4))
    np.savez_compressed(OUT, **out)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
