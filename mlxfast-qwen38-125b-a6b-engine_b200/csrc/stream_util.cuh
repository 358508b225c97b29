// stream_util.cuh -- device helpers shared by the single-column decode kernels:
// activation staging (scaled, permuted fp16 columns and their group sums),
// the nibble x activation MMA step, and the softmax over the k routed logits.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace b2q {
namespace su {

constexpr int SU_MAXK = 8;  // activation columns / routed slots

// Activation staging: stage_cols writes `ncols` columns of K values as scaled,
// permuted fp16 chunks (x0 S, x4 S) (x1 S/16, x5 S/16) (x2 S, x6 S)
// (x3 S/16, x7 S/16) and per group: xs = sum of x S, xo = 1024 * sum_even +
// 1024 * sum_odd / 16 (the offset the nibble decode adds), inv = 1 / S.
// Region layout: xs [cap][G], xo [cap][G], inv [SU_MAXK], colmax [SU_MAXK],
// S [SU_MAXK], S / 16 [SU_MAXK].
__device__ __forceinline__ float* c_xs(float* sums, int G, int col) { return sums + (size_t)col * G; }
__device__ __forceinline__ float* c_xo(float* sums, int cap, int G, int col) { return sums + (size_t)(cap + col) * G; }
__device__ __forceinline__ float* c_inv(float* sums, int cap, int G) { return sums + (size_t)2 * cap * G; }

__device__ __forceinline__ uint32_t h2pack(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float lbf(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hbf(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// A 16-byte load issued where it stands (volatile: not sunk towards its use),
// L2-coherent (.cg) or through the non-coherent path (.nc).
__device__ __forceinline__ uint4 ld_v4_now(const void* ptr, bool coherent) {
  uint4 v;
  if (coherent)
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ptr));
  else
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ptr));
  return v;
}

// max |value| of 8 bf16 as bf16 bits << 16, NaN clamped to +inf's bits
__device__ __forceinline__ unsigned chunk_max(uint4 v) {
  unsigned m = max(max(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu), max(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu));
  m = max(m & 0xffffu, m >> 16) << 16;
  return m > 0x7f800000u ? 0x7f800000u : m;
}

// Activation staging. All NCT consumer threads call this (named barrier 1).
// Column j is the K values at base + j * rstride. A max pass finds each
// column's max |value| (every CTA stages the same rows, so every CTA finds the
// same scales); the store pass writes the scaled, permuted fp16 chunks and
// forms the group sums by a shuffle reduction over the gs / 8 lanes that hold
// a group's chunks. Up to SC_REG chunks per thread stay in registers between
// the passes (their loads all issued first), else each pass loads them.
constexpr int SC_REG = 8;
template <int NCT>
__device__ void stage_cols(uint8_t* dst, float* sums, int cap, int XS, const uint16_t* base, size_t rstride, int ncols,
                           int K, int gs, bool coherent) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int nch = K / 8, G = K / gs, CPG = gs / 8;
  const int total = ncols * nch;
  float* inv = c_inv(sums, cap, G);
  unsigned* colmax = reinterpret_cast<unsigned*>(inv + SU_MAXK);
  float* colS = inv + 2 * SU_MAXK;
  float* colS16 = inv + 3 * SU_MAXK;
  // a warp's 32 consecutive chunks stay inside one column when nch is a multiple of 32
  const bool warp_col = (nch % 32) == 0;
  // q / nch by multiply-high: exact while q * nch < 2^32 / 8 (q < SU_MAXK * nch)
  const unsigned mdiv = 0xffffffffu / (unsigned)nch + 1u;
  auto col_of = [&](int q) { return (int)__umulhi((unsigned)q, mdiv); };
  auto src = [&](int q) {
    const int col = col_of(q);
    return base + (size_t)col * rstride + (size_t)(q - col * nch) * 8;
  };
  // max pass step over chunks q0 + [0, NCT) (q0 uniform)
  auto max_step = [&](int q0, uint4 v) {
    const int q = q0 + tid;
    unsigned m = q < total ? chunk_max(v) : 0u;
    const int col = col_of(q < total ? q : q0 + (tid & ~31));
    if (warp_col) {
      m = __reduce_max_sync(0xffffffffu, m);
      if (lane == 0 && q0 + (tid & ~31) < total) atomicMax(&colmax[col], m);
    } else if (q < total) {
      atomicMax(&colmax[col], m);
    }
  };
  // store pass step (q0 uniform; every lane takes part in the shuffles)
  auto store_step = [&](int q0, uint4 v) {
    const int q = q0 + tid;
    const bool live = q < total;
    const int col = live ? col_of(q) : 0, ch = live ? q - col * nch : 0;
    const float S = colS[col], S16 = colS16[col];
    uint4 o;
    o.x = h2pack(lbf(v.x) * S, lbf(v.z) * S);
    o.y = h2pack(hbf(v.x) * S16, hbf(v.z) * S16);
    o.z = h2pack(lbf(v.y) * S, lbf(v.w) * S);
    o.w = h2pack(hbf(v.y) * S16, hbf(v.w) * S16);
    if (live) *reinterpret_cast<uint4*>(dst + (size_t)col * XS + (size_t)ch * 16) = o;
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&o.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&o.y));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&o.z));
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&o.w));
    float se = ((a.x + c.x) + a.y) + c.y;
    float so = ((b.x + d.x) + b.y) + d.y;
    for (int off = 1; off < CPG; off <<= 1) {
      se += __shfl_xor_sync(0xffffffffu, se, off);
      so += __shfl_xor_sync(0xffffffffu, so, off);
    }
    if (live && (ch % CPG) == 0) {
      const int g = ch / CPG;
      c_xs(sums, G, col)[g] = se + 16.0f * so;
      c_xo(sums, cap, G, col)[g] = 1024.0f * se + 1024.0f * so;
    }
  };
  // the power of two S = 2^e of each column from its max |value| bits: for a
  // normal max with biased exponent x, max * 2^(137 - x) lies in [1024, 2048);
  // e stays in [-100, 100] (0 for a zero, infinite or NaN max)
  auto set_scales = [&]() {
    if (tid < ncols) {
      const unsigned mb = colmax[tid];
      int e = 0;
      if (mb != 0u && mb < 0x7f800000u) e = min(100, max(-100, 137 - (int)(mb >> 23)));
      inv[tid] = __int_as_float((127 - e) << 23);
      colS[tid] = __int_as_float((127 + e) << 23);
      colS16[tid] = __int_as_float((123 + e) << 23);
    }
  };
  if (tid < SU_MAXK) colmax[tid] = 0u;
  if (total <= SC_REG * NCT) {
    uint4 keep[SC_REG];
#pragma unroll
    for (int i = 0; i < SC_REG; ++i) {
      const int q = i * NCT + tid;
      keep[i] = q < total ? ld_v4_now(src(q), coherent) : make_uint4(0u, 0u, 0u, 0u);
    }
    named_bar_sync(1, NCT);
#pragma unroll
    for (int i = 0; i < SC_REG; ++i)
      if (i * NCT < total) max_step(i * NCT, keep[i]);
    named_bar_sync(1, NCT);
    set_scales();
    named_bar_sync(1, NCT);
#pragma unroll
    for (int i = 0; i < SC_REG; ++i)
      if (i * NCT < total) store_step(i * NCT, keep[i]);
  } else {
    auto load = [&](int q) {
      if (q >= total) return make_uint4(0u, 0u, 0u, 0u);
      const uint4* sp = reinterpret_cast<const uint4*>(src(q));
      return coherent ? __ldcg(sp) : __ldg(sp);
    };
    named_bar_sync(1, NCT);
    for (int q0 = 0; q0 < total; q0 += NCT) max_step(q0, load(q0 + tid));
    named_bar_sync(1, NCT);
    set_scales();
    named_bar_sync(1, NCT);
    for (int q0 = 0; q0 < total; q0 += NCT) store_step(q0, load(q0 + tid));
  }
  named_bar_sync(1, NCT);
}

// One packed word of row r (P) and of row r + 8 (Q) against the matching
// 8-value activation chunk: two m16n8k16 steps (fp16 x fp16 -> fp32).
__device__ __forceinline__ void word_mma(const uint8_t* wp, int qoff, const uint4 xv, bool first, float (&d)[4]) {
  const uint32_t W0 = *reinterpret_cast<const uint32_t*>(wp);
  const uint32_t W8 = *reinterpret_cast<const uint32_t*>(wp + qoff);
  uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
  decode_word_h(W0, p0, p1, p2, p3);
  decode_word_h(W8, q0, q1, q2, q3);
  if (first)
    mma_f16_16816_zero(d, p0, q0, p1, q1, xv.x, xv.y);
  else
    mma_f16_16816(d, p0, q0, p1, q1, xv.x, xv.y);
  mma_f16_16816(d, p2, q2, p3, q3, xv.z, xv.w);
}

// softmax over the k selected logits held by lanes 0..k-1 (slot order): max,
// exp, per-lane partial sums of 4 then a butterfly, as the reference's
// softmax over its k values (Runner/FastModel/TrackFastMoE.swift:846-880)
__device__ void softmax_k(float selv, int k, float* sw) {
  const int lane = threadIdx.x & 31;
  float mx = (lane < k) ? selv : -INFINITY;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float ex = (lane < k) ? expf(selv - mx) : 0.0f;
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float t = __shfl_sync(0xffffffffu, ex, (4 * lane + i) & 31);
    part += (lane < 8) ? t : 0.0f;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  const float inv = 1.0f / part;
  if (lane < k) sw[lane] = ex * inv;
}

}  // namespace su
}  // namespace b2q
