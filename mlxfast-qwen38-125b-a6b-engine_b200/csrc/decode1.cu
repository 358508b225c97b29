// decode1.cu -- single-column streaming products: qmv for one row of x
// (M = 1) and the fused one-token MoE decode layer.
//
// Reference operators (paths relative to the reference project):
//   qmv_fast_impl / qdot       Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/metal/kernels/quantized.h:28-105,191-290,757-822
//   gateUpAct / downCombine    Runner/FastModel/TrackFastMoE.swift:1192-1590
//   route (top-k + softmax)    Runner/FastModel/TrackFastMoE.swift:767-911
//
// Organisation (one persistent CTA per SM, 8 consumer warps + 2 producer warps):
//  * A unit is 16 weight rows (P: 8 rows, Q: 8 rows; for gate|up P are gate
//    rows and Q the up rows of the same 8 outputs) over the whole reduction
//    length. It is split into T tasks of 1024 reduction values (4 x 128-byte
//    row pieces); T consecutive consumer warps take the T tasks of a unit and
//    the CTA runs 8 / T units side by side.
//  * Every consumer warp owns two stage slots; two producer warps fill them in
//    task order with TMA tensor copies (an 8-row weight block P, an 8-row
//    block Q, and their scale / bias rows), one full / empty mbarrier pair
//    per slot. A warp processes 4 pieces per wait.
//  * A task's partial row sums go to shared memory; the last of the T warps
//    (a shared-memory arrival count) adds them in task order and finishes
//    the unit: bf16 store (qmv), SwiGLU into the activation rows (gate|up),
//    or the weighted expert combine (down). No finisher warp, no per-unit
//    handshake beyond that count.
//  * Fused decode: router rows (CTA b takes experts b, b + grid, ...) -> a grid
//    counter -> every CTA computes the same top-k -> gate|up units -> a grid
//    counter of finished units -> activation staging -> down units (8 output
//    rows x 8 slots: 4 slot pairs x 2 halves of F = 8 tasks). The producer
//    issues the copies of DOWN_AHEAD down units before that counter
//    completes, the rest once the activations are staged (named barrier 3).
//    Gate|up and down units are handed out by two grid-wide counters (the
//    producer asks for its next round while it issues the current one) and
//    published to the consumers with the slot fill. The last CTA out
//    re-arms the counters.
//  * The dot products use the engine's arithmetic: nibbles OR-ed into fp16
//    1024.0 give 1024 + q (and 1024 + 16 q from the upper nibble of a byte);
//    activations are staged as fp16 scaled by a power of two per column so
//    that max |x| * 2^e lies in [1024, 2048); mma.sync m16n8k16 (fp16 x fp16
//    -> fp32) per 16 weight rows; per group: s * (D - xoff) + b * sum(x),
//    then the power of two is undone.
// All waits are bounded; a wait that runs out records B2Q_ETIMEOUT and raises
// an abort flag; every role then runs to the end of its loops without
// waiting or computing, so all barriers still see every thread.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "decode1.cuh"
#include "host.hpp"
#include "tc.cuh"
#include "tmap.hpp"

namespace b2q {
namespace d1 {

constexpr int NCW = 8;                  // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NPW = 2;                  // producer warps
constexpr int NTH = NCT + 32 * NPW;
constexpr int SPW = 2;                  // stage slots per consumer warp
constexpr int NSLOT = NCW * SPW;
constexpr int SLOT = 10240;             // bytes per slot
constexpr int TK = 1024;                // reduction values per gate|up / qmv task
constexpr int RR = 4;                   // reduction-slot ring per warp group
constexpr int MAXK = 8;                 // routed slots (fused decode)
// Down units whose copies the producer issues before the activations are
// staged: copies issued earlier queue in front of the staging loads.
constexpr int DOWN_AHEAD = 1;

// tensor-map slots
enum : int { MW = 0, MS = 1, MB = 2, MWG = 0, MSG = 1, MBG = 2, MWU = 3, MSU = 4, MBU = 5, MWD = 6, MSD = 7, MBD = 8 };

// ---------------------------------------------------------------------------
// shared-memory plan (byte offsets from the 1024-aligned base)
// ---------------------------------------------------------------------------
struct Plan {
  int slots;     // NSLOT x SLOT
  int x;         // staged activation column(s) of the gate|up / qmv family
  int xs;        // its group sums
  int act;       // staged activation columns of the down family (fused)
  int acts;
  int red;       // task partials
  int misc;      // barriers, counters, routing
  int bytes;
  int XS1, XS2;  // activation column strides
};

// Activation staging: stage_cols writes `ncols` columns of K values as scaled,
// permuted fp16 chunks (x0 S, x4 S) (x1 S/16, x5 S/16) (x2 S, x6 S)
// (x3 S/16, x7 S/16) and per group: xs = sum of x S, xo = 1024 * sum_even +
// 1024 * sum_odd / 16 (the offset the nibble decode adds), inv = 1 / S.
// Region layout: xs [cap][G], xo [cap][G], inv [MAXK], colmax [MAXK],
// S [MAXK], S / 16 [MAXK].
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
__device__ void stage_cols(uint8_t* dst, float* sums, int cap, int XS, const uint16_t* base, size_t rstride, int ncols,
                           int K, int gs, bool coherent) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int nch = K / 8, G = K / gs, CPG = gs / 8;
  const int total = ncols * nch;
  float* inv = c_inv(sums, cap, G);
  unsigned* colmax = reinterpret_cast<unsigned*>(inv + MAXK);
  float* colS = inv + 2 * MAXK;
  float* colS16 = inv + 3 * MAXK;
  // a warp's 32 consecutive chunks stay inside one column when nch is a multiple of 32
  const bool warp_col = (nch % 32) == 0;
  // q / nch by multiply-high: exact while q * nch < 2^32 / 8 (q < MAXK * nch)
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
  if (tid < MAXK) colmax[tid] = 0u;
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

// ---------------------------------------------------------------------------
// consumers: one task = npc 128-byte pieces of the 16 rows
// ---------------------------------------------------------------------------
// Slot layout: [P: npc atoms of 1024 bytes][Q: npc atoms][sP][bP][sQ][bQ], a
// meta block = 8 rows x GB groups of bf16 (row stride GB * 2). Atom j holds
// piece j of the 8 rows, 16-byte unit u of row r at unit position u ^ r.
// Lane (r = lane / 4, c = lane % 4) takes word 4u + c of row r of P and of Q
// (MMA rows r and r + 8).
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

// Single activation column (qmv, gate|up): the quad lanes finish groups c of
// each batch of NB groups; acc[0] row r (P), acc[2] row r + 8 (Q).
// gb0: group index inside the slot's meta rows of the task's first group;
// gabs0: absolute group index (for xs / xo) of the task's first group.
template <int WPT>
__device__ __forceinline__ void task_col(const uint8_t* st, int npc, int GB, int gb0, int gabs0,
                                         const uint8_t* xc, const float* xs, const float* xo, float (&acc)[4]) {
  constexpr int GPC = 8 / WPT;
  constexpr int NB = GPC < 4 ? GPC : 4;
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const int qoff = npc * 1024;
  const uint8_t* mP = st + 2 * qoff;
  const int mblk = 8 * GB * 2;
  const uint8_t* wl = st + r * 128 + c * 4;
  const uint8_t* xl = xc + c * 16;
  for (int pc = 0; pc < npc; ++pc) {
    const uint8_t* pw = wl + pc * 1024;
    const uint8_t* px = xl + pc * 512;
#pragma unroll
    for (int b0 = 0; b0 < GPC; b0 += NB) {
      float D[NB][4];
#pragma unroll
      for (int j = 0; j < WPT; ++j) {
#pragma unroll
        for (int gi = 0; gi < NB; ++gi) {
          const int u = (b0 + gi) * WPT + j;
          word_mma(pw + ((u ^ r) << 4), qoff, *reinterpret_cast<const uint4*>(px + u * 64), j == 0, D[gi]);
        }
      }
      float e0 = D[0][0], e2 = D[0][2];
#pragma unroll
      for (int gi = 1; gi < NB; ++gi) {
        e0 = (c == gi) ? D[gi][0] : e0;
        e2 = (c == gi) ? D[gi][2] : e2;
      }
      const int gl = pc * GPC + b0 + (c < NB ? c : NB - 1);  // group inside the task
      const int mo = r * GB * 2 + (gb0 + gl) * 2;
      const float sP = bf2f(*reinterpret_cast<const uint16_t*>(mP + mo));
      const float bP = bf2f(*reinterpret_cast<const uint16_t*>(mP + mblk + mo));
      const float sQ = bf2f(*reinterpret_cast<const uint16_t*>(mP + 2 * mblk + mo));
      const float bQ = bf2f(*reinterpret_cast<const uint16_t*>(mP + 3 * mblk + mo));
      const float xa = xs[gabs0 + gl], xoa = xo[gabs0 + gl];
      if (c < NB) {
        acc[0] = fmaf(sP, e0 - xoa, fmaf(bP, xa, acc[0]));
        acc[2] = fmaf(sQ, e2 - xoa, fmaf(bQ, xa, acc[2]));
      }
    }
  }
}

// Down pair: P = slot 2 * pair, Q = slot 2 * pair + 1. The B operand's column
// n is activation slot 2 * pair + (n & 1), so every lane (r, c) holds row r
// against slot 2 * pair in D[0] and row r + 8 against slot 2 * pair + 1 in
// D[3]; as in task_col, the quad lanes finish groups c of each batch of NB
// groups (acc[0]: P, acc[3]: Q). gabs0: the task's first group inside the
// full-length meta rows and staged sums.
template <int WPT>
__device__ __forceinline__ void task_pair(const uint8_t* st, int npc, int GB, int gabs0, const uint8_t* acol0, int XS,
                                          const float* xsP, const float* xoP, const float* xsQ, const float* xoQ,
                                          int pair, float (&acc)[4]) {
  constexpr int GPC = 8 / WPT;
  constexpr int NB = GPC < 4 ? GPC : 4;
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const int qoff = npc * 1024;
  const uint8_t* mP = st + 2 * qoff;
  const int mblk = 8 * GB * 2;
  const uint8_t* wl = st + r * 128 + c * 4;
  const uint8_t* xl = acol0 + (size_t)(2 * pair + (r & 1)) * XS + c * 16;
  for (int pc = 0; pc < npc; ++pc) {
    const uint8_t* pw = wl + pc * 1024;
    const uint8_t* px = xl + pc * 512;
#pragma unroll
    for (int b0 = 0; b0 < GPC; b0 += NB) {
      float D[NB][4];
#pragma unroll
      for (int j = 0; j < WPT; ++j) {
#pragma unroll
        for (int gi = 0; gi < NB; ++gi) {
          const int u = (b0 + gi) * WPT + j;
          word_mma(pw + ((u ^ r) << 4), qoff, *reinterpret_cast<const uint4*>(px + u * 64), j == 0, D[gi]);
        }
      }
      float e0 = D[0][0], e3 = D[0][3];
#pragma unroll
      for (int gi = 1; gi < NB; ++gi) {
        e0 = (c == gi) ? D[gi][0] : e0;
        e3 = (c == gi) ? D[gi][3] : e3;
      }
      const int ga = gabs0 + pc * GPC + b0 + (c < NB ? c : NB - 1);
      const int mo = r * GB * 2 + ga * 2;
      const float sP = bf2f(*reinterpret_cast<const uint16_t*>(mP + mo));
      const float bP = bf2f(*reinterpret_cast<const uint16_t*>(mP + mblk + mo));
      const float sQ = bf2f(*reinterpret_cast<const uint16_t*>(mP + 2 * mblk + mo));
      const float bQ = bf2f(*reinterpret_cast<const uint16_t*>(mP + 3 * mblk + mo));
      if (c < NB) {
        acc[0] = fmaf(sP, e0 - xoP[ga], fmaf(bP, xsP[ga], acc[0]));
        acc[3] = fmaf(sQ, e3 - xoQ[ga], fmaf(bQ, xsQ[ga], acc[3]));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// routing (Runner/FastModel/TrackFastMoE.swift:767-911)
// ---------------------------------------------------------------------------
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

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar,
                                     uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch3(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch2(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

struct Shape {
  int T;      // tasks per unit
  int units;  // units of the phase (grid-wide)
};

template <int WPT, int MODE>
__global__ void __launch_bounds__(NTH, 1) d1_kernel(const __grid_constant__ D1Params p) {
  extern __shared__ uint8_t smem_raw[];
  // aligned by pointer arithmetic on the shared array (an integer round trip
  // would hide the address space and turn every shared access generic)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* slots = smem + p.off_slots;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_misc);
  uint64_t* empty = full + NSLOT;
  unsigned* cnt = reinterpret_cast<unsigned*>(empty + NSLOT);  // [9 groups][RR] arrival counts
  unsigned* gen = cnt + 9 * RR;                                // [9 groups][RR] consumed uses
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gen + 9 * RR);
  uint32_t* sidx = reinterpret_cast<uint32_t*>(const_cast<int*>(abort_flag) + 4);
  float* sw = reinterpret_cast<float*>(sidx + MAXK);
  float* rsum = sw + MAXK;  // [NCW]
  int* lastfill = reinterpret_cast<int*>(rsum + NCW);  // [NSLOT] ordinal of the last fill issued per slot
  volatile int* slot_unit = lastfill + NSLOT;            // [NSLOT] unit of the task in the slot (-1: no more work)
  int* p1n = lastfill + 2 * NSLOT;                       // [NCW] phase-1 task count of each consumer warp
  unsigned* fin_cta = reinterpret_cast<unsigned*>(p1n + NCW);  // gate|up units this CTA finished
  int* lslot = reinterpret_cast<int*>(fin_cta + 1);  // [MAXK] routed slots whose expert this rank holds, in slot order
  int* nloc_sm = lslot + MAXK;                      // their count
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  const uint64_t deadline = globaltimer() + (uint64_t)p.timeout_ns;
  const bool fused = MODE != D1_QMV;
  constexpr bool EP = MODE == D1_FUSED_EP;  // local slots only, fp32 partial out
  const int G1 = p.K1 / p.gs, G2 = fused ? p.F / p.gs : 0;

  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 9 * RR; ++i) cnt[i] = gen[i] = 0;
    for (int i = 0; i < NSLOT; ++i) lastfill[i] = -1;
    *fin_cta = 0u;
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // phase geometry
  const Shape ph1{p.K1 / TK, fused ? p.k * (p.F / 8) : p.N / 16};
  const Shape ph2{8, fused ? p.H / 8 : 0};
  auto local_units = [&](int units) { return units > (int)blockIdx.x ? (units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0; };
  const int nl1 = local_units(ph1.units);
  const int G1grp = NCW / ph1.T;  // units side by side in phase 1
  const int rounds1 = (nl1 + G1grp - 1) / G1grp;

  if (warp >= NCW) {
    // ------------------------------ producers ------------------------------
    // Producer pw fills the slots of the phase-1 groups gi with gi % NPW == pw
    // and, in the down phase, of consumer warps [4 pw, 4 pw + 4).
    const int pw = warp - NCW;
    if (fused) named_bar_sync(2, NTH);  // routing done
    const uint64_t pol = policy_evict_first();
    if (tc::elect_one())
      for (int i = 0; i < (fused ? 9 : 3); ++i)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.map[i])) : "memory");
    __syncwarp();
    // n: the warp's task ordinal (its round in phase 1; then phase-1 count + round)
    // waits until slot (w, n) is free: its fill of ordinal n - SPW was consumed
    auto wait_empty = [&](int w, int n) -> bool {
      const int si = w * SPW + (n % SPW);
      if (n >= SPW && !__all_sync(0xffffffffu, tc::wait(&empty[si], ((n / SPW) - 1) & 1, deadline, abort_flag))) {
        if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        return false;
      }
      return true;
    };
    auto issue = [&](int w, int n, bool valid, int rowP, int rowQ, int pieceP, int npc, int mwP, int msP, int mbP,
                     int mwQ, int msQ, int mbQ, int gcol, int GB, int unit) -> bool {
      const int si = w * SPW + (n % SPW);
      if (!wait_empty(w, n)) return false;
      if (tc::elect_one()) {
        uint8_t* st = slots + (size_t)si * SLOT;
        lastfill[si] = n;
        slot_unit[si] = unit;  // published by the arrive below
        if (!valid || *abort_flag) {
          mbar_arrive_expect_tx(&full[si], 0u);
        } else {
          const uint32_t mb = 8u * (uint32_t)GB * 2u;
          mbar_arrive_expect_tx(&full[si], 2u * (uint32_t)npc * 1024u + 4u * mb);
          tma3(st, &p.map[mwP], 0, rowP, pieceP, &full[si], pol);
          tma3(st + npc * 1024, &p.map[mwQ], 0, rowQ, pieceP, &full[si], pol);
          uint8_t* m = st + 2 * npc * 1024;
          tc::tma_load_2d(m, &p.map[msP], gcol, rowP, &full[si], pol);
          tc::tma_load_2d(m + mb, &p.map[mbP], gcol, rowP, &full[si], pol);
          tc::tma_load_2d(m + 2 * mb, &p.map[msQ], gcol, rowQ, &full[si], pol);
          tc::tma_load_2d(m + 3 * mb, &p.map[mbQ], gcol, rowQ, &full[si], pol);
        }
      }
      __syncwarp();
      return true;
    };
    bool ok = true;
    const int GB1 = TK / p.gs;
    if (!fused) {
      // qmv: static round-robin units, T tasks of TK values (4 pieces) each
      for (int j = 0; ok && j < rounds1; ++j)
        for (int gi = 0; ok && gi < G1grp; ++gi) {
          const int li = j * G1grp + gi;
          if (li >= nl1) break;
          if (gi % NPW != pw) continue;
          const int u = blockIdx.x + li * gridDim.x;
          // the issue order rotates with the round, so the warp whose data lands
          // last (and that usually finishes the unit) changes from unit to unit
          for (int i = 0; ok && i < ph1.T; ++i) {
            const int t = (i + j) % ph1.T;
            ok = issue(gi * ph1.T + t, j, true, u * 16, u * 16 + 8, t * (TK / 256), TK / 256, MW, MS, MB, MW, MS, MB,
                       t * GB1, GB1, u);
          }
        }
    } else {
      // fused, phase 1: units come from a grid-wide counter, so CTAs that
      // stream faster take more. A round takes one unit per group of this
      // producer with one atomic (unit base + k for its k-th group), and the
      // next round's atomic is issued as soon as the current one is known, so
      // its latency overlaps the round's copies. A unit past the end (a fill
      // without copies, published as -1) ends a group's phase.
      int jr[NCW];
      bool gdone[NCW];
      int ng = 0;
      for (int gi = 0; gi < G1grp; ++gi) {
        jr[gi] = 0;
        gdone[gi] = gi % NPW != pw;
        ng += gdone[gi] ? 0 : 1;
      }
      if (ng > 0) {
        const unsigned U1 = (unsigned)((EP ? *nloc_sm : p.k) * (p.F / 8));  // units of the (local) slots
        unsigned nxt = (lane == 0) ? atomicAdd(&p.sched[0], (unsigned)ng) : 0u;
        int left = ng;
        while (ok && left > 0) {
          const unsigned base = __shfl_sync(0xffffffffu, nxt, 0);
          if (lane == 0 && base < U1) nxt = atomicAdd(&p.sched[0], (unsigned)ng);
          for (int gi = pw, k = 0; ok && gi < G1grp; gi += NPW, ++k) {
            if (gdone[gi]) continue;
            const int u = base + k < U1 ? (int)(base + k) : -1;
            if (u >= 0) {
              const int z = u / (p.F / 8), rb = u % (p.F / 8);
              const int row = EP ? (int)((sidx[lslot[z]] - (uint32_t)p.e_lo) * (uint32_t)p.F) + rb * 8
                                 : (int)(sidx[z] * (uint32_t)p.F) + rb * 8;
              for (int i = 0; ok && i < ph1.T; ++i) {  // rotated issue order, as in qmv
                const int t = (i + jr[gi]) % ph1.T;
                ok = issue(gi * ph1.T + t, jr[gi], true, row, row, t * (TK / 256), TK / 256, MWG, MSG, MBG, MWU,
                           MSU, MBU, t * GB1, GB1, u);
              }
            } else {
              for (int t = 0; ok && t < ph1.T; ++t)
                ok = issue(gi * ph1.T + t, jr[gi], false, 0, 0, 0, 1, MWG, MSG, MBG, MWU, MSU, MBU, 0, GB1, -1);
              gdone[gi] = true;
              --left;
            }
            ++jr[gi];
          }
        }
      }
      // phase-1 fill counts of every consumer warp, for the down ordinals
      if (lane == 0)
        for (int gi = pw; gi < G1grp; gi += NPW)
          for (int t = 0; t < ph1.T; ++t) p1n[gi * ph1.T + t] = jr[gi];
      named_bar_sync(4, 32 * NPW);
      // phase 2: down rows, 4 slot pairs x 2 halves of F (meta rows whole) for
      // consumer warps 0..7; units round-robin over the CTAs (every CTA gets
      // H / 8 / grid of them, within one); warp t's ordinals continue from its
      // phase-1 count; a -1 unit ends the phase
      const int npc2 = p.F / 2 / 256;
      const int nl2 = local_units(ph2.units);
      uint32_t ex[MAXK];
#pragma unroll
      const int nloc = EP ? *nloc_sm : p.k;
      for (int s2 = 0; s2 < MAXK; ++s2)
        ex[s2] = s2 < nloc ? (EP ? sidx[lslot[s2]] - (uint32_t)p.e_lo : sidx[s2]) : 0u;
      int n0[8 / NPW];
#pragma unroll
      for (int i = 0; i < 8 / NPW; ++i) n0[i] = p1n[pw * (8 / NPW) + i];
      bool staged = false;  // barrier 3: the consumers staged the activations
      for (int j2 = 0; ok && j2 <= nl2; ++j2) {
        if (j2 == DOWN_AHEAD) {
          named_bar_sync(3, NTH);
          staged = true;
        }
        const int u = j2 < nl2 ? (int)blockIdx.x + j2 * (int)gridDim.x : -1;
#pragma unroll
        for (int i0 = 0; i0 < 8 / NPW; ++i0) {
          if (!ok) break;
          const int i = (i0 + j2) % (8 / NPW);  // rotated issue order
          const int t = pw * (8 / NPW) + i;
          const int pair = t >> 1, half = t & 1;
          const bool v0 = 2 * pair < nloc, v1 = 2 * pair + 1 < nloc;
          const uint32_t e0 = v0 ? ex[2 * pair] : 0u, e1 = v1 ? ex[2 * pair + 1] : e0;
          const int n = n0[i] + j2;
          ok = u >= 0 ? issue(t, n, v0, (int)(e0 * (uint32_t)p.H) + u * 8, (int)(e1 * (uint32_t)p.H) + u * 8,
                              half * npc2, npc2, MWD, MSD, MBD, MWD, MSD, MBD, 0, G2, u)
                      : issue(t, n, false, 0, 0, 0, 1, MWD, MSD, MBD, MWD, MSD, MBD, 0, G2, -1);
        }
      }
      if (!staged) named_bar_sync(3, NTH);
    }
    // let every copy issued land before the CTA may exit: once both producers
    // are done, a slot's last fill is the only one that can still be in
    // flight (a fill is issued only after the previous one was consumed)
    named_bar_sync(4, 32 * NPW);
    const uint64_t dl = globaltimer() + 200000000ull;
    if (lane < NSLOT && lane % NPW == pw && lastfill[lane] >= 0)
      tc::wait_until(&full[lane], (lastfill[lane] / SPW) & 1, dl);
  } else {
    // ------------------------------ consumers ------------------------------
    uint8_t* xbuf = smem + p.off_x;
    float* xsum = reinterpret_cast<float*>(smem + p.off_xs);
    uint8_t* abuf = smem + p.off_act;
    float* asum = reinterpret_cast<float*>(smem + p.off_acts);
    const int r = lane >> 2, c = lane & 3;

    if (fused) {
      // router rows of this CTA, then a grid-wide count of finished rows
      const int nvec = p.H / 8;
      int rows_done = 0;
      for (int e = blockIdx.x; e < p.E; e += gridDim.x) {
        float part = 0.0f;
        for (int v = tid; v < nvec; v += NCT) {
          const uint4 xv = __ldg(reinterpret_cast<const uint4*>(p.x) + v);
          const uint4 wv = __ldg(reinterpret_cast<const uint4*>(p.wr + (size_t)e * p.H) + v);
          part += lbf(xv.x) * lbf(wv.x) + hbf(xv.x) * hbf(wv.x);
          part += lbf(xv.y) * lbf(wv.y) + hbf(xv.y) * hbf(wv.y);
          part += lbf(xv.z) * lbf(wv.z) + hbf(xv.z) * hbf(wv.z);
          part += lbf(xv.w) * lbf(wv.w) + hbf(xv.w) * hbf(wv.w);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        if (lane == 0) rsum[warp] = part;
        named_bar_sync(1, NCT);
        if (tid == 0) {
          float lg = 0.0f;
          for (int w = 0; w < NCW; ++w) lg += rsum[w];
          p.ws_logits[e] = lg;
        }
        named_bar_sync(1, NCT);
        ++rows_done;
      }
      if (tid == 0 && rows_done) {
        __threadfence();
        atomicAdd(&p.counters[0], (unsigned)rows_done);
      }
      {
        // stage x while the other CTAs finish their router rows
        stage_cols(xbuf, xsum, 1, p.XS1, p.x, 0, 1, p.K1, p.gs, false);
      }
      if (tid == 0) {
        // acquire load of the count; the CTA barrier below orders the
        // other threads' reads after it
        if (!wait_counter_geq(&p.counters[0], (unsigned)p.E, deadline, abort_flag)) {
          record_error(p.err, B2Q_ETIMEOUT);
          *abort_flag = 1;
        }
      }
      named_bar_sync(1, NCT);
      // top-k by rank: expert e is selected at slot rank(e) when rank(e) < k,
      // rank(e) = #{j : v_j > v_e or (v_j == v_e and j < e)} (largest first, ties
      // to the lower index, as the sequential selection); NaN ranks as -inf
      float* lgs = reinterpret_cast<float*>(abuf);  // scratch before the down phase
      float* sval = lgs + p.E;
      for (int e = tid; e < p.E; e += NCT) {
        const float v = *abort_flag ? 0.0f : __ldcg(p.ws_logits + e);
        lgs[e] = (v != v) ? -INFINITY : v;
      }
      named_bar_sync(1, NCT);
      for (int e = tid; e < p.E; e += NCT) {
        const float v = lgs[e];
        int rank = 0;
        for (int j = 0; j < p.E; ++j) {
          const float vj = lgs[j];
          rank += (vj > v || (vj == v && j < e)) ? 1 : 0;
        }
        if (rank < p.k) {
          sidx[rank] = (uint32_t)e;
          sval[rank] = v;
        }
      }
      named_bar_sync(1, NCT);
      if (warp == 0) {
        softmax_k(lane < p.k ? sval[lane] : -INFINITY, p.k, sw);
        __syncwarp();
        if (blockIdx.x == 0 && lane < p.k) {
          if (p.idx_out) p.idx_out[lane] = sidx[lane];
          if (p.w_out) p.w_out[lane] = sw[lane];
        }
        if (blockIdx.x == 0 && p.logits_out)
          for (int e = lane; e < p.E; e += 32) p.logits_out[e] = __ldcg(p.ws_logits + e);
        // the slots this rank computes: all of them, or (expert parallel) those
        // whose expert lies in [e_lo, e_lo + e_local)
        if (EP && lane == 0) {
          int n = 0;
          for (int s = 0; s < p.k; ++s) {
            const int e = (int)sidx[s];
            if (e >= p.e_lo && e < p.e_lo + p.e_local) lslot[n++] = s;
          }
          *nloc_sm = n;
        }
      }
      named_bar_sync(2, NTH);  // releases the producer
    }
    if (!fused) {
      stage_cols(xbuf, xsum, 1, p.XS1, p.x, 0, 1, p.K1, p.gs, false);
    }
    const float* xs1 = c_xs(xsum, G1, 0);
    const float* xo1 = c_xo(xsum, 1, G1, 0);
    const float inv1 = c_inv(xsum, 1, G1)[0];

    // this warp's slot ring
    int n = 0;
    auto take = [&](int& si) -> bool {
      si = warp * SPW + (n % SPW);
      const bool got = __all_sync(0xffffffffu, tc::wait(&full[si], (n / SPW) & 1, deadline, abort_flag));
      if (!got && !*abort_flag) {
        record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
      }
      return got && !*abort_flag;
    };
    auto give = [&](int si) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[si]);
      ++n;
    };
    // Reduction through shared memory: returns true in the warp that arrived
    // last. The unit's partial rows are [T][16] (or [8][16] for down).
    auto arrive_last = [&](int grp, int use, int T) -> bool {
      unsigned* cn = cnt + grp * RR + (use % RR);
      unsigned old = 0;
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        old = atomicAdd(cn, 1u);
      }
      old = __shfl_sync(0xffffffffu, old, 0);
      const bool last = old == (unsigned)(T - 1);
      if (last) __threadfence_block();
      return last;
    };
    auto release_use = [&](int grp, int use) {
      __syncwarp();
      if (lane == 0) {
        cnt[grp * RR + (use % RR)] = 0;
        __threadfence_block();
        atomicAdd(&gen[grp * RR + (use % RR)], 1u);
      }
      __syncwarp();
    };
    // writers wait until the previous use of the reduction slot was consumed
    auto slot_free = [&](int grp, int use) {
      if (use < RR) return;
      const unsigned want = (unsigned)(use / RR);
      if (lane == 0) {
        volatile unsigned* g = &gen[grp * RR + (use % RR)];
        while (*g < want && !*abort_flag) {
          if (globaltimer() > deadline) {
            record_error(p.err, B2Q_ETIMEOUT);
            *abort_flag = 1;
          }
        }
      }
      __syncwarp();
    };

    // ---------------- phase 1 ----------------
    {
      const int T = ph1.T, grp = warp / T, t = warp % T;
      const int GB1 = TK / p.gs;
      int finished = 0;  // gate|up units this warp finished (fused)
      for (int j = 0;; ++j) {
        int u = 0;
        if (!fused) {
          const int li = j * G1grp + grp;
          if (li >= nl1) break;
          u = blockIdx.x + li * gridDim.x;
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int si;
        const bool got = take(si);
        if (fused) {
          // the producer publishes the unit with the fill; -1 ends the phase
          u = got ? slot_unit[si] : -1;
          if (u < 0) {
            give(si);
            break;
          }
        }
        if (got) {
          const uint8_t* st = slots + (size_t)si * SLOT;
          task_col<WPT>(st, 4, GB1, 0, t * GB1, xbuf + (size_t)t * (TK / 8) * 16, xs1, xo1, acc);
        }
        give(si);
        // the four lanes of a quad hold different groups: add them
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 1);
        acc[2] += __shfl_xor_sync(0xffffffffu, acc[2], 1);
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 2);
        acc[2] += __shfl_xor_sync(0xffffffffu, acc[2], 2);
        float* rp = red + ((size_t)(grp * RR + (j % RR)) * 8 + t) * 16;  // [grp][RR][T<=8][16]
        if (__any_sync(0xffffffffu, *abort_flag != 0)) continue;
        slot_free(grp, j);
        if (c == 0) {
          rp[r] = acc[0];
          rp[r + 8] = acc[2];
        }
        if (!arrive_last(grp, j, T)) continue;
        // last warp of the unit: rows r (P) and r + 8 (Q) in task order
        const float* rbuf = red + (size_t)(grp * RR + (j % RR)) * 8 * 16;
        float tot = 0.0f;
        if (lane < 16) {
          for (int q = 0; q < T; ++q) tot += rbuf[q * 16 + lane];
          tot *= inv1;
        }
        // the reduction slot is free once read (its release fences shared
        // memory only, so it goes before the global stores)
        release_use(grp, j);
        if (fused) {
          // lanes 0..7: gate row f = rb*8 + lane and its up row (lane + 8)
          const float up = __shfl_sync(0xffffffffu, tot, (lane + 8) & 31);
          const int z = u / (p.F / 8), rbk = u % (p.F / 8);
          if (lane < 8) p.ws_act[(size_t)z * p.F + rbk * 8 + lane] = swiglu_bf16(f2bf(tot), f2bf(up));
          ++finished;
        } else {
          if (lane < 16) p.y[(size_t)u * 16 + lane] = f2bf(tot);
        }
      }
      if (fused && lane == 0 && finished) atomicAdd(fin_cta, (unsigned)finished);
    }

    // ---------------- phase 2 (fused): down + weighted combine ----------------
    if (fused) {
      const int nloc = EP ? *nloc_sm : p.k;
      // the CTA's finished units are published once (after the barrier, one
      // fence covers every warp's activation rows); then every gate|up unit
      // of the grid must have been published
      named_bar_sync(1, NCT);
      if (tid == 0) {
        const unsigned nfin = *fin_cta;
        if (nfin) {
          __threadfence();
          atomicAdd(&p.counters[1], nfin);
        }
        if (!*abort_flag &&
            !wait_counter_geq(&p.counters[1], (unsigned)(nloc * (p.F / 8)), deadline, abort_flag)) {
          record_error(p.err, B2Q_ETIMEOUT);
          *abort_flag = 1;
        }
      }
      named_bar_sync(1, NCT);
      {
        // the activation rows of the local slots (compact, local order)
        if (nloc > 0) stage_cols(abuf, asum, p.k, p.XS2, p.ws_act, (size_t)p.F, nloc, p.F, p.gs, true);
      }
      named_bar_arrive(3, NTH);  // the producer may issue the remaining down copies
      const int pair = warp >> 1, half = warp & 1;
      const int s0 = max(0, min(2 * pair, nloc - 1)), s1 = max(0, min(2 * pair + 1, nloc - 1));
      const float* xsP = c_xs(asum, G2, s0);
      const float* xoP = c_xo(asum, p.k, G2, s0);
      const float* xsQ = c_xs(asum, G2, s1);
      const float* xoQ = c_xo(asum, p.k, G2, s1);
      const float* ainv = c_inv(asum, p.k, G2);
      const int npc2 = p.F / 2 / 256;
      const int gh = (p.F / 2) / p.gs;  // groups per half
      constexpr int G_DOWN = 8;  // reduction group of the down units
      for (int use = 0;; ++use) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int si;
        const bool got = take(si);
        const int u = got ? slot_unit[si] : -1;
        if (u < 0) {
          give(si);
          break;
        }
        {
          const uint8_t* st = slots + (size_t)si * SLOT;
          if (2 * pair < nloc)
            task_pair<WPT>(st, npc2, G2, half * gh, abuf + (size_t)half * (p.F / 2 / 8) * 16, p.XS2, xsP, xoP, xsQ,
                           xoQ, pair, acc);
        }
        give(si);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) continue;
        float* rp = red + ((size_t)(G_DOWN * RR + (use % RR)) * 8 + warp) * 16;
        slot_free(G_DOWN, use);
        // the four lanes of a quad hold different groups: add them
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 1);
        acc[3] += __shfl_xor_sync(0xffffffffu, acc[3], 1);
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 2);
        acc[3] += __shfl_xor_sync(0xffffffffu, acc[3], 2);
        if (c == 0) {  // row r against slot 2p (P), row r against slot 2p+1 (Q)
          rp[r] = acc[0];
          rp[r + 8] = acc[3];
        }
        if (!arrive_last(G_DOWN, use, 8)) continue;
        const float* rbuf = red + (size_t)(G_DOWN * RR + (use % RR)) * 8 * 16;
        // row h = u*8 + lane: y_j = (half 0 + half 1) / S_j, prod_j = rb(y_j) * w_j,
        // combined in the mlx_colsum_small_f32 association
        float prod[MAXK];
#pragma unroll
        for (int s = 0; s < MAXK; ++s) {
          if (s < nloc && lane < 8) {
            const int pr = s >> 1, q = s & 1;
            const float y = (rbuf[(2 * pr) * 16 + q * 8 + lane] + rbuf[(2 * pr + 1) * 16 + q * 8 + lane]) * ainv[s];
            prod[s] = b2q::rb(y) * sw[EP ? lslot[s] : s];
          } else {
            prod[s] = 0.0f;
          }
        }
        release_use(G_DOWN, use);  // partials read; fences shared memory only
        if (lane < 8) {
          const int TY = nloc < 8 ? nloc : 8;
          float total = 0.0f;
#pragma unroll
          for (int q = 0; q < MAXK; ++q) {
            if (q < TY) {
              float a = 0.0f;
              for (int s = q; s < nloc; s += TY) a = prod[s] + a;
              total = (q == 0) ? a : a + total;
            }
          }
          if (EP)
            p.out_f32[(size_t)u * 8 + lane] = total;  // this rank's partial
          else
            p.out[(size_t)u * 8 + lane] = f2bf(total);
        }
      }
    }
  }

  // ---- exit: the last CTA out re-arms the grid counters for the next call ----
  __syncthreads();
  if (fused && tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&p.counters[2], 1u);
    if (prev == gridDim.x - 1) {
      p.counters[0] = 0;
      p.counters[1] = 0;
      p.counters[2] = 0;
      p.sched[0] = p.sched[1] = 0;
      __threadfence();
    }
  }
}

}  // namespace d1
}  // namespace b2q

namespace b2q {
namespace d1 {

static int round_up(int v, int a) { return (v + a - 1) / a * a; }

static int plan(D1Params& p, int mode) {
  const int G1 = p.K1 / p.gs;
  int off = 0;
  p.off_slots = off;
  off += NSLOT * SLOT;
  p.XS1 = round_up(p.K1 * 2, 128) + 64;
  p.off_x = off;
  off = round_up(off + p.XS1, 128);
  p.off_xs = off;
  off = round_up(off + (2 * G1 + 4 * MAXK) * 4, 128);
  if (mode != D1_QMV) {
    const int G2 = p.F / p.gs;
    p.XS2 = round_up(p.F * 2, 128) + 64;
    p.off_act = off;
    off = round_up(off + MAXK * p.XS2, 128);
    p.off_acts = off;
    off = round_up(off + (2 * MAXK * G2 + 4 * MAXK) * 4, 128);
  } else {
    p.XS2 = 0;
    p.off_act = p.off_acts = off;
  }
  p.off_red = off;
  off = round_up(off + 9 * RR * 8 * 16 * 4, 128);
  p.off_misc = off;
  off = round_up(off + 2 * NSLOT * 8 + 2 * 9 * RR * 4 + 16 + (2 * MAXK + 2 * NCW + 2 * NSLOT) * 4 + 64, 128);
  p.smem_bytes = off + 1024;
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (p.smem_bytes > di.smem_optin)
    return set_error(B2Q_EUNSUPPORTED, "decode kernel: %d bytes of shared memory", p.smem_bytes);
  return B2Q_OK;
}

template <int WPT, int MODE>
static int launch_t(const D1Params& p, cudaStream_t st, int grid) {
  static int attr_done[64] = {};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (!attr_done[di.device & 63]) {
    B2Q_TRY_CUDA(cudaFuncSetAttribute(d1_kernel<WPT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_done[di.device & 63] = 1;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTH);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (MODE != D1_QMV) ? 1 : 0;
  B2Q_TRY_CUDA(cudaLaunchKernelEx(&cfg, d1_kernel<WPT, MODE>, p));
  return B2Q_OK;
}

static int launch(const D1Params& p, int mode, cudaStream_t st) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int grid = di.sm_count;
  const int wpt = p.gs / 32;
  switch (wpt * 4 + mode) {
    case 1 * 4 + D1_QMV: return launch_t<1, D1_QMV>(p, st, grid);
    case 2 * 4 + D1_QMV: return launch_t<2, D1_QMV>(p, st, grid);
    case 4 * 4 + D1_QMV: return launch_t<4, D1_QMV>(p, st, grid);
    case 1 * 4 + D1_FUSED: return launch_t<1, D1_FUSED>(p, st, grid);
    case 2 * 4 + D1_FUSED: return launch_t<2, D1_FUSED>(p, st, grid);
    case 4 * 4 + D1_FUSED: return launch_t<4, D1_FUSED>(p, st, grid);
    case 1 * 4 + D1_FUSED_EP: return launch_t<1, D1_FUSED_EP>(p, st, grid);
    case 2 * 4 + D1_FUSED_EP: return launch_t<2, D1_FUSED_EP>(p, st, grid);
    case 4 * 4 + D1_FUSED_EP: return launch_t<4, D1_FUSED_EP>(p, st, grid);
    default: return set_error(B2Q_EUNSUPPORTED, "decode kernel: group size %d", p.gs);
  }
}

// Tensor maps of recently used weight sets. Encoding the (up to nine) maps of
// a call costs microseconds of host time, while a model calls the same layers
// over and over; maps depend only on addresses, shapes and boxes, so an entry
// keyed by those stays valid whatever the buffers hold. Least recently used
// entries are replaced.
struct MapKey {
  const void* ptr[9];
  int device, mode, a, b, c, gs;
};
struct MapEntry {
  MapKey key;
  CUtensorMap map[9];
  uint64_t stamp;
};
constexpr int MAP_CACHE = 128;
static std::mutex g_map_mu;
static MapEntry g_maps[MAP_CACHE];
static uint64_t g_map_clock = 0;

static MapKey map_key(int mode, const void* const* ptrs, int n, int a, int b, int c, int gs) {
  MapKey k;
  std::memset(&k, 0, sizeof(k));  // padding included: keys compare bytewise
  for (int i = 0; i < n; ++i) k.ptr[i] = ptrs[i];
  cudaGetDevice(&k.device);
  k.mode = mode;
  k.a = a;
  k.b = b;
  k.c = c;
  k.gs = gs;
  return k;
}
static bool find_maps(const MapKey& k, CUtensorMap* out, int n) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (MapEntry& e : g_maps) {
    if (e.stamp && std::memcmp(&e.key, &k, sizeof(k)) == 0) {
      std::memcpy(out, e.map, sizeof(CUtensorMap) * n);
      e.stamp = ++g_map_clock;
      return true;
    }
  }
  return false;
}
static void put_maps(const MapKey& k, const CUtensorMap* m, int n) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  MapEntry* victim = &g_maps[0];
  for (MapEntry& e : g_maps)
    if (e.stamp < victim->stamp) victim = &e;
  victim->key = k;
  std::memcpy(victim->map, m, sizeof(CUtensorMap) * n);
  victim->stamp = ++g_map_clock;
}

// weights: 3-D 128-byte-swizzled map, box of 8 rows x `box_bytes` of each row;
// scales / biases: 2-D map, box of 8 rows x `mbox_bytes`
static int set_family(D1Params& p, int mw, int ms, int mb, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                      uint64_t rows, int K, int box_bytes, int mbox_bytes) {
  int rc = make_row_block_map(&p.map[mw], w, rows, (uint64_t)K / 2, box_bytes, true);
  if (rc) return rc;
  const uint64_t mrow = (uint64_t)(K / p.gs) * 2;
  rc = make_row_block_map(&p.map[ms], s, rows, mrow, mbox_bytes, false);
  if (rc) return rc;
  return make_row_block_map(&p.map[mb], b, rows, mrow, mbox_bytes, false);
}

}  // namespace d1

using namespace d1;

bool d1_qmv_eligible(int N, int K, int gs, const void* x, const void* w, const void* s, const void* b) {
  return (gs == 32 || gs == 64 || gs == 128) && N > 0 && N % 16 == 0 && K % TK == 0 && K <= 8 * TK &&
         aligned16(x) && aligned16(w) && aligned16(s) && aligned16(b);
}

int d1_qmv(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b, uint16_t* y, int N, int K,
           int gs, cudaStream_t st) {
  D1Params p;
  std::memset(&p, 0, sizeof(p));
  p.gs = gs;
  p.K1 = K;
  p.N = N;
  p.x = x;
  p.y = y;
  p.timeout_ns = 2000000000ll;
  int rc = plan(p, D1_QMV);
  if (rc) return rc;
  const void* ptrs[3] = {w, s, b};
  const MapKey key = map_key(D1_QMV, ptrs, 3, N, K, 0, gs);
  if (!find_maps(key, p.map, 3)) {
    rc = set_family(p, MW, MS, MB, w, s, b, (uint64_t)N, K, TK / 2, (TK / gs) * 2);
    if (rc) return rc;
    put_maps(key, p.map, 3);
  }
  return launch(p, D1_QMV, st);
}

bool d1_moe_eligible(int H, int E, int F, int k, int gs) {
  if (!((gs == 32 || gs == 64 || gs == 128) && H % TK == 0 && H <= 8 * TK && F % 512 == 0 && F <= 2048 &&
        (F / gs) % 8 == 0 && k >= 1 && k <= MAXK && E >= k && E <= 1024))
    return false;
  // a down task (half of F for 16 rows) and a gate|up task with their scale / bias rows fit one slot
  const int down_bytes = 2 * (F / 2 / 256) * 1024 + 4 * 8 * (F / gs) * 2;
  const int gu_bytes = 2 * (TK / 256) * 1024 + 4 * 8 * (TK / gs) * 2;
  return down_bytes <= SLOT && gu_bytes <= SLOT;
}

int d1_moe_decode(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                  const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd, const uint16_t* sd,
                  const uint16_t* bd, uint16_t* out, uint32_t* idx, float* w, float* logits, int H, int E, int F,
                  int k, int gs, int* err, unsigned* counters, unsigned* sched, float* ws_logits,
                  uint16_t* ws_act, cudaStream_t st, int e_lo, int e_local, float* out_f32) {
  D1Params p;
  std::memset(&p, 0, sizeof(p));
  p.gs = gs;
  p.K1 = H;
  p.x = x;
  p.wr = wr;
  p.out = out;
  p.idx_out = idx;
  p.w_out = w;
  p.logits_out = logits;
  p.H = H;
  p.E = E;
  p.F = F;
  p.k = k;
  p.err = err;
  p.counters = counters;
  p.sched = sched;
  p.ws_logits = ws_logits;
  p.ws_act = ws_act;
  p.e_lo = e_lo;
  p.e_local = e_local;
  p.out_f32 = out_f32;
  p.timeout_ns = 2000000000ll;
  const int mode = out_f32 ? D1_FUSED_EP : D1_FUSED;
  int rc = plan(p, mode);
  if (rc) return rc;
  const void* ptrs[9] = {wg, sg, bg, wu, su, bu, wd, sd, bd};
  const int Eh = e_local > 0 ? e_local : E;  // experts in the stacks this call reads
  const MapKey key = map_key(D1_FUSED, ptrs, 9, H, Eh, F, gs);
  if (!find_maps(key, p.map, 9)) {
    const uint64_t rgu = (uint64_t)Eh * F, rd = (uint64_t)Eh * H;
    rc = set_family(p, MWG, MSG, MBG, wg, sg, bg, rgu, H, TK / 2, (TK / gs) * 2);
    if (rc) return rc;
    rc = set_family(p, MWU, MSU, MBU, wu, su, bu, rgu, H, TK / 2, (TK / gs) * 2);
    if (rc) return rc;
    rc = set_family(p, MWD, MSD, MBD, wd, sd, bd, rd, F, F / 4, (F / gs) * 2);
    if (rc) return rc;
    put_maps(key, p.map, 9);
  }
  return launch(p, mode, st);
}

}  // namespace b2q
