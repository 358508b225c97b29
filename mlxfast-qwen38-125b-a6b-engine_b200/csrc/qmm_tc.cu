// qmm_tc.cu -- grouped 4-bit affine GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), the prefill side of the MoE layer.
//
// Reference operators (paths relative to the reference project):
//   affine_gather_qmm_rhs + expert tiles   Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/metal/kernels/quantized.h:2785-3207
//   TrackPrefillIndirect.apply / .down     Runner/FastModel/TrackPrefillIndirect.swift:83-227
//   tile loader dequantisation             .../metal/kernels/quantized.h:485-530
//
// Problem: rows (tokens) are grouped by expert: group e owns rows
// [offsets[e], offsets[e+1]) of a row-major bf16 matrix X [R, K]; each group
// is multiplied by the transposed dequantised weight of its expert,
// W_e [Nw, K] (MLX packing: uint32 [E, Nw, K/8], bf16 scales/biases
// [E, Nw, K/gs]). Two forms:
//   GLU  : gate and up weights; out = silu(bf16 g) * bf16 u in bf16, written
//          in the K-permuted column order the down product reads.
//   PLAIN: one weight; out = bf16(X W^T), row r written to out_rows[r] (or r).
//
// Mapping onto tcgen05 (weights are the M side, tokens the N side, so an
// expert's token count only has to be rounded to 16):
//   * a work unit is (expert, chunk of <= 192 rows of that expert, 128-row
//     weight tile); a GLU tile holds 64 gate rows and the same 64 up rows,
//     16 gate rows then their 16 up rows in every 32-lane quarter;
//   * two producer warps stream the packed weight tile (TMA, 128 bytes of
//     every row = 4 K steps per stage, 128-byte swizzle) and, per 64-wide K
//     step, the token rows (TMA, 128-byte swizzle);
//   * eight dequant warps (two groups of four taking alternate K steps) turn
//     packed nibbles into bf16 (mask into bf16 128.0, subtract 128, one bf16x2
//     fma with scale and bias: one rounding of s*q + b) and store them to
//     TMEM as the MMA's A operand;
//   * one warp issues tcgen05.mma (A from TMEM, B from shared memory) into
//     one of two 128 x N fp32 accumulators in TMEM, so the epilogue of one
//     unit overlaps the main loop of the next. Token rows and dequantized A
//     of a K step complete ONE operand barrier (one wait, one commit per
//     step), and the issuing warps stay converged with one elected lane per
//     instruction: a single divergent lane issuing MMAs next to busy dequant
//     warps reached well under half the tensor rate;
//   * four epilogue warps read the accumulator back (tcgen05.ld) and write
//     bf16 outputs; GLU pairs a gate lane with its up lane by one shuffle,
//     PLAIN transposes 32x32 tiles through shared memory for 16-byte stores.
// K order: inside every 8-element block the token rows carry the order
// (0,4,1,5,2,6,3,7), which is the order in which the nibble decode produces
// weight pairs; both operands use it, so the dot products are unchanged.
//
// All waits are bounded (globaltimer deadline); a wait that runs out records
// B2Q_ETIMEOUT, raises an in-CTA abort flag, and every role drains its
// in-flight copies / MMAs before TMEM is released.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "host.hpp"
#include "qmm_tc.cuh"
#include "tc.cuh"
#include "tmap.hpp"

namespace b2q {
namespace qtc {

constexpr int KSTEP = 64;          // K elements per pipeline step
constexpr int TILE_M = 128;        // weight rows per unit (TMEM lanes)
constexpr int MAX_N = 192;         // token rows per unit (accumulator columns)
constexpr int NS = 4;              // operand stages: token rows (smem) + dequantized A (TMEM), one K step each
constexpr int NP = 4;              // packed-weight stages (4 K steps each)
constexpr int PK = 4;              // K steps per packed-weight stage (128 bytes of every row)
constexpr int B_STAGE = MAX_N * KSTEP * 2;   // 24 KB of token rows per operand stage
constexpr int P_STAGE = TILE_M * PK * KSTEP / 2;  // 16 KB
constexpr int TMEM_COLS = 512;
constexpr int D_COL1 = MAX_N;      // accumulators at columns [0, 192) and [192, 384)
constexpr int A_COL = 2 * MAX_N;   // A ring at [384, 512)
constexpr int NWARPS = 14;         // warps before the token-row producer (see the role list below)
constexpr int NTHREADS = NWARPS * 32;
constexpr int MAX_E = 1024;
static_assert(A_COL + NS * 32 == TMEM_COLS, "TMEM plan");

struct Smem {
  uint8_t b[NS][B_STAGE];          // 1024-aligned (first member)
  uint8_t p[NP][P_STAGE];
  uint16_t stg[4][32 * 32];        // PLAIN epilogue transpose, one 32x32 tile per warp
  uint32_t prefix[MAX_E + 1];
  uint32_t offs[MAX_E + 1];
  uint64_t ofull[NS], oempty[NS], pfull[NP], pempty[NP];
  uint64_t dfull[2], dempty[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct Unit {
  int e, mt, row0, len;
};

__device__ __forceinline__ Unit decode_unit(const Smem& sm, int E, int MT, int u) {
  int lo = 0, hi = E;  // prefix[lo] <= u < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if ((int)sm.prefix[mid] <= u) lo = mid; else hi = mid;
  }
  Unit r;
  r.e = lo;
  const int l = u - (int)sm.prefix[lo];
  const int chunk = l / MT;
  r.mt = l - chunk * MT;
  const int Re = (int)(sm.offs[lo + 1] - sm.offs[lo]);
  const int nch = (Re + MAX_N - 1) / MAX_N;
  const int rpc = (Re + nch - 1) / nch;
  r.row0 = (int)sm.offs[lo] + chunk * rpc;
  r.len = min(rpc, Re - chunk * rpc);
  return r;
}

// AND of `v` over the `n` threads of named barrier `id` (all of them wait).
__device__ __forceinline__ bool bar_red_and(int id, int n, bool v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n barrier.red.and.pred q, %2, %3, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((int)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// position of K index f inside its 8-block after the (0,4,1,5,2,6,3,7) reorder
__device__ __forceinline__ int kperm(int f) {
  const int j = f & 7;
  return (f & ~7) | (j < 4 ? 2 * j : 2 * (j - 4) + 1);
}

// SwiGLU with the bf16 rounding points of the decode path; exp through the
// fast hardware exponential (results can differ from expf in the last bf16
// place of the sigmoid, well inside the layer tolerance) and the reciprocal
// through the correctly rounded rcp (identical to 1/x).
// Round to bf16 (nearest even) with the conversion instruction; differs from
// f2bf only in the NaN payload.
__device__ __forceinline__ uint16_t f2bf_hw(float f) {
  uint16_t h;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return h;
}
__device__ __forceinline__ float rb_hw(float f) { return __uint_as_float((uint32_t)f2bf_hw(f) << 16); }

__device__ __forceinline__ uint16_t swiglu_bf16_fast(float g, float u) {
  const float x = rb_hw(g);
  const float e = rb_hw(__expf(rb_hw(fabsf(x))));
  const float y = rb_hw(__frcp_rn(rb_hw(1.0f + e)));
  const float sg = x < 0.0f ? y : rb_hw(1.0f - y);
  const float si = rb_hw(x * sg);
  return f2bf_hw(si * rb_hw(u));
}

// Scale or bias of group gi (0..7) of an 8-group block held as 16 bytes.
template <int GI>
__device__ __forceinline__ uint32_t meta_pair(const uint4& v) {
  const uint32_t w = (GI >> 1) == 0 ? v.x : (GI >> 1) == 1 ? v.y : (GI >> 1) == 2 ? v.z : v.w;
  // both halves of the result hold the group's bf16 value
  return __byte_perm(w, 0, (GI & 1) ? 0x3232 : 0x1010);
}

// One dequant warp of group GROUP (0 or 1): the group handles every other K
// step (the two groups keep two steps in flight); per step the warp turns the
// 64 packed values of its A row into bf16 s*q + b and stores them to TMEM.
// The group arithmetic is compile-time: GS / 8 K steps share one 16-byte
// block of 8 scales / biases.
template <int MODE, int GS, int GROUP>
__device__ __forceinline__ void dequant_role(const TcParams& p, Smem& sm, uint32_t tbase, int warp, int lane, int E,
                                             int MT, int nk, int U, uint64_t deadline, volatile int* abort_flag) {
  constexpr int SPB = GS / 8;  // K steps per block of 8 groups (even)
  static_assert(SPB % 2 == 0, "each block holds an even number of K steps");
  const int quarter = warp & 3;
  const int r = quarter * 32 + lane;  // A row = TMEM lane
  // GLU rows: each 32-lane quarter holds 16 gate rows then the same 16 up rows
  const int fo = quarter * 16 + (lane & 15);
  const bool up_row = (MODE == TC_GLU) && (lane >= 16);
  const int prow = (MODE == TC_GLU) ? (up_row ? 64 + fo : fo) : r;  // row in the packed stage
  const uint32_t prow_off = prow * 128, sw = prow & 7;  // 128-byte swizzle: unit c at (c ^ row % 8)
  const uint32_t t_col = tbase + ((uint32_t)(quarter * 32) << 16) + A_COL;
  const int G = p.K / GS;
  const int nblk = G / 8;
  uint32_t ks = GROUP;  // running K-step index (stage counters), this group's steps only
  for (int u = blockIdx.x; u < U && !__any_sync(0xffffffffu, *abort_flag != 0); u += gridDim.x) {
    const Unit t = decode_unit(sm, E, MT, u);
    const size_t row = (MODE == TC_GLU) ? (size_t)t.e * p.Nw + t.mt * 64 + fo : (size_t)t.e * p.Nw + t.mt * TILE_M + r;
    const uint4* s4 = reinterpret_cast<const uint4*>((up_row ? p.s1 : p.s0) + row * G);
    const uint4* b4 = reinterpret_cast<const uint4*>((up_row ? p.b1 : p.b0) + row * G);
    uint4 s_nxt = __ldg(s4), b_nxt = __ldg(b4);
    bool ok = true;
    for (int blk = 0; blk < nblk && ok; ++blk) {
      const uint4 sc = s_nxt, bc = b_nxt;
      if (blk + 1 < nblk) {
        s_nxt = __ldg(s4 + blk + 1);
        b_nxt = __ldg(b4 + blk + 1);
      }
#pragma unroll
      for (int j = GROUP; j < SPB; j += 2, ks += 2) {
        const uint32_t pst = ks / PK, ps = pst % NP, as = ks % NS;
        const uint32_t sub = j % PK;  // K step inside the packed stage (compile-time after unrolling)
        if (!__all_sync(0xffffffffu, tc::wait(&sm.pfull[ps], (pst / NP) & 1, deadline, abort_flag))) {
          ok = false;
          break;
        }
        const uint4 w0 = *reinterpret_cast<const uint4*>(sm.p[ps] + prow_off + (((2 * sub) ^ sw) << 4));
        const uint4 w1 = *reinterpret_cast<const uint4*>(sm.p[ps] + prow_off + (((2 * sub + 1) ^ sw) << 4));
        __syncwarp();
        // each warp reads a packed stage in two of its K steps; it releases it after the second
        if (sub >= 2 && lane == 0) mbar_arrive(&sm.pempty[ps]);
        if (ks >= NS &&
            !__all_sync(0xffffffffu, tc::wait(&sm.oempty[as], ((ks / NS) - 1) & 1, deadline, abort_flag))) {
          ok = false;
          break;
        }
        tc::fence_after();
        // groups of the two 32-value halves of this K step inside the block
        uint32_t s2[2], b2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          switch ((j * 64 + h * 32) / GS) {
            case 0: s2[h] = meta_pair<0>(sc); b2[h] = meta_pair<0>(bc); break;
            case 1: s2[h] = meta_pair<1>(sc); b2[h] = meta_pair<1>(bc); break;
            case 2: s2[h] = meta_pair<2>(sc); b2[h] = meta_pair<2>(bc); break;
            case 3: s2[h] = meta_pair<3>(sc); b2[h] = meta_pair<3>(bc); break;
            case 4: s2[h] = meta_pair<4>(sc); b2[h] = meta_pair<4>(bc); break;
            case 5: s2[h] = meta_pair<5>(sc); b2[h] = meta_pair<5>(bc); break;
            case 6: s2[h] = meta_pair<6>(sc); b2[h] = meta_pair<6>(bc); break;
            default: s2[h] = meta_pair<7>(sc); b2[h] = meta_pair<7>(bc); break;
          }
        }
        uint32_t a[32];
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint32_t k128 = 0x43004300u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t w = words[i];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint32_t q = tc::bf2_sub(lop_or_and(w >> (4 * jj), 0x000F000Fu, k128), k128);
            a[i * 4 + jj] = tc::bf2_fma(q, s2[i >> 2], b2[i >> 2]);
          }
        }
        tc::tmem_st32(t_col + as * 32, a);
        tc::tmem_wait_st();
        tc::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.ofull[as]);
      }
    }
    if (!ok) {
      if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
      *abort_flag = 1;
      break;
    }
  }
}

// Roles (warp: role). A warp may only touch TMEM lanes 32*(warp%4) ...+31.
//   0      producer of packed weight tiles (elected lane)
//   1      TMEM allocation; MMA issue (elected lane)
//   2..9   dequant: A row = 32*(warp%4) + lane; warps 2..5 even K steps, 6..9 odd
//   10..13 epilogue: accumulator lanes 32*(warp%4) ... +31
//   14     producer of token-row tiles (elected lane)
template <int MODE, int GS>
__global__ void __launch_bounds__(NTHREADS + 32, 1) qmm_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  // aligned by pointer arithmetic on the shared array (an integer round trip
  // would hide the address space and turn every shared access generic)
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = p.E;
  const int MT = (MODE == TC_GLU) ? p.Nw / 64 : p.Nw / TILE_M;
  const int nk = p.K / KSTEP;
  volatile int* abort_flag = &sm.abort_flag;
  const uint64_t deadline = globaltimer() + (uint64_t)p.timeout_ns;

  if (tid == 0) {
    // operand stage full: 4 dequant warps of one group + the token-row producer (with its bytes)
    for (int i = 0; i < NS; ++i) { mbar_init(&sm.ofull[i], 5); mbar_init(&sm.oempty[i], 1); }
    for (int i = 0; i < NP; ++i) { mbar_init(&sm.pfull[i], 1); mbar_init(&sm.pempty[i], 8); }
    for (int i = 0; i < 2; ++i) { mbar_init(&sm.dfull[i], 1); mbar_init(&sm.dempty[i], 4); }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = tid; i <= E; i += blockDim.x) {
    sm.prefix[i] = p.prefix[i];
    sm.offs[i] = p.offsets[i];
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = sm.tmem_base;
  const int U = (int)sm.prefix[E];

  if (warp == 0 || warp == NWARPS) {
    // ---------------- producers (one converged warp each; an elected lane issues) ----------------
    const bool weights = (warp == 0);
    const uint64_t pol = weights ? policy_evict_first() : policy_evict_last();
    uint32_t nfill = 0;
    const uint32_t NSTG = weights ? NP : NS;
    uint64_t* full = weights ? sm.pfull : sm.ofull;
    uint64_t* empty = weights ? sm.pempty : sm.oempty;
    for (int u = blockIdx.x; u < U && !__any_sync(0xffffffffu, *abort_flag != 0); u += gridDim.x) {
      const Unit t = decode_unit(sm, E, MT, u);
      const int nbox = (t.len + 31) / 32;
      bool ok = true;
      const int nfills = weights ? nk / PK : nk;
      for (int s = 0; s < nfills; ++s, ++nfill) {
        const uint32_t st = nfill % NSTG;
        if (nfill >= NSTG &&
            !__all_sync(0xffffffffu, tc::wait(&empty[st], ((nfill / NSTG) - 1) & 1, deadline, abort_flag))) {
          ok = false;
          break;
        }
        if (tc::elect_one()) {
          if (weights) {
            // 128 bytes (4 K steps) of each of the tile's weight rows
            mbar_arrive_expect_tx(&full[st], P_STAGE);
            uint8_t* dst = sm.p[st];
            if (MODE == TC_GLU) {
              const int r0 = t.e * p.Nw + t.mt * 64;
              tc::tma_load_2d(dst, &p.map_w0, s * 64, r0, &full[st], pol);
              tc::tma_load_2d(dst + P_STAGE / 2, &p.map_w1, s * 64, r0, &full[st], pol);
            } else {
              tc::tma_load_2d(dst, &p.map_w0, s * 64, t.e * p.Nw + t.mt * TILE_M, &full[st], pol);
            }
          } else {
            // token rows of this K step; one of the five arrivals of the operand barrier
            mbar_arrive_expect_tx(&full[st], nbox * 4096);
            for (int b = 0; b < nbox; ++b)
              tc::tma_load_2d(sm.b[st] + b * 4096, &p.map_b, s * KSTEP, t.row0 + b * 32, &full[st], pol);
          }
        }
        __syncwarp();
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
    }
    if (*abort_flag) {
      // let every copy already issued land before the CTA can exit
      const uint64_t dl = globaltimer() + 200000000ull;
      for (uint32_t i = (nfill > NSTG ? nfill - NSTG : 0); i < nfill; ++i)
        tc::wait_until(&full[i % NSTG], (i / NSTG) & 1, dl);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (converged warp; an elected lane issues) ----------------
    uint32_t ks = 0, units = 0;
    bool issued = false;
    for (int u = blockIdx.x; u < U && !__any_sync(0xffffffffu, *abort_flag != 0); u += gridDim.x, ++units) {
      const Unit t = decode_unit(sm, E, MT, u);
      const int N = ((t.len + 15) / 16) * 16;
      const uint32_t idesc = tc::idesc_bf16_f32(TILE_M, N);
      const uint32_t d = units & 1;
      if (units >= 2 &&
          !__all_sync(0xffffffffu, tc::wait(&sm.dempty[d], ((units >> 1) - 1) & 1, deadline, abort_flag))) {
        if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc::fence_after();
      const uint32_t dcol = tbase + (d ? D_COL1 : 0);
      bool ok = true;
      for (int s = 0; s < nk; ++s, ++ks) {
        const uint32_t st = ks % NS;
        if (!__all_sync(0xffffffffu, tc::wait(&sm.ofull[st], (ks / NS) & 1, deadline, abort_flag))) {
          ok = false;
          break;
        }
        tc::fence_after();
        const uint64_t bdesc = tc::smem_desc_sw128(smem_u32(sm.b[st]));
#pragma unroll
        for (int kk = 0; kk < KSTEP / 16; ++kk)
          tc::mma_ts_elect(dcol, tbase + A_COL + st * 32 + kk * 8, bdesc + 2 * kk, idesc, (s | kk) != 0);
        issued = true;
        tc::commit_elect(&sm.oempty[st]);
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc::commit_elect(&sm.dfull[d]);
    }
    if (issued) {
      // every MMA done before TMEM can be released
      tc::commit_elect(&sm.drain);
      tc::wait_until(&sm.drain, 0, globaltimer() + 200000000ull);
    }
  } else if (warp < 10) {
    // ---------------- dequant (8 warps: quarter = warp % 4, K half) ----------------
    if (warp < 6)
      dequant_role<MODE, GS, 0>(p, sm, tbase, warp, lane, E, MT, nk, U, deadline, abort_flag);
    else
      dequant_role<MODE, GS, 1>(p, sm, tbase, warp, lane, E, MT, nk, U, deadline, abort_flag);
  } else if (warp < NWARPS) {
    // ---------------- epilogue (4 warps, quarter = warp % 4) ----------------
    const int quarter = warp & 3;
    const uint32_t t_lane = tbase + ((uint32_t)(quarter * 32) << 16);
    uint16_t* stg = sm.stg[warp - 10];
    uint32_t units = 0;
    // the loop bound is uniform and every exit is decided by one barrier
    // reduction over the four warps
    for (int u = blockIdx.x; u < U; u += gridDim.x, ++units) {
      const Unit t = decode_unit(sm, E, MT, u);
      const uint32_t d = units & 1;
      const bool got = tc::wait(&sm.dfull[d], (units >> 1) & 1, deadline, abort_flag);
      if (!bar_red_and(1, 128, got)) {
        if (!got && !*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc::fence_after();
      const uint32_t dcol = t_lane + (d ? D_COL1 : 0);
      const int nchunk = (t.len + 31) / 32;
      for (int c = 0; c < nchunk; ++c) {
        uint32_t v[32];
        tc::tmem_ld32(dcol + c * 32, v);
        tc::tmem_wait_ld();
        if (c == nchunk - 1) {
          // accumulator fully read: hand it back to the MMA issuer
          tc::fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.dempty[d]);
        }
        if (MODE == TC_GLU) {
          // lane l < 16: gate row f, lane l + 16: up row f; pair through a shuffle
          const int f = t.mt * 64 + quarter * 16 + (lane & 15);
          const int pf = kperm(f);
          const bool lo = lane < 16;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t send = lo ? v[i + 16] : v[i];
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 16);
            const float gv = __uint_as_float(lo ? v[i] : recv);
            const float uv = __uint_as_float(lo ? recv : v[i + 16]);
            const int tok = c * 32 + (lo ? i : 16 + i);
            if (tok < t.len)
              p.out[(size_t)(t.row0 + tok) * p.out_ld + pf] = swiglu_bf16_fast(gv, uv);
          }
        } else {
          // transpose the 32 x 32 tile through shared memory for 16-byte row stores
#pragma unroll
          for (int i = 0; i < 32; ++i) stg[i * 32 + lane] = f2bf_hw(__uint_as_float(v[i]));
          __syncwarp();
          const int h = t.mt * TILE_M + quarter * 32 + (lane & 3) * 8;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int tl = j * 8 + (lane >> 2);
            const int tok = c * 32 + tl;
            if (tok < t.len) {
              const int row = t.row0 + tok;
              const size_t orow = p.out_rows ? p.out_rows[row] : (size_t)row;
              *reinterpret_cast<uint4*>(p.out + orow * p.out_ld + h) =
                  *reinterpret_cast<const uint4*>(stg + tl * 32 + (lane & 3) * 8);
            }
          }
          __syncwarp();
        }
      }
    }
  }

  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == 1) tc::tmem_dealloc(tbase, TMEM_COLS);
}

// Units per expert: ceil(R_e / 192) chunks times the weight tiles.
__global__ void unit_table_kernel(const uint32_t* __restrict__ offsets, int E, int MT0, int MT1,
                                  uint32_t* __restrict__ prefix0, uint32_t* __restrict__ prefix1) {
  __shared__ uint32_t c0[MAX_E + 1], c1[MAX_E + 1];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const uint32_t Re = offsets[e + 1] - offsets[e];
    const uint32_t nch = (Re + MAX_N - 1) / MAX_N;
    c0[e] = nch * MT0;
    c1[e] = nch * MT1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t a = 0, b = 0;
    for (int e = 0; e < E; ++e) {
      prefix0[e] = a;
      if (prefix1) prefix1[e] = b;
      a += c0[e];
      b += c1[e];
    }
    prefix0[E] = a;
    if (prefix1) prefix1[E] = b;
  }
}

// xs[i, :] = x[rows[i], :] with every 8-block reordered (0,4,1,5,2,6,3,7);
// with `range`, only rows in [range[0], range[range_n]) are written.
__global__ void gather_rows_perm_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ rows,
                                        uint16_t* __restrict__ xs, int R, int K, int n_src,
                                        const uint32_t* __restrict__ range, int range_n) {
  const int i = blockIdx.x;
  if (i >= R) return;
  if (range && ((uint32_t)i < range[0] || (uint32_t)i >= range[range_n])) return;
  const uint32_t src = rows ? rows[i] : (uint32_t)i;
  const int nv = K / 8;
  uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)i * K);
  if (src >= (uint32_t)n_src) {
    for (int v = threadIdx.x; v < nv; v += blockDim.x) dst[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(x + (size_t)src * K);
  for (int v = threadIdx.x; v < nv; v += blockDim.x) dst[v] = perm_x8(__ldg(s + v));
}

}  // namespace qtc

using namespace qtc;

size_t tc_smem_bytes() { return sizeof(Smem) + 1024; }

bool tc_shape_ok(int Nw, int K, int gs, int mode) {
  // whole 64-wide K steps; metadata rows in 16-byte blocks of 8 groups
  if (K <= 0 || K % KSTEP || K % (8 * gs)) return false;
  if (mode == TC_GLU) return Nw > 0 && Nw % 64 == 0;
  return Nw > 0 && Nw % TILE_M == 0;
}

int tc_unit_tables(const uint32_t* offsets, int E, int mt0, int mt1, uint32_t* prefix0, uint32_t* prefix1,
                   cudaStream_t st) {
  if (E < 1 || E > MAX_E) return set_error(B2Q_EUNSUPPORTED, "tensor-core qmm: E=%d (1..%d)", E, MAX_E);
  unit_table_kernel<<<1, 256, 0, st>>>(offsets, E, mt0, mt1, prefix0, prefix1);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int tc_gather_rows(const uint16_t* x, const uint32_t* rows, uint16_t* xs, int R, int K, int n_src,
                   cudaStream_t st) {
  if (R <= 0) return B2Q_OK;
  gather_rows_perm_kernel<<<R, 128, 0, st>>>(x, rows, xs, R, K, n_src, nullptr, 0);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int tc_gather_rows_range(const uint16_t* x, const uint32_t* rows, uint16_t* xs, int R, int K, int n_src,
                         const uint32_t* offsets, int n_groups, cudaStream_t st) {
  if (R <= 0) return B2Q_OK;
  gather_rows_perm_kernel<<<R, 128, 0, st>>>(x, rows, xs, R, K, n_src, offsets, n_groups);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int tc_setup(TcParams& p, int mode, const uint16_t* xs, int R, const uint32_t* w0, const uint32_t* w1) {
  // packed weights: uint16 view [E*Nw rows, K/4], boxes {64 (128 bytes = 4 K steps), 64 or 128 rows},
  // 128-byte swizzle
  const int box_rows = (mode == TC_GLU) ? 64 : TILE_M;
  int rc = make_2d_map(&p.map_w0, w0, (uint64_t)p.E * p.Nw, (uint64_t)p.K / 2, 128, box_rows, 128);
  if (rc) return rc;
  if (mode == TC_GLU) {
    rc = make_2d_map(&p.map_w1, w1, (uint64_t)p.E * p.Nw, (uint64_t)p.K / 2, 128, box_rows, 128);
    if (rc) return rc;
  }
  // token rows: bf16 [R, K], boxes {64 (128 bytes), 32 rows}, 128-byte swizzle
  return make_2d_map(&p.map_b, xs, (uint64_t)R, (uint64_t)p.K * 2, 128, 32, 128);
}

int tc_launch(const TcParams& p, int mode, cudaStream_t st) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const size_t smem = tc_smem_bytes();
  if ((int)smem > di.smem_optin) return set_error(B2Q_EUNSUPPORTED, "tensor-core qmm: %zu bytes of shared memory", smem);
  const int grid = di.sm_count;
  const int threads = NTHREADS + 32;
#define B2Q_TC_CASE(M, G)                                                                                   \
  if (mode == M && p.gs == G) {                                                                             \
    static int attr_done[64] = {};                                                                          \
    if (!attr_done[di.device & 63]) {                                                                       \
      B2Q_TRY_CUDA(cudaFuncSetAttribute(qmm_tc_kernel<M, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
      attr_done[di.device & 63] = 1;                                                                        \
    }                                                                                                       \
    qmm_tc_kernel<M, G><<<grid, threads, smem, st>>>(p);                                                    \
  } else
  B2Q_TC_CASE(TC_GLU, 32) B2Q_TC_CASE(TC_GLU, 64) B2Q_TC_CASE(TC_GLU, 128)
  B2Q_TC_CASE(TC_PLAIN, 32) B2Q_TC_CASE(TC_PLAIN, 64) B2Q_TC_CASE(TC_PLAIN, 128)
  return set_error(B2Q_EUNSUPPORTED, "tensor-core qmm: group size %d", p.gs);
#undef B2Q_TC_CASE
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // namespace b2q
