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
//   * a work unit is (expert, chunk of <= 256 rows of that expert, 128-row
//     weight tile); GLU tiles stack 64 gate rows over the same 64 up rows;
//   * a producer warp streams, per 64-wide K step, the packed weight tile
//     (TMA, 32-byte swizzle) and the token rows (TMA, 128-byte swizzle);
//   * eight dequant warps turn packed nibbles into bf16 (mask into bf16 128.0,
//     subtract 128, one bf16x2 fma with scale and bias: one rounding of
//     s*q + b) and store them to TMEM as the MMA's A operand;
//   * one thread issues tcgen05.mma (A from TMEM, B from shared memory) into a
//     128 x N fp32 accumulator in TMEM;
//   * four epilogue warps read the accumulator back (tcgen05.ld) and write
//     bf16 outputs; GLU pairs gate and up lanes through shared memory.
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

constexpr int KSTEP = 64;         // K elements per pipeline step
constexpr int TILE_M = 128;       // weight rows per unit (TMEM lanes)
constexpr int MAX_N = 256;        // token rows per unit
constexpr int NB = 3;             // token-row stages
constexpr int NP = 8;             // packed-weight stages
constexpr int NA = 8;             // TMEM A stages (32 columns each)
constexpr int B_STAGE = MAX_N * KSTEP * 2;   // 32 KB
constexpr int P_STAGE = TILE_M * KSTEP / 2;  // 4 KB
constexpr int EXCH_BYTES = 2 * MAX_N * 64 * 2;  // GLU gate/up bf16 exchange: 64 KB
constexpr int TMEM_COLS = 512;
constexpr int A_COL = 256;        // first TMEM column of the A ring
constexpr int NWARPS = 14;        // 0 producer, 1 MMA, 2..9 dequant, 10..13 epilogue
constexpr int NTHREADS = NWARPS * 32;
constexpr int MAX_E = 1024;

struct Smem {
  uint8_t b[NB][B_STAGE];          // 1024-aligned (first member)
  uint8_t p[NP][P_STAGE];
  uint8_t exch[EXCH_BYTES];
  uint32_t prefix[MAX_E + 1];
  uint32_t offs[MAX_E + 1];
  uint64_t bfull[NB], bempty[NB], pfull[NP], pempty[NP], afull[NA], aempty[NA];
  uint64_t dfull, dempty, drain;
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

template <int MODE>
__global__ void __launch_bounds__(NTHREADS, 1) qmm_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = p.E;
  const int MT = (MODE == TC_GLU) ? p.Nw / 64 : p.Nw / TILE_M;
  const int nk = p.K / KSTEP;
  volatile int* abort_flag = &sm.abort_flag;
  const uint64_t deadline = globaltimer() + (uint64_t)p.timeout_ns;

  if (tid == 0) {
    for (int i = 0; i < NB; ++i) { mbar_init(&sm.bfull[i], 1); mbar_init(&sm.bempty[i], 1); }
    for (int i = 0; i < NP; ++i) { mbar_init(&sm.pfull[i], 1); mbar_init(&sm.pempty[i], 8); }
    for (int i = 0; i < NA; ++i) { mbar_init(&sm.afull[i], 8); mbar_init(&sm.aempty[i], 1); }
    mbar_init(&sm.dfull, 1);
    mbar_init(&sm.dempty, 4);
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = tid; i <= E; i += NTHREADS) {
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

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
      uint32_t nbfill = 0, npfill = 0;
      for (int u = blockIdx.x; u < U && !*abort_flag; u += gridDim.x) {
        const Unit t = decode_unit(sm, E, MT, u);
        const int nbox = (t.len + 31) / 32;
        for (int s = 0; s < nk; ++s) {
          {
            const uint32_t ps = npfill % NP;
            if (npfill >= NP && !tc::wait(&sm.pempty[ps], ((npfill / NP) - 1) & 1, deadline, abort_flag)) {
              record_error(p.err, B2Q_ETIMEOUT);
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&sm.pfull[ps], P_STAGE);
            uint8_t* dst = sm.p[ps];
            if (MODE == TC_GLU) {
              const int r0 = t.e * p.Nw + t.mt * 64;
              tc::tma_load_2d(dst, &p.map_w0, s * 16, r0, &sm.pfull[ps], pol_w);
              tc::tma_load_2d(dst + P_STAGE / 2, &p.map_w1, s * 16, r0, &sm.pfull[ps], pol_w);
            } else {
              tc::tma_load_2d(dst, &p.map_w0, s * 16, t.e * p.Nw + t.mt * TILE_M, &sm.pfull[ps], pol_w);
            }
            ++npfill;
          }
          {
            const uint32_t bs = nbfill % NB;
            if (nbfill >= NB && !tc::wait(&sm.bempty[bs], ((nbfill / NB) - 1) & 1, deadline, abort_flag)) {
              record_error(p.err, B2Q_ETIMEOUT);
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&sm.bfull[bs], nbox * 4096);
            for (int b = 0; b < nbox; ++b)
              tc::tma_load_2d(sm.b[bs] + b * 4096, &p.map_b, s * KSTEP, t.row0 + b * 32, &sm.bfull[bs], pol_x);
            ++nbfill;
          }
        }
      }
      if (*abort_flag) {
        // let every copy already issued land before the CTA can exit
        const uint64_t dl = globaltimer() + 200000000ull;
        for (uint32_t i = (npfill > NP ? npfill - NP : 0); i < npfill; ++i) tc::wait_until(&sm.pfull[i % NP], (i / NP) & 1, dl);
        for (uint32_t i = (nbfill > NB ? nbfill - NB : 0); i < nbfill; ++i) tc::wait_until(&sm.bfull[i % NB], (i / NB) & 1, dl);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t nb = 0, na = 0, units = 0;
      bool issued = false;
      for (int u = blockIdx.x; u < U && !*abort_flag; u += gridDim.x, ++units) {
        const Unit t = decode_unit(sm, E, MT, u);
        const int N = ((t.len + 15) / 16) * 16;
        const uint32_t idesc = tc::idesc_bf16_f32(TILE_M, N);
        if (units > 0 && !tc::wait(&sm.dempty, (units - 1) & 1, deadline, abort_flag)) {
          record_error(p.err, B2Q_ETIMEOUT);
          *abort_flag = 1;
          break;
        }
        tc::fence_after();
        bool ok = true;
        for (int s = 0; s < nk; ++s, ++nb, ++na) {
          const uint32_t as = na % NA, bs = nb % NB;
          if (!tc::wait(&sm.afull[as], (na / NA) & 1, deadline, abort_flag) ||
              !tc::wait(&sm.bfull[bs], (nb / NB) & 1, deadline, abort_flag)) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint64_t bdesc = tc::smem_desc_sw128(smem_u32(sm.b[bs]));
#pragma unroll
          for (int kk = 0; kk < KSTEP / 16; ++kk)
            tc::mma_ts(tbase, tbase + A_COL + as * 32 + kk * 8, bdesc + 2 * kk, idesc, (s | kk) != 0);
          issued = true;
          tc::commit(&sm.aempty[as]);
          tc::commit(&sm.bempty[bs]);
        }
        if (!ok) {
          record_error(p.err, B2Q_ETIMEOUT);
          *abort_flag = 1;
          break;
        }
        tc::commit(&sm.dfull);
      }
      if (issued) {
        // every MMA done before TMEM can be released
        tc::commit(&sm.drain);
        tc::wait_until(&sm.drain, 0, globaltimer() + 200000000ull);
      }
    }
  } else if (warp < 10) {
    // ---------------- dequant (8 warps: quarter = warp % 4, K half) ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // A row = TMEM lane
    const uint32_t t_lane = tbase + ((uint32_t)(quarter * 32) << 16);
    const int G = p.K / p.gs;
    uint32_t np = 0, na = 0;
    for (int u = blockIdx.x; u < U && !__any_sync(0xffffffffu, *abort_flag != 0); u += gridDim.x) {
      const Unit t = decode_unit(sm, E, MT, u);
      // weight row of this thread and its metadata rows
      const uint16_t* srow;
      const uint16_t* brow;
      if (MODE == TC_GLU) {
        const int f = t.mt * 64 + (r & 63);
        const size_t row = (size_t)t.e * p.Nw + f;
        srow = (r < 64 ? p.s0 : p.s1) + row * G;
        brow = (r < 64 ? p.b0 : p.b1) + row * G;
      } else {
        const size_t row = (size_t)t.e * p.Nw + t.mt * TILE_M + r;
        srow = p.s0 + row * G;
        brow = p.b0 + row * G;
      }
      // scales / biases in blocks of 8 groups (16 bytes), the next block in flight
      int blk = -1;
      uint4 s_cur = make_uint4(0, 0, 0, 0), b_cur = s_cur, s_nxt = s_cur, b_nxt = s_cur;
      const uint4* s4 = reinterpret_cast<const uint4*>(srow);
      const uint4* b4 = reinterpret_cast<const uint4*>(brow);
      const int nblk = G / 8;
      bool ok = true;
      for (int s = 0; s < nk; ++s, ++np, ++na) {
        const uint32_t ps = np % NP, as = na % NA;
        // group of this thread's 32 K values
        const int g = (s * KSTEP + half * 32) / p.gs;
        if ((g >> 3) != blk) {
          if (blk < 0) {
            s_cur = __ldg(s4 + (g >> 3));
            b_cur = __ldg(b4 + (g >> 3));
          } else {
            s_cur = s_nxt;
            b_cur = b_nxt;
          }
          blk = g >> 3;
          if (blk + 1 < nblk) {
            s_nxt = __ldg(s4 + blk + 1);
            b_nxt = __ldg(b4 + blk + 1);
          }
        }
        const int gi = g & 7;
        const uint32_t sw = (gi & 4) ? ((gi & 2) ? s_cur.w : s_cur.z) : ((gi & 2) ? s_cur.y : s_cur.x);
        const uint32_t bw = (gi & 4) ? ((gi & 2) ? b_cur.w : b_cur.z) : ((gi & 2) ? b_cur.y : b_cur.x);
        const uint32_t sv = (gi & 1) ? (sw >> 16) : (sw & 0xFFFFu);
        const uint32_t bv = (gi & 1) ? (bw >> 16) : (bw & 0xFFFFu);
        const uint32_t s2 = sv | (sv << 16), b2 = bv | (bv << 16);
        if (!__all_sync(0xffffffffu, tc::wait(&sm.pfull[ps], (np / NP) & 1, deadline, abort_flag))) {
          ok = false;
          break;
        }
        const uint4 wv = *reinterpret_cast<const uint4*>(sm.p[ps] + r * 32 + ((half ^ ((r >> 2) & 1)) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.pempty[ps]);
        if (na >= NA &&
            !__all_sync(0xffffffffu, tc::wait(&sm.aempty[as], ((na / NA) - 1) & 1, deadline, abort_flag))) {
          ok = false;
          break;
        }
        tc::fence_after();
        uint32_t a[16];
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint32_t k128 = 0x43004300u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w = words[i];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t q = tc::bf2_sub(lop_or_and(w >> (4 * j), 0x000F000Fu, k128), k128);
            a[i * 4 + j] = tc::bf2_fma(q, s2, b2);
          }
        }
        tc::tmem_st16(t_lane + A_COL + as * 32 + half * 16, a);
        tc::tmem_wait_st();
        tc::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.afull[as]);
      }
      if (!ok) {
        record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
    }
  } else {
    // ---------------- epilogue (4 warps, quarter = warp % 4) ----------------
    const int quarter = warp & 3;
    const int etid = tid - 10 * 32;  // 0..127
    const uint32_t t_lane = tbase + ((uint32_t)(quarter * 32) << 16);
    uint16_t* exg = reinterpret_cast<uint16_t*>(sm.exch);  // [MAX_N][64] gate
    uint16_t* exu = exg + MAX_N * 64;                      // [MAX_N][64] up
    uint32_t units = 0;
    // the loop bound is uniform and every exit is decided by one barrier
    // reduction over the four warps, so the named barriers below always see
    // all 128 threads
    for (int u = blockIdx.x; u < U; u += gridDim.x, ++units) {
      const Unit t = decode_unit(sm, E, MT, u);
      const bool got = tc::wait(&sm.dfull, units & 1, deadline, abort_flag);
      if (!bar_red_and(1, 128, got)) {
        if (!got && !*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc::fence_after();
      const int nchunk = (t.len + 31) / 32;
      for (int c = 0; c < nchunk; ++c) {
        uint32_t v[32];
        tc::tmem_ld32(t_lane + c * 32, v);
        tc::tmem_wait_ld();
        if (MODE == TC_GLU) {
          uint16_t* ex = (quarter < 2) ? exg : exu;
          const int fl = (quarter & 1) * 32 + lane;
#pragma unroll
          for (int i = 0; i < 32; ++i) ex[(c * 32 + i) * 64 + fl] = f2bf(__uint_as_float(v[i]));
        } else {
          const int h = t.mt * TILE_M + quarter * 32 + lane;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int tok = c * 32 + i;
            if (tok < t.len) {
              const int row = t.row0 + tok;
              const size_t orow = p.out_rows ? p.out_rows[row] : (size_t)row;
              p.out[orow * p.out_ld + h] = f2bf(__uint_as_float(v[i]));
            }
          }
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dempty);
      if (MODE == TC_GLU) {
        named_bar_sync(1, 128);
        const int fl = etid & 63;
        const int pf = kperm(t.mt * 64 + fl);
        for (int tok = etid >> 6; tok < t.len; tok += 2) {
          const uint16_t gv = exg[tok * 64 + fl], uv = exu[tok * 64 + fl];
          p.out[(size_t)(t.row0 + tok) * p.out_ld + pf] = swiglu_bf16(gv, uv);
        }
        named_bar_sync(1, 128);
      }
    }
  }

  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == 1) tc::tmem_dealloc(tbase, TMEM_COLS);
}

// Units per expert: ceil(R_e / 256) chunks times the weight tiles.
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

// xs[i, :] = x[rows[i], :] with every 8-block reordered (0,4,1,5,2,6,3,7).
__global__ void gather_rows_perm_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ rows,
                                        uint16_t* __restrict__ xs, int R, int K, int n_src) {
  const int i = blockIdx.x;
  if (i >= R) return;
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
  gather_rows_perm_kernel<<<R, 128, 0, st>>>(x, rows, xs, R, K, n_src);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int tc_setup(TcParams& p, int mode, const uint16_t* xs, int R, const uint32_t* w0, const uint32_t* w1) {
  // packed weights: uint16 view [E*Nw rows, K/4], boxes {16 (32 bytes), 64 or 128 rows}, 32-byte swizzle
  const int box_rows = (mode == TC_GLU) ? 64 : TILE_M;
  int rc = make_2d_map(&p.map_w0, w0, (uint64_t)p.E * p.Nw, (uint64_t)p.K / 2, 32, box_rows, 32);
  if (rc) return rc;
  if (mode == TC_GLU) {
    rc = make_2d_map(&p.map_w1, w1, (uint64_t)p.E * p.Nw, (uint64_t)p.K / 2, 32, box_rows, 32);
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
  static int attr_done[64] = {};
  const int slot = (di.device & 63);
  if (!(attr_done[slot] & (1 << mode))) {
    if (mode == TC_GLU)
      B2Q_TRY_CUDA(cudaFuncSetAttribute(qmm_tc_kernel<TC_GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    else
      B2Q_TRY_CUDA(cudaFuncSetAttribute(qmm_tc_kernel<TC_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_done[slot] |= 1 << mode;
  }
  const int grid = di.sm_count;
  if (mode == TC_GLU)
    qmm_tc_kernel<TC_GLU><<<grid, NTHREADS, smem, st>>>(p);
  else
    qmm_tc_kernel<TC_PLAIN><<<grid, NTHREADS, smem, st>>>(p);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // namespace b2q
