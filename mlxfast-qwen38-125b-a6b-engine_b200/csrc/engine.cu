// engine.cu -- the streaming (decode) product engine for sm_100a.
//
// Reference arithmetic it stands in for (paths relative to the reference
// project, QH = Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/metal/kernels/quantized.h):
//   qmv_fast_impl / qmv_impl       QH:757-987   (per-group s*sum(xq) + b*sum(x), fp32)
//   affine_gather_qmv_fast         QH:2444-2505 (per-item expert offset)
//   track_moe_gate_up_act          Runner/FastModel/TrackFastMoE.swift:1192-1410
//   track_moe_down_combine         Runner/FastModel/TrackFastMoE.swift:1412-1590
//   track_moe_route                Runner/FastModel/TrackFastMoE.swift:767-911
// The design is this file's own: TMA tensor-copy producer, MMA consumers,
// static persistent schedule, fixed-order cross-warp reduction.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "tc.cuh"
#include "engine.cuh"
#include "host.hpp"
#include "tmap.hpp"

namespace b2q {
namespace eng {

// ---------------------------------------------------------------------------
// PTX: 3-D tiled TMA load into shared memory, completion on an mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 prefetch of a tensor-map box (no shared-memory destination).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Wait with a suspend-time hint so a waiting warp sleeps instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 100000;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline, volatile int* abort) {
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (abort && *abort) return false;
    if (globaltimer() > deadline) return false;
  }
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ float lo_bf(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_bf(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// ---------------------------------------------------------------------------
// unit / pass enumeration (shared by producer and consumers)
// ---------------------------------------------------------------------------
struct Sched {
  int U;      // total units
  int U_gu;   // FUSED: gate|up units before the down units
  int RB;     // QMV: row blocks per item
  int FB;     // gate|up row blocks per slot (F / 8)
  int HB;     // down row blocks per token (H / 8)
  int npair;  // down slot pairs (ceil(k / 2))
};

__device__ __forceinline__ Sched make_sched(const Params& p) {
  Sched s{};
  s.FB = p.F / 8;
  s.HB = p.H / 8;
  s.npair = (p.k + 1) / 2;
  switch (p.mode) {
    case MODE_QMV:
      s.RB = (p.N + 15) / 16;
      s.U = p.batch * s.RB;
      break;
    case MODE_GU:
      s.U = p.n_slots * s.FB;
      break;
    case MODE_DOWN:
      s.U = p.S * s.HB;
      break;
    default:  // FUSED, one token
      s.U_gu = p.k * s.FB;
      s.U = s.U_gu + s.HB;
      break;
  }
  return s;
}

__device__ __forceinline__ bool unit_is_down(const Params& p, const Sched& s, int u) {
  return p.mode == MODE_DOWN || (p.mode == MODE_FUSED && u >= s.U_gu);
}

__device__ __forceinline__ int unit_passes(const Params& p, const Sched& s, int u) {
  return unit_is_down(p, s, u) ? s.npair * p.g2.nkc : p.g1.nkc;
}

__device__ __forceinline__ uint32_t clamp_expert(uint32_t e, int E, int* err) {
  if (e >= (uint32_t)E) {
    record_error(err, B2Q_EINVAL);
    return 0;
  }
  return e;
}

// Which maps and rows one pass reads.
struct LoadDesc {
  int mwP, msP, mbP, mwQ, msQ, mbQ;  // tensor-map slots
  int rowP, rowQ;                    // first row of each 8-row block (in the map's row space)
  int kc;                            // reduction chunk index
  bool valid;
};

__device__ __forceinline__ LoadDesc describe(const Params& p, const Sched& s, int u, int pass, const uint32_t* sidx,
                                             int* err) {
  LoadDesc d{};
  d.valid = true;
  if (p.mode == MODE_QMV) {
    const int item = u / s.RB, rb = u % s.RB;
    const uint32_t e = p.rhs ? __ldg(p.rhs + item) : (uint32_t)item;
    const uint32_t xi = p.lhs ? __ldg(p.lhs + item) : (uint32_t)item;
    d.valid = e < (uint32_t)p.n_w && xi < (uint32_t)p.n_x;
    d.mwP = d.mwQ = M_W;
    d.msP = d.msQ = M_S;
    d.mbP = d.mbQ = M_B;
    d.rowP = (int)(e * (uint32_t)p.N) + rb * 16;
    d.rowQ = d.rowP + 8;
    d.kc = pass;
    return d;
  }
  if (!unit_is_down(p, s, u)) {
    const int z = u / s.FB, rb = u % s.FB;
    const uint32_t e = (p.mode == MODE_FUSED) ? sidx[z] : clamp_expert(__ldg(p.idx_in + z), p.E, err);
    d.mwP = M_WG;
    d.msP = M_SG;
    d.mbP = M_BG;
    d.mwQ = M_WU;
    d.msQ = M_SU;
    d.mbQ = M_BU;
    d.rowP = d.rowQ = (int)(e * (uint32_t)p.F) + rb * 8;
    d.kc = pass;
    return d;
  }
  const int ud = (p.mode == MODE_FUSED) ? u - s.U_gu : u;
  const int t = ud / s.HB, hb = ud % s.HB;
  const int pair = pass / p.g2.nkc;
  const int j0 = 2 * pair, j1 = 2 * pair + 1;
  uint32_t e0, e1;
  if (p.mode == MODE_FUSED) {
    e0 = sidx[j0];
    e1 = (j1 < p.k) ? sidx[j1] : e0;
  } else {
    e0 = clamp_expert(__ldg(p.idx_in + (size_t)t * p.k + j0), p.E, err);
    e1 = (j1 < p.k) ? clamp_expert(__ldg(p.idx_in + (size_t)t * p.k + j1), p.E, err) : e0;
  }
  d.mwP = d.mwQ = M_WD;
  d.msP = d.msQ = M_SD;
  d.mbP = d.mbQ = M_BD;
  d.rowP = (int)(e0 * (uint32_t)p.H) + hb * 8;
  d.rowQ = (int)(e1 * (uint32_t)p.H) + hb * 8;
  d.kc = pass % p.g2.nkc;
  return d;
}

// ---------------------------------------------------------------------------
// activation staging: bf16 rows -> scaled, permuted fp16 chunks + group sums
// ---------------------------------------------------------------------------
// The MMA B operand is fp16. Column c is scaled by S_c = 2^e_c chosen so that
// max|x| * S_c lies in [1024, 2048): every bf16 value converts to fp16
// exactly (bf16 has 8 significant bits, fp16 11) without overflow, and only
// values below 2^-24 of the column's maximum lose bits. The 16-byte chunk of
// values x0..x7 is stored as fp16 pairs
//   (x0 S, x4 S) (x1 S/16, x5 S/16) (x2 S, x6 S) (x3 S/16, x7 S/16)
// to meet the decoded weight pairs (1024+q0, 1024+q4) (1024+16q1, 1024+16q5)
// (1024+q2, 1024+q6) (1024+16q3, 1024+16q7). Per group g:
//   xs[c][g]   = sum of x S
//   xoff[c][g] = 1024 * sum_even x S + 64 * sum_odd x S  (the offset the decode adds)
// and inv[c] = 1 / S_c. Region layout: xs [cap][G], xoff [cap][G], inv [MAX_COLS],
// colmax [MAX_COLS] (scratch).
__device__ __forceinline__ float* cols_xs(float* sums, int G, int col) { return sums + (size_t)col * G; }
__device__ __forceinline__ float* cols_xo(float* sums, int cap, int G, int col) {
  return sums + (size_t)(cap + col) * G;
}
__device__ __forceinline__ float* cols_inv(float* sums, int cap, int G) { return sums + (size_t)2 * cap * G; }

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ void stage_columns(uint8_t* dst, float* sums, int cap, int XS, const uint16_t* const* src_rows, int ncols,
                              int K, int gs, bool coherent) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int nch = K / 8;
  const int G = K / gs;
  float* inv = cols_inv(sums, cap, G);
  unsigned* colmax = reinterpret_cast<unsigned*>(inv + MAX_COLS);
  if (tid < MAX_COLS) colmax[tid] = 0u;
  named_bar_sync(1, NCT);
  // pass 1: max |x| per column (non-negative floats order like their bits)
  for (int q0 = 0; q0 < ncols * nch; q0 += NCT) {
    const int q = q0 + tid;
    unsigned m = 0u;
    int col = q0 / nch;  // warp-uniform when a warp stays inside one column
    if (q < ncols * nch) {
      col = q / nch;
      const int ch = q % nch;
      const uint4* src = reinterpret_cast<const uint4*>(src_rows[col] + (size_t)ch * 8);
      const uint4 v = coherent ? __ldcg(src) : __ldg(src);
      m = max(max(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu), max(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu));
      m = max(m & 0xffffu, m >> 16) << 16;  // largest |bf16| of the chunk as float bits
      if (m > 0x7f800000u) m = 0x7f800000u;  // NaN never sets the scale
      atomicMax(&colmax[col], m);
    }
  }
  named_bar_sync(1, NCT);
  if (tid < ncols) {
    const float mx = __uint_as_float(colmax[tid]);
    int e = 0;
    if (mx > 0.0f && mx < INFINITY) {
      int E;
      frexpf(mx, &E);  // mx = m * 2^E, m in [0.5, 1)
      e = 11 - E;      // mx * 2^e in [1024, 2048)
    }
    inv[tid] = ldexpf(1.0f, -e);
    colmax[tid] = (unsigned)(e + 1000);  // the exponent for pass 2
  }
  named_bar_sync(1, NCT);
  // pass 2: scaled fp16 pairs
  for (int q = tid; q < ncols * nch; q += NCT) {
    const int col = q / nch, ch = q % nch;
    const uint4* src = reinterpret_cast<const uint4*>(src_rows[col] + (size_t)ch * 8);
    const uint4 v = coherent ? __ldcg(src) : __ldg(src);
    const int e = (int)colmax[col] - 1000;
    const float S = ldexpf(1.0f, e), S16 = ldexpf(1.0f, e - 4);
    uint4 o;
    o.x = pack_h2(lo_bf(v.x) * S, lo_bf(v.z) * S);      // (x0, x4)
    o.y = pack_h2(hi_bf(v.x) * S16, hi_bf(v.z) * S16);  // (x1/16, x5/16)
    o.z = pack_h2(lo_bf(v.y) * S, lo_bf(v.w) * S);      // (x2, x6)
    o.w = pack_h2(hi_bf(v.y) * S16, hi_bf(v.w) * S16);  // (x3/16, x7/16)
    *reinterpret_cast<uint4*>(dst + (size_t)col * XS + (size_t)ch * 16) = o;
  }
  named_bar_sync(1, NCT);
  // pass 3: group sums of the scaled values (k order within a chunk)
  for (int q = tid; q < ncols * G; q += NCT) {
    const int col = q / G, g = q % G;
    const uint8_t* base = dst + (size_t)col * XS + (size_t)g * (gs / 8) * 16;
    float se = 0.0f, so = 0.0f;
    for (int ch = 0; ch < gs / 8; ++ch) {
      const uint4 v = *reinterpret_cast<const uint4*>(base + ch * 16);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
      const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
      const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
      se += ((a.x + c.x) + a.y) + c.y;              // x0 + x2 + x4 + x6
      so += ((b.x + d.x) + b.y) + d.y;              // (x1 + x3 + x5 + x7) / 16
    }
    cols_xs(sums, G, col)[g] = se + 16.0f * so;
    cols_xo(sums, cap, G, col)[g] = 1024.0f * se + 1024.0f * so;  // 64 * (16 * so)
  }
  named_bar_sync(1, NCT);
}

// ---------------------------------------------------------------------------
// one pass of MMAs over this warp's share of the 128-byte row pieces
// ---------------------------------------------------------------------------
// Stage layout: [P weights][Q weights][sP][bP][sQ][bQ]. A weight block is one
// 1024-byte atom per 128-byte piece of the 8 rows, 16-byte unit u of row r at
// unit position u ^ r (TMA 128-byte swizzle). Lane (r = lane/4, c = lane%4)
// takes packed word 4*u + c of row r of P and of Q -> MMA rows r and r + 8.
// A piece holds 256 values = 8 / WPT quantization groups; the unrolled loop
// over its 8 units keeps every swizzle offset a per-lane constant.
//
// KIND 0: one activation column matters for every lane (gate|up, qmv M = 1):
//         elements 0 (row r) and 2 (row r + 8) against column sums xs0.
// KIND 1: two columns per lane (qmv M >= 2): elements 0..3, xs0 / xs1.
// KIND 2: down pass of slot pair `pair`: lanes c == pair own element 0
//         (P slot, column 2c) and element 3 (Q slot, column 2c + 1).
// Shared per-pass lane context (plain values, so everything stays in registers).
struct PassCtx {
  const uint8_t* st;
  const uint8_t* mP;  // sP; bP at +blkm
  const uint8_t* mQ;  // sQ; bQ at +blkm
  int blkw, blkm, mswz, mrow;
  int r, c;
};

// byte offset of the 16-bit scale / bias of group gl (within the pass) for row r
__device__ __forceinline__ int meta_off(const PassCtx& x, int gl) {
  if (x.mswz) {
    const int gg = gl & 63;
    return (gl >> 6) * 1024 + x.r * 128 + (((gg >> 3) ^ x.r) << 4) + (gg & 7) * 2;
  }
  return x.r * x.mrow + gl * 2;
}

// One word step: P word at wp, Q word at wp + blkw, activation chunk xv.
__device__ __forceinline__ void word_step(const uint8_t* wp, int blkw, const uint4 xv, bool first, float (&d)[4]) {
  const uint32_t W0 = lds32(wp);
  const uint32_t W8 = lds32(wp + blkw);
  uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
  decode_word_h(W0, p0, p1, p2, p3);
  decode_word_h(W8, q0, q1, q2, q3);
  if (first)
    mma_f16_16816_zero(d, p0, q0, p1, q1, xv.x, xv.y);
  else
    mma_f16_16816(d, p0, q0, p1, q1, xv.x, xv.y);
  mma_f16_16816(d, p2, q2, p3, q3, xv.z, xv.w);
}

// A single-column (KIND 0) piece: every column of B holds the same activation,
// so the four lanes of a quad hold identical D: lane c finishes group c of
// each batch of NB groups. `pw` points at this lane's word of unit 0 of the
// piece before swizzling; unit u lives at pw + ((u ^ r) << 4). The activation
// chunks come from xv (registers) when XREG, else from px (shared memory).
template <int WPT, bool XREG>
__device__ __forceinline__ void piece_kind0(const PassCtx& x, const uint8_t* pw, const uint8_t* px,
                                            const uint4 (&xv)[8], int pc, int gabs0,
                                            const float* __restrict__ xs0, const float* __restrict__ xo0,
                                            float (&acc)[4]) {
  constexpr int GPC = 8 / WPT;
  constexpr int NB = GPC < 4 ? GPC : 4;
#pragma unroll
  for (int b0 = 0; b0 < GPC; b0 += NB) {
    float D[NB][4];
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
#pragma unroll
      for (int gi = 0; gi < NB; ++gi) {
        const int u = (b0 + gi) * WPT + j;
        const uint4 xu = XREG ? xv[u] : lds128(px + u * 64);
        word_step(pw + ((u ^ x.r) << 4), x.blkw, xu, j == 0, D[gi]);
      }
    }
    float e0 = D[0][0], e2 = D[0][2];
#pragma unroll
    for (int gi = 1; gi < NB; ++gi) {
      e0 = (x.c == gi) ? D[gi][0] : e0;
      e2 = (x.c == gi) ? D[gi][2] : e2;
    }
    const int gl = pc * GPC + b0 + (x.c < NB ? x.c : NB - 1);
    const int mo = meta_off(x, gl);
    const float sP = bf2f(*reinterpret_cast<const uint16_t*>(x.mP + mo));
    const float bP = bf2f(*reinterpret_cast<const uint16_t*>(x.mP + x.blkm + mo));
    const float sQ = bf2f(*reinterpret_cast<const uint16_t*>(x.mQ + mo));
    const float bQ = bf2f(*reinterpret_cast<const uint16_t*>(x.mQ + x.blkm + mo));
    const float xa = xs0[gabs0 + gl], xoa = xo0[gabs0 + gl];
    if (x.c < NB) {
      acc[0] = fmaf(sP, e0 - xoa, fmaf(bP, xa, acc[0]));
      acc[2] = fmaf(sQ, e2 - xoa, fmaf(bQ, xa, acc[2]));
    }
  }
}

// One pass of MMAs over this warp's share of the pass's 128-byte row pieces.
//
// Stage layout: [P weights][Q weights][sP][bP][sQ][bQ]. A weight block is one
// 1024-byte atom per 128-byte piece of the 8 rows, 16-byte unit u of row r at
// unit position u ^ r (TMA 128-byte swizzle). Lane (r = lane/4, c = lane%4)
// takes packed word 4*u + c of row r of P and of Q -> MMA rows r and r + 8.
//
// KIND 0: one activation column matters for every lane (gate|up, qmv M = 1):
//         elements 0 (row r) and 2 (row r + 8) against column sums xs0.
//         With XR = 2 the warp's (at most two) pieces take their activation
//         chunks from registers (xr), loaded once per kernel.
// KIND 1: two columns per lane (qmv M >= 2): elements 0..3, xs0 / xs1.
// KIND 2: down pass of slot pair `pair`: lanes c == pair own element 0
//         (P slot, column 2c) and element 3 (Q slot, column 2c + 1).
template <int WPT, int KIND, int XR>
__device__ __forceinline__ void consume_pass(const uint8_t* __restrict__ st, const Geo& g, int pc_lo, int pc_hi,
                                             int g_lo, int g_hi, int gabs0, const uint8_t* __restrict__ xcol,
                                             const float* __restrict__ xs0, const float* __restrict__ xs1,
                                             const float* __restrict__ xo0, const float* __restrict__ xo1,
                                             bool on, const uint4 (&xr)[2][8], float (&acc)[4]) {
  constexpr int GPC = 8 / WPT;  // groups per 128-byte piece
  const int lane = threadIdx.x & 31;
  PassCtx x;
  x.st = st;
  x.blkw = g.blkw;
  x.blkm = g.blkm;
  x.mswz = g.mswz;
  x.mrow = g.mrow;
  x.r = lane >> 2;
  x.c = lane & 3;
  x.mP = st + 2 * x.blkw;
  x.mQ = x.mP + 2 * x.blkm;
  const uint8_t* wbase = st + x.r * 128 + x.c * 4;
  const uint8_t* xbase = xcol + x.c * 16;
  if (KIND == 0 && XR > 0) {
    if (pc_lo < pc_hi) piece_kind0<WPT, true>(x, wbase + pc_lo * 1024, nullptr, xr[0], pc_lo, gabs0, xs0, xo0, acc);
    if (pc_lo + 1 < pc_hi)
      piece_kind0<WPT, true>(x, wbase + (pc_lo + 1) * 1024, nullptr, xr[1], pc_lo + 1, gabs0, xs0, xo0, acc);
    return;
  }
  for (int pc = pc_lo; pc < pc_hi; ++pc) {
    const uint8_t* pw = wbase + pc * 1024;
    const uint8_t* px = xbase + pc * 512;
    if (KIND == 0) {
      piece_kind0<WPT, false>(x, pw, px, xr[0], pc, gabs0, xs0, xo0, acc);
      continue;
    }
#pragma unroll
    for (int gi = 0; gi < GPC; ++gi) {
      const int gl = pc * GPC + gi;
      if (gl < g_lo || gl >= g_hi) continue;
      float D[4];
#pragma unroll
      for (int j = 0; j < WPT; ++j) {
        const int u = gi * WPT + j;
        word_step(pw + ((u ^ x.r) << 4), x.blkw, lds128(px + u * 64), j == 0, D);
      }
      const int mo = meta_off(x, gl);
      const float sP = bf2f(*reinterpret_cast<const uint16_t*>(x.mP + mo));
      const float bP = bf2f(*reinterpret_cast<const uint16_t*>(x.mP + x.blkm + mo));
      const float sQ = bf2f(*reinterpret_cast<const uint16_t*>(x.mQ + mo));
      const float bQ = bf2f(*reinterpret_cast<const uint16_t*>(x.mQ + x.blkm + mo));
      const float xa = xs0[gabs0 + gl], xb = xs1[gabs0 + gl];
      const float xoa = xo0[gabs0 + gl], xob = xo1[gabs0 + gl];
      if (KIND == 1) {
        acc[0] = fmaf(sP, D[0] - xoa, fmaf(bP, xa, acc[0]));
        acc[1] = fmaf(sP, D[1] - xob, fmaf(bP, xb, acc[1]));
        acc[2] = fmaf(sQ, D[2] - xoa, fmaf(bQ, xa, acc[2]));
        acc[3] = fmaf(sQ, D[3] - xob, fmaf(bQ, xb, acc[3]));
      } else {
        const float e0 = fmaf(sP, D[0] - xoa, bP * xa);
        const float e3 = fmaf(sQ, D[3] - xob, bQ * xb);
        acc[0] += on ? e0 : 0.0f;
        acc[3] += on ? e3 : 0.0f;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// routing (one warp): top-k, ties to the lower index, softmax over the k
// ---------------------------------------------------------------------------
__device__ void warp_route(const float* lr, int E, int k, bool coherent, uint32_t* sidx, float* sw) {
  const int lane = threadIdx.x & 31;
  float v[32];
  bool taken[32];
  const int EP = (E + 31) / 32;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int e = lane + 32 * j;
    const bool ok = j < EP && e < E;
    v[j] = ok ? (coherent ? __ldcg(lr + e) : __ldg(lr + e)) : -INFINITY;
    taken[j] = !ok;
  }
  float selv = -INFINITY;
  uint32_t seli = 0xffffffffu;
  for (int kk = 0; kk < k; ++kk) {
    float bv = -INFINITY;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (!taken[j] && v[j] > bv) {
        bv = v[j];
        bj = j;
      }
    float gmax = bv;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
    uint32_t cand = (bj >= 0 && bv == gmax) ? (uint32_t)(lane + 32 * bj) : 0xffffffffu;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, off));
    if (lane == kk) {
      selv = gmax;
      seli = cand;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j == bj && cand == (uint32_t)(lane + 32 * bj)) taken[j] = true;
  }
  // softmax_single_row over k values, N_READS = 4 per lane (slot order)
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
  if (lane < k) {
    sidx[lane] = seli;
    sw[lane] = ex * inv;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// KMODE: MODE_QMV (one token), MODE_GU, MODE_DOWN, MODE_FUSED, or KMODE_QMVM
// (qmv with 2..8 tokens); one instance per mode keeps each kernel's code small.
constexpr int KMODE_QMVM = 4;

template <int WPT, int KMODE>
__global__ void __launch_bounds__(NTHREADS, 1) engine_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // swizzled TMA destinations need 1024-byte alignment
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_misc);
  uint64_t* empty = full + NSTAGE_MAX;
  uint64_t* red_full = empty + NSTAGE_MAX;    // consumers -> finisher, per ring slot
  uint64_t* red_free = red_full + NRED;   // finisher -> consumers
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red_free + NRED);
  uint32_t* sidx = reinterpret_cast<uint32_t*>(smem + p.off_misc + (2 * NSTAGE_MAX + 2 * NRED) * 8 + 16);
  float* sw = reinterpret_cast<float*>(sidx + MAX_COLS);
  float* rsum = sw + MAX_COLS;  // [NC_WARPS] router partials
  float* red = reinterpret_cast<float*>(smem + p.off_red);  // [NRED][NC_WARPS][16][8] partials
  int* err = p.err;
  const Sched sch = make_sched(p);
  const uint64_t deadline = globaltimer() + (uint64_t)p.timeout_ns;

  if (tid == 0) {
    for (int i = 0; i < p.nstage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NC_WARPS);
    }
    for (int i = 0; i < NRED; ++i) {
      mbar_init(&red_full[i], NC_WARPS);
      mbar_init(&red_free[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const bool fused = p.mode == MODE_FUSED;

  if (warp == NC_WARPS) {
    // ------------------------------- producer -------------------------------
    if (fused) named_bar_sync(2, NTHREADS);  // wait for the routing
    // The whole warp runs the schedule (its values stay warp-uniform) and one
    // elected lane issues each group of copies.
    {
      if (tc::elect_one())
        for (int i = 0; i < N_MAPS; ++i)
          asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.map[i])) : "memory");
      const uint64_t pol = policy_evict_first();
      // L2 prefetch cursor, PF_AHEAD passes ahead of the shared-memory loads:
      // it keeps more bytes in flight than the stage ring alone can hold.
      const int PF_AHEAD = p.nstage + 2;
      int pf_u = blockIdx.x, pf_pass = 0, pf_np = (pf_u < sch.U) ? unit_passes(p, sch, pf_u) : 0;
      auto prefetch_next = [&]() {
        if (pf_u >= sch.U) return;
        const Geo& pg = unit_is_down(p, sch, pf_u) ? p.g2 : p.g1;
        const LoadDesc d = describe(p, sch, pf_u, pf_pass, sidx, nullptr);
        if (d.valid && tc::elect_one()) {
          const int cw = d.kc * (pg.KC / 256);
          tma_prefetch_3d(&p.map[d.mwP], 0, d.rowP, cw);
          tma_prefetch_3d(&p.map[d.mwQ], 0, d.rowQ, cw);
          if (pg.mswz) {
            const int cm = d.kc * (pg.GC / 64);
            tma_prefetch_3d(&p.map[d.msP], 0, d.rowP, cm);
            tma_prefetch_3d(&p.map[d.mbP], 0, d.rowP, cm);
            tma_prefetch_3d(&p.map[d.msQ], 0, d.rowQ, cm);
            tma_prefetch_3d(&p.map[d.mbQ], 0, d.rowQ, cm);
          } else {
            const int cm = d.kc * pg.GC;
            tma_prefetch_2d(&p.map[d.msP], cm, d.rowP);
            tma_prefetch_2d(&p.map[d.mbP], cm, d.rowP);
            tma_prefetch_2d(&p.map[d.msQ], cm, d.rowQ);
            tma_prefetch_2d(&p.map[d.mbQ], cm, d.rowQ);
          }
        }
        if (++pf_pass >= pf_np) {
          pf_pass = 0;
          pf_u += gridDim.x;
          pf_np = (pf_u < sch.U) ? unit_passes(p, sch, pf_u) : 0;
        }
      };
      for (int i = 0; i < PF_AHEAD; ++i) prefetch_next();
      int L = 0;
      bool ok = !*abort_flag;
      for (int u = blockIdx.x; ok && u < sch.U; u += gridDim.x) {
        const int np = unit_passes(p, sch, u);
        const Geo& g = unit_is_down(p, sch, u) ? p.g2 : p.g1;
        for (int pass = 0; pass < np; ++pass, ++L) {
          const int NS = p.nstage;
          const int si = L % NS;
          if (L >= NS && !__all_sync(0xffffffffu, bar_wait(&empty[si], ((L / NS) - 1) & 1, deadline, abort_flag))) {
            if (!*abort_flag) record_error(err, B2Q_ETIMEOUT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const LoadDesc d = describe(p, sch, u, pass, sidx, err);
          prefetch_next();
          uint8_t* st = stages + (size_t)si * p.stage_bytes;
          if (!d.valid) {
            if (tc::elect_one()) mbar_arrive_expect_tx(&full[si], 0u);
            __syncwarp();
            continue;
          }
          if (tc::elect_one()) {
          // a box always delivers its full size (out-of-range parts of a last,
          // shorter chunk are zero-filled), so the byte count is per box
          const uint32_t mbox = g.mswz ? (uint32_t)(g.GC / 64) * 1024u : 8u * (uint32_t)g.GC * 2u;
          mbar_arrive_expect_tx(&full[si], 2u * (uint32_t)g.blkw + 4u * mbox);
          const int cw = d.kc * (g.KC / 256);  // 128-byte piece index of the chunk start
          tma_load_3d(st, &p.map[d.mwP], 0, d.rowP, cw, &full[si], pol);
          tma_load_3d(st + g.blkw, &p.map[d.mwQ], 0, d.rowQ, cw, &full[si], pol);
          uint8_t* mb = st + 2 * g.blkw;
          if (g.mswz) {
            const int cm = d.kc * (g.GC / 64);
            tma_load_3d(mb, &p.map[d.msP], 0, d.rowP, cm, &full[si], pol);
            tma_load_3d(mb + g.blkm, &p.map[d.mbP], 0, d.rowP, cm, &full[si], pol);
            tma_load_3d(mb + 2 * g.blkm, &p.map[d.msQ], 0, d.rowQ, cm, &full[si], pol);
            tma_load_3d(mb + 3 * g.blkm, &p.map[d.mbQ], 0, d.rowQ, cm, &full[si], pol);
          } else {
            const int cm = d.kc * g.GC;  // element index along the meta row
            tma_load_2d(mb, &p.map[d.msP], cm, d.rowP, &full[si], pol);
            tma_load_2d(mb + g.blkm, &p.map[d.mbP], cm, d.rowP, &full[si], pol);
            tma_load_2d(mb + 2 * g.blkm, &p.map[d.msQ], cm, d.rowQ, &full[si], pol);
            tma_load_2d(mb + 3 * g.blkm, &p.map[d.mbQ], cm, d.rowQ, &full[si], pol);
          }
          }
          __syncwarp();
        }
      }
      // Drain: no copy may still be landing when the CTA exits.
      const uint64_t dl2 = globaltimer() + 200000000ull;
      for (int l = max(0, L - p.nstage); l < L; ++l) {
        if (!bar_wait(&full[l % p.nstage], (l / p.nstage) & 1, dl2, nullptr) && lane == 0) record_error(err, B2Q_ETIMEOUT);
      }
    }
    __syncwarp();
  } else if (warp == NC_WARPS + 1) {
    // ------------------------------- finisher -------------------------------
    // Per unit: wait for the NC_WARPS partials, sum them in warp order (a fixed
    // association), write the unit's outputs, release the ring slot.
    if (fused) named_bar_sync(2, NTHREADS);
    int ui = 0;
    for (int u = blockIdx.x; u < sch.U; u += gridDim.x, ++ui) {
      const int rs = ui % NRED;
      if (!bar_wait(&red_full[rs], (ui / NRED) & 1, deadline, abort_flag)) {
        if (!*abort_flag) record_error(err, B2Q_ETIMEOUT);
        *abort_flag = 1;
      }
      const float* rr = red + (size_t)rs * NC_WARPS * 128;
      auto wsum = [&](int i, int n) -> float {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < NC_WARPS; ++w) v += rr[w * 128 + i * 8 + n];
        return v;
      };
      const bool down = unit_is_down(p, sch, u);
      if constexpr (KMODE == MODE_QMV || KMODE == KMODE_QMVM) {
        const int item = u / sch.RB, rb = u % sch.RB;
        const uint32_t xi = p.lhs ? __ldg(p.lhs + item) : (uint32_t)item;
        const uint32_t e = p.rhs ? __ldg(p.rhs + item) : (uint32_t)item;
        const bool item_ok = xi < (uint32_t)p.n_x && e < (uint32_t)p.n_w && !*abort_flag;
        for (int o = lane; o < 16 * p.M; o += 32) {
          const int i = o & 15, n = o >> 4;
          const int row = rb * 16 + i;
          if (row < p.N) p.y[((size_t)item * p.M + n) * p.N + row] = item_ok ? f2bf(wsum(i, n)) : (uint16_t)0;
        }
      } else if (!down) {
        const int zslot = u / sch.FB, rb = u % sch.FB;
        if (lane < 8) {
          uint16_t* dst = (KMODE == MODE_FUSED) ? p.ws_act : p.act_out;
          dst[(size_t)zslot * p.F + rb * 8 + lane] = swiglu_bf16(f2bf(wsum(lane, 0)), f2bf(wsum(lane + 8, 0)));
          if (KMODE == MODE_FUSED) __threadfence();
        }
        if (KMODE == MODE_FUSED) {
          __syncwarp();
          if (lane == 0) {
            __threadfence();
            atomicAdd(&p.counters[1], 1u);
          }
        }
      } else {
        // 8 rows x k slots: lane (row = lane / 4, q = lane % 4) owns slots 2q (P
        // rows) and 2q + 1 (Q rows); the products meet in lane 4 * row, which
        // folds them in slot order (mlx_colsum_small_f32<K>).
        const int ud = (KMODE == MODE_FUSED) ? u - sch.U_gu : u;
        const int tok = ud / sch.HB, hb = ud % sch.HB;
        const int row = lane >> 2, q = lane & 3;
        const int j0 = 2 * q, j1 = 2 * q + 1;
        float pr0 = 0.0f, pr1 = 0.0f;
        if (j0 < p.k) {
          const float wj = (KMODE == MODE_FUSED) ? sw[j0] : __ldg(p.w_in + (size_t)tok * p.k + j0);
          pr0 = b2q::rb(wsum(row, j0)) * wj;  // f32(bf16(y_j)) * w_j
        }
        if (j1 < p.k) {
          const float wj = (KMODE == MODE_FUSED) ? sw[j1] : __ldg(p.w_in + (size_t)tok * p.k + j1);
          pr1 = b2q::rb(wsum(row + 8, j1)) * wj;
        }
        float prod[MAX_COLS];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          prod[2 * qq] = __shfl_sync(0xffffffffu, pr0, (lane & ~3) | qq);
          prod[2 * qq + 1] = __shfl_sync(0xffffffffu, pr1, (lane & ~3) | qq);
        }
        if (q == 0) {
          const int TY = p.k < 8 ? p.k : 8;
          float t[MAX_COLS];
#pragma unroll
          for (int y = 0; y < MAX_COLS; ++y) t[y] = 0.0f;
          for (int y = 0; y < TY; ++y) {
            float a = 0.0f;
            for (int qq = y; qq < p.k; qq += TY) a = prod[qq] + a;
            t[y] = a;
          }
          float total = t[0];
          for (int j = 1; j < TY; ++j) total = t[j] + total;
          p.out[(size_t)tok * p.H + hb * 8 + row] = f2bf(total);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_free[rs]);
    }
  } else {
    // ------------------------------- consumers ------------------------------
    uint8_t* xbuf = smem + p.off_x;
    float* xsum = reinterpret_cast<float*>(smem + p.off_xs);
    uint8_t* abuf = smem + p.off_act;
    float* asum = reinterpret_cast<float*>(smem + p.off_acts);
    const int r = lane >> 2, c = lane & 3;
    int cur_item = -1;  // QMV gather: item whose activations are staged
    // Register-resident activation chunks (single-column units): every pass
    // of the gate|up / qmv family has one chunk, so a warp always takes pieces
    // [xr_lo, xr_hi) and can keep their activations for the whole kernel.
    uint4 xr[2][8];
    const int np1 = p.g1.KC / 256;
    const int xr_lo = (warp * np1) / NC_WARPS, xr_hi = ((warp + 1) * np1) / NC_WARPS;
    const bool xreg = (KMODE == MODE_FUSED || KMODE == MODE_QMV || (KMODE == MODE_GU && p.S == 1)) &&
                      p.mode != MODE_DOWN && p.g1.nkc == 1 && (xr_hi - xr_lo) <= 2;
    auto load_xr = [&](const uint8_t* col) {
#pragma unroll
      for (int pl = 0; pl < 2; ++pl)
#pragma unroll
        for (int u = 0; u < 8; ++u)
          xr[pl][u] = (xr_lo + pl < xr_hi) ? lds128(col + c * 16 + (xr_lo + pl) * 512 + u * 64)
                                           : make_uint4(0u, 0u, 0u, 0u);
    };
    int cur_tok = -1;   // DOWN: token whose slot activations are staged
    bool act_ready = false;

    if (fused) {
      // --- router logits for this CTA's rows, then a grid-wide count ---
      const int nvec = p.H / 8;
      int rows_done = 0;
      for (int e = blockIdx.x; e < p.E; e += gridDim.x) {
        float part = 0.0f;
        for (int v = tid; v < nvec; v += NCT) {
          const uint4 xv = __ldg(reinterpret_cast<const uint4*>(p.x) + v);
          const uint4 wv = __ldg(reinterpret_cast<const uint4*>(p.wr + (size_t)e * p.H) + v);
          part += lo_bf(xv.x) * lo_bf(wv.x) + hi_bf(xv.x) * hi_bf(wv.x);
          part += lo_bf(xv.y) * lo_bf(wv.y) + hi_bf(xv.y) * hi_bf(wv.y);
          part += lo_bf(xv.z) * lo_bf(wv.z) + hi_bf(xv.z) * hi_bf(wv.z);
          part += lo_bf(xv.w) * lo_bf(wv.w) + hi_bf(xv.w) * hi_bf(wv.w);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        if (lane == 0) rsum[warp] = part;
        named_bar_sync(1, NCT);
        if (tid == 0) {
          float lg = 0.0f;
          for (int w = 0; w < NC_WARPS; ++w) lg += rsum[w];
          p.ws_logits[e] = lg;
        }
        named_bar_sync(1, NCT);
        ++rows_done;
      }
      if (tid == 0 && rows_done) {
        __threadfence();
        atomicAdd(&p.counters[0], (unsigned)rows_done);
      }
      if (tid == 0) {
        if (!wait_counter_geq(&p.counters[0], (unsigned)p.E, deadline, abort_flag)) {
          record_error(err, B2Q_ETIMEOUT);
          *abort_flag = 1;
        }
        __threadfence();
      }
      named_bar_sync(1, NCT);
      if (warp == 0) {
        if (!*abort_flag) {
          warp_route(p.ws_logits, p.E, p.k, true, sidx, sw);
        } else if (lane < p.k) {
          sidx[lane] = 0;
          sw[lane] = 0.0f;
        }
        __syncwarp();
        if (blockIdx.x == 0 && lane < p.k) {
          if (p.idx_out) p.idx_out[lane] = sidx[lane];
          if (p.w_out) p.w_out[lane] = sw[lane];
        }
        if (blockIdx.x == 0 && p.logits_out)
          for (int e = lane; e < p.E; e += 32) p.logits_out[e] = __ldcg(p.ws_logits + e);
      }
      named_bar_sync(2, NTHREADS);  // releases the producer
      // stage x (token 0) while the first expert tiles are in flight
      {
        const uint16_t* rows[1] = {p.x};
        stage_columns(xbuf, xsum, p.xcols, p.g1.XS, rows, 1, p.H, p.gs, false);
      }
      if (xreg) load_xr(xbuf);
    } else if (p.mode == MODE_GU) {
      const uint16_t* rows[MAX_COLS];
      for (int t = 0; t < p.S; ++t) rows[t] = p.x + (size_t)t * p.H;
      stage_columns(xbuf, xsum, p.xcols, p.g1.XS, rows, p.S, p.H, p.gs, false);
      if (xreg) load_xr(xbuf);
    }

    int L = 0;
    for (int u = blockIdx.x; u < sch.U; u += gridDim.x) {
      const bool down = unit_is_down(p, sch, u);
      const Geo& g = down ? p.g2 : p.g1;
      // ---- per-unit activation setup ----
      const uint8_t* xcol;
      const float* xs0;
      const float* xs1;
      const float* xo0;
      const float* xo1;
      float inv0, inv1;  // 1 / S of the columns of acc[0|2] and acc[1|3]
      int item = 0, zslot = 0, tok = 0, rb = 0, hb = 0;
      bool item_ok = true;
      if (p.mode == MODE_QMV) {
        item = u / sch.RB;
        rb = u % sch.RB;
        const uint32_t xi = p.lhs ? __ldg(p.lhs + item) : (uint32_t)item;
        const uint32_t e = p.rhs ? __ldg(p.rhs + item) : (uint32_t)item;
        item_ok = xi < (uint32_t)p.n_x && e < (uint32_t)p.n_w;
        const int xkey = item_ok ? (int)xi : -2;
        if (xkey != cur_item) {
          if (item_ok) {
            const uint16_t* rows[MAX_COLS];
            for (int m = 0; m < p.M; ++m) rows[m] = p.x + ((size_t)xi * p.M + m) * g.K;
            stage_columns(xbuf, xsum, p.xcols, g.XS, rows, p.M, g.K, p.gs, false);
            if (xreg) load_xr(xbuf);
          }
          cur_item = xkey;
        }
        xcol = xbuf + (size_t)((r < p.M) ? r : 0) * g.XS;
        const int c0 = min(2 * c, p.M - 1), c1 = min(2 * c + 1, p.M - 1);
        xs0 = cols_xs(xsum, g.G, c0);
        xs1 = cols_xs(xsum, g.G, c1);
        xo0 = cols_xo(xsum, p.xcols, g.G, c0);
        xo1 = cols_xo(xsum, p.xcols, g.G, c1);
        inv0 = cols_inv(xsum, p.xcols, g.G)[c0];
        inv1 = cols_inv(xsum, p.xcols, g.G)[c1];
      } else if (!down) {
        zslot = u / sch.FB;
        rb = u % sch.FB;
        // slot -> token: the xrow table, else z / k when the slots are token-major
        tok = (p.mode == MODE_FUSED) ? 0
                                     : (p.xrow_in ? (int)__ldg(p.xrow_in + zslot) : (p.k > 0 ? zslot / p.k : 0));
        if (tok < 0 || tok >= p.S) {
          record_error(err, B2Q_EINVAL);
          tok = 0;
        }
        xcol = xbuf + (size_t)tok * g.XS;
        xs0 = xs1 = cols_xs(xsum, g.G, tok);
        xo0 = xo1 = cols_xo(xsum, p.xcols, g.G, tok);
        inv0 = inv1 = cols_inv(xsum, p.xcols, g.G)[tok];
      } else {
        const int ud = (p.mode == MODE_FUSED) ? u - sch.U_gu : u;
        tok = ud / sch.HB;
        hb = ud % sch.HB;
        if (p.mode == MODE_FUSED) {
          if (!act_ready) {
            // all gate|up units of the grid must have published their activations
            if (tid == 0) {
              if (!wait_counter_geq(&p.counters[1], (unsigned)sch.U_gu, deadline, abort_flag)) {
                record_error(err, B2Q_ETIMEOUT);
                *abort_flag = 1;
              }
              __threadfence();
            }
            named_bar_sync(1, NCT);
            const uint16_t* rows[MAX_COLS];
            for (int j = 0; j < p.k; ++j) rows[j] = p.ws_act + (size_t)j * p.F;
            stage_columns(abuf, asum, p.k, g.XS, rows, p.k, p.F, p.gs, true);
            act_ready = true;
          }
        } else if (tok != cur_tok) {
          const uint16_t* rows[MAX_COLS];
          for (int j = 0; j < p.k; ++j) rows[j] = p.act_in + ((size_t)tok * p.k + j) * p.F;
          stage_columns(abuf, asum, p.k, g.XS, rows, p.k, p.F, p.gs, false);
          cur_tok = tok;
        }
        xcol = abuf + (size_t)((r < p.k) ? r : 0) * g.XS;
        const int c0 = min(2 * c, p.k - 1), c1 = min(2 * c + 1, p.k - 1);
        xs0 = cols_xs(asum, g.G, c0);
        xs1 = cols_xs(asum, g.G, c1);
        xo0 = cols_xo(asum, p.k, g.G, c0);
        xo1 = cols_xo(asum, p.k, g.G, c1);
        inv0 = cols_inv(asum, p.k, g.G)[c0];
        inv1 = cols_inv(asum, p.k, g.G)[c1];
      }

      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int np = unit_passes(p, sch, u);
      for (int pass = 0; pass < np; ++pass, ++L) {
        const int si = L % p.nstage;
        const bool ok = bar_wait(&full[si], (L / p.nstage) & 1, deadline, abort_flag);
        if (!ok && !*abort_flag) {
          record_error(err, B2Q_ETIMEOUT);
          *abort_flag = 1;
        }
        if (ok && !*abort_flag) {
          const int kc = down ? pass % g.nkc : pass;
          const int pair = down ? pass / g.nkc : 0;
          const int kcw = min(g.KC, g.K - kc * g.KC);
          const int npieces = kcw / 256;  // 128-byte pieces of each row in this chunk
          // single-column passes split by whole pieces; the others by groups
          // (pieces [plo, phi) cover groups [glo, ghi), partial at the ends)
          int plo, phi, glo = 0, ghi = 1 << 30;
          if (down || KMODE == KMODE_QMVM) {
            const int ng = kcw / p.gs, gpc = 8 / WPT;
            glo = (warp * ng) / NC_WARPS;
            ghi = ((warp + 1) * ng) / NC_WARPS;
            plo = glo / gpc;
            phi = (ghi + gpc - 1) / gpc;
          } else {
            plo = (warp * npieces) / NC_WARPS;
            phi = ((warp + 1) * npieces) / NC_WARPS;
          }
          const uint8_t* st = stages + (size_t)si * p.stage_bytes;
          const uint8_t* xc = xcol + (size_t)kc * (g.KC / 8) * 16;
          const int gabs0 = kc * g.GC;  // blocks keep the full-pass box layout, also for a shorter last chunk
          if constexpr (KMODE == MODE_DOWN) {
            consume_pass<WPT, 2, 0>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, c == pair, xr, acc);
          } else if constexpr (KMODE == MODE_FUSED) {
            if (down)
              consume_pass<WPT, 2, 0>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, c == pair, xr, acc);
            else
              {
              if (xreg)
                consume_pass<WPT, 0, 2>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, true, xr, acc);
              else
                consume_pass<WPT, 0, 0>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, true, xr, acc);
            }
          } else if constexpr (KMODE == KMODE_QMVM) {
            consume_pass<WPT, 1, 0>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, true, xr, acc);
          } else {
            {
              if (xreg)
                consume_pass<WPT, 0, 2>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, true, xr, acc);
              else
                consume_pass<WPT, 0, 0>(st, g, plo, phi, glo, ghi, gabs0, xc, xs0, xs1, xo0, xo1, true, xr, acc);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[si]);
      }
      // ---- unit epilogue: fixed-order reduction over the warps ----
      // undo the activation scaling (a power of two: exact)
      acc[0] *= inv0;
      acc[1] *= inv1;
      acc[2] *= inv0;
      acc[3] *= inv1;
      // single-column units: the four lanes of a quad hold different groups
      const bool quad_groups = (KMODE == MODE_QMV || KMODE == MODE_GU || (KMODE == MODE_FUSED && !down));
      if (quad_groups) {
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 1);
        acc[2] += __shfl_xor_sync(0xffffffffu, acc[2], 1);
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 2);
        acc[2] += __shfl_xor_sync(0xffffffffu, acc[2], 2);
      }
      // hand the partials to the finisher warp through the ring
      const int ui = (u - (int)blockIdx.x) / (int)gridDim.x;  // this CTA's unit ordinal
      const int rs = ui % NRED;
      if (ui >= NRED && !bar_wait(&red_free[rs], ((ui / NRED) - 1) & 1, deadline, abort_flag)) {
        if (!*abort_flag) record_error(err, B2Q_ETIMEOUT);
        *abort_flag = 1;
      }
      float* rw = red + ((size_t)rs * NC_WARPS + warp) * 128;
      rw[r * 8 + 2 * c] = acc[0];
      rw[r * 8 + 2 * c + 1] = acc[1];
      rw[(r + 8) * 8 + 2 * c] = acc[2];
      rw[(r + 8) * 8 + 2 * c + 1] = acc[3];
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[rs]);
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
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// standalone router kernels
// ---------------------------------------------------------------------------
// logits[t, e] = f32(x[t]) . f32(wr[e]); one warp per (t, e), 8 bf16 per load.
__global__ void router_logits_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
                                     float* __restrict__ logits, int T, int E, int H) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= T * E) return;
  const int t = gw / E, e = gw % E;
  const uint4* xv = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  const uint4* wv = reinterpret_cast<const uint4*>(wr + (size_t)e * H);
  float part = 0.0f;
  for (int v = lane; v < H / 8; v += 32) {
    const uint4 a = __ldg(xv + v), b = __ldg(wv + v);
    part += lo_bf(a.x) * lo_bf(b.x) + hi_bf(a.x) * hi_bf(b.x);
    part += lo_bf(a.y) * lo_bf(b.y) + hi_bf(a.y) * hi_bf(b.y);
    part += lo_bf(a.z) * lo_bf(b.z) + hi_bf(a.z) * hi_bf(b.z);
    part += lo_bf(a.w) * lo_bf(b.w) + hi_bf(a.w) * hi_bf(b.w);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  if (lane == 0) logits[(size_t)t * E + e] = part;
}

// One warp per token row.
__global__ void route_kernel(const float* __restrict__ logits, uint32_t* __restrict__ idx,
                             float* __restrict__ w, int T, int E, int k) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  warp_route(logits + (size_t)t * E, E, k, false, idx + (size_t)t * k, w + (size_t)t * k);
}

// Tiled router GEMM for token windows: CTA tile 32 tokens x 128 experts, K in
// steps of 64 through double-buffered shared memory (cp.async), 8 warps each
// 16 tokens x 32 experts with mma.sync m16n8k16 (bf16 products are exact in
// fp32; fp32 accumulation).
// 16 tokens x 128 experts per CTA (2048 tokens: 128 CTAs); padded rows: 144 bytes
constexpr int RT_BM = 16, RT_BN = 128, RT_BK = 64, RT_LD = RT_BK + 8;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__global__ void __launch_bounds__(256) router_gemm_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ wr,
                                                          float* __restrict__ logits, int T, int E, int H) {
  __shared__ __align__(16) uint16_t xs[2][RT_BM * RT_LD];
  __shared__ __align__(16) uint16_t ws[2][RT_BN * RT_LD];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * RT_BM, e0 = blockIdx.y * RT_BN;
  const int wn = warp * 16;  // 8 warps x 16 experts
  auto load = [&](int buf, int k0) {
    // x: 32 rows x 8 chunks of 16 bytes; wr: 128 rows x 8 chunks
    for (int i = tid; i < RT_BM * 8; i += 256) {
      const int r = i >> 3, c = i & 7;
      const bool ok = t0 + r < T;
      cp_async16(&xs[buf][r * RT_LD + c * 8], x + (size_t)(ok ? t0 + r : 0) * H + k0 + c * 8, ok);
    }
    for (int i = tid; i < RT_BN * 8; i += 256) {
      const int r = i >> 3, c = i & 7;
      const bool ok = e0 + r < E;
      cp_async16(&ws[buf][r * RT_LD + c * 8], wr + (size_t)(ok ? e0 + r : 0) * H + k0 + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[2][4] = {};
  const int nk = H / RT_BK;
  load(0, 0);
  for (int kt = 0; kt < nk; ++kt) {
    if (kt + 1 < nk) {
      load((kt + 1) & 1, (kt + 1) * RT_BK);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint16_t* xb = xs[kt & 1];
    const uint16_t* wb = ws[kt & 1];
#pragma unroll
    for (int kk = 0; kk < RT_BK; kk += 16) {
      uint32_t a[4];
      ldmatrix_x4(a, xb + (lane & 15) * RT_LD + kk + (lane >> 4) * 8);
      uint32_t b[4];
      const int m = lane >> 3, r = lane & 7;
      ldmatrix_x4(b, wb + (wn + (m >> 1) * 8 + r) * RT_LD + kk + (m & 1) * 8);
      mma_bf16_16816(acc[0], a[0], a[1], a[2], a[3], b[0], b[1]);
      mma_bf16_16816(acc[1], a[0], a[1], a[2], a[3], b[2], b[3]);
    }
    __syncthreads();
  }
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int e = e0 + wn + nt * 8 + 2 * q;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = t0 + g + h * 8;
      if (t < T) {
        if (e < E) logits[(size_t)t * E + e] = acc[nt][2 * h];
        if (e + 1 < E) logits[(size_t)t * E + e + 1] = acc[nt][2 * h + 1];
      }
    }
  }
}

// Split-K router GEMM for long token windows (prefill): a CTA computes 64
// tokens x 128 experts over one of S slices of the hidden size through a
// 4-stage cp.async ring; 8 warps each 64 tokens x 16 experts (mma.sync
// m16n8k16, bf16 products exact in fp32, fp32 accumulation). Every CTA writes
// its fp32 partial tile; router_reduce_kernel adds the S partials in slice
// order. Fewer re-reads of the router matrix per token than the 16-token
// tiles, and a deeper pipeline.
constexpr int RS_BM = 64, RS_BN = 128, RS_BK = 64, RS_LD = RS_BK + 8, RS_ST = 4;
constexpr int RS_SMEM = RS_ST * (RS_BM + RS_BN) * RS_LD * 2;

__global__ void __launch_bounds__(256) router_gemm_sk_kernel(const uint16_t* __restrict__ x,
                                                             const uint16_t* __restrict__ wr,
                                                             float* __restrict__ partial, int T, int E, int H,
                                                             int S) {
  extern __shared__ __align__(16) uint16_t rsm[];
  uint16_t* xs = rsm;                           // [RS_ST][RS_BM * RS_LD]
  uint16_t* wsm = rsm + RS_ST * RS_BM * RS_LD;  // [RS_ST][RS_BN * RS_LD]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * RS_BM, e0 = blockIdx.y * RS_BN, sl = blockIdx.z;
  const int kslice = H / S, kbase = sl * kslice, nk = kslice / RS_BK;
  const int wn = warp * 16;
  auto load = [&](int buf, int kt) {
    const int k0 = kbase + kt * RS_BK;
    for (int i = tid; i < RS_BM * 8; i += 256) {
      const int r = i >> 3, c = i & 7;
      const bool ok = t0 + r < T;
      cp_async16(&xs[buf * RS_BM * RS_LD + r * RS_LD + c * 8], x + (size_t)(ok ? t0 + r : 0) * H + k0 + c * 8, ok);
    }
    for (int i = tid; i < RS_BN * 8; i += 256) {
      const int r = i >> 3, c = i & 7;
      const bool ok = e0 + r < E;
      cp_async16(&wsm[buf * RS_BN * RS_LD + r * RS_LD + c * 8], wr + (size_t)(ok ? e0 + r : 0) * H + k0 + c * 8,
                 ok);
    }
  };
  float acc[4][2][4] = {};
#pragma unroll
  for (int st = 0; st < RS_ST - 1; ++st) {
    if (st < nk) load(st, st);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int kt = 0; kt < nk; ++kt) {
    asm volatile("cp.async.wait_group %0;" ::"n"(RS_ST - 2) : "memory");
    __syncthreads();
    if (kt + RS_ST - 1 < nk) load((kt + RS_ST - 1) % RS_ST, kt + RS_ST - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint16_t* xb = xs + (kt % RS_ST) * RS_BM * RS_LD;
    const uint16_t* wb = wsm + (kt % RS_ST) * RS_BN * RS_LD;
#pragma unroll
    for (int kk = 0; kk < RS_BK; kk += 16) {
      uint32_t b[4];
      const int m = lane >> 3, r = lane & 7;
      ldmatrix_x4(b, wb + (wn + (m >> 1) * 8 + r) * RS_LD + kk + (m & 1) * 8);
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        uint32_t a[4];
        ldmatrix_x4(a, xb + (mi * 16 + (lane & 15)) * RS_LD + kk + (lane >> 4) * 8);
        mma_bf16_16816(acc[mi][0], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_bf16_16816(acc[mi][1], a[0], a[1], a[2], a[3], b[2], b[3]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  const int g = lane >> 2, q = lane & 3;
  float* part = partial + (size_t)sl * T * E;
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int e = e0 + wn + nt * 8 + 2 * q;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = t0 + mi * 16 + g + h * 8;
        if (t < T) {
          if (e < E) part[(size_t)t * E + e] = acc[mi][nt][2 * h];
          if (e + 1 < E) part[(size_t)t * E + e + 1] = acc[mi][nt][2 * h + 1];
        }
      }
    }
}

__global__ void router_reduce_kernel(const float* __restrict__ partial, float* __restrict__ logits, long long n,
                                     int S) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float a = partial[i];
  for (int s = 1; s < S; ++s) a += partial[(size_t)s * n + i];
  logits[i] = a;
}

int launch_router_logits_sk(const uint16_t* x, const uint16_t* wr, float* logits, float* scratch,
                            size_t scratch_bytes, int T, int E, int H, cudaStream_t s) {
  const int mt = (T + RS_BM - 1) / RS_BM, nt = (E + RS_BN - 1) / RS_BN;
  int S = 1;
  // slices until the grid fills the GPU about twice (two CTAs fit per SM)
  while (S < 8 && mt * nt * S * 2 <= 296 && H % (RS_BK * S * 2) == 0) S *= 2;
  if (T < RS_BM || H % (RS_BK * S) || !scratch || scratch_bytes < (size_t)S * T * E * sizeof(float))
    return launch_router_logits(x, wr, logits, T, E, H, s);
  static bool attr_done[64] = {};
  int dev = 0;
  B2Q_TRY_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    B2Q_TRY_CUDA(cudaFuncSetAttribute(router_gemm_sk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RS_SMEM));
    attr_done[dev & 63] = true;
  }
  router_gemm_sk_kernel<<<dim3(mt, nt, S), 256, RS_SMEM, s>>>(x, wr, S > 1 ? scratch : logits, T, E, H, S);
  B2Q_TRY_CUDA(cudaGetLastError());
  if (S > 1) {
    const long long n = (long long)T * E;
    router_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(scratch, logits, n, S);
    B2Q_TRY_CUDA(cudaGetLastError());
  }
  return B2Q_OK;
}

int launch_router_logits(const uint16_t* x, const uint16_t* wr, float* logits, int T, int E, int H,
                         cudaStream_t s) {
  if (T >= RT_BM && H % RT_BK == 0) {
    dim3 grid((T + RT_BM - 1) / RT_BM, (E + RT_BN - 1) / RT_BN);
    router_gemm_kernel<<<grid, 256, 0, s>>>(x, wr, logits, T, E, H);
    B2Q_TRY_CUDA(cudaGetLastError());
    return B2Q_OK;
  }
  const long long warps = (long long)T * E;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  if (blocks <= 0) return B2Q_OK;
  router_logits_kernel<<<(unsigned)blocks, threads, 0, s>>>(x, wr, logits, T, E, H);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int launch_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k, cudaStream_t s) {
  const int threads = 128;
  const long long blocks = ((long long)T * 32 + threads - 1) / threads;
  if (blocks <= 0) return B2Q_OK;
  route_kernel<<<(unsigned)blocks, threads, 0, s>>>(logits, idx, w, T, E, k);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

// ---------------------------------------------------------------------------
// host: geometry, shared-memory plan, tensor maps, launch
// ---------------------------------------------------------------------------
static int round_up(int v, int a) { return (v + a - 1) / a * a; }

// Reduction-chunk geometry for one product family (K elements per row);
// returns the stage bytes one full pass needs.
static int make_geo(Geo& g, int K, int gs) {
  g.K = K;
  g.G = K / gs;
  // chunk granularity: whole 128-byte row pieces and whole 16-byte meta units
  const int unit = std::max(256, 8 * gs);
  int kc = (K <= 4096) ? K : 4096;
  kc = std::max(unit, kc / unit * unit);
  g.KC = kc;
  g.nkc = (K + kc - 1) / kc;
  g.GC = kc / gs;
  g.blkw = 8 * (kc / 2);
  // meta rows take the swizzled 128-byte layout when every chunk is whole 128-byte pieces
  g.mswz = (g.GC % 64 == 0 && g.G % 64 == 0) ? 1 : 0;
  g.mrow = g.GC * 2;
  g.blkm = g.mswz ? (g.GC / 64) * 1024 : round_up(8 * g.GC * 2, 128);
  const int xb = (K / 8) * 16;
  g.XS = xb + ((64 - xb % 128) + 128) % 128;  // XS % 128 == 64: 8 columns hit distinct bank quads
  return 2 * g.blkw + 4 * g.blkm;
}

int plan(Params& p) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  int st1 = 0, st2 = 0;
  const bool uses_down = p.mode == MODE_DOWN || p.mode == MODE_FUSED;
  const bool uses_g1 = p.mode != MODE_DOWN;
  if (uses_g1) st1 = make_geo(p.g1, p.mode == MODE_QMV ? p.g1.K : p.H, p.gs);
  if (uses_down) st2 = make_geo(p.g2, p.F, p.gs);
  p.stage_bytes = round_up(std::max(st1, st2), 1024);
  if (p.stage_bytes > STAGE_MAX) return set_error(B2Q_EUNSUPPORTED, "engine: stage of %d bytes", p.stage_bytes);
  // shared memory besides the stage ring
  p.xcols = (p.mode == MODE_QMV) ? p.M : (p.mode == MODE_GU ? p.S : (p.mode == MODE_FUSED ? 1 : 0));
  int fixed = 0;
  fixed += round_up(p.xcols * (uses_g1 ? p.g1.XS : 0), 128);
  fixed += round_up((2 * p.xcols * (uses_g1 ? p.g1.G : 0) + 2 * MAX_COLS) * 4, 128);
  fixed += round_up(uses_down ? p.k * p.g2.XS : 0, 128);
  fixed += round_up(uses_down ? (2 * p.k * p.g2.G + 2 * MAX_COLS) * 4 : 0, 128);
  fixed += NRED * NC_WARPS * 128 * 4;
  fixed += round_up((2 * NSTAGE_MAX + 2 * NRED) * 8 + 16 + MAX_COLS * 8 + NC_WARPS * 4 + 64 * 4, 128);
  fixed += 1024;  // alignment slack of the 1024-byte base
  p.nstage = std::min(NSTAGE_MAX, (di.smem_optin - fixed) / p.stage_bytes);
  if (p.nstage < 2)
    return set_error(B2Q_EUNSUPPORTED, "engine: shared memory holds only %d stages of %d bytes", p.nstage,
                     p.stage_bytes);
  int off = p.nstage * p.stage_bytes;
  p.off_x = off;
  off += round_up(p.xcols * (uses_g1 ? p.g1.XS : 0), 128);
  p.off_xs = off;
  off += round_up((2 * p.xcols * (uses_g1 ? p.g1.G : 0) + 2 * MAX_COLS) * 4, 128);
  p.off_act = off;
  off += round_up(uses_down ? p.k * p.g2.XS : 0, 128);
  p.off_acts = off;
  off += round_up(uses_down ? (2 * p.k * p.g2.G + 2 * MAX_COLS) * 4 : 0, 128);
  p.off_red = off;
  off += NRED * NC_WARPS * 128 * 4;
  p.off_misc = off;
  off += (2 * NSTAGE_MAX + 2 * NRED) * 8 + 16 + MAX_COLS * 8 + NC_WARPS * 4 + 64 * 4;
  p.smem_bytes = round_up(off, 128) + 1024;  // + alignment slack of the 1024-byte base
  if (p.smem_bytes > di.smem_optin)
    return set_error(B2Q_EUNSUPPORTED, "engine: needs %d bytes of shared memory, device allows %d", p.smem_bytes,
                     di.smem_optin);
  if (p.timeout_ns <= 0) p.timeout_ns = 2000000000ll;
  return B2Q_OK;
}

// maps for a weight tensor [rows, K/8] and its scales / biases [rows, K/gs]
static int set_triplet(Params& p, int slot_w, int slot_s, int slot_b, const uint32_t* w, const uint16_t* s,
                       const uint16_t* b, uint64_t rows, const Geo& g) {
  int rc = make_row_block_map(&p.map[slot_w], w, rows, (uint64_t)g.K / 2, (uint32_t)g.KC / 2, true);
  if (rc) return rc;
  rc = make_row_block_map(&p.map[slot_s], s, rows, (uint64_t)g.G * 2, (uint32_t)g.GC * 2, g.mswz != 0);
  if (rc) return rc;
  return make_row_block_map(&p.map[slot_b], b, rows, (uint64_t)g.G * 2, (uint32_t)g.GC * 2, g.mswz != 0);
}

int set_maps_qmv(Params& p, const uint32_t* w, const uint16_t* s, const uint16_t* b) {
  return set_triplet(p, M_W, M_S, M_B, w, s, b, (uint64_t)p.n_w * p.N, p.g1);
}
int set_maps_gu(Params& p, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg, const uint32_t* wu,
                const uint16_t* su, const uint16_t* bu) {
  int rc = set_triplet(p, M_WG, M_SG, M_BG, wg, sg, bg, (uint64_t)p.E * p.F, p.g1);
  if (rc) return rc;
  return set_triplet(p, M_WU, M_SU, M_BU, wu, su, bu, (uint64_t)p.E * p.F, p.g1);
}
int set_maps_down(Params& p, const uint32_t* wd, const uint16_t* sd, const uint16_t* bd) {
  return set_triplet(p, M_WD, M_SD, M_BD, wd, sd, bd, (uint64_t)p.E * p.H, p.g2);
}

template <int WPT, int KMODE>
static int launch_t(const Params& p, cudaStream_t stream, bool cooperative, int grid) {
  auto kern = engine_kernel<WPT, KMODE>;
  // The shared-memory opt-in is a per-device function attribute: raise it to
  // the device maximum once instead of on every launch.
  static int opted[64] = {0};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (!opted[di.device]) {
    B2Q_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, di.smem_optin));
    opted[di.device] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cooperative ? 1 : 0;
  B2Q_TRY_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
  return B2Q_OK;
}

int launch(const Params& p, void* stream, bool cooperative) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  int U = 0;
  switch (p.mode) {
    case MODE_QMV: U = p.batch * ((p.N + 15) / 16); break;
    case MODE_GU: U = p.n_slots * (p.F / 8); break;
    case MODE_DOWN: U = p.S * (p.H / 8); break;
    default: U = di.sm_count; break;
  }
  if (U <= 0) return B2Q_OK;
  const int grid = (p.mode == MODE_FUSED) ? di.sm_count : std::min(U, di.sm_count);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int km = (p.mode == MODE_QMV && p.M > 1) ? KMODE_QMVM : p.mode;
  switch (p.wpt * 8 + km) {
#define B2Q_ENGINE_CASE(W, KM) \
  case W * 8 + KM:             \
    return launch_t<W, KM>(p, s, cooperative, grid);
    B2Q_ENGINE_CASE(1, MODE_QMV) B2Q_ENGINE_CASE(1, MODE_GU) B2Q_ENGINE_CASE(1, MODE_DOWN)
    B2Q_ENGINE_CASE(1, MODE_FUSED) B2Q_ENGINE_CASE(1, KMODE_QMVM)
    B2Q_ENGINE_CASE(2, MODE_QMV) B2Q_ENGINE_CASE(2, MODE_GU) B2Q_ENGINE_CASE(2, MODE_DOWN)
    B2Q_ENGINE_CASE(2, MODE_FUSED) B2Q_ENGINE_CASE(2, KMODE_QMVM)
    B2Q_ENGINE_CASE(4, MODE_QMV) B2Q_ENGINE_CASE(4, MODE_GU) B2Q_ENGINE_CASE(4, MODE_DOWN)
    B2Q_ENGINE_CASE(4, MODE_FUSED) B2Q_ENGINE_CASE(4, KMODE_QMVM)
#undef B2Q_ENGINE_CASE
    default:
      return set_error(B2Q_EUNSUPPORTED, "engine: group size %d / mode %d", p.gs, p.mode);
  }
}

}  // namespace eng
}  // namespace b2q
