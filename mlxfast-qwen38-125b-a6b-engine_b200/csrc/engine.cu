// engine.cu -- the streaming (decode) product engine for sm_100a.
//
// Reference arithmetic it stands in for (paths relative to the reference
// project, QH = Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/metal/kernels/quantized.h):
//   qmv_fast_impl / qmv_impl       QH:757-987   (per-group s*sum(xq) + b*sum(x), fp32)
//   affine_gather_qmv_fast         QH:2444-2505 (per-item expert offset)
//   track_moe_gate_up_act          Runner/FastModel/TrackFastMoE.swift:1192-1410
//   track_moe_down_combine         Runner/FastModel/TrackFastMoE.swift:1412-1590
//   track_moe_route                Runner/FastModel/TrackFastMoE.swift:767-911
// The design is this file's own: bulk-copy producer, MMA consumers, static
// persistent schedule, fixed-order cross-warp reduction.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "engine.cuh"
#include "host.hpp"

namespace b2q {
namespace eng {

// ---------------------------------------------------------------------------
// unit / pass enumeration (shared by producer and consumers)
// ---------------------------------------------------------------------------
struct Sched {
  int U;       // total units
  int U_gu;    // FUSED: gate|up units before the down units
  int RB;      // QMV: row blocks per item
  int FB;      // gate|up row blocks per slot (F / 8)
  int HB;      // down row blocks per token (H / 8)
  int npair;   // down slot pairs (ceil(k / 2))
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

// Where one pass's rows come from.
struct LoadDesc {
  const uint8_t* wP;
  const uint8_t* wQ;
  const uint8_t* sP;
  const uint8_t* bP;
  const uint8_t* sQ;
  const uint8_t* bQ;
  int nP, nQ;
  int row_bytes, meta_bytes;  // per row in this pass
  int wstride, mstride;       // global row strides (bytes)
};

__device__ __forceinline__ uint32_t clamp_expert(uint32_t e, int E, int* err) {
  if (e >= (uint32_t)E) {
    record_error(err, B2Q_EINVAL);
    return 0;
  }
  return e;
}

// expert ids of the current CTA's routed slots (FUSED) live in shared memory
__device__ __forceinline__ LoadDesc describe(const Params& p, const Sched& s, int u, int pass,
                                             const uint32_t* sidx, int* err) {
  LoadDesc d{};
  if (!unit_is_down(p, s, u) && p.mode != MODE_QMV) {
    // gate|up: P = gate rows, Q = up rows of expert e
    const int z = u / s.FB, rb = u % s.FB;
    const uint32_t e = (p.mode == MODE_FUSED) ? sidx[z] : clamp_expert(__ldg(p.idx_in + z), p.E, err);
    const Geo& g = p.g1;
    const int c = pass;
    const size_t row0 = (size_t)e * p.F + (size_t)rb * 8;
    d.wstride = g.K / 2;
    d.mstride = g.G * 2;
    d.row_bytes = min(g.KC, g.K - c * g.KC) / 2;
    d.meta_bytes = d.row_bytes * 2 / p.gs * 2;
    const size_t wo = row0 * d.wstride + (size_t)c * g.KC / 2;
    const size_t mo = row0 * d.mstride + (size_t)c * (g.KC / p.gs) * 2;
    d.wP = reinterpret_cast<const uint8_t*>(p.wg) + wo;
    d.wQ = reinterpret_cast<const uint8_t*>(p.wu) + wo;
    d.sP = reinterpret_cast<const uint8_t*>(p.sg) + mo;
    d.bP = reinterpret_cast<const uint8_t*>(p.bg) + mo;
    d.sQ = reinterpret_cast<const uint8_t*>(p.su) + mo;
    d.bQ = reinterpret_cast<const uint8_t*>(p.bu) + mo;
    d.nP = d.nQ = 8;
    return d;
  }
  if (p.mode == MODE_QMV) {
    const int item = u / s.RB, rb = u % s.RB;
    const uint32_t e = p.rhs ? __ldg(p.rhs + item) : (uint32_t)item;
    const uint32_t xi = p.lhs ? __ldg(p.lhs + item) : (uint32_t)item;
    const Geo& g = p.g1;
    const int c = pass;
    d.wstride = g.K / 2;
    d.mstride = g.G * 2;
    d.row_bytes = min(g.KC, g.K - c * g.KC) / 2;
    d.meta_bytes = d.row_bytes * 2 / p.gs * 2;
    if (e >= (uint32_t)p.n_w || xi >= (uint32_t)p.n_x) {
      d.nP = d.nQ = 0;  // the finisher writes zeros for this item
      return d;
    }
    const int r0 = rb * 16;
    d.nP = max(0, min(8, p.N - r0));
    d.nQ = max(0, min(8, p.N - r0 - 8));
    const size_t base = (size_t)e * p.N + r0;
    const size_t wo = base * d.wstride + (size_t)c * g.KC / 2;
    const size_t mo = base * d.mstride + (size_t)c * (g.KC / p.gs) * 2;
    d.wP = reinterpret_cast<const uint8_t*>(p.w) + wo;
    d.wQ = d.wP + (size_t)8 * d.wstride;
    d.sP = reinterpret_cast<const uint8_t*>(p.s) + mo;
    d.bP = reinterpret_cast<const uint8_t*>(p.b) + mo;
    d.sQ = d.sP + (size_t)8 * d.mstride;
    d.bQ = d.bP + (size_t)8 * d.mstride;
    return d;
  }
  // down: unit = (token t, 8 output rows hb); pass = (slot pair, reduction chunk)
  const int ud = (p.mode == MODE_FUSED) ? u - s.U_gu : u;
  const int t = ud / s.HB, hb = ud % s.HB;
  const Geo& g = p.g2;
  const int pair = pass / g.nkc, c = pass % g.nkc;
  const int j0 = 2 * pair, j1 = 2 * pair + 1;
  uint32_t e0, e1;
  if (p.mode == MODE_FUSED) {
    e0 = sidx[j0];
    e1 = (j1 < p.k) ? sidx[j1] : e0;
  } else {
    e0 = clamp_expert(__ldg(p.idx_in + (size_t)t * p.k + j0), p.E, err);
    e1 = (j1 < p.k) ? clamp_expert(__ldg(p.idx_in + (size_t)t * p.k + j1), p.E, err) : e0;
  }
  d.wstride = g.K / 2;
  d.mstride = g.G * 2;
  d.row_bytes = min(g.KC, g.K - c * g.KC) / 2;
  d.meta_bytes = d.row_bytes * 2 / p.gs * 2;
  const size_t r0P = (size_t)e0 * p.H + (size_t)hb * 8;
  const size_t r0Q = (size_t)e1 * p.H + (size_t)hb * 8;
  const size_t cw = (size_t)c * g.KC / 2, cm = (size_t)c * (g.KC / p.gs) * 2;
  d.wP = reinterpret_cast<const uint8_t*>(p.wd) + r0P * d.wstride + cw;
  d.wQ = reinterpret_cast<const uint8_t*>(p.wd) + r0Q * d.wstride + cw;
  d.sP = reinterpret_cast<const uint8_t*>(p.sd) + r0P * d.mstride + cm;
  d.bP = reinterpret_cast<const uint8_t*>(p.bd) + r0P * d.mstride + cm;
  d.sQ = reinterpret_cast<const uint8_t*>(p.sd) + r0Q * d.mstride + cm;
  d.bQ = reinterpret_cast<const uint8_t*>(p.bd) + r0Q * d.mstride + cm;
  d.nP = 8;
  d.nQ = (j1 < p.k) ? 8 : 0;
  return d;
}

// ---------------------------------------------------------------------------
// activation staging: bf16 rows -> permuted chunks + fp32 group sums
// ---------------------------------------------------------------------------
// col c of `dst` (stride XS bytes) receives row src_rows[c]; sums[c * G + g].
__device__ void stage_columns(uint8_t* dst, float* sums, int XS, const uint16_t* const* src_rows, int ncols,
                              int K, int gs, bool coherent) {
  const int tid = threadIdx.x;
  const int nch = K / 8;
  for (int q = tid; q < ncols * nch; q += NCT) {
    const int col = q / nch, ch = q % nch;
    const uint4* src = reinterpret_cast<const uint4*>(src_rows[col] + (size_t)ch * 8);
    uint4 v = coherent ? __ldcg(src) : __ldg(src);
    *reinterpret_cast<uint4*>(dst + (size_t)col * XS + (size_t)ch * 16) = perm_x8(v);
  }
  named_bar_sync(1, NCT);
  const int G = K / gs;
  for (int q = tid; q < ncols * G; q += NCT) {
    const int col = q / G, g = q % G;
    const uint8_t* base = dst + (size_t)col * XS + (size_t)g * (gs / 8) * 16;
    float acc = 0.0f;
    for (int ch = 0; ch < gs / 8; ++ch) {
      const uint4 v = *reinterpret_cast<const uint4*>(base + ch * 16);
      // permuted (x0,x4)(x1,x5)(x2,x6)(x3,x7): sum in k order x0..x7
      const float x0 = __uint_as_float(v.x << 16), x4 = __uint_as_float(v.x & 0xffff0000u);
      const float x1 = __uint_as_float(v.y << 16), x5 = __uint_as_float(v.y & 0xffff0000u);
      const float x2 = __uint_as_float(v.z << 16), x6 = __uint_as_float(v.z & 0xffff0000u);
      const float x3 = __uint_as_float(v.w << 16), x7 = __uint_as_float(v.w & 0xffff0000u);
      acc += ((((((x0 + x1) + x2) + x3) + x4) + x5) + x6) + x7;
    }
    sums[(size_t)col * G + g] = acc;
  }
  named_bar_sync(1, NCT);
}

// ---------------------------------------------------------------------------
// one pass of MMAs over this warp's share of the groups
// ---------------------------------------------------------------------------
struct LaneCols {
  const uint8_t* xcol;  // this lane's B column (permuted chunks) at the pass start
  const float* xs0;     // group sums of column 2c (absolute group index)
  const float* xs1;     // group sums of column 2c+1
  bool a00, a01, a10, a11;
};

template <int WPT>
__device__ __forceinline__ void consume_pass(const uint8_t* __restrict__ st, const Geo& g, int gs, int g_lo,
                                             int g_hi, int gabs0, const LaneCols& lc, float (&acc)[4]) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const uint8_t* wrow0 = st + r * g.RS + c * 4;
  const uint8_t* wrow8 = st + (r + 8) * g.RS + c * 4;
  const uint8_t* meta = st + 16 * g.RS;
  const uint16_t* sPm = reinterpret_cast<const uint16_t*>(meta + (0 + r) * g.MS);
  const uint16_t* bPm = reinterpret_cast<const uint16_t*>(meta + (8 + r) * g.MS);
  const uint16_t* sQm = reinterpret_cast<const uint16_t*>(meta + (16 + r) * g.MS);
  const uint16_t* bQm = reinterpret_cast<const uint16_t*>(meta + (24 + r) * g.MS);
  const bool actP = lc.a00 || lc.a01, actQ = lc.a10 || lc.a11;
#pragma unroll 2
  for (int gi = g_lo; gi < g_hi; ++gi) {
    float dA[4] = {0.f, 0.f, 0.f, 0.f};
    float dB[4] = {0.f, 0.f, 0.f, 0.f};
    const int wbase = gi * (gs / 8);  // first packed word of the group within the pass
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
      const int wi = wbase + j * 4;  // lane c takes word wi + c
      const uint32_t W0 = *reinterpret_cast<const uint32_t*>(wrow0 + wi * 4);
      const uint32_t W8 = *reinterpret_cast<const uint32_t*>(wrow8 + wi * 4);
      const uint4 xv = *reinterpret_cast<const uint4*>(lc.xcol + (size_t)(wi + c) * 16);
      uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
      decode_word(W0, p0, p1, p2, p3);
      decode_word(W8, q0, q1, q2, q3);
      mma_bf16_16816(dA, p0, q0, p1, q1, xv.x, xv.y);
      mma_bf16_16816(dB, p2, q2, p3, q3, xv.z, xv.w);
    }
    const int ga = gabs0 + gi;
    if (actP) {
      const float sv = bf2f(sPm[gi]);
      const float bv = bf2f(bPm[gi]) - 128.0f * sv;
      if (lc.a00) acc[0] += sv * (dA[0] + dB[0]) + bv * lc.xs0[ga];
      if (lc.a01) acc[1] += sv * (dA[1] + dB[1]) + bv * lc.xs1[ga];
    }
    if (actQ) {
      const float sv = bf2f(sQm[gi]);
      const float bv = bf2f(bQm[gi]) - 128.0f * sv;
      if (lc.a10) acc[2] += sv * (dA[2] + dB[2]) + bv * lc.xs0[ga];
      if (lc.a11) acc[3] += sv * (dA[3] + dB[3]) + bv * lc.xs1[ga];
    }
  }
}

// ---------------------------------------------------------------------------
// routing (one warp): top-k, ties to the lower index, softmax over the k
// ---------------------------------------------------------------------------
// lr: logits row (global, read with ld.cg when `coherent`); results to
// sidx/sw (lane j < k writes slot j).
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
template <int WPT>
__global__ void __launch_bounds__(NTHREADS, 1) engine_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_misc);
  uint64_t* empty = full + NSTAGE;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NSTAGE);
  uint32_t* sidx = reinterpret_cast<uint32_t*>(smem + p.off_misc + 2 * NSTAGE * 8 + 16);
  float* sw = reinterpret_cast<float*>(sidx + MAX_COLS);
  float* rsum = sw + MAX_COLS;  // [NC_WARPS] router partials
  int* err = p.err;
  const Sched sch = make_sched(p);
  const uint64_t t0 = globaltimer();
  const uint64_t deadline = t0 + (uint64_t)p.timeout_ns;

  if (tid == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NC_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const bool fused = p.mode == MODE_FUSED;

  if (warp == NC_WARPS) {
    // ------------------------------- producer -------------------------------
    if (fused) named_bar_sync(2, NTHREADS);  // wait for the routing
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int L = 0;
      bool ok = !*abort_flag;
      for (int u = blockIdx.x; ok && u < sch.U; u += gridDim.x) {
        const int np = unit_passes(p, sch, u);
        for (int pass = 0; pass < np; ++pass, ++L) {
          const int sidx_s = L % NSTAGE;
          if (L >= NSTAGE && !mbar_wait(&empty[sidx_s], ((L / NSTAGE) - 1) & 1, deadline, abort_flag)) {
            if (!*abort_flag) record_error(err, B2Q_ETIMEOUT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const bool down = unit_is_down(p, sch, u);
          const Geo& g = down ? p.g2 : p.g1;
          const LoadDesc d = describe(p, sch, u, pass, sidx, err);
          uint8_t* st = stages + (size_t)sidx_s * p.stage_bytes;
          const uint32_t bytes = (uint32_t)(d.nP + d.nQ) * (d.row_bytes + 2 * d.meta_bytes);
          mbar_arrive_expect_tx(&full[sidx_s], bytes);
          for (int r = 0; r < d.nP; ++r) {
            bulk_g2s(st + r * g.RS, d.wP + (size_t)r * d.wstride, d.row_bytes, &full[sidx_s], pol);
            bulk_g2s(st + 16 * g.RS + (0 + r) * g.MS, d.sP + (size_t)r * d.mstride, d.meta_bytes, &full[sidx_s], pol);
            bulk_g2s(st + 16 * g.RS + (8 + r) * g.MS, d.bP + (size_t)r * d.mstride, d.meta_bytes, &full[sidx_s], pol);
          }
          for (int r = 0; r < d.nQ; ++r) {
            bulk_g2s(st + (8 + r) * g.RS, d.wQ + (size_t)r * d.wstride, d.row_bytes, &full[sidx_s], pol);
            bulk_g2s(st + 16 * g.RS + (16 + r) * g.MS, d.sQ + (size_t)r * d.mstride, d.meta_bytes, &full[sidx_s], pol);
            bulk_g2s(st + 16 * g.RS + (24 + r) * g.MS, d.bQ + (size_t)r * d.mstride, d.meta_bytes, &full[sidx_s], pol);
          }
        }
      }
      // Drain: no bulk copy may still be landing when the CTA exits.
      const uint64_t dl2 = globaltimer() + 200000000ull;
      for (int l = max(0, L - NSTAGE); l < L; ++l) {
        if (!mbar_wait(&full[l % NSTAGE], (l / NSTAGE) & 1, dl2, nullptr)) record_error(err, B2Q_ETIMEOUT);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------- consumers ------------------------------
    uint8_t* xbuf = smem + p.off_x;
    float* xsum = reinterpret_cast<float*>(smem + p.off_xs);
    uint8_t* abuf = smem + p.off_act;
    float* asum = reinterpret_cast<float*>(smem + p.off_acts);
    float* red = reinterpret_cast<float*>(smem + p.off_red);  // [2][NC_WARPS][16][8]
    const int r = lane >> 2, c = lane & 3;
    int cur_item = -1;  // QMV gather: item whose activations are staged
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
          const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            part += __uint_as_float(xa[i] << 16) * __uint_as_float(wa[i] << 16);
            part += __uint_as_float(xa[i] & 0xffff0000u) * __uint_as_float(wa[i] & 0xffff0000u);
          }
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
      // stage x (token 0) while the other CTAs finish their router rows
      {
        const uint16_t* rows[1] = {p.x};
        stage_columns(xbuf, xsum, p.g1.XS, rows, 1, p.H, p.gs, false);
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
    } else if (p.mode == MODE_GU) {
      // stage all S tokens once
      const uint16_t* rows[MAX_COLS];
      for (int t = 0; t < p.S; ++t) rows[t] = p.x + (size_t)t * p.H;
      stage_columns(xbuf, xsum, p.g1.XS, rows, p.S, p.H, p.gs, false);
    }

    int L = 0, buf = 0;
    for (int u = blockIdx.x; u < sch.U; u += gridDim.x) {
      const bool down = unit_is_down(p, sch, u);
      const Geo& g = down ? p.g2 : p.g1;
      // ---- per-unit activation setup ----
      LaneCols lc{};
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
            stage_columns(xbuf, xsum, g.XS, rows, p.M, g.K, p.gs, false);
          }
          cur_item = xkey;
        }
        const int n = r;  // B column of this lane = token n
        const int ncol = (n < p.M) ? n : 0;
        lc.xcol = xbuf + (size_t)ncol * g.XS;
        const int c0 = min(2 * c, p.M - 1), c1 = min(2 * c + 1, p.M - 1);
        lc.xs0 = xsum + (size_t)c0 * g.G;
        lc.xs1 = xsum + (size_t)c1 * g.G;
        lc.a00 = lc.a10 = (2 * c < p.M);
        lc.a01 = lc.a11 = (2 * c + 1 < p.M);
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
        lc.xcol = xbuf + (size_t)tok * g.XS;
        lc.xs0 = lc.xs1 = xsum + (size_t)tok * g.G;
        lc.a00 = lc.a10 = (c == 0);
        lc.a01 = lc.a11 = false;
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
            stage_columns(abuf, asum, g.XS, rows, p.k, p.F, p.gs, true);
            act_ready = true;
          }
        } else if (tok != cur_tok) {
          const uint16_t* rows[MAX_COLS];
          for (int j = 0; j < p.k; ++j) rows[j] = p.act_in + ((size_t)tok * p.k + j) * p.F;
          stage_columns(abuf, asum, g.XS, rows, p.k, p.F, p.gs, false);
          cur_tok = tok;
        }
        const int n = r;
        const int ncol = (n < p.k) ? n : 0;
        lc.xcol = abuf + (size_t)ncol * g.XS;
        const int c0 = min(2 * c, p.k - 1), c1 = min(2 * c + 1, p.k - 1);
        lc.xs0 = asum + (size_t)c0 * g.G;
        lc.xs1 = asum + (size_t)c1 * g.G;
      }

      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int np = unit_passes(p, sch, u);
      for (int pass = 0; pass < np; ++pass, ++L) {
        const int si = L % NSTAGE;
        const bool ok = mbar_wait(&full[si], (L / NSTAGE) & 1, deadline, abort_flag);
        if (!ok && !*abort_flag) {
          record_error(err, B2Q_ETIMEOUT);
          *abort_flag = 1;
        }
        if (ok && !*abort_flag) {
          int kc = pass;
          LaneCols lcp = lc;
          if (down) {
            const int pair = pass / g.nkc;
            kc = pass % g.nkc;
            lcp.a00 = (c == pair) && (2 * pair < p.k);
            lcp.a11 = (c == pair) && (2 * pair + 1 < p.k);
            lcp.a01 = lcp.a10 = false;
          }
          const int Gc = min(g.KC, g.K - kc * g.KC) / p.gs;
          const int glo = (warp * Gc) / NC_WARPS, ghi = ((warp + 1) * Gc) / NC_WARPS;
          lcp.xcol += (size_t)kc * (g.KC / 8) * 16;
          consume_pass<WPT>(stages + (size_t)si * p.stage_bytes, g, p.gs, glo, ghi, kc * (g.KC / p.gs), lcp, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[si]);
      }
      // ---- unit epilogue: fixed-order reduction over the 8 warps ----
      float* rw = red + ((size_t)buf * NC_WARPS + warp) * 128;
      rw[r * 8 + 2 * c] = acc[0];
      rw[r * 8 + 2 * c + 1] = acc[1];
      rw[(r + 8) * 8 + 2 * c] = acc[2];
      rw[(r + 8) * 8 + 2 * c + 1] = acc[3];
      named_bar_sync(1, NCT);
      const float* rr = red + (size_t)buf * NC_WARPS * 128;
      if (p.mode == MODE_QMV) {
        if (tid < 16 * p.M) {
          const int i = tid & 15, n = tid >> 4;
          const int row = rb * 16 + i;
          if (row < p.N) {
            float v = 0.0f;
            for (int w = 0; w < NC_WARPS; ++w) v += rr[w * 128 + i * 8 + n];
            p.y[((size_t)item * p.M + n) * p.N + row] = (item_ok && !*abort_flag) ? f2bf(v) : (uint16_t)0;
          }
        }
      } else if (!down) {
        if (tid < 8) {
          float gv = 0.0f, uv = 0.0f;
          for (int w = 0; w < NC_WARPS; ++w) {
            gv += rr[w * 128 + tid * 8];
            uv += rr[w * 128 + (tid + 8) * 8];
          }
          uint16_t* dst = (p.mode == MODE_FUSED) ? p.ws_act : p.act_out;
          dst[(size_t)zslot * p.F + rb * 8 + tid] = swiglu_bf16(f2bf(gv), f2bf(uv));
          if (p.mode == MODE_FUSED) __threadfence();
        }
        if (p.mode == MODE_FUSED) {
          named_bar_sync(1, NCT);
          if (tid == 0) {
            __threadfence();
            atomicAdd(&p.counters[1], 1u);
          }
        }
      } else {
        if (tid < 8) {
          const float* wts = (p.mode == MODE_FUSED) ? sw : nullptr;
          float prod[MAX_COLS];
          for (int j = 0; j < p.k; ++j) {
            const int i = (j & 1) ? tid + 8 : tid;
            float v = 0.0f;
            for (int w = 0; w < NC_WARPS; ++w) v += rr[w * 128 + i * 8 + j];
            const float wj = wts ? wts[j] : __ldg(p.w_in + (size_t)tok * p.k + j);
            prod[j] = b2q::rb(v) * wj;  // f32(bf16(y_j)) * w_j
          }
          // mlx_colsum_small_f32<K>: TY = min(8, K) chains, then folded in order
          const int TY = p.k < 8 ? p.k : 8;
          float t[MAX_COLS];
          for (int y = 0; y < TY; ++y) {
            float a = 0.0f;
            for (int q = y; q < p.k; q += TY) a = prod[q] + a;
            t[y] = a;
          }
          float total = t[0];
          for (int j = 1; j < TY; ++j) total = t[j] + total;
          p.out[(size_t)tok * p.H + hb * 8 + tid] = f2bf(total);
        }
      }
      buf ^= 1;
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
    const uint32_t xa[4] = {a.x, a.y, a.z, a.w}, wa[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      part += __uint_as_float(xa[i] << 16) * __uint_as_float(wa[i] << 16);
      part += __uint_as_float(xa[i] & 0xffff0000u) * __uint_as_float(wa[i] & 0xffff0000u);
    }
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

int launch_router_logits(const uint16_t* x, const uint16_t* wr, float* logits, int T, int E, int H,
                         cudaStream_t s) {
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
// host: geometry, shared-memory plan, launch
// ---------------------------------------------------------------------------
static int round_up(int v, int a) { return (v + a - 1) / a * a; }

// Reduction-chunk geometry for one product family (K elements per row).
static int make_geo(Geo& g, int K, int gs) {
  g.K = K;
  g.G = K / gs;
  const int unit = 8 * gs;  // chunk granularity keeps meta rows 16-byte sized and aligned
  // largest chunk whose 16 rows + 32 meta rows fit one stage
  int kc = (K <= 4096) ? K : 4096;
  kc = std::max(unit, kc / unit * unit);
  g.KC = kc;
  g.nkc = (K + kc - 1) / kc;
  const int row_bytes = kc / 2;
  g.RS = row_bytes + ((16 - row_bytes % 128) + 128) % 128;  // RS % 128 == 16
  int ms = round_up((kc / gs) * 2, 16);
  if ((ms / 16) % 2 == 0) ms += 16;  // odd multiple of 16: 8 meta rows hit 8 bank quads
  g.MS = ms;
  const int xb = (K / 8) * 16;
  g.XS = xb + ((64 - xb % 128) + 128) % 128;  // XS % 128 == 64
  return 16 * g.RS + 32 * g.MS;
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
  p.stage_bytes = round_up(std::max(st1, st2), 128);
  if (p.stage_bytes > STAGE_MAX) return set_error(B2Q_EUNSUPPORTED, "engine: stage of %d bytes", p.stage_bytes);
  int off = NSTAGE * p.stage_bytes;
  p.xcols = (p.mode == MODE_QMV) ? p.M : (p.mode == MODE_GU ? p.S : (p.mode == MODE_FUSED ? 1 : 0));
  p.off_x = off;
  off += round_up(p.xcols * (uses_g1 ? p.g1.XS : 0), 128);
  p.off_xs = off;
  off += round_up(p.xcols * (uses_g1 ? p.g1.G : 0) * 4, 128);
  p.off_act = off;
  off += round_up(uses_down ? p.k * p.g2.XS : 0, 128);
  p.off_acts = off;
  off += round_up(uses_down ? p.k * p.g2.G * 4 : 0, 128);
  p.off_red = off;
  off += 2 * NC_WARPS * 128 * 4;
  p.off_misc = off;
  off += 2 * NSTAGE * 8 + 16 + MAX_COLS * 8 + NC_WARPS * 4;
  p.smem_bytes = round_up(off, 128);
  if (p.smem_bytes > di.smem_optin)
    return set_error(B2Q_EUNSUPPORTED, "engine: needs %d bytes of shared memory, device allows %d", p.smem_bytes,
                     di.smem_optin);
  if (p.timeout_ns <= 0) p.timeout_ns = 2000000000ll;
  return B2Q_OK;
}

template <int WPT>
static int launch_t(const Params& p, cudaStream_t stream, bool cooperative, int grid) {
  auto kern = engine_kernel<WPT>;
  B2Q_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem_bytes));
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
  switch (p.wpt) {
    case 1: return launch_t<1>(p, s, cooperative, grid);
    case 2: return launch_t<2>(p, s, cooperative, grid);
    case 4: return launch_t<4>(p, s, cooperative, grid);
    default: return set_error(B2Q_EUNSUPPORTED, "engine: group size %d", p.gs);
  }
}

}  // namespace eng
}  // namespace b2q
