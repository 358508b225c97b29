// prefill.cu -- the prefill MoE layer: router, route, expert sort, expert
// products over the sorted rows, SwiGLU, and the weighted combine through the
// inverse permutation.
//
// Reference flow (paths relative to the reference project):
//   TrackP12Prefill.sortedMoE            Runner/FastModel/TrackP12Prefill.swift:198-237
//   TrackPrefillIndirect.apply / .down   Runner/FastModel/TrackPrefillIndirect.swift:83-227
//   track_p12_moe_sorted_combine         Runner/FastModel/TrackP12Prefill.swift:180-197
//   compiled silu * up                   Runner/FastModel/TrackFastKernels2.swift:547-600
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "engine.cuh"
#include "host.hpp"
#include "misc.cuh"
#include "prefill.cuh"
#include "qmm_tc.cuh"

namespace b2q {

// act[p, f] = silu(bf16 g) * bf16 u, all in bf16 (compiledSiluProduct).
__global__ void swiglu_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                              uint16_t* __restrict__ act, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = swiglu_bf16(g[i], u[i]);
}

// out[t, h] = bf16(colsum_j f32(y[inverse[t*k + j], h]) * w[t, j]) with the
// mlx_colsum_small_f32 association (TrackFastKernels2.swift:36-47).
__global__ void sorted_combine_kernel(const uint16_t* __restrict__ y, const uint32_t* __restrict__ inverse,
                                      const float* __restrict__ w, uint16_t* __restrict__ out, int T, int H,
                                      int k) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  const int t = blockIdx.y;
  if (h >= H || t >= T) return;
  float prod[32];
  for (int j = 0; j < k; ++j) {
    const uint32_t pj = __ldg(inverse + (size_t)t * k + j);
    prod[j] = bf2f(y[(size_t)pj * H + h]) * __ldg(w + (size_t)t * k + j);
  }
  const int TY = k < 8 ? k : 8;
  float tt[8];
  for (int q = 0; q < TY; ++q) {
    float a = 0.0f;
    for (int r = q; r < k; r += TY) a = prod[r] + a;
    tt[q] = a;
  }
  float total = tt[0];
  for (int q = 1; q < TY; ++q) total = tt[q] + total;
  out[(size_t)t * H + h] = f2bf(total);
}

// The same combine for 8 consecutive outputs per thread (16-byte loads of the
// k rows and one 16-byte store); H % 8 == 0, 16-byte aligned rows, k <= 8.
// All k row loads are issued before any is used (up to 8 x 16 bytes in flight
// per thread); with k <= 8 each slot is its own chain of the colsum
// association, and the chains fold in slot order.
__global__ void sorted_combine8_kernel(const uint16_t* __restrict__ y, const uint32_t* __restrict__ inverse,
                                       const float* __restrict__ w, uint16_t* __restrict__ out, int T, int H,
                                       int k) {
  const int h0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int t = blockIdx.y;
  if (h0 >= H || t >= T) return;
  uint4 r[8];
  float wj[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < k) {
      const uint32_t pj = __ldg(inverse + (size_t)t * k + j);
      wj[j] = __ldg(w + (size_t)t * k + j);
      r[j] = __ldg(reinterpret_cast<const uint4*>(y + (size_t)pj * H + h0));
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int v = 0; v < 8; v += 2) {
    float t0 = 0.0f, t1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < k) {
        const uint32_t word = (v >> 1) == 0 ? r[j].x : (v >> 1) == 1 ? r[j].y : (v >> 1) == 2 ? r[j].z : r[j].w;
        // product rounded, then a chain starting from 0 (c = p + 0, as the
        // colsum's running sums do), chains folded in slot order
        const float c0 = __fmul_rn(__uint_as_float(word << 16), wj[j]) + 0.0f;
        const float c1 = __fmul_rn(__uint_as_float(word & 0xffff0000u), wj[j]) + 0.0f;
        t0 = (j == 0) ? c0 : c0 + t0;
        t1 = (j == 0) ? c1 : c1 + t1;
      }
    }
    o[v >> 1] = (uint32_t)f2bf(t0) | ((uint32_t)f2bf(t1) << 16);
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * H + h0) = make_uint4(o[0], o[1], o[2], o[3]);
}

static void launch_sorted_combine(const uint16_t* y, const uint32_t* inverse, const float* w, uint16_t* out, int T,
                                  int H, int k, cudaStream_t st) {
  if (k <= 8 && H % 8 == 0 && aligned16(y) && aligned16(out)) {
    dim3 grid((H / 8 + 255) / 256, T);
    sorted_combine8_kernel<<<grid, 256, 0, st>>>(y, inverse, w, out, T, H, k);
  } else {
    dim3 grid((H + 255) / 256, T);
    sorted_combine_kernel<<<grid, 256, 0, st>>>(y, inverse, w, out, T, H, k);
  }
}

// ---------------------------------------------------------------------------
// gather_qmm / quantized_matmul with many rows per weight matrix (M > 8): the
// tcgen05 grouped GEMM over rows grouped by weight matrix.
// Item i multiplies x[lhs[i]] (M rows; lhs null: x[i]) by w[rhs[i]] (rhs null:
// w[i]) into y[i]; items whose indices are out of range produce zeros, as the
// shape-general kernel does.
// ---------------------------------------------------------------------------
bool prefill_qmm_eligible(int batch, int M, int N, int K, int gs, const void* x, const void* w, const void* s,
                          const void* b, const void* y) {
  (void)batch;
  return M > 8 && tc_shape_ok(N, K, gs, TC_PLAIN) && aligned16(x) && aligned16(w) && aligned16(s) &&
         aligned16(b) && aligned16(y);
}

// ids[i] = rhs[i] (or i)
__global__ void item_ids_kernel(const uint32_t* __restrict__ rhs, uint32_t* __restrict__ ids, int batch) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < batch) ids[i] = rhs ? rhs[i] : (uint32_t)i;
}

// Row tables of the sorted items: sorted row p*M + m reads x row
// lhs[item]*M + m (0xFFFFFFFF when lhs is out of range: zeros) and is written
// to y row item*M + m. Row offsets per weight matrix = item offsets * M.
__global__ void item_rows_kernel(const uint32_t* __restrict__ item_of, const uint32_t* __restrict__ lhs,
                                 const uint32_t* __restrict__ offsets, uint32_t* __restrict__ src_row,
                                 uint32_t* __restrict__ out_row, uint32_t* __restrict__ row_offsets, int n_sorted,
                                 int M, int n_x, int E) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t <= E && row_offsets) row_offsets[t] = offsets[t] * (uint32_t)M;
  if (t >= n_sorted * M) return;
  const int p = t / M, m = t % M;
  const uint32_t item = item_of[p];
  if (item >= (uint32_t)n_sorted) {  // a position past the valid items: never multiplied
    src_row[t] = 0xFFFFFFFFu;
    out_row[t] = 0;
    return;
  }
  const uint32_t xi = lhs ? lhs[item] : item;
  src_row[t] = xi < (uint32_t)n_x ? xi * (uint32_t)M + (uint32_t)m : 0xFFFFFFFFu;
  out_row[t] = item * (uint32_t)M + (uint32_t)m;
}

// Temporaries of the tensor-core gather GEMM, in one region: ids, sorted ids,
// item order, inverse, offsets, row offsets, unit prefix, error word, source /
// output row tables, sorted x rows.
struct GatherQmmWs {
  size_t o_ids, o_sid, o_item, o_inv, o_off, o_roff, o_pre, o_err, o_src, o_out, o_xs, bytes;
};

static GatherQmmWs gather_qmm_ws_layout(int batch, int M, int K, int E) {
  auto a256 = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t R = (size_t)batch * M;
  GatherQmmWs l{};
  size_t off = 0;
  l.o_ids = off; off = a256(off + 4 * (size_t)batch);
  l.o_sid = off; off = a256(off + 4 * (size_t)batch);
  l.o_item = off; off = a256(off + 4 * (size_t)batch);
  l.o_inv = off; off = a256(off + 4 * (size_t)batch);
  l.o_off = off; off = a256(off + 4 * ((size_t)E + 1));
  l.o_roff = off; off = a256(off + 4 * ((size_t)E + 1));
  l.o_pre = off; off = a256(off + 4 * ((size_t)E + 1));
  l.o_err = off; off = a256(off + 4);
  l.o_src = off; off = a256(off + 4 * R);
  l.o_out = off; off = a256(off + 4 * R);
  l.o_xs = off; off = a256(off + 2 * R * (size_t)K);
  l.bytes = off;
  return l;
}

size_t prefill_gather_qmm_ws_bytes(int batch, int M, int K, int n_w) {
  if (batch <= 0 || M <= 0 || K <= 0 || n_w <= 0) return 0;
  return gather_qmm_ws_layout(batch, M, K, n_w).bytes;
}

int launch_prefill_gather_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                              const uint32_t* lhs, const uint32_t* rhs, uint16_t* y, int batch, int M, int N, int K,
                              int n_x, int n_w, int gs, int sorted, void* workspace, size_t workspace_bytes,
                              cudaStream_t st) {
  (void)sorted;  // the items are grouped by a stable sort either way
  const int E = n_w;
  if (E < 1 || E > 1024) return set_error(B2Q_EUNSUPPORTED, "gather_qmm: %d weight matrices on tensor cores", E);
  const size_t R = (size_t)batch * M;
  const GatherQmmWs l = gather_qmm_ws_layout(batch, M, K, E);
  const size_t o_ids = l.o_ids, o_sid = l.o_sid, o_item = l.o_item, o_inv = l.o_inv, o_off = l.o_off,
               o_roff = l.o_roff, o_pre = l.o_pre, o_err = l.o_err, o_src = l.o_src, o_out = l.o_out, o_xs = l.o_xs;
  // caller's workspace when given (256-byte aligned, at least l.bytes), else a
  // stream-ordered temporary freed at the end of the call
  char* tmp = static_cast<char*>(workspace);
  const bool owned = tmp == nullptr;
  if (!owned) {
    if (workspace_bytes < l.bytes || (reinterpret_cast<uintptr_t>(tmp) & 255))
      return set_error(B2Q_EINVAL, "gather_qmm: workspace of %zu bytes (256-byte aligned) needed, %zu given",
                       l.bytes, workspace_bytes);
  } else {
    B2Q_TRY_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&tmp), l.bytes, st));
  }
  auto U32 = [&](size_t o) { return reinterpret_cast<uint32_t*>(tmp + o); };
  int rc = B2Q_OK;
  do {
    if (cudaMemsetAsync(tmp + o_err, 0, 4, st) != cudaSuccess || cudaMemsetAsync(y, 0, R * (size_t)N * 2, st) != cudaSuccess) {
      rc = cuda_check(cudaGetLastError(), "gather_qmm: memset");
      break;
    }
    item_ids_kernel<<<(batch + 255) / 256, 256, 0, st>>>(rhs, U32(o_ids), batch);
    // stable grouping of the items by weight matrix; out-of-range ids are left out
    rc = launch_expert_sort(U32(o_ids), U32(o_sid), U32(o_item), U32(o_inv), U32(o_off), batch, E, 1,
                            reinterpret_cast<int*>(tmp + o_err), st);
    if (rc) break;
    // row tables over every sorted position (positions of left-out items are never reached:
    // the row offsets stop at the valid items)
    const int nthreads = (int)std::max<size_t>(R, (size_t)E + 1);
    item_rows_kernel<<<(nthreads + 255) / 256, 256, 0, st>>>(U32(o_item), lhs, U32(o_off), U32(o_src), U32(o_out),
                                                              U32(o_roff), batch, M, n_x, E);
    rc = tc_unit_tables(U32(o_roff), E, tc_m_tiles(N, TC_PLAIN), 0, U32(o_pre), nullptr, st);
    if (rc) break;
    rc = tc_gather_rows(x, U32(o_src), reinterpret_cast<uint16_t*>(tmp + o_xs), (int)R, K, n_x * M, st);
    if (rc) break;
    TcParams p{};
    p.E = E;
    p.K = K;
    p.Nw = N;
    p.gs = gs;
    p.s0 = s;
    p.b0 = b;
    p.offsets = U32(o_roff);
    p.prefix = U32(o_pre);
    p.out = y;
    p.out_rows = U32(o_out);
    p.out_ld = N;
    p.err = reinterpret_cast<int*>(tmp + o_err);
    p.timeout_ns = 2000000000ll;
    rc = tc_setup(p, TC_PLAIN, reinterpret_cast<uint16_t*>(tmp + o_xs), (int)R, w, nullptr);
    if (rc) break;
    rc = tc_launch(p, TC_PLAIN, st);
  } while (0);
  if (owned) cudaFreeAsync(tmp, st);
  return rc;
}

struct PrefillWs {
  int* err;
  float* logits;
  uint32_t* idx;
  float* w;
  uint32_t* sorted_ids;
  uint32_t* token_rows;
  uint32_t* inverse;
  uint32_t* offsets;
  uint32_t* prefix_gu;  // tensor-core unit ranges per expert (gate|up, down)
  uint32_t* prefix_dn;
  uint16_t* g;   // per-slot path: gate [R, F] and up [R, F] ...
  uint16_t* u;
  uint16_t* xs;  // ... or, tensor-core path, the sorted token rows [R, H] (same region)
  uint16_t* act;
  uint16_t* y;
  size_t bytes;
};

static size_t a256(size_t v) { return (v + 255) / 256 * 256; }

static PrefillWs prefill_ws_layout(void* base, int T, int H, int E, int F, int k) {
  PrefillWs d{};
  char* b = static_cast<char*>(base);
  const size_t R = (size_t)T * k;
  size_t off = 0;
  d.err = reinterpret_cast<int*>(b);
  off = 256;
  d.logits = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * (size_t)T * E);
  d.idx = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.w = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * R);
  d.sorted_ids = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.token_rows = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.inverse = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.offsets = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * ((size_t)E + 1));
  d.prefix_gu = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * ((size_t)E + 1));
  d.prefix_dn = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * ((size_t)E + 1));
  d.g = reinterpret_cast<uint16_t*>(b + off);
  d.u = d.g + R * F;
  d.xs = d.g;
  off = a256(off + 2 * std::max(2 * R * F, R * (size_t)H));
  d.act = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * F);
  d.y = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * H);
  d.bytes = off;
  return d;
}

// The tensor-core path: both products fit the tcgen05 kernel's shape rules
// and every operand is 16-byte aligned.
static bool prefill_tc_ok(int H, int E, int F, int gs, const void* const* ptrs, int nptr) {
  if (E > 1024 || !tc_shape_ok(F, H, gs, TC_GLU) || !tc_shape_ok(H, F, gs, TC_PLAIN)) return false;
  for (int i = 0; i < nptr; ++i)
    if (!aligned16(ptrs[i])) return false;
  return true;
}

}  // namespace b2q

using namespace b2q;

extern "C" {

int b2q_swiglu(const uint16_t* g, const uint16_t* u, uint16_t* act, int64_t n, void* stream) {
  clear_error();
  if (n < 0) return set_error(B2Q_EINVAL, "swiglu: n < 0");
  if (n == 0) return B2Q_OK;
  if (!g || !u || !act) return set_error(B2Q_EINVAL, "swiglu: null pointer");
  swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(g, u, act, n);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int b2q_moe_sorted_combine(const uint16_t* y, const uint32_t* inverse, const float* w, uint16_t* out, int T, int H,
                           int k, void* stream) {
  clear_error();
  if (T < 0 || H <= 0 || k < 1 || k > 32) return set_error(B2Q_EINVAL, "sorted_combine: bad shape");
  if (T == 0) return B2Q_OK;
  if (!y || !inverse || !w || !out) return set_error(B2Q_EINVAL, "sorted_combine: null pointer");
  launch_sorted_combine(y, inverse, w, out, T, H, k, static_cast<cudaStream_t>(stream));
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

size_t b2q_sort_workspace_size(int R, int E) {
  (void)R;
  (void)E;
  return 256;  // the error word; the sort itself keeps its state in shared memory
}

int b2q_moe_sort(const uint32_t* ids, uint32_t* sorted_ids, uint32_t* token_rows, uint32_t* inverse,
                 uint32_t* offsets, int R, int E, int k, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (R < 0 || E < 1 || E > 1024 || k < 1) return set_error(B2Q_EINVAL, "moe_sort: bad shape");
  if (!ids || !workspace || workspace_bytes < 256) return set_error(B2Q_EINVAL, "moe_sort: null pointer/workspace");
  if (R == 0) return B2Q_OK;
  return launch_expert_sort(ids, sorted_ids, token_rows, inverse, offsets, R, E, k, static_cast<int*>(workspace),
                            static_cast<cudaStream_t>(stream));
}

size_t b2q_moe_prefill_workspace_size(int T, int H, int E, int F, int k) {
  if (T < 1 || H < 1 || E < 1 || F < 1 || k < 1) return 0;
  return prefill_ws_layout(nullptr, T, H, E, F, k).bytes;
}

int b2q_moe_prefill(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg,
                    const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                    const uint32_t* wd, const uint16_t* sd, const uint16_t* bd, uint16_t* out, uint32_t* idx,
                    float* w, int T, int H, int E, int F, int k, int group_size, int bits, void* workspace,
                    size_t workspace_bytes, void* stream) {
  clear_error();
  if (bits != 4) return set_error(B2Q_EUNSUPPORTED, "moe_prefill: bits=%d", bits);
  if (!(group_size == 32 || group_size == 64 || group_size == 128))
    return set_error(B2Q_EUNSUPPORTED, "moe_prefill: group_size=%d", group_size);
  if (T < 0 || H <= 0 || E < 1 || E > 1024 || F <= 0 || k < 1 || k > 32 || k > E || H % group_size ||
      F % group_size || H % 8 || F % 8)
    return set_error(B2Q_EINVAL, "moe_prefill: bad shape");
  if (T == 0) return B2Q_OK;
  if (!x || !wr || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !out)
    return set_error(B2Q_EINVAL, "moe_prefill: null pointer");
  const PrefillWs ws = prefill_ws_layout(workspace, T, H, E, F, k);
  if (!workspace || workspace_bytes < ws.bytes || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "moe_prefill: workspace of %zu bytes needed", ws.bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int R = T * k;
  uint32_t* ix = idx ? idx : ws.idx;
  float* ww = w ? w : ws.w;
  // the split-K router GEMM keeps its partials in the down-output region,
  // which is not in use before the expert products
  int rc = eng::launch_router_logits_sk(x, wr, ws.logits, reinterpret_cast<float*>(ws.y), 2 * (size_t)T * k * H, T,
                                        E, H, st);
  if (rc) return rc;
  rc = eng::launch_route(ws.logits, ix, ww, T, E, k, st);
  if (rc) return rc;
  rc = launch_expert_sort(ix, ws.sorted_ids, ws.token_rows, ws.inverse, ws.offsets, R, E, k, ws.err, st);
  if (rc) return rc;
  const void* wptrs[9] = {wg, sg, bg, wu, su, bu, wd, sd, bd};
  if (prefill_tc_ok(H, E, F, group_size, wptrs, 9)) {
    // tensor cores: sorted token rows -> gate|up + SwiGLU -> down, per expert
    rc = tc_unit_tables(ws.offsets, E, tc_m_tiles(F, TC_GLU), tc_m_tiles(H, TC_PLAIN), ws.prefix_gu, ws.prefix_dn, st);
    if (rc) return rc;
    rc = tc_gather_rows(x, ws.token_rows, ws.xs, R, H, T, st);
    if (rc) return rc;
    TcParams pg{};
    pg.E = E;
    pg.K = H;
    pg.Nw = F;
    pg.gs = group_size;
    pg.s0 = sg;
    pg.b0 = bg;
    pg.s1 = su;
    pg.b1 = bu;
    pg.offsets = ws.offsets;
    pg.prefix = ws.prefix_gu;
    pg.out = ws.act;
    pg.out_ld = F;
    pg.err = ws.err;
    pg.timeout_ns = 2000000000ll;
    rc = tc_setup(pg, TC_GLU, ws.xs, R, wg, wu);
    if (rc) return rc;
    rc = tc_launch(pg, TC_GLU, st);
    if (rc) return rc;
    TcParams pd{};
    pd.E = E;
    pd.K = F;
    pd.Nw = H;
    pd.gs = group_size;
    pd.s0 = sd;
    pd.b0 = bd;
    pd.offsets = ws.offsets;
    pd.prefix = ws.prefix_dn;
    pd.out = ws.y;
    pd.out_ld = H;
    pd.err = ws.err;
    pd.timeout_ns = 2000000000ll;
    rc = tc_setup(pd, TC_PLAIN, ws.act, R, wd, nullptr);
    if (rc) return rc;
    rc = tc_launch(pd, TC_PLAIN, st);
    if (rc) return rc;
    launch_sorted_combine(ws.y, ws.inverse, ww, out, T, H, k, st);
    B2Q_TRY_CUDA(cudaGetLastError());
    return B2Q_OK;
  }
  // per-slot products through the streaming engine: gate, up (x rows through token_rows)
  rc = b2q_gather_qmm(x, wg, sg, bg, ws.token_rows, ws.sorted_ids, ws.g, R, 1, F, H, T, E, group_size, bits, 1, 1,
                      stream);
  if (rc) return rc;
  rc = b2q_gather_qmm(x, wu, su, bu, ws.token_rows, ws.sorted_ids, ws.u, R, 1, F, H, T, E, group_size, bits, 1, 1,
                      stream);
  if (rc) return rc;
  {
    const int64_t n = (int64_t)R * F;
    swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ws.g, ws.u, ws.act, n);
    B2Q_TRY_CUDA(cudaGetLastError());
  }
  rc = b2q_gather_qmm(ws.act, wd, sd, bd, nullptr, ws.sorted_ids, ws.y, R, 1, H, F, R, E, group_size, bits, 1, 1,
                      stream);
  if (rc) return rc;
  {
    launch_sorted_combine(ws.y, ws.inverse, ww, out, T, H, k, st);
    B2Q_TRY_CUDA(cudaGetLastError());
  }
  return B2Q_OK;
}

}  // extern "C"
