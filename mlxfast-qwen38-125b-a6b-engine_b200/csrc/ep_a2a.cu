// ep_a2a.cu -- expert-parallel prefill over an all-to-all token exchange.
//
// Tokens are owned by ranks (each rank passes its own rows); experts are
// sharded by the contiguous-block rule (ep_expert_block). One layer is
//
//   dispatch (token owner)  route its T tokens; for every destination rank d
//                           that holds at least one of a token's k experts,
//                           copy the token row once (deduplicated per rank)
//                           and its k (expert, weight) pairs into block d of
//                           the send buffers; pos[t, d] = row in block d, or -1
//   exchange                counts all-gathered, then grouped NCCL send / recv
//                           of each block to its rank (self: a device copy)
//   experts (expert rank)   for the received rows: keep the slots whose expert
//                           is local, stable-sort them by expert, gate|up +
//                           SwiGLU and down on the tensor cores, and fold the
//                           weighted local slots of each row into an fp32
//                           partial row (colsum association)
//   exchange back           each partial row returns to its owner, into the
//                           block of the rank that made it
//   combine (token owner)   out[t] = bf16(sum over d in rank order of the
//                           partial rows of t)
//
// The reference has no expert parallelism: all experts of a layer share one
// Apple GPU's memory (its MoE layer is moeForwardShared,
// Runner/FastModel/TrackFastModel.swift:867-1009, with the sorted prefill of
// Runner/FastModel/TrackP12Prefill.swift:180-237). This is the sharded form
// of that layer; per-rank partial sums then the sum over ranks change the
// combine association, so outputs match the one-GPU layer to rounding.
//
// The three phases are separate entry points (a runtime with its own
// transport moves the blocks itself; the tests emulate ranks on one GPU
// through them); b2q_ep_moe_prefill_a2a chains them over the library's NCCL
// communicator. The count exchange is read on the host (NCCL needs the sizes
// when the transfers are enqueued), so that call waits for the dispatch.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "common.cuh"
#include "engine.cuh"
#include "ep.cuh"
#include "host.hpp"
#include "prefill.cuh"
#include "qmm_tc.cuh"

namespace b2q {
namespace a2a {

constexpr int MAXR = B2Q_EP_MAX_RANKS;
constexpr int PLAN_THREADS = 1024;

size_t a256(size_t v) { return (v + 255) / 256 * 256; }

// rank holding expert e under the contiguous-block rule
__device__ __forceinline__ int owner_of(uint32_t e, int E, int nranks) {
  const int base = E / nranks, extra = E % nranks;
  const int split = extra * (base + 1);
  return (int)e < split ? (int)e / (base + 1) : extra + ((int)e - split) / base;
}

__device__ __forceinline__ unsigned dest_mask(const uint32_t* idx, int t, int k, int E, int nranks, int* err) {
  unsigned m = 0;
  for (int j = 0; j < k; ++j) {
    const uint32_t e = idx[(size_t)t * k + j];
    if (e < (uint32_t)E)
      m |= 1u << owner_of(e, E, nranks);
    else
      record_error(err, B2Q_EINVAL);
  }
  return m;
}

// One CTA: pos[t, d] = number of earlier tokens sent to d (or -1), counts[d].
// Each thread owns a contiguous run of tokens; a block-wide exclusive scan of
// the per-thread counts gives the run's first position for every rank.
__global__ void __launch_bounds__(PLAN_THREADS, 1)
    plan_kernel(const uint32_t* __restrict__ idx, int T, int k, int E, int nranks, int32_t* __restrict__ pos,
                int32_t* __restrict__ counts, int* err) {
  __shared__ unsigned wsum[PLAN_THREADS / 32][MAXR];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (T + PLAN_THREADS - 1) / PLAN_THREADS;
  const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
  unsigned cnt[MAXR];
#pragma unroll
  for (int d = 0; d < MAXR; ++d) cnt[d] = 0;
  for (int t = t0; t < t1; ++t) {
    const unsigned m = dest_mask(idx, t, k, E, nranks, err);
#pragma unroll
    for (int d = 0; d < MAXR; ++d) cnt[d] += (m >> d) & 1u;
  }
  unsigned excl[MAXR];
#pragma unroll
  for (int d = 0; d < MAXR; ++d) {
    unsigned v = cnt[d];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned u = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += u;
    }
    if (lane == 31) wsum[warp][d] = v;
    excl[d] = v - cnt[d];
  }
  __syncthreads();
#pragma unroll
  for (int d = 0; d < MAXR; ++d) {
    unsigned pre = 0;
    for (int w = 0; w < warp; ++w) pre += wsum[w][d];
    excl[d] += pre;
  }
  if (tid < nranks) {
    unsigned tot = 0;
    for (int w = 0; w < PLAN_THREADS / 32; ++w) tot += wsum[w][tid];
    counts[tid] = (int32_t)tot;
  }
  for (int t = t0; t < t1; ++t) {
    const unsigned m = dest_mask(idx, t, k, E, nranks, err);
#pragma unroll
    for (int d = 0; d < MAXR; ++d) {
      if (d < nranks) {
        const bool sent = (m >> d) & 1u;
        pos[(size_t)t * nranks + d] = sent ? (int32_t)excl[d] : -1;
        excl[d] += sent;
      }
    }
  }
}

// Block t copies token t's row and its k (expert, weight-bits) pairs into
// every destination block it goes to.
__global__ void pack_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ idx,
                            const float* __restrict__ w, const int32_t* __restrict__ pos,
                            uint16_t* __restrict__ send_x, uint32_t* __restrict__ send_meta, int T, int H, int k,
                            int nranks) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  const int nv = H / 8;
  for (int d = 0; d < nranks; ++d) {
    const int p = pos[(size_t)t * nranks + d];
    if (p < 0) continue;
    const size_t row = (size_t)d * T + p;
    uint4* dst = reinterpret_cast<uint4*>(send_x + row * H);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) dst[v] = __ldg(src + v);
    uint32_t* meta = send_meta + row * 2 * k;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      meta[j] = idx[(size_t)t * k + j];
      meta[k + j] = __float_as_uint(w[(size_t)t * k + j]);
    }
  }
}

// Received slots -> local expert id (e_local for experts held elsewhere: a
// trailing bucket the products skip) and the fp32 weight.
__global__ void localize_kernel(const uint32_t* __restrict__ meta, int R, int k, int E, int e_lo, int e_local,
                                uint32_t* __restrict__ ids, float* __restrict__ w, int* err) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)R * k) return;
  const size_t r = i / k, j = i % k;
  const uint32_t e = meta[r * 2 * k + j];
  if (e >= (uint32_t)E) record_error(err, B2Q_EINVAL);
  const uint32_t le = e - (uint32_t)e_lo;  // wraps for experts below e_lo
  ids[i] = le < (uint32_t)e_local ? le : (uint32_t)e_local;
  w[i] = __uint_as_float(meta[r * 2 * k + k + j]);
}

// out[t, h] = bf16(sum over d (rank order) of ret[d*T + pos[t, d], h]), 4 columns per thread
__global__ void combine_kernel(const float* __restrict__ ret, const int32_t* __restrict__ pos,
                               uint16_t* __restrict__ out, int T, int H, int nranks) {
  const int t = blockIdx.y;
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (t >= T || h >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  bool first = true;
  for (int d = 0; d < nranks; ++d) {
    const int p = pos[(size_t)t * nranks + d];
    if (p < 0) continue;
    const float4 v = *reinterpret_cast<const float4*>(ret + ((size_t)d * T + p) * H + h);
    if (first) {
      acc = v;
      first = false;
    } else {
      acc.x = acc.x + v.x;
      acc.y = acc.y + v.y;
      acc.z = acc.z + v.z;
      acc.w = acc.w + v.w;
    }
  }
  uint2 o;
  o.x = (uint32_t)f2bf(acc.x) | ((uint32_t)f2bf(acc.y) << 16);
  o.y = (uint32_t)f2bf(acc.z) | ((uint32_t)f2bf(acc.w) << 16);
  *reinterpret_cast<uint2*>(out + (size_t)t * H + h) = o;
}

// ---- workspaces ---------------------------------------------------------------
struct DispatchWs {
  int* err;
  float* logits;
  uint32_t* idx;
  float* w;
  size_t bytes;
};

DispatchWs dispatch_layout(void* base, int T, int E, int k) {
  DispatchWs d{};
  char* b = static_cast<char*>(base);
  size_t off = 0;
  d.err = reinterpret_cast<int*>(b);
  off = 256;
  d.logits = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * (size_t)T * E);
  d.idx = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * (size_t)T * k);
  d.w = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * (size_t)T * k);
  d.bytes = off;
  return d;
}

struct ExpertsWs {
  int* err;
  uint32_t *ids, *sorted_ids, *token_rows, *inverse, *offsets, *prefix_gu, *prefix_dn;
  float* w;
  uint16_t *xs, *act, *y;
  size_t bytes;
};

ExpertsWs experts_layout(void* base, int R, int H, int E, int F, int k) {
  ExpertsWs d{};
  char* b = static_cast<char*>(base);
  const size_t S = (size_t)R * k;  // received slots
  size_t off = 0;
  d.err = reinterpret_cast<int*>(b);
  off = 256;
  uint32_t** slot_arrays[] = {&d.ids, &d.sorted_ids, &d.token_rows, &d.inverse};
  for (uint32_t** q : slot_arrays) {
    *q = reinterpret_cast<uint32_t*>(b + off);
    off = a256(off + 4 * S);
  }
  d.w = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * S);
  uint32_t** per_e[] = {&d.offsets, &d.prefix_gu, &d.prefix_dn};
  for (uint32_t** q : per_e) {
    *q = reinterpret_cast<uint32_t*>(b + off);
    off = a256(off + 4 * ((size_t)E + 2));
  }
  d.xs = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * S * H);
  d.act = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * S * F);
  d.y = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * S * H);
  d.bytes = off;
  return d;
}

struct FullWs {
  int* err;
  int32_t *counts, *matrix, *pos;
  uint16_t *send_x, *recv_x;
  uint32_t *send_meta, *recv_meta;
  float *partial, *ret;
  void* dispatch;
  void* experts;
  size_t dispatch_bytes, experts_bytes, bytes;
};

// T_max tokens per rank at most, so a rank receives at most nranks * T_max rows
FullWs full_layout(void* base, int T_max, int H, int E, int F, int k, int nranks) {
  FullWs d{};
  char* b = static_cast<char*>(base);
  const size_t rows = (size_t)nranks * T_max;
  size_t off = 0;
  d.err = reinterpret_cast<int*>(b);
  off = 256;
  d.counts = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + 4 * (size_t)(nranks + 1));
  d.matrix = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + 4 * (size_t)nranks * (nranks + 1));
  d.pos = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + 4 * (size_t)T_max * nranks);
  d.send_x = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * rows * H);
  d.recv_x = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * rows * H);
  d.send_meta = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 8 * rows * k);
  d.recv_meta = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 8 * rows * k);
  d.partial = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * rows * H);
  d.ret = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * rows * H);
  d.dispatch = b + off;
  d.dispatch_bytes = dispatch_layout(nullptr, T_max, E, k).bytes;
  off = a256(off + d.dispatch_bytes);
  d.experts = b + off;
  d.experts_bytes = experts_layout(nullptr, (int)rows, H, E, F, k).bytes;
  off = a256(off + d.experts_bytes);
  d.bytes = off;
  return d;
}

bool shape_ok_dispatch(int T, int H, int E, int k, int nranks) {
  return T >= 0 && H > 0 && H % 8 == 0 && E >= 1 && E <= 1024 && k >= 1 && k <= 32 && k <= E && nranks >= 1 &&
         nranks <= MAXR && nranks <= E;
}

int dispatch(const uint16_t* x, const uint16_t* wr, uint16_t* send_x, uint32_t* send_meta, int32_t* send_counts,
             int32_t* pos, uint32_t* idx, float* w, int T, int H, int E, int k, int nranks, void* workspace,
             int* err, cudaStream_t st) {
  const DispatchWs ws = dispatch_layout(workspace, T, E, k);
  B2Q_TRY_CUDA(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * nranks, st));
  if (T == 0) return B2Q_OK;
  uint32_t* ix = idx ? idx : ws.idx;
  float* ww = w ? w : ws.w;
  int rc = eng::launch_router_logits(x, wr, ws.logits, T, E, H, st);
  if (rc) return rc;
  rc = eng::launch_route(ws.logits, ix, ww, T, E, k, st);
  if (rc) return rc;
  plan_kernel<<<1, PLAN_THREADS, 0, st>>>(ix, T, k, E, nranks, pos, send_counts, err);
  B2Q_TRY_CUDA(cudaGetLastError());
  pack_kernel<<<T, 128, 0, st>>>(x, ix, ww, pos, send_x, send_meta, T, H, k, nranks);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int experts(const uint16_t* recv_x, const uint32_t* recv_meta, const uint32_t* wg, const uint16_t* sg,
            const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd,
            const uint16_t* sd, const uint16_t* bd, float* partial, int R, int H, int E, int F, int k, int e_lo,
            int e_local, int gs, void* workspace, int* err, cudaStream_t st) {
  if (R == 0) return B2Q_OK;
  const ExpertsWs ws = experts_layout(workspace, R, H, E, F, k);
  const int S = R * k;
  localize_kernel<<<(S + 255) / 256, 256, 0, st>>>(recv_meta, R, k, E, e_lo, e_local, ws.ids, ws.w, err);
  B2Q_TRY_CUDA(cudaGetLastError());
  // buckets 0..e_local-1 are the local experts, bucket e_local the slots held elsewhere
  int rc = launch_expert_sort(ws.ids, ws.sorted_ids, ws.token_rows, ws.inverse, ws.offsets, S, e_local + 1, k,
                              err, st);
  if (rc) return rc;
  rc = tc_unit_tables(ws.offsets, e_local, tc_m_tiles(F, TC_GLU), tc_m_tiles(H, TC_PLAIN), ws.prefix_gu,
                      ws.prefix_dn, st);
  if (rc) return rc;
  rc = tc_gather_rows_range(recv_x, ws.token_rows, ws.xs, S, H, R, ws.offsets, e_local, st);
  if (rc) return rc;
  TcParams pg{};
  pg.E = e_local;
  pg.K = H;
  pg.Nw = F;
  pg.gs = gs;
  pg.s0 = sg;
  pg.b0 = bg;
  pg.s1 = su;
  pg.b1 = bu;
  pg.offsets = ws.offsets;
  pg.prefix = ws.prefix_gu;
  pg.out = ws.act;
  pg.out_ld = F;
  pg.err = err;
  pg.timeout_ns = 2000000000ll;
  rc = tc_setup(pg, TC_GLU, ws.xs, S, wg, wu);
  if (rc) return rc;
  rc = tc_launch(pg, TC_GLU, st);
  if (rc) return rc;
  TcParams pd{};
  pd.E = e_local;
  pd.K = F;
  pd.Nw = H;
  pd.gs = gs;
  pd.s0 = sd;
  pd.b0 = bd;
  pd.offsets = ws.offsets;
  pd.prefix = ws.prefix_dn;
  pd.out = ws.y;
  pd.out_ld = H;
  pd.err = err;
  pd.timeout_ns = 2000000000ll;
  rc = tc_setup(pd, TC_PLAIN, ws.act, S, wd, nullptr);
  if (rc) return rc;
  rc = tc_launch(pd, TC_PLAIN, st);
  if (rc) return rc;
  return launch_ep_sorted_combine(ws.y, ws.inverse, ws.w, ws.offsets, 0, e_local, partial, R, H, k, st);
}

int combine(const float* ret, const int32_t* pos, uint16_t* out, int T, int H, int nranks, cudaStream_t st) {
  for (int t0 = 0; t0 < T; t0 += 65535) {
    const int n = T - t0 < 65535 ? T - t0 : 65535;
    dim3 grid((H / 4 + 127) / 128, n);
    // ret blocks keep the stride T: shift the token range, not the blocks
    combine_kernel<<<grid, 128, 0, st>>>(ret, pos + (size_t)t0 * nranks, out + (size_t)t0 * H, T, H, nranks);
    B2Q_TRY_CUDA(cudaGetLastError());
  }
  return B2Q_OK;
}

}  // namespace a2a
}  // namespace b2q

using namespace b2q;
using namespace b2q::a2a;

extern "C" {

int b2q_ep_expert_range(int E, int nranks, int rank, int* e_lo, int* e_local) {
  clear_error();
  if (E < 1 || nranks < 1 || nranks > E || rank < 0 || rank >= nranks || !e_lo || !e_local)
    return set_error(B2Q_EINVAL, "ep_expert_range: cannot shard %d experts over %d ranks (rank %d)", E, nranks, rank);
  ep_expert_block(E, nranks, rank, e_lo, e_local);
  return B2Q_OK;
}

size_t b2q_ep_a2a_dispatch_workspace_size(int T, int H, int E, int k, int nranks) {
  if (T < 1 || !shape_ok_dispatch(T, H, E, k, nranks)) return 0;
  return dispatch_layout(nullptr, T, E, k).bytes;
}

int b2q_ep_a2a_dispatch(const uint16_t* x, const uint16_t* wr, uint16_t* send_x, uint32_t* send_meta,
                        int32_t* send_counts, int32_t* pos, uint32_t* idx, float* w, int T, int H, int E, int k,
                        int nranks, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!shape_ok_dispatch(T, H, E, k, nranks))
    return set_error(B2Q_EINVAL, "ep_a2a_dispatch: bad shape (T=%d H=%d E=%d k=%d nranks=%d, at most %d ranks)", T,
                     H, E, k, nranks, MAXR);
  if (!send_counts) return set_error(B2Q_EINVAL, "ep_a2a_dispatch: null send_counts");
  if (T > 0 && (!x || !wr || !send_x || !send_meta || !pos))
    return set_error(B2Q_EINVAL, "ep_a2a_dispatch: null pointer");
  if (T > 0 && (!aligned16(x) || !aligned16(send_x)))
    return set_error(B2Q_EINVAL, "ep_a2a_dispatch: x and send_x must be 16-byte aligned");
  if (T > 0) {
    const size_t need = dispatch_layout(nullptr, T, E, k).bytes;
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
      return set_error(B2Q_EINVAL, "ep_a2a_dispatch: workspace of %zu bytes needed", need);
  }
  int* err = T > 0 ? dispatch_layout(workspace, T, E, k).err : nullptr;
  return dispatch(x, wr, send_x, send_meta, send_counts, pos, idx, w, T, H, E, k, nranks, workspace, err,
                  static_cast<cudaStream_t>(stream));
}

size_t b2q_ep_a2a_experts_workspace_size(int R, int H, int E, int F, int k) {
  if (R < 1 || H < 1 || E < 1 || F < 1 || k < 1) return 0;
  return experts_layout(nullptr, R, H, E, F, k).bytes;
}

int b2q_ep_a2a_experts(const uint16_t* recv_x, const uint32_t* recv_meta, const uint32_t* wg, const uint16_t* sg,
                       const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                       const uint32_t* wd, const uint16_t* sd, const uint16_t* bd, float* partial, int R, int H, int E,
                       int F, int k, int e_lo, int e_local, int group_size, int bits, void* workspace,
                       size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = ep_check_common("ep_a2a_experts", R, H, E, F, k, e_lo, e_local, group_size, bits);
  if (rc) return rc;
  if (R == 0) return B2Q_OK;
  if ((size_t)R * k > 0x7fffffff) return set_error(B2Q_EINVAL, "ep_a2a_experts: %d rows", R);
  if (!tc_shape_ok(F, H, group_size, TC_GLU) || !tc_shape_ok(H, F, group_size, TC_PLAIN))
    return set_error(B2Q_EUNSUPPORTED, "ep_a2a_experts: H %% 128, F %% 64 and K %% (8 * group_size) are required");
  const void* ptrs[] = {recv_x, recv_meta, wg, sg, bg, wu, su, bu, wd, sd, bd, partial};
  for (const void* q : ptrs) {
    if (!q) return set_error(B2Q_EINVAL, "ep_a2a_experts: null pointer");
    if (!aligned16(q)) return set_error(B2Q_EINVAL, "ep_a2a_experts: tensors must be 16-byte aligned");
  }
  const size_t need = experts_layout(nullptr, R, H, E, F, k).bytes;
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "ep_a2a_experts: workspace of %zu bytes needed", need);
  return experts(recv_x, recv_meta, wg, sg, bg, wu, su, bu, wd, sd, bd, partial, R, H, E, F, k, e_lo, e_local,
                 group_size, workspace, experts_layout(workspace, R, H, E, F, k).err, static_cast<cudaStream_t>(stream));
}

int b2q_ep_a2a_combine(const float* ret, const int32_t* pos, uint16_t* out, int T, int H, int nranks, void* stream) {
  clear_error();
  if (T < 0 || H <= 0 || H % 4 || nranks < 1 || nranks > MAXR)
    return set_error(B2Q_EINVAL, "ep_a2a_combine: bad shape (T=%d H=%d nranks=%d)", T, H, nranks);
  if (T == 0) return B2Q_OK;
  if (!ret || !pos || !out) return set_error(B2Q_EINVAL, "ep_a2a_combine: null pointer");
  if (!aligned16(ret) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return set_error(B2Q_EINVAL, "ep_a2a_combine: ret must be 16-byte and out 8-byte aligned");
  return combine(ret, pos, out, T, H, nranks, static_cast<cudaStream_t>(stream));
}

size_t b2q_ep_moe_prefill_a2a_workspace_size(int T_max, int H, int E, int F, int k, int nranks) {
  if (T_max < 1 || F < 1 || !shape_ok_dispatch(T_max, H, E, k, nranks) || (size_t)nranks * T_max * k > 0x7fffffff)
    return 0;
  return full_layout(nullptr, T_max, H, E, F, k, nranks).bytes;
}

int b2q_ep_moe_prefill_a2a(void* comm, const uint16_t* x, const uint16_t* wr, const uint32_t* wg,
                           const uint16_t* sg, const uint16_t* bg, const uint32_t* wu, const uint16_t* su,
                           const uint16_t* bu, const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                           uint16_t* out, uint32_t* idx, float* w, int T, int T_max, int H, int E, int F, int k,
                           int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  EpComm* c = static_cast<EpComm*>(comm);
  const int nranks = c ? c->nranks : 1, me = c ? c->rank : 0;
  if (!shape_ok_dispatch(T, H, E, k, nranks) || T_max < 1 || T > T_max ||
      (size_t)nranks * T_max * k > 0x7fffffff)
    return set_error(B2Q_EINVAL, "ep_moe_prefill_a2a: bad shape (T=%d T_max=%d nranks=%d, at most %d ranks)", T,
                     T_max, nranks, MAXR);
  int e_lo, e_local;
  ep_expert_block(E, nranks, me, &e_lo, &e_local);
  int rc = ep_check_common("ep_moe_prefill_a2a", T, H, E, F, k, e_lo, e_local, group_size, bits);
  if (rc) return rc;
  if (!tc_shape_ok(F, H, group_size, TC_GLU) || !tc_shape_ok(H, F, group_size, TC_PLAIN))
    return set_error(B2Q_EUNSUPPORTED, "ep_moe_prefill_a2a: H %% 128, F %% 64 and K %% (8 * group_size) are required");
  const void* ptrs[] = {wr, wg, sg, bg, wu, su, bu, wd, sd, bd};
  for (const void* q : ptrs)
    if (!q || !aligned16(q)) return set_error(B2Q_EINVAL, "ep_moe_prefill_a2a: null or unaligned weight pointer");
  if (T > 0 && (!x || !out || !aligned16(x) || (reinterpret_cast<uintptr_t>(out) & 7u)))
    return set_error(B2Q_EINVAL, "ep_moe_prefill_a2a: null or unaligned x / out");
  const FullWs ws = full_layout(workspace, T_max, H, E, F, k, nranks);
  if (!workspace || workspace_bytes < ws.bytes || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "ep_moe_prefill_a2a: workspace of %zu bytes needed", ws.bytes);
  if (nranks > 1 && !nccl().p2p_ok)
    return set_error(B2Q_ENCCL, "ep_moe_prefill_a2a: NCCL all-gather / send / recv not available");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // 1. dispatch: route, plan and pack this rank's tokens (block d at row d * T)
  // device-side errors of every phase land in this workspace's header
  rc = dispatch(x, wr, ws.send_x, ws.send_meta, ws.counts, ws.pos, idx, w, T, H, E, k, nranks, ws.dispatch, ws.err,
                st);
  if (rc) return rc;
  // 2. counts of every rank (with its T_max) to every rank: matrix[s][d] = rows s sends to d
  const int32_t tmax = T_max;
  B2Q_TRY_CUDA(cudaMemcpyAsync(ws.counts + nranks, &tmax, sizeof(int32_t), cudaMemcpyHostToDevice, st));
  if (nranks > 1) {
    rc = nccl_check(nccl().all_gather(ws.counts, ws.matrix, nranks + 1, kNcclInt32, c->comm, st),
                    "ep_moe_prefill_a2a: ncclAllGather");
    if (rc) return rc;
  } else {
    B2Q_TRY_CUDA(cudaMemcpyAsync(ws.matrix, ws.counts, sizeof(int32_t) * 2, cudaMemcpyDeviceToDevice, st));
  }
  std::vector<int32_t> m((size_t)nranks * (nranks + 1));
  B2Q_TRY_CUDA(cudaMemcpyAsync(m.data(), ws.matrix, sizeof(int32_t) * m.size(), cudaMemcpyDeviceToHost, st));
  B2Q_TRY_CUDA(cudaStreamSynchronize(st));
  const int W = nranks + 1;
  auto cnt = [&](int s, int d) { return (size_t)m[(size_t)s * W + d]; };
  // every rank checks every rank's receive capacity, so all take the same branch
  for (int d = 0; d < nranks; ++d) {
    size_t rows = 0;
    for (int s = 0; s < nranks; ++s) rows += cnt(s, d);
    if (rows > (size_t)nranks * (size_t)m[(size_t)d * W + nranks])
      return set_error(B2Q_EINVAL, "ep_moe_prefill_a2a: rank %d would receive %zu rows (T_max too small)", d, rows);
  }
  std::vector<size_t> rdispl(nranks + 1, 0);
  for (int s = 0; s < nranks; ++s) rdispl[s + 1] = rdispl[s] + cnt(s, me);
  const size_t R = rdispl[nranks];
  const size_t xrow = (size_t)H * 2, mrow = (size_t)k * 8, prow = (size_t)H * 4;
  // 3. token rows and their (expert, weight) pairs to the expert ranks
  if (cnt(me, me)) {
    B2Q_TRY_CUDA(cudaMemcpyAsync(ws.recv_x + rdispl[me] * H, ws.send_x + (size_t)me * T * H, cnt(me, me) * xrow,
                                 cudaMemcpyDeviceToDevice, st));
    B2Q_TRY_CUDA(cudaMemcpyAsync(ws.recv_meta + rdispl[me] * 2 * k, ws.send_meta + (size_t)me * T * 2 * k,
                                 cnt(me, me) * mrow, cudaMemcpyDeviceToDevice, st));
  }
  if (nranks > 1) {
    const Nccl& n = nccl();
    rc = nccl_check(n.group_start(), "ncclGroupStart");
    if (rc) return rc;
    for (int p = 0; p < nranks && rc == B2Q_OK; ++p) {
      if (p == me) continue;
      if (cnt(me, p)) {
        rc = nccl_check(n.send(ws.send_x + (size_t)p * T * H, cnt(me, p) * xrow, kNcclUint8, p, c->comm, st),
                        "ncclSend");
        if (!rc)
          rc = nccl_check(n.send(ws.send_meta + (size_t)p * T * 2 * k, cnt(me, p) * mrow, kNcclUint8, p, c->comm, st),
                          "ncclSend");
      }
      if (!rc && cnt(p, me)) {
        rc = nccl_check(n.recv(ws.recv_x + rdispl[p] * H, cnt(p, me) * xrow, kNcclUint8, p, c->comm, st),
                        "ncclRecv");
        if (!rc)
          rc = nccl_check(n.recv(ws.recv_meta + rdispl[p] * 2 * k, cnt(p, me) * mrow, kNcclUint8, p, c->comm, st),
                          "ncclRecv");
      }
    }
    const int rc_end = nccl_check(n.group_end(), "ncclGroupEnd");
    if (rc) return rc;
    if (rc_end) return rc_end;
  }
  // 4. the local experts over the received rows
  rc = experts(ws.recv_x, ws.recv_meta, wg, sg, bg, wu, su, bu, wd, sd, bd, ws.partial, (int)R, H, E, F, k, e_lo,
               e_local, group_size, ws.experts, ws.err, st);
  if (rc) return rc;
  // 5. partial rows back to their owners (block p of ret holds what rank p made)
  if (cnt(me, me))
    B2Q_TRY_CUDA(cudaMemcpyAsync(ws.ret + (size_t)me * T * H, ws.partial + rdispl[me] * H, cnt(me, me) * prow,
                                 cudaMemcpyDeviceToDevice, st));
  if (nranks > 1) {
    const Nccl& n = nccl();
    rc = nccl_check(n.group_start(), "ncclGroupStart");
    if (rc) return rc;
    for (int p = 0; p < nranks && rc == B2Q_OK; ++p) {
      if (p == me) continue;
      if (cnt(p, me))
        rc = nccl_check(n.send(ws.partial + rdispl[p] * H, cnt(p, me) * prow, kNcclUint8, p, c->comm, st),
                        "ncclSend");
      if (!rc && cnt(me, p))
        rc = nccl_check(n.recv(ws.ret + (size_t)p * T * H, cnt(me, p) * prow, kNcclUint8, p, c->comm, st),
                        "ncclRecv");
    }
    const int rc_end = nccl_check(n.group_end(), "ncclGroupEnd");
    if (rc) return rc;
    if (rc_end) return rc_end;
  }
  // 6. the weighted partial rows of each token, summed in rank order
  if (T == 0) return B2Q_OK;
  return combine(ws.ret, ws.pos, out, T, H, nranks, st);
}

}  // extern "C"
