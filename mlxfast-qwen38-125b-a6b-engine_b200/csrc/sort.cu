// sort.cu -- stable counting sort of routed assignments by expert.
//
// The unique stable permutation that groups R = T*k assignment slots by
// expert id (Runner/FastModel/TrackPrefillSort.swift:17-44 argues MLX's
// argsort is stable, so this permutation equals argSort(flatIDs)); outputs
// sorted_ids[p], token_rows[p] = order[p] / k, inverse[order[p]] = p and the
// per-expert offsets [E + 1].
//
// One CTA of 32 warps; warp w owns the contiguous slot range
// [w * R / 32, (w + 1) * R / 32), so slot order is (warp, position in the
// warp's range). Pass 1: every warp counts its range per expert (ranks inside
// 32 consecutive slots from __match_any_sync, the lowest lane of each peer set
// adds the set's size). Scan: base[w][e] = the counts of e in warps before w;
// offsets = exclusive scan of the per-expert totals. Pass 2: every warp walks
// its range again, placing slot i at offsets[e] + base[w][e] + (earlier slots
// of e in the warp's range). Three block barriers in all.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"
#include "prefill.cuh"

namespace b2q {

constexpr int SORT_THREADS = 1024;
constexpr int SORT_WARPS = SORT_THREADS / 32;
constexpr int BATCH = 8;  // chunks of 32 ids loaded together

__global__ void __launch_bounds__(SORT_THREADS, 1)
    expert_sort_kernel(const uint32_t* __restrict__ ids, uint32_t* __restrict__ sorted_ids,
                       uint32_t* __restrict__ token_rows, uint32_t* __restrict__ inverse,
                       uint32_t* __restrict__ offsets, int R, int E, int k, int* err) {
  extern __shared__ unsigned sm[];
  unsigned* cnt = sm;                   // [SORT_WARPS][E] counts, then running positions
  unsigned* tot = sm + SORT_WARPS * E;  // [E] per-expert totals, then offsets
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i = tid; i < SORT_WARPS * E; i += SORT_THREADS) cnt[i] = 0;
  __syncthreads();
  // this warp's slot range
  const int per = (R + SORT_WARPS - 1) / SORT_WARPS;
  const int i0 = min(R, warp * per), i1 = min(R, i0 + per);
  unsigned* wc = cnt + warp * E;
  // ---- pass 1: counts per expert of the warp's range (the ids of BATCH
  // chunks of 32 are loaded together: one memory latency per batch) ----
  for (int b0 = i0; b0 < i1; b0 += 32 * BATCH) {
    uint32_t ev[BATCH];
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int i = b0 + 32 * j + lane;
      ev[j] = (i < i1) ? __ldg(ids + i) : 0xffffffffu;
    }
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int i = b0 + 32 * j + lane;
      uint32_t e = ev[j];
      if (i < i1 && e >= (uint32_t)E) {
        record_error(err, B2Q_EINVAL);
        e = 0xffffffffu;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e != 0xffffffffu && (peers & lt_mask) == 0) wc[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  // ---- scan: base[w][e] over warps, offsets over experts ----
  for (int e = tid; e < E; e += SORT_THREADS) {
    unsigned run = 0;
    for (int w = 0; w < SORT_WARPS; ++w) {
      const unsigned c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  __syncthreads();
  if (warp == 0) {
    const int pe = (E + 31) / 32;
    const int e0 = lane * pe, e1 = min(E, e0 + pe);
    unsigned run = 0;
    for (int e = e0; e < e1; ++e) run += tot[e];
    unsigned incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    unsigned acc = incl - run;
    for (int e = e0; e < e1; ++e) {
      const unsigned c = tot[e];
      tot[e] = acc;
      if (offsets) offsets[e] = acc;
      acc += c;
    }
    if (lane == 31 && offsets) offsets[E] = incl;
  }
  __syncthreads();
  // ---- pass 2: place the warp's range in slot order ----
  for (int b0 = i0; b0 < i1; b0 += 32 * BATCH) {
    uint32_t ev[BATCH];
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int i = b0 + 32 * j + lane;
      ev[j] = (i < i1) ? __ldg(ids + i) : 0xffffffffu;
    }
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int i = b0 + 32 * j + lane;
      uint32_t e = ev[j];
      if (e >= (uint32_t)E) e = 0xffffffffu;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e != 0xffffffffu) {
        const unsigned pos = tot[e] + wc[e] + __popc(peers & lt_mask);
        if (sorted_ids) sorted_ids[pos] = e;
        if (token_rows) token_rows[pos] = (uint32_t)(i / k);
        if (inverse) inverse[i] = pos;
      }
      __syncwarp();
      if (e != 0xffffffffu && (peers & lt_mask) == 0) wc[e] += __popc(peers);
      __syncwarp();
    }
  }
}

int launch_expert_sort(const uint32_t* ids, uint32_t* sorted_ids, uint32_t* token_rows, uint32_t* inverse,
                       uint32_t* offsets, int R, int E, int k, int* err, cudaStream_t st) {
  const size_t smem = sizeof(unsigned) * (size_t)E * (SORT_WARPS + 1);
  B2Q_TRY_CUDA(cudaFuncSetAttribute(expert_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  expert_sort_kernel<<<1, SORT_THREADS, smem, st>>>(ids, sorted_ids, token_rows, inverse, offsets, R, E, k, err);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // namespace b2q
