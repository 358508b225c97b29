// sort.cu -- stable counting sort of routed assignments by expert.
//
// The unique stable permutation that groups R = T*k assignment slots by
// expert id (Runner/FastModel/TrackPrefillSort.swift:17-44 argues MLX's
// argsort is stable, so this permutation equals argSort(flatIDs)); outputs
// sorted_ids[p], token_rows[p] = order[p] / k, inverse[order[p]] = p and the
// per-expert offsets [E + 1]. One CTA of 1024 threads walks the slots in
// chunks of 1024; inside a chunk, ranks among equal ids come from
// __match_any_sync within a warp plus per-warp counts of earlier warps, so the
// order among equal ids is slot order.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"
#include "prefill.cuh"

namespace b2q {

constexpr int SORT_THREADS = 1024;
constexpr int SORT_WARPS = SORT_THREADS / 32;

__global__ void __launch_bounds__(SORT_THREADS, 1)
    expert_sort_kernel(const uint32_t* __restrict__ ids, uint32_t* __restrict__ sorted_ids,
                       uint32_t* __restrict__ token_rows, uint32_t* __restrict__ inverse,
                       uint32_t* __restrict__ offsets, int R, int E, int k, int* err) {
  extern __shared__ unsigned sm[];
  unsigned* base = sm;         // [E] running bucket start
  unsigned* wcnt = sm + E;     // [SORT_WARPS][E] counts of the current chunk
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E; e += SORT_THREADS) base[e] = 0;
  for (int i = tid; i < SORT_WARPS * E; i += SORT_THREADS) wcnt[i] = 0;
  __syncthreads();
  for (int i = tid; i < R; i += SORT_THREADS) {
    const uint32_t e = __ldg(ids + i);
    if (e < (uint32_t)E)
      atomicAdd(&base[e], 1u);
    else
      record_error(err, B2Q_EINVAL);
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scan of the E bucket sizes: each lane owns a contiguous run
    const int per = (E + 31) / 32;
    const int e0 = lane * per, e1 = min(E, e0 + per);
    unsigned run = 0;
    for (int e = e0; e < e1; ++e) run += base[e];
    unsigned incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    unsigned acc = incl - run;
    for (int e = e0; e < e1; ++e) {
      const unsigned c = base[e];
      base[e] = acc;
      if (offsets) offsets[e] = acc;
      acc += c;
    }
    if (lane == 31 && offsets) offsets[E] = incl;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c0 = 0; c0 < R; c0 += SORT_THREADS) {
    const int i = c0 + tid;
    uint32_t e = (i < R) ? __ldg(ids + i) : 0xffffffffu;
    if (e >= (uint32_t)E) e = 0xffffffffu;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const unsigned rank = __popc(peers & lt_mask);
    const bool valid = e != 0xffffffffu;
    if (valid && rank == 0) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    if (valid) {
      unsigned pre = 0;
      for (int w = 0; w < warp; ++w) pre += wcnt[w * E + e];
      const unsigned pos = base[e] + pre + rank;
      if (sorted_ids) sorted_ids[pos] = e;
      if (token_rows) token_rows[pos] = (uint32_t)(i / k);
      if (inverse) inverse[i] = pos;
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += SORT_THREADS) {
      unsigned tot = 0;
      for (int w = 0; w < SORT_WARPS; ++w) {
        tot += wcnt[w * E + ee];
        wcnt[w * E + ee] = 0;
      }
      base[ee] += tot;
    }
    __syncthreads();
  }
}

int launch_expert_sort(const uint32_t* ids, uint32_t* sorted_ids, uint32_t* token_rows, uint32_t* inverse,
                       uint32_t* offsets, int R, int E, int k, int* err, cudaStream_t st) {
  const size_t smem = sizeof(unsigned) * (size_t)E * (1 + SORT_WARPS);
  B2Q_TRY_CUDA(cudaFuncSetAttribute(expert_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  expert_sort_kernel<<<1, SORT_THREADS, smem, st>>>(ids, sorted_ids, token_rows, inverse, offsets, R, E, k, err);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // namespace b2q
