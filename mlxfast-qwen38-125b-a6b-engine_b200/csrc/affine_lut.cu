// affine_lut.cu -- load-time pair index of the affine metadata of a 4-bit
// tensor, and the one-row product that reads its metadata through it.
//
// Reference: Runner/FastModel/TrackAffineLUT.swift:1-110 (TrackAffineLUT.build,
// buildOnDevice, verified) and :114-368 (TrackLUTGemv). A tensor whose groups
// carry only a few thousand distinct (scale, bias) bf16 bit pairs is given a
// table of those pairs (entry = scale_bits | bias_bits << 16) and a u16 index
// per group; the one-token product then streams 2 bytes of metadata per group
// instead of 4. The table order is the reference's: first occurrence for
// tensors of fewer than 2^20 groups (its host loop), ascending pair value
// otherwise (its on-device sort and run ranks). Every group is checked to
// reconstruct its exact bit pair before the index is reported usable; a tensor
// with more distinct pairs than the limit, or whose round trip fails, is
// reported as not indexed (count -1), as the reference returns nil.
//
// Build on the device, in one region of caller workspace:
//   1. insert every pair into an open-addressing hash set (64-bit slots,
//      key = pair + 1, 0 = empty), keeping the first group index of each pair
//      (first-occurrence order only);
//   2. compact the occupied slots into a list; the host reads the count;
//   3. rank each distinct pair among all of them (by value or by first
//      occurrence: the keys are distinct, so ranks are a permutation) and
//      write table[rank] = pair, slot -> rank;
//   4. index[g] = rank of group g's pair (a second probe);
//   5. count groups with table[index[g]] != pair; the host reads it.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "decode2.cuh"
#include "host.hpp"

namespace b2q {
namespace lut {

constexpr int MAX_ENTRIES = 65536;  // a u16 index names at most 2^16 pairs
constexpr int64_t FIRST_ORDER_LIMIT = int64_t(1) << 20;  // below: first-occurrence order

__device__ __forceinline__ uint32_t pair_of(const uint16_t* s, const uint16_t* b, int64_t g) {
  return (uint32_t)s[g] | ((uint32_t)b[g] << 16);
}

// 32-bit mixing function (the finaliser of MurmurHash3, a published hash)
__device__ __forceinline__ uint32_t mix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h;
}

struct Ws {
  unsigned long long* keys;  // [cap]
  uint32_t* first;           // [cap]
  uint32_t* srank;           // [cap]
  uint32_t* lkey;            // [max]
  uint32_t* lfirst;          // [max]
  uint32_t* lslot;           // [max]
  uint32_t* ctr;             // [0] listed pairs, [1] not indexable, [2] round-trip mismatches, [3] inserted pairs
  size_t bytes;
};

static int cap_for(int max_entries) {
  int cap = 1024;
  while (cap < 4 * max_entries) cap <<= 1;
  return cap;
}

static Ws layout(void* base, int max_entries) {
  auto a256 = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t cap = (size_t)cap_for(max_entries);
  char* b = static_cast<char*>(base);
  Ws w{};
  size_t off = 0;
  w.ctr = reinterpret_cast<uint32_t*>(b + off);
  off = 256;
  w.keys = reinterpret_cast<unsigned long long*>(b + off);
  off = a256(off + 8 * cap);
  w.first = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * cap);
  w.srank = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * cap);
  w.lkey = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * (size_t)max_entries);
  w.lfirst = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * (size_t)max_entries);
  w.lslot = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * (size_t)max_entries);
  w.bytes = off;
  return w;
}

// 1. Insert. A slot holding this key already is read first (most groups) so
// only a pair's first arrivals contend on the compare-and-swap. The set is 4x
// the entry limit, so probe sequences stay short while the pairs fit; once more
// pairs than the limit were inserted, or a probe runs past PROBE_LIMIT slots,
// the tensor is not indexed and every thread stops at its next group.
constexpr uint32_t PROBE_LIMIT = 512;

__global__ void insert_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int64_t G, Ws w,
                              uint32_t mask, int max_entries, int track_first) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < G; g += (int64_t)gridDim.x * blockDim.x) {
    if (__ldcg(&w.ctr[1])) return;
    const uint32_t p = pair_of(s, b, g);
    const unsigned long long key = (unsigned long long)p + 1ull;
    uint32_t h = mix32(p) & mask;
    bool placed = false;
    for (uint32_t i = 0; i < PROBE_LIMIT; ++i) {
      unsigned long long cur = __ldcg(&w.keys[h]);
      if (cur == 0ull) {
        cur = atomicCAS(&w.keys[h], 0ull, key);
        if (cur == 0ull && atomicAdd(&w.ctr[3], 1u) >= (uint32_t)max_entries) atomicOr(&w.ctr[1], 1u);
      }
      if (cur == 0ull || cur == key) {
        placed = true;
        break;
      }
      h = (h + 1) & mask;
    }
    if (!placed) {
      atomicOr(&w.ctr[1], 1u);
      return;
    }
    if (track_first && (uint32_t)g < __ldcg(&w.first[h])) atomicMin(&w.first[h], (uint32_t)g);
  }
}

// 2. Compact the occupied slots (list order is arbitrary; ranks fix the order).
__global__ void compact_kernel(Ws w, uint32_t cap, int max_entries) {
  const uint32_t h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= cap) return;
  const unsigned long long k = w.keys[h];
  if (k == 0ull) return;
  const uint32_t pos = atomicAdd(&w.ctr[0], 1u);
  if (pos < (uint32_t)max_entries) {
    w.lkey[pos] = (uint32_t)(k - 1ull);
    w.lfirst[pos] = w.first[h];
    w.lslot[pos] = h;
  }
}

// 3. Rank of entry i = number of entries ordered before it (by value, or by
// first occurrence); the list is staged through shared memory in tiles.
__global__ void rank_kernel(Ws w, int n, int by_first, uint32_t* __restrict__ table) {
  constexpr int TILE = 4096;
  __shared__ uint32_t tile[TILE];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t* ord = by_first ? w.lfirst : w.lkey;
  const uint32_t mine = i < n ? ord[i] : 0u;
  uint32_t rank = 0;
  for (int t0 = 0; t0 < n; t0 += TILE) {
    const int m = min(TILE, n - t0);
    __syncthreads();
    for (int j = threadIdx.x; j < m; j += blockDim.x) tile[j] = ord[t0 + j];
    __syncthreads();
    if (i < n)
      for (int j = 0; j < m; ++j) rank += tile[j] < mine ? 1u : 0u;
  }
  if (i < n) {
    table[rank] = w.lkey[i];
    w.srank[w.lslot[i]] = rank;
  }
}

// 4. index[g] = rank of group g's pair; 5. round-trip check.
__global__ void index_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int64_t G, Ws w,
                             uint32_t mask, uint16_t* __restrict__ index) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < G; g += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t p = pair_of(s, b, g);
    const unsigned long long key = (unsigned long long)p + 1ull;
    uint32_t h = mix32(p) & mask;
    uint32_t r = 0xffffffffu;
    for (uint32_t i = 0; i < PROBE_LIMIT; ++i) {
      const unsigned long long cur = w.keys[h];
      if (cur == key) {
        r = w.srank[h];
        break;
      }
      if (cur == 0ull) break;
      h = (h + 1) & mask;
    }
    index[g] = (uint16_t)r;  // a pair not found leaves a wrong index: the check below counts it
  }
}

__global__ void verify_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int64_t G,
                              const uint16_t* __restrict__ index, const uint32_t* __restrict__ table, int count,
                              uint32_t* __restrict__ mismatches) {
  uint32_t bad = 0;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < G; g += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t i = index[g];
    bad += (i >= (uint32_t)count || table[i] != pair_of(s, b, g)) ? 1u : 0u;
  }
  if (bad) atomicAdd(mismatches, bad);
}

__global__ void pad_kernel(uint32_t* table, int from, int to) {
  const int i = from + (int)threadIdx.x;
  if (i < to) table[i] = 0u;
}

__global__ void expand_kernel(const uint16_t* __restrict__ index, const uint32_t* __restrict__ table, int64_t G,
                              uint16_t* __restrict__ s, uint16_t* __restrict__ b) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < G; g += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t p = table[index[g]];
    s[g] = (uint16_t)(p & 0xffffu);
    b[g] = (uint16_t)(p >> 16);
  }
}

static int grid_for(int64_t n, int threads) {
  DeviceInfo di;
  const int sms = device_info(&di) == B2Q_OK ? di.sm_count : 148;
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, (int64_t)sms * 8));
}

}  // namespace lut
}  // namespace b2q

using namespace b2q;

extern "C" {

size_t b2q_affine_lut_workspace_size(int max_entries) {
  if (max_entries < 1 || max_entries > lut::MAX_ENTRIES) return 0;
  return lut::layout(nullptr, max_entries).bytes;
}

int b2q_affine_lut_build(const uint16_t* scales, const uint16_t* biases, int64_t n_groups, uint16_t* index,
                         uint32_t* table, int max_entries, int* count_out, void* workspace, size_t workspace_bytes,
                         void* stream) {
  clear_error();
  if (!count_out) return set_error(B2Q_EINVAL, "affine_lut_build: null count_out");
  *count_out = -1;
  if (n_groups <= 0 || n_groups >= (int64_t(1) << 31) || max_entries < 4 || max_entries > lut::MAX_ENTRIES ||
      max_entries % 4)
    return set_error(B2Q_EINVAL, "affine_lut_build: bad size (groups %lld, max_entries %d: 4..65536, a multiple of 4)",
                     (long long)n_groups, max_entries);
  if (!scales || !biases || !index || !table || !workspace)
    return set_error(B2Q_EINVAL, "affine_lut_build: null pointer");
  const lut::Ws w = lut::layout(workspace, max_entries);
  if (workspace_bytes < w.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(B2Q_EINVAL, "affine_lut_build: workspace of %zu bytes (256-byte aligned) needed", w.bytes);
  if (!aligned16(table)) return set_error(B2Q_EINVAL, "affine_lut_build: table must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t cap = (uint32_t)lut::cap_for(max_entries);
  const int by_first = n_groups < lut::FIRST_ORDER_LIMIT ? 1 : 0;
  B2Q_TRY_CUDA(cudaMemsetAsync(w.ctr, 0, 256, st));
  B2Q_TRY_CUDA(cudaMemsetAsync(w.keys, 0, 8 * (size_t)cap, st));
  B2Q_TRY_CUDA(cudaMemsetAsync(w.first, 0xff, 4 * (size_t)cap, st));
  lut::insert_kernel<<<lut::grid_for(n_groups, 256), 256, 0, st>>>(scales, biases, n_groups, w, cap - 1,
                                                                     max_entries, by_first);
  lut::compact_kernel<<<(cap + 255) / 256, 256, 0, st>>>(w, cap, max_entries);
  B2Q_TRY_CUDA(cudaGetLastError());
  uint32_t hc[2] = {0, 0};
  B2Q_TRY_CUDA(cudaMemcpyAsync(hc, w.ctr, 8, cudaMemcpyDeviceToHost, st));
  B2Q_TRY_CUDA(cudaStreamSynchronize(st));
  if (hc[1] || hc[0] > (uint32_t)max_entries) return B2Q_OK;  // more distinct pairs than the limit: not indexed
  const int n = (int)hc[0];
  lut::rank_kernel<<<(n + 255) / 256, 256, 0, st>>>(w, n, by_first, table);
  lut::pad_kernel<<<1, 4, 0, st>>>(table, n, std::min((n + 3) / 4 * 4, max_entries));
  lut::index_kernel<<<lut::grid_for(n_groups, 256), 256, 0, st>>>(scales, biases, n_groups, w, cap - 1, index);
  lut::verify_kernel<<<lut::grid_for(n_groups, 256), 256, 0, st>>>(scales, biases, n_groups, index, table, n,
                                                                     w.ctr + 2);
  B2Q_TRY_CUDA(cudaGetLastError());
  uint32_t bad = 0;
  B2Q_TRY_CUDA(cudaMemcpyAsync(&bad, w.ctr + 2, 4, cudaMemcpyDeviceToHost, st));
  B2Q_TRY_CUDA(cudaStreamSynchronize(st));
  if (bad == 0) *count_out = n;  // fail closed: any group that does not reconstruct its bits
  return B2Q_OK;
}

int b2q_affine_lut_expand(const uint16_t* index, const uint32_t* table, int64_t n_groups, uint16_t* scales,
                          uint16_t* biases, void* stream) {
  clear_error();
  if (n_groups < 0) return set_error(B2Q_EINVAL, "affine_lut_expand: bad size");
  if (n_groups == 0) return B2Q_OK;
  if (!index || !table || !scales || !biases) return set_error(B2Q_EINVAL, "affine_lut_expand: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  lut::expand_kernel<<<lut::grid_for(n_groups, 256), 256, 0, st>>>(index, table, n_groups, scales, biases);
  return cuda_check(cudaGetLastError(), "affine_lut_expand");
}

int b2q_qmv_lut(const uint16_t* x, const uint32_t* w, const uint16_t* index, const uint32_t* table, int count,
                uint16_t* y, int N, int K, int group_size, int bits, void* stream) {
  clear_error();
  if (bits != 4) return set_error(B2Q_EUNSUPPORTED, "qmv_lut: bits=%d (only 4-bit)", bits);
  if (N <= 0 || K <= 0 || count < 1 || count > lut::MAX_ENTRIES) return set_error(B2Q_EINVAL, "qmv_lut: bad shape");
  if (!x || !w || !index || !table || !y) return set_error(B2Q_EINVAL, "qmv_lut: null pointer");
  if (!d2_qmv_lut_eligible(N, K, group_size, count, x, w, index, table) || !aligned16(y))
    return set_error(B2Q_EUNSUPPORTED,
                     "qmv_lut: shape outside the kernel (N %% 16 == 0, N >= 32, K %% 512 == 0, gs 32/64/128, "
                     "16-byte aligned tensors, a table that fits in shared memory)");
  return d2_qmv_lut(x, w, index, table, count, y, N, K, group_size, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
