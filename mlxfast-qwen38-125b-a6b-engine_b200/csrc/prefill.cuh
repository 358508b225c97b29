// prefill.cuh -- the prefill side: expert sort and tensor-core gather GEMMs.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

// True when the tensor-core gather GEMM handles this product.
bool prefill_qmm_eligible(int batch, int M, int N, int K, int gs, const void* x, const void* w, const void* s,
                          const void* b, const void* y);
int launch_prefill_gather_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                              const uint32_t* lhs, const uint32_t* rhs, uint16_t* y, int batch, int M, int N, int K,
                              int n_x, int n_w, int gs, int sorted, cudaStream_t st);

// Stable counting sort of R expert ids into E buckets (one CTA).
int launch_expert_sort(const uint32_t* ids, uint32_t* sorted_ids, uint32_t* token_rows, uint32_t* inverse,
                       uint32_t* offsets, int R, int E, int k, int* err, cudaStream_t st);

}  // namespace b2q
