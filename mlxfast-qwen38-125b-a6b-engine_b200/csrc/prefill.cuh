// prefill.cuh -- the prefill side: expert sort and tensor-core gather GEMMs.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

// True when the tensor-core gather GEMM handles this product.
bool prefill_qmm_eligible(int batch, int M, int N, int K, int gs, const void* x, const void* w, const void* s,
                          const void* b, const void* y);
// workspace == nullptr: the call takes a stream-ordered temporary of
// prefill_gather_qmm_ws_bytes() bytes and frees it at its end.
size_t prefill_gather_qmm_ws_bytes(int batch, int M, int K, int n_w);
int launch_prefill_gather_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                              const uint32_t* lhs, const uint32_t* rhs, uint16_t* y, int batch, int M, int N, int K,
                              int n_x, int n_w, int gs, int sorted, void* workspace, size_t workspace_bytes,
                              cudaStream_t st);

// Stable counting sort of R expert ids into E buckets (one CTA).
int launch_expert_sort(const uint32_t* ids, uint32_t* sorted_ids, uint32_t* token_rows, uint32_t* inverse,
                       uint32_t* offsets, int R, int E, int k, int* err, cudaStream_t st);

}  // namespace b2q
