// misc.cuh -- packing kernels and the shape-general product kernel (launchers).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

struct GenericArgs {
  const uint16_t* x;
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  const uint32_t* lhs;
  const uint32_t* rhs;
  uint16_t* y;
  int batch, M, N, K, n_x, n_w, gs;
};

int launch_dequantize(const uint32_t* w, const uint16_t* s, const uint16_t* b, uint16_t* out, int64_t rows, int K,
                      int gs, cudaStream_t st);
int launch_quantize(const uint16_t* w, uint32_t* wq, uint16_t* s, uint16_t* b, int64_t rows, int K, int gs,
                    cudaStream_t st);
int launch_generic_qmv(const GenericArgs& a, cudaStream_t st);

}  // namespace b2q
