// ref_mlx_cpu.cpp -- C entry points over the reference's OWN MLX CPU quantized
// kernels, compiled from the reference tree where it lies (never copied).
//
// Test infrastructure only: this translation unit #includes
//   Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/cpu/quantized.cpp
// from the reference checkout (path given with -I by oracle/Makefile), so its
// anonymous-namespace kernels are visible here and are called unchanged:
//   _qmm_dispatch_typed<bfloat16_t>(T*, ...)  backend/cpu/quantized.cpp:341
//       (pointer-level; on x86 simd::max_size == 1 so the scalar `_qmm_t`
//        at backend/cpu/quantized.cpp:155 runs, with a bf16 running sum)
//   quantize<bfloat16_t, uint32_t>(...)        backend/cpu/quantized.cpp:1158
// The output goes to oracle/_ref/libmlxref.so (git-ignored).  Only tests/,
// bench.py's CPU-baseline legs and __graft_entry__.smoke() load it.
#include "mlx/backend/cpu/quantized.cpp"

#include <cstdint>
#include <cstring>

#define MLXREF_API __attribute__((visibility("default")))

extern "C" {

// y[M,N] = x[M,K] . dequant(w)^T  (transposed=1) in MLX's CPU arithmetic.
// All buffers are host memory; bf16 values are passed as raw uint16 bits.
MLXREF_API int mlxref_qmm_bf16(
    uint16_t* y,
    const uint16_t* x,
    const uint32_t* w,
    const uint16_t* scales,
    const uint16_t* biases,
    int M,
    int N,
    int K,
    int group_size,
    int bits,
    int transposed) {
  using namespace mlx::core;
  try {
    _qmm_dispatch_typed<bfloat16_t>(
        reinterpret_cast<bfloat16_t*>(y),
        reinterpret_cast<const bfloat16_t*>(x),
        w,
        reinterpret_cast<const bfloat16_t*>(scales),
        reinterpret_cast<const bfloat16_t*>(biases),
        M,
        N,
        K,
        group_size,
        bits,
        transposed != 0);
  } catch (...) {
    return 1;
  }
  return 0;
}

// MLX affine quantize of a bf16 matrix (n_el elements, groups along the last
// axis): packed uint32 words, bf16 scales and biases.
MLXREF_API int mlxref_quantize_bf16(
    const uint16_t* w,
    uint32_t* wq,
    uint16_t* scales,
    uint16_t* biases,
    int bits,
    int group_size,
    long long n_el) {
  using namespace mlx::core;
  try {
    quantize<bfloat16_t, uint32_t>(
        reinterpret_cast<const bfloat16_t*>(w),
        wq,
        reinterpret_cast<bfloat16_t*>(scales),
        reinterpret_cast<bfloat16_t*>(biases),
        bits,
        group_size,
        static_cast<size_t>(n_el));
  } catch (...) {
    return 1;
  }
  return 0;
}

} // extern "C"
