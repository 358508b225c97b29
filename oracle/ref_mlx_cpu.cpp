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
//   _qmm_dispatch_typed<float>(T*, ...)       backend/cpu/quantized.cpp:341
//       (the same kernel over fp32 operands: every product and the running
//        sum in fp32 -- the reference's own fp32-accumulating arithmetic)
//   quantize<bfloat16_t, uint32_t>(...)        backend/cpu/quantized.cpp:1158
// The gather entry points walk (lhs, rhs) index pairs the way
// _bs_qmm_dispatch_typed does (backend/cpu/quantized.cpp:701-747) for
// row-contiguous operands (elem_to_loc(i) == i) and call the reference's
// pointer-level _qmm_dispatch_typed<T> for each pair; the array-level
// function itself needs MLX's array class, which is not compiled here.
// The output goes to oracle/_ref/libmlxref.so (git-ignored).  Only tests/,
// bench.py's CPU-baseline legs and __graft_entry__.smoke() load it.
#include "mlx/backend/cpu/quantized.cpp"

#include <cstdint>
#include <cstring>

#define MLXREF_API __attribute__((visibility("default")))

// gather_qmm over `pairs` index pairs: y[i] = x[lhs[i]] . dequant(w[rhs[i]])^T,
// x [n_x, M, K], w [n_w, N, K*bits/32], scales / biases [n_w, N, K/gs],
// y [pairs, M, N]; indices outside [0, n_x) / [0, n_w) are refused (the
// reference does not check them).
template <typename T>
static int gather_pairs(
    T* y,
    const T* x,
    const uint32_t* w,
    const T* scales,
    const T* biases,
    const uint32_t* lhs,
    const uint32_t* rhs,
    int pairs,
    int M,
    int N,
    int K,
    int n_x,
    int n_w,
    int group_size,
    int bits) {
  using namespace mlx::core;
  const long long w_els = (long long)N * (K * bits / 32);
  const long long g_els = (long long)N * (K / group_size);
  try {
    for (int i = 0; i < pairs; i++) {
      const uint32_t x_idx = lhs ? lhs[i] : (uint32_t)(i % n_x);
      const uint32_t w_idx = rhs ? rhs[i] : (uint32_t)(i % n_w);
      if (x_idx >= (uint32_t)n_x || w_idx >= (uint32_t)n_w) return 2;
      _qmm_dispatch_typed<T>(
          y + (long long)i * M * N,
          x + (long long)x_idx * M * K,
          w + (long long)w_idx * w_els,
          scales + (long long)w_idx * g_els,
          biases + (long long)w_idx * g_els,
          M,
          N,
          K,
          group_size,
          bits,
          true);
    }
  } catch (...) {
    return 1;
  }
  return 0;
}

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

// y[M,N] = x[M,K] . dequant(w)^T with fp32 x, scales, biases and result: the
// reference kernel instantiated for float (fp32 accumulation).
MLXREF_API int mlxref_qmm_f32(
    float* y,
    const float* x,
    const uint32_t* w,
    const float* scales,
    const float* biases,
    int M,
    int N,
    int K,
    int group_size,
    int bits,
    int transposed) {
  using namespace mlx::core;
  try {
    _qmm_dispatch_typed<float>(
        y, x, w, scales, biases, M, N, K, group_size, bits, transposed != 0);
  } catch (...) {
    return 1;
  }
  return 0;
}

MLXREF_API int mlxref_gather_qmm_bf16(
    uint16_t* y,
    const uint16_t* x,
    const uint32_t* w,
    const uint16_t* scales,
    const uint16_t* biases,
    const uint32_t* lhs,
    const uint32_t* rhs,
    int pairs,
    int M,
    int N,
    int K,
    int n_x,
    int n_w,
    int group_size,
    int bits) {
  using mlx::core::bfloat16_t;
  return gather_pairs<bfloat16_t>(
      reinterpret_cast<bfloat16_t*>(y),
      reinterpret_cast<const bfloat16_t*>(x),
      w,
      reinterpret_cast<const bfloat16_t*>(scales),
      reinterpret_cast<const bfloat16_t*>(biases),
      lhs, rhs, pairs, M, N, K, n_x, n_w, group_size, bits);
}

MLXREF_API int mlxref_gather_qmm_f32(
    float* y,
    const float* x,
    const uint32_t* w,
    const float* scales,
    const float* biases,
    const uint32_t* lhs,
    const uint32_t* rhs,
    int pairs,
    int M,
    int N,
    int K,
    int n_x,
    int n_w,
    int group_size,
    int bits) {
  return gather_pairs<float>(
      y, x, w, scales, biases, lhs, rhs, pairs, M, N, K, n_x, n_w, group_size, bits);
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
