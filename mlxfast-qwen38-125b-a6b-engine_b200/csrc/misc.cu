// misc.cu -- packing kernels and the shape-general product kernel.
//
//   dequantize  : the Metal affine dequantizer's arithmetic,
//                 bf16(fp32(s)*q + fp32(b)) (Vendor/mlx-swift/Source/Cmlx/mlx/mlx/
//                 backend/metal/kernels/quantized.h:3314-3373 and :485-530).
//   quantize    : MLX affine quantize (.../backend/cpu/quantized.cpp:1158-1236),
//                 same fp32 operations in the same order, one thread per group.
//   generic_qmv : y = x . dequant(w)^T for shapes outside the streaming
//                 engine's fast path (any K multiple of the group size); per
//                 group s*sum(x*q) + b*sum(x) in fp32 like the Metal qmv.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"
#include "misc.cuh"

namespace b2q {

__global__ void dequantize_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                  const uint16_t* __restrict__ b, uint16_t* __restrict__ out, int64_t n_words,
                                  int K, int gs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  const int wpr = K / 8;
  const int64_t row = i / wpr;
  const int kw = (int)(i % wpr);
  const int G = K / gs;
  const int64_t gidx = row * G + (kw * 8) / gs;
  const float sc = bf2f(__ldg(s + gidx)), bi = bf2f(__ldg(b + gidx));
  const uint32_t W = __ldg(w + i);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __fadd_rn(__fmul_rn(sc, (float)((W >> (8 * j)) & 0xF)), bi);
    const float hi = __fadd_rn(__fmul_rn(sc, (float)((W >> (8 * j + 4)) & 0xF)), bi);
    o[j] = (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
  }
  reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void quantize_kernel(const uint16_t* __restrict__ w, uint32_t* __restrict__ wq, uint16_t* __restrict__ s,
                                uint16_t* __restrict__ b, int64_t n_groups, int gs) {
  const int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= n_groups) return;
  const uint16_t* wg = w + gi * gs;
  const float n_bins = 15.0f, eps = 1e-7f;
  float w_min = INFINITY, w_max = -INFINITY;
  for (int j = 0; j < gs; ++j) {
    const float v = bf2f(wg[j]);
    w_max = (w_max < v) ? v : w_max;
    w_min = (v < w_min) ? v : w_min;
  }
  const bool mask = fabsf(w_min) > fabsf(w_max);
  float scale = __fdiv_rn(__fsub_rn(w_max, w_min), n_bins);
  scale = (scale < eps) ? eps : scale;
  scale = mask ? scale : -scale;
  const float edge = mask ? w_min : w_max;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  uint32_t* dst = wq + gi * (gs / 8);
  for (int j = 0; j < gs / 8; ++j) {
    uint32_t word = 0;
    for (int kk = 0; kk < 8; ++kk) {
      float q = rintf(__fdiv_rn(__fsub_rn(bf2f(wg[j * 8 + kk]), bias), scale));
      q = (q < 0.0f) ? 0.0f : q;
      q = (n_bins < q) ? n_bins : q;
      word |= (uint32_t)q << (4 * kk);
    }
    dst[j] = word;
  }
  s[gi] = f2bf(scale);
  b[gi] = f2bf(bias);
}

// One warp per (item, output row); up to 8 tokens of the item at a time.
__global__ void generic_qmv_kernel(GenericArgs a) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)a.batch * a.N) return;
  const int item = (int)(gw / a.N), n = (int)(gw % a.N);
  const uint32_t xi = a.lhs ? __ldg(a.lhs + item) : (uint32_t)item;
  const uint32_t e = a.rhs ? __ldg(a.rhs + item) : (uint32_t)item;
  const bool ok = xi < (uint32_t)a.n_x && e < (uint32_t)a.n_w;
  const int G = a.K / a.gs;
  const int wpr = a.K / 8;
  const uint32_t* wrow = a.w + ((size_t)e * a.N + n) * wpr;
  const uint16_t* srow = a.s + ((size_t)e * a.N + n) * G;
  const uint16_t* brow = a.b + ((size_t)e * a.N + n) * G;
  for (int m0 = 0; m0 < a.M; m0 += 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int mc = min(8, a.M - m0);
    if (ok) {
      for (int g = lane; g < G; g += 32) {
        const float sc = bf2f(__ldg(srow + g)), bi = bf2f(__ldg(brow + g));
        for (int m = 0; m < mc; ++m) {
          const uint16_t* xr = a.x + ((size_t)xi * a.M + m0 + m) * a.K + (size_t)g * a.gs;
          float sq = 0.0f, sx = 0.0f;
          for (int kw = 0; kw < a.gs / 8; ++kw) {
            const uint32_t W = __ldg(wrow + (size_t)g * (a.gs / 8) + kw);
            const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr) + kw);
            const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float x0 = __uint_as_float(xa[j] << 16), x1 = __uint_as_float(xa[j] & 0xffff0000u);
              sq += x0 * (float)((W >> (8 * j)) & 0xF) + x1 * (float)((W >> (8 * j + 4)) & 0xF);
              sx += x0 + x1;
            }
          }
          acc[m] += sc * sq + bi * sx;
        }
      }
    }
    for (int m = 0; m < mc; ++m) {
      float v = acc[m];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) a.y[((size_t)item * a.M + m0 + m) * a.N + n] = ok ? f2bf(v) : (uint16_t)0;
    }
  }
}

int launch_dequantize(const uint32_t* w, const uint16_t* s, const uint16_t* b, uint16_t* out, int64_t rows, int K,
                      int gs, cudaStream_t st) {
  const int64_t n_words = rows * (K / 8);
  if (n_words <= 0) return B2Q_OK;
  const int threads = 256;
  dequantize_kernel<<<(unsigned)((n_words + threads - 1) / threads), threads, 0, st>>>(w, s, b, out, n_words, K, gs);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int launch_quantize(const uint16_t* w, uint32_t* wq, uint16_t* s, uint16_t* b, int64_t rows, int K, int gs,
                    cudaStream_t st) {
  const int64_t n_groups = rows * (K / gs);
  if (n_groups <= 0) return B2Q_OK;
  const int threads = 128;
  quantize_kernel<<<(unsigned)((n_groups + threads - 1) / threads), threads, 0, st>>>(w, wq, s, b, n_groups, gs);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int launch_generic_qmv(const GenericArgs& a, cudaStream_t st) {
  const int64_t warps = (int64_t)a.batch * a.N;
  if (warps <= 0) return B2Q_OK;
  const int threads = 256;
  generic_qmv_kernel<<<(unsigned)((warps * 32 + threads - 1) / threads), threads, 0, st>>>(a);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // namespace b2q
