// decoder.cu -- the small kernels of a decoder around the 4-bit path: token
// embedding from the tied 4-bit table, RMSNorm, rotary position embedding.
//
//   embed_gather : out[t] = dequant(table[ids[t]]), the quantized embedding
//                  lookup (MLXNN QuantizedEmbedding, Vendor/mlx-swift/Source/
//                  MLXNN/Quantized.swift:238-300: gather the packed rows, then
//                  dequantize) with the Metal dequantizer's arithmetic
//                  bf16(fp32(s)*q + fp32(b)) (backend/metal/kernels/quantized.h:
//                  3314-3373), 8 values per thread from one packed word.
//   rms_norm     : out = bf16(w * x * rsqrt(mean(x^2) + eps)), fp32 inside and
//                  one rounding at the end (MLX fast::rms_norm rounds the
//                  normalized x before the weight product; the decoder is
//                  outside the parity path and is checked against fp32 math).
//   rope         : the non-interleaved rotary embedding (MLX fast::rope with
//                  traditional = false): for pair (i, i + d/2) of a head at
//                  position p, angle = p * theta^(-2i/d), fp32 inside.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"

namespace b2q {
namespace dec {

__global__ void embed_gather_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                    const uint16_t* __restrict__ b, const int32_t* __restrict__ ids,
                                    uint16_t* __restrict__ out, int T, int V, int K, int gs, int* err) {
  const int t = blockIdx.y;
  const int kw = blockIdx.x * blockDim.x + threadIdx.x;  // packed word of the row
  const int wpr = K / 8;
  if (t >= T || kw >= wpr) return;
  const int id = ids[t];
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * K) + kw;
  if (id < 0 || id >= V) {  // out-of-range token id: zero row, recorded
    if (kw == 0) record_error(err, B2Q_EINVAL);
    *dst = make_uint4(0, 0, 0, 0);
    return;
  }
  const int G = K / gs;
  const size_t gidx = (size_t)id * G + (kw * 8) / gs;
  const float sc = bf2f(__ldg(s + gidx)), bi = bf2f(__ldg(b + gidx));
  const uint32_t W = __ldg(w + (size_t)id * wpr + kw);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __fadd_rn(__fmul_rn(sc, (float)((W >> (8 * j)) & 0xF)), bi);
    const float hi = __fadd_rn(__fmul_rn(sc, (float)((W >> (8 * j + 4)) & 0xF)), bi);
    o[j] = (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
  }
  *dst = make_uint4(o[0], o[1], o[2], o[3]);
}

constexpr int NORM_THREADS = 256;

// one CTA per row; 8 bf16 values per 16-byte load
__global__ void __launch_bounds__(NORM_THREADS)
    rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wt, uint16_t* __restrict__ out,
                    int H, float eps) {
  __shared__ float red[NORM_THREADS / 32];
  const int t = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  const int nv = H / 8;
  float ss = 0.0f;
  for (int v = threadIdx.x; v < nv; v += NORM_THREADS) {
    const uint4 q = __ldg(xr + v);
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = bf2f((uint16_t)(u[j] & 0xFFFF)), c = bf2f((uint16_t)(u[j] >> 16));
      ss = fmaf(a, a, ss);
      ss = fmaf(c, c, ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < NORM_THREADS / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)H + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(wt);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int v = threadIdx.x; v < nv; v += NORM_THREADS) {
    const uint4 q = __ldg(xr + v), g = __ldg(wr + v);
    const uint32_t u[4] = {q.x, q.y, q.z, q.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = bf2f((uint16_t)(u[j] & 0xFFFF)) * r * bf2f((uint16_t)(gw[j] & 0xFFFF));
      const float c = bf2f((uint16_t)(u[j] >> 16)) * r * bf2f((uint16_t)(gw[j] >> 16));
      o[j] = (uint32_t)f2bf(a) | ((uint32_t)f2bf(c) << 16);
    }
    orow[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// x [T, heads, d] in place; thread = (t, head, pair i)
__global__ void rope_kernel(uint16_t* __restrict__ x, int T, int heads, int d, const int32_t* __restrict__ positions,
                            int pos0, float log2_theta) {
  const int half = d / 2;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n = (size_t)T * heads * half;
  if (i >= n) return;
  const int p = (int)(i % half);
  const size_t th = i / half;  // t * heads + head
  const int t = (int)(th / heads);
  const int pos = positions ? positions[t] : pos0 + t;
  const float inv_freq = exp2f(-((float)p / (float)half) * log2_theta);
  float sn, cs;
  sincosf((float)pos * inv_freq, &sn, &cs);
  uint16_t* row = x + th * d;
  const float a = bf2f(row[p]), c = bf2f(row[p + half]);
  row[p] = f2bf(a * cs - c * sn);
  row[p + half] = f2bf(a * sn + c * cs);
}

}  // namespace dec
}  // namespace b2q

using namespace b2q;
using namespace b2q::dec;

extern "C" {

int b2q_embed_gather(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const int32_t* ids,
                     uint16_t* out, int T, int V, int K, int group_size, int bits, int* status, void* stream) {
  clear_error();
  if (bits != 4) return set_error(B2Q_EUNSUPPORTED, "embed_gather: bits=%d", bits);
  if (!(group_size == 32 || group_size == 64 || group_size == 128))
    return set_error(B2Q_EUNSUPPORTED, "embed_gather: group_size=%d", group_size);
  if (T < 0 || T > 65535 || V < 1 || K <= 0 || K % group_size)
    return set_error(B2Q_EINVAL, "embed_gather: bad shape (T=%d V=%d K=%d)", T, V, K);
  if (T == 0) return B2Q_OK;
  if (!w || !scales || !biases || !ids || !out) return set_error(B2Q_EINVAL, "embed_gather: null pointer");
  if (!aligned16(out)) return set_error(B2Q_EINVAL, "embed_gather: out must be 16-byte aligned");
  const int wpr = K / 8;
  dim3 grid((wpr + 127) / 128, T);
  embed_gather_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(w, scales, biases, ids, out, T, V, K,
                                                                           group_size, status);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int b2q_rms_norm(const uint16_t* x, const uint16_t* weight, uint16_t* out, int T, int H, float eps, void* stream) {
  clear_error();
  if (T < 0 || H <= 0 || H % 8 || !(eps >= 0.0f)) return set_error(B2Q_EINVAL, "rms_norm: bad shape (H=%d)", H);
  if (T == 0) return B2Q_OK;
  if (!x || !weight || !out) return set_error(B2Q_EINVAL, "rms_norm: null pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out))
    return set_error(B2Q_EINVAL, "rms_norm: tensors must be 16-byte aligned");
  rms_norm_kernel<<<T, NORM_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(x, weight, out, H, eps);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int b2q_rope(uint16_t* x, int T, int heads, int head_dim, const int32_t* positions, int pos0, float theta,
             void* stream) {
  clear_error();
  if (T < 0 || heads < 1 || head_dim < 2 || head_dim % 2 || !(theta > 1.0f))
    return set_error(B2Q_EINVAL, "rope: bad shape (heads=%d head_dim=%d theta=%g)", heads, head_dim, theta);
  if (T == 0) return B2Q_OK;
  if (!x) return set_error(B2Q_EINVAL, "rope: null pointer");
  const size_t n = (size_t)T * heads * (head_dim / 2);
  rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, T, heads, head_dim, positions, pos0, log2f(theta));
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // extern "C"
