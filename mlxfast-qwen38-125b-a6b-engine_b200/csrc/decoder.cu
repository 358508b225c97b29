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
//   add_rms_norm : h' = bf16(h + delta) (one rounding, as a bf16 add), then
//                  rms_norm(h'): the residual add fused into the next norm.
//   rope_kv      : rope on the q and k rows of a fused q|k|v product in place,
//                  then k and v appended to the bf16 KV cache at each row's
//                  position (one launch instead of copies, two ropes and two
//                  scatters).
//   gqa_decode   : attention of a few query rows over the KV cache rows
//                  [0, position] (decode and short windows): split over key
//                  chunks of 128, each CTA one kv head and chunk with the g
//                  query heads that share it, fp32 scores / exp / sums; a second
//                  kernel merges the chunks (max-rescaled sums) and rounds once.
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


// ---- fused residual add + RMSNorm -------------------------------------------
__global__ void __launch_bounds__(NORM_THREADS)
    add_rms_norm_kernel(const uint16_t* h, const uint16_t* __restrict__ delta, const uint16_t* __restrict__ wt,
                        uint16_t* h_out, uint16_t* __restrict__ out, int H, float eps) {
  // h_out may be h (in place): each thread re-reads only the words it wrote
  __shared__ float red[NORM_THREADS / 32];
  const int t = blockIdx.x;
  const uint4* hr = reinterpret_cast<const uint4*>(h + (size_t)t * H);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + (size_t)t * H) : nullptr;
  uint4* hw = reinterpret_cast<uint4*>(h_out + (size_t)t * H);
  const int nv = H / 8;
  float ss = 0.0f;
  // pass 1: h' = bf16(h + delta) written out, sum of squares of h'
  for (int v = threadIdx.x; v < nv; v += NORM_THREADS) {
    const uint4 q = hr[v];
    uint32_t u[4] = {q.x, q.y, q.z, q.w};
    if (dr) {
      const uint4 dq = dr[v];
      const uint32_t du[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf2f((uint16_t)(u[j] & 0xFFFF)) + bf2f((uint16_t)(du[j] & 0xFFFF));
        const float c = bf2f((uint16_t)(u[j] >> 16)) + bf2f((uint16_t)(du[j] >> 16));
        u[j] = (uint32_t)f2bf(a) | ((uint32_t)f2bf(c) << 16);
      }
      hw[v] = make_uint4(u[0], u[1], u[2], u[3]);
    }
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
  const uint4* src = dr ? reinterpret_cast<const uint4*>(hw) : hr;
  const uint4* wr = reinterpret_cast<const uint4*>(wt);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int v = threadIdx.x; v < nv; v += NORM_THREADS) {
    const uint4 q = src[v], g = __ldg(wr + v);
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

// ---- rope on q|k rows in place + KV append ------------------------------------
// qkv [T, (nq + 2 nk) * d]; thread = (t, head of q or k, pair i); the k-head
// threads also copy their roped k pair and the v pair into the cache.
__global__ void rope_kv_kernel(uint16_t* __restrict__ qkv, int T, int nq, int nk, int d,
                               const int32_t* __restrict__ positions, float log2_theta,
                               uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int max_seq, int* err) {
  const int half = d / 2;
  const int heads = nq + nk;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n = (size_t)T * heads * half;
  if (i >= n) return;
  const int p = (int)(i % half);
  const int hh = (int)((i / half) % heads);
  const int t = (int)(i / ((size_t)half * heads));
  const int pos = positions[t];
  const size_t row = (size_t)t * (nq + 2 * nk) * d;
  uint16_t* x = qkv + row + (size_t)hh * d;
  const float inv_freq = exp2f(-((float)p / (float)half) * log2_theta);
  float sn, cs;
  sincosf((float)pos * inv_freq, &sn, &cs);
  const float a = bf2f(x[p]), c = bf2f(x[p + half]);
  const uint16_t r0 = f2bf(a * cs - c * sn), r1 = f2bf(a * sn + c * cs);
  x[p] = r0;
  x[p + half] = r1;
  if (hh < nq) return;
  const int kh = hh - nq;
  if (pos < 0 || pos >= max_seq) {
    if (p == 0) record_error(err, B2Q_EINVAL);
    return;
  }
  uint16_t* kdst = kc + ((size_t)pos * nk + kh) * d;
  kdst[p] = r0;
  kdst[p + half] = r1;
  const uint16_t* vsrc = qkv + row + (size_t)(nq + nk + kh) * d;
  uint16_t* vdst = vc + ((size_t)pos * nk + kh) * d;
  vdst[p] = vsrc[p];
  vdst[p + half] = vsrc[p + half];
}

// ---- GQA attention of a few query rows over the cache ------------------------------
#ifndef B2Q_ATT_CHUNK
#define B2Q_ATT_CHUNK 128
#endif
constexpr int ATT_CHUNK = B2Q_ATT_CHUNK;  // keys per CTA (one per thread in the score phase)
constexpr int ATT_MAXG = 16;    // query heads per kv head
constexpr int ATT_MAXD = 256;   // head_dim

// Shared memory of one chunk CTA: K rows padded by 8 values (16-byte reads of
// consecutive rows fall in distinct banks), V rows, the g query rows (fp32) and
// the g x 128 probabilities.
__host__ __device__ inline int gqa_kld(int d) { return d + 8; }
__host__ __device__ inline size_t gqa_smem_bytes(int g, int d) {
  return (size_t)ATT_CHUNK * gqa_kld(d) * 2 + (size_t)ATT_CHUNK * d * 2 + (size_t)g * d * 4 +
         (size_t)g * ATT_CHUNK * 4;
}

// partial layout per (t, kv head, chunk): [g] max, [g] sum, [g][d] weighted values
__global__ void __launch_bounds__(ATT_CHUNK)
    gqa_chunk_kernel(const uint16_t* __restrict__ q, int q_ld, const uint16_t* __restrict__ kc,
                     const uint16_t* __restrict__ vc, const int32_t* __restrict__ positions, int nk, int g, int d,
                     int n_chunks, int window, float scale_log2, float* __restrict__ part, int* err) {
  extern __shared__ __align__(16) unsigned char gsm[];
  const int kld = gqa_kld(d);
  uint16_t* ks = reinterpret_cast<uint16_t*>(gsm);
  uint16_t* vs = ks + (size_t)ATT_CHUNK * kld;
  float* qs = reinterpret_cast<float*>(vs + (size_t)ATT_CHUNK * d);
  float* ps = qs + (size_t)g * d;
  __shared__ float red[ATT_MAXG][ATT_CHUNK / 32];
  __shared__ float stat[ATT_MAXG];
  const int kh = blockIdx.x, chunk = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int pos = positions[t];
  if (pos < 0 || pos >= window) {  // outside the cache window: recorded, attends row 0 only
    if (kh == 0 && chunk == 0 && tid == 0) record_error(err, B2Q_EINVAL);
    pos = 0;
  }
  const int k0 = chunk * ATT_CHUNK;
  const int nkeys = min(ATT_CHUNK, pos + 1 - k0);  // <= 0: chunk entirely after the position
  float* out = part + (((size_t)t * nk + kh) * n_chunks + chunk) * (size_t)g * (d + 2);
  if (nkeys <= 0) {
    for (int j = tid; j < g; j += ATT_CHUNK) {
      out[j] = -INFINITY;
      out[g + j] = 0.0f;
    }
    return;
  }
  // stage the chunk's K and V rows (16-byte loads, many in flight per thread) and q
  const int vpr = d / 8;  // 16-byte vectors per row
  const int nvec = nkeys * vpr;
#pragma unroll 4
  for (int i = tid; i < nvec; i += ATT_CHUNK) {
    const int key = i / vpr, c = i % vpr;
    const size_t src = ((size_t)(k0 + key) * nk + kh) * d + (size_t)c * 8;
    const uint4 kv = __ldg(reinterpret_cast<const uint4*>(kc + src));
    const uint4 vv = __ldg(reinterpret_cast<const uint4*>(vc + src));
    *reinterpret_cast<uint4*>(ks + (size_t)key * kld + c * 8) = kv;
    *reinterpret_cast<uint4*>(vs + (size_t)key * d + c * 8) = vv;
  }
  for (int idx = tid; idx < g * d; idx += ATT_CHUNK) {
    const int j = idx / d, e = idx % d;
    qs[idx] = bf2f(q[(size_t)t * q_ld + (size_t)(kh * g + j) * d + e]);
  }
  __syncthreads();
  // scores: thread = key
  float s[ATT_MAXG];
#pragma unroll
  for (int j = 0; j < ATT_MAXG; ++j) s[j] = -INFINITY;
  if (tid < nkeys) {
#pragma unroll
    for (int j = 0; j < ATT_MAXG; ++j) s[j] = 0.0f;
    const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)tid * kld);
    for (int v = 0; v < vpr; ++v) {
      const uint4 kv = kr[v];
      const uint32_t u[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float a = bf2f((uint16_t)(u[m] & 0xFFFF)), c = bf2f((uint16_t)(u[m] >> 16));
        const int e = v * 8 + 2 * m;
#pragma unroll
        for (int j = 0; j < ATT_MAXG; ++j)
          if (j < g) s[j] = fmaf(c, qs[j * d + e + 1], fmaf(a, qs[j * d + e], s[j]));
      }
    }
#pragma unroll
    for (int j = 0; j < ATT_MAXG; ++j) s[j] *= scale_log2;  // log2-domain scores
  }
  // per head: chunk max and sum of 2^(s - max)
#pragma unroll
  for (int j = 0; j < ATT_MAXG; ++j) {
    if (j < g) {
      float m = s[j];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (lane == 0) red[j][warp] = m;
    }
  }
  __syncthreads();
  if (tid < g) {
    float m = red[tid][0];
    for (int w = 1; w < ATT_CHUNK / 32; ++w) m = fmaxf(m, red[tid][w]);
    stat[tid] = m;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < ATT_MAXG; ++j) {
    if (j < g) {
      const float pj = (tid < nkeys) ? exp2f(s[j] - stat[j]) : 0.0f;
      ps[j * ATT_CHUNK + tid] = pj;
      float l = pj;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) red[j][warp] = l;
    }
  }
  __syncthreads();
  if (tid < g) {
    float l = 0.0f;
    for (int w = 0; w < ATT_CHUNK / 32; ++w) l += red[tid][w];
    out[tid] = stat[tid];
    out[g + tid] = l;
  }
  // weighted values from shared memory: thread = dimension
  for (int e = tid; e < d; e += ATT_CHUNK) {
    float acc[ATT_MAXG];
#pragma unroll
    for (int j = 0; j < ATT_MAXG; ++j) acc[j] = 0.0f;
#pragma unroll 4
    for (int key = 0; key < nkeys; ++key) {
      const float vv = bf2f(vs[(size_t)key * d + e]);
#pragma unroll
      for (int j = 0; j < ATT_MAXG; ++j)
        if (j < g) acc[j] = fmaf(ps[j * ATT_CHUNK + key], vv, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < ATT_MAXG; ++j)  // static indices keep acc in registers
      if (j < g) out[2 * g + (size_t)j * d + e] = acc[j];
  }
}

// out[t, (kh*g + j)*d + e] = bf16(sum_c 2^(m_c - M) acc_c / sum_c 2^(m_c - M) l_c)
__global__ void gqa_merge_kernel(const float* __restrict__ part, uint16_t* __restrict__ out, int nk, int g, int d,
                                 int n_chunks) {
  const int kh = blockIdx.x, j = blockIdx.y, t = blockIdx.z;
  const size_t stride = (size_t)g * (d + 2);
  const float* base = part + ((size_t)t * nk + kh) * n_chunks * stride;
  float M = -INFINITY;
  for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, base[c * stride + j]);
  float L = 0.0f;
  for (int c = 0; c < n_chunks; ++c) {
    const float m = base[c * stride + j];
    if (m != -INFINITY) L += exp2f(m - M) * base[c * stride + g + j];
  }
  const float invL = 1.0f / L;
  for (int e = threadIdx.x; e < d; e += blockDim.x) {
    float a = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
      const float m = base[c * stride + j];
      if (m != -INFINITY) a += exp2f(m - M) * base[c * stride + 2 * g + (size_t)j * d + e];
    }
    out[(size_t)t * nk * g * d + (size_t)(kh * g + j) * d + e] = f2bf(a * invL);
  }
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


int b2q_add_rms_norm(const uint16_t* h, const uint16_t* delta, const uint16_t* weight, uint16_t* h_out, uint16_t* out,
                     int T, int H, float eps, void* stream) {
  clear_error();
  if (T < 0 || H <= 0 || H % 8 || !(eps >= 0.0f)) return set_error(B2Q_EINVAL, "add_rms_norm: bad shape (H=%d)", H);
  if (T == 0) return B2Q_OK;
  if (!h || !weight || !out || (delta && !h_out)) return set_error(B2Q_EINVAL, "add_rms_norm: null pointer");
  if (!aligned16(h) || !aligned16(weight) || !aligned16(out) || (delta && (!aligned16(delta) || !aligned16(h_out))))
    return set_error(B2Q_EINVAL, "add_rms_norm: tensors must be 16-byte aligned");
  add_rms_norm_kernel<<<T, NORM_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(h, delta, weight, h_out, out, H, eps);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

int b2q_rope_kv(uint16_t* qkv, int T, int nq, int nk, int head_dim, const int32_t* positions, float theta,
                uint16_t* k_cache, uint16_t* v_cache, int max_seq, int* status, void* stream) {
  clear_error();
  if (T < 0 || nq < 1 || nk < 1 || head_dim < 2 || head_dim % 2 || !(theta > 1.0f) || max_seq < 1)
    return set_error(B2Q_EINVAL, "rope_kv: bad shape (nq=%d nk=%d head_dim=%d)", nq, nk, head_dim);
  if (T == 0) return B2Q_OK;
  if (!qkv || !positions || !k_cache || !v_cache) return set_error(B2Q_EINVAL, "rope_kv: null pointer");
  const size_t n = (size_t)T * (nq + nk) * (head_dim / 2);
  rope_kv_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qkv, T, nq, nk, head_dim, positions, log2f(theta), k_cache, v_cache, max_seq, status);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

size_t b2q_gqa_decode_workspace_size(int T, int nq, int nk, int head_dim, int window) {
  if (T < 1 || nq < 1 || nk < 1 || nq % nk || head_dim < 1 || window < 1) return 0;
  const size_t chunks = (size_t)(window + ATT_CHUNK - 1) / ATT_CHUNK;
  return sizeof(float) * (size_t)T * nk * chunks * (size_t)(nq / nk) * (head_dim + 2);
}

int b2q_gqa_decode(const uint16_t* q, int q_ld, const uint16_t* k_cache, const uint16_t* v_cache,
                   const int32_t* positions, uint16_t* out, int T, int nq, int nk, int head_dim, int window,
                   int* status, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (T < 0 || T > 65535 || nq < 1 || nk < 1 || nq % nk || nq / nk > ATT_MAXG || head_dim < 8 || head_dim % 8 ||
      head_dim > ATT_MAXD || window < 1 || q_ld < nq * head_dim)
    return set_error(B2Q_EINVAL, "gqa_decode: bad shape (nq=%d nk=%d head_dim=%d window=%d)", nq, nk, head_dim,
                     window);
  if (T == 0) return B2Q_OK;
  if (!q || !k_cache || !v_cache || !positions || !out) return set_error(B2Q_EINVAL, "gqa_decode: null pointer");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return set_error(B2Q_EINVAL, "gqa_decode: k_cache and v_cache must be 16-byte aligned");
  const size_t need = b2q_gqa_decode_workspace_size(T, nq, nk, head_dim, window);
  if (!workspace || workspace_bytes < need)
    return set_error(B2Q_EINVAL, "gqa_decode: workspace of %zu bytes needed", need);
  const int g = nq / nk;
  const int chunks = (window + ATT_CHUNK - 1) / ATT_CHUNK;
  if (chunks > 65535) return set_error(B2Q_EINVAL, "gqa_decode: window %d", window);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  // scores in the log2 domain: q.k / sqrt(d) * log2(e)
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  const size_t smem = gqa_smem_bytes(g, head_dim);
  static int attr_done[64] = {};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if ((int)smem > di.smem_optin) return set_error(B2Q_EUNSUPPORTED, "gqa_decode: %zu bytes of shared memory", smem);
  if (!attr_done[di.device & 63]) {  // the largest shape's need, once per device
    B2Q_TRY_CUDA(cudaFuncSetAttribute(gqa_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)gqa_smem_bytes(ATT_MAXG, ATT_MAXD)));
    attr_done[di.device & 63] = 1;
  }
  gqa_chunk_kernel<<<dim3(nk, chunks, T), ATT_CHUNK, smem, st>>>(q, q_ld, k_cache, v_cache, positions, nk, g,
                                                                head_dim, chunks, window, scale_log2, part, status);
  B2Q_TRY_CUDA(cudaGetLastError());
  gqa_merge_kernel<<<dim3(nk, g, T), 128, 0, st>>>(part, out, nk, g, head_dim, chunks);
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // extern "C"
