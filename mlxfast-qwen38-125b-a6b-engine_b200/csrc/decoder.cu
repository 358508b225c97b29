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
//   attn_decode  : rope_kv + gqa_decode in one launch for windows of up to 8
//                  rows, the chunks merged by the last CTA of each kv head.
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

// Programmatic dependent launch for the per-layer kernels of a decode step: a
// kernel waits for its predecessor in the stream before reading anything
// (griddepcontrol.wait), then lets its own successor start launching, so each
// launch's set-up overlaps the previous kernel's tail.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

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
  pdl_enter();
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

// ---- one-launch attention of a decode window -----------------------------------
// rope_kv + gqa_chunk + gqa_merge in one kernel for windows of at most 8 rows
// (the graph decode step and the MTP verify windows). CTA (kv head kh, chunk c,
// row t) covers keys [c * AD_CH, c * AD_CH + AD_CH) up to row t's position:
//  * keys at positions of the window's own rows are taken from the q|k|v rows
//    (k roped here), not from the cache, so no CTA waits for another's append;
//    the CTA whose chunk holds row t's position appends row t's k / v of head kh
//    to the cache (one writer per row and head);
//  * cache keys are staged with cp.async (every 16-byte piece in flight at once);
//  * scores and weighted values on the tensor cores (mma.sync m16n8k16 bf16,
//    fp32 accumulation): warp w takes keys [16 w, 16 w + 16) of the chunk, the
//    g query heads (zero-padded to 16) are the M rows; S = Q K^T, then the
//    chunk's per-head max and 2^(S - max) in fp32, rounded to bf16 as the A
//    operand of P V (the score fragments are the A fragments: no shuffle);
//    V fragments by ldmatrix.trans; the four warps' P V partials are added in
//    warp order (deterministic);
//  * the last CTA of (t, kh) to finish (a counter per (t, kh) in the workspace,
//    re-armed by that CTA) merges the chunks and writes the bf16 output.
// q and k are rounded to bf16 after the rotation and v is read as bf16, as the
// separate kernels store them, so the cache rows are bit-identical to rope_kv's.
constexpr int AD_CH = 64;        // keys per CTA
constexpr int AD_THREADS = 128;  // four warps of 16 keys
constexpr int AD_MAXT = 8;       // window rows

// K and V rows padded by 8 values (ldmatrix / fragment reads of 8 consecutive
// rows fall in distinct banks), 16 q rows, each warp's g x d P V partial (fp32), and
// the merge's per-(head, chunk) maxima, sums and weights
__host__ __device__ inline size_t ad_smem_bytes(int g, int d, int n_chunks) {
  return (size_t)2 * AD_CH * gqa_kld(d) * 2 + (size_t)16 * gqa_kld(d) * 2 + (size_t)(AD_THREADS / 32) * g * d * 4 +
         (size_t)3 * g * n_chunks * 4;
}

// partial of one (row, kv head, chunk): [g][d] weighted values (16-byte
// aligned for the merge's vector loads), then [g] maxima, [g] sums, padding
__host__ __device__ inline int ad_stride(int g, int d) { return g * d + (2 * g + 3) / 4 * 4; }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// roped pair (p, p + half) of one head row at position pos, rounded to bf16
__device__ __forceinline__ void rope_pair(const uint16_t* x, int p, int half, int pos, float log2_theta,
                                          uint16_t& r0, uint16_t& r1) {
  const float inv_freq = exp2f(-((float)p / (float)half) * log2_theta);
  float sn, cs;
  sincosf((float)pos * inv_freq, &sn, &cs);
  const float a = bf2f(x[p]), c = bf2f(x[p + half]);
  r0 = f2bf(a * cs - c * sn);
  r1 = f2bf(a * sn + c * cs);
}

__global__ void __launch_bounds__(AD_THREADS)
    attn_decode_kernel(const uint16_t* __restrict__ qkv, int q_ld, int T, const int32_t* __restrict__ positions,
                       int nq, int nk, int d, float log2_theta, uint16_t* __restrict__ kc, uint16_t* __restrict__ vc,
                       int window, int n_chunks, float scale_log2, float* __restrict__ part, unsigned* __restrict__ cnt,
                       uint16_t* __restrict__ out, int* err) {
  extern __shared__ __align__(16) unsigned char asm_[];
  const int kld = gqa_kld(d);
  uint16_t* ks = reinterpret_cast<uint16_t*>(asm_);
  uint16_t* vs = ks + (size_t)AD_CH * kld;
  uint16_t* qb = vs + (size_t)AD_CH * kld;                     // [16][kld] bf16 q rows (rows >= g zero)
  float* ob = reinterpret_cast<float*>(qb + (size_t)16 * kld);  // [warp][g][d] P V partials
  __shared__ float red[AD_THREADS / 32][16];
  __shared__ float stat[16];
  __shared__ float2 rot[ATT_MAXD / 2];  // (cos, sin) of row t's angles
  __shared__ int wpos[AD_MAXT];
  __shared__ int last_sm;
  const int kh = blockIdx.x, chunk = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = nq / nk, half = d / 2, vpr = d / 8;
  pdl_enter();
  if (tid < T) wpos[tid] = positions[tid];
  __syncthreads();
  int pos = wpos[t];
  const bool bad = pos < 0 || pos >= window;
  if (bad) {  // outside the cache window: recorded, attends row 0 only, appends nothing
    if (kh == 0 && chunk == 0 && tid == 0) record_error(err, B2Q_EINVAL);
    pos = 0;
  }
  const uint16_t* row_t = qkv + (size_t)t * q_ld;
  const int k0 = chunk * AD_CH;
  const int nkeys = min(AD_CH, pos + 1 - k0);  // <= 0: chunk entirely after the position
  // the window row whose position is key j (the last such row), or -1
  auto window_row = [&](int j) {
    int w = -1;
    for (int u = 0; u < T; ++u)
      if (wpos[u] == j) w = u;
    return w;
  };
  // row t's k / v of head kh into the cache, by the chunk holding its position
  if (!bad && chunk == pos / AD_CH) {
    const uint16_t* krow = row_t + (size_t)(nq + kh) * d;
    const uint16_t* vrow = row_t + (size_t)(nq + nk + kh) * d;
    uint16_t* kdst = kc + ((size_t)pos * nk + kh) * d;
    uint16_t* vdst = vc + ((size_t)pos * nk + kh) * d;
    for (int p = tid; p < half; p += AD_THREADS) {
      uint16_t r0, r1;
      rope_pair(krow, p, half, pos, log2_theta, r0, r1);
      kdst[p] = r0;
      kdst[p + half] = r1;
      vdst[p] = vrow[p];
      vdst[p + half] = vrow[p + half];
    }
  }
  const int stride = ad_stride(g, d);
  float* pout = part + (((size_t)t * nk + kh) * n_chunks + chunk) * (size_t)stride;
  float* pm = pout + (size_t)g * d;  // maxima, then sums
  if (nkeys <= 0) {
    for (int j = tid; j < g; j += AD_THREADS) {
      pm[j] = -INFINITY;
      pm[g + j] = 0.0f;
    }
  } else {
    // cache keys: every 16-byte piece in flight at once; key rows past nkeys zeroed
    for (int i = tid; i < AD_CH * vpr; i += AD_THREADS) {
      const int key = i / vpr, c = i % vpr;
      uint16_t* kd = ks + (size_t)key * kld + c * 8;
      uint16_t* vd = vs + (size_t)key * kld + c * 8;
      if (key >= nkeys) {
        *reinterpret_cast<uint4*>(kd) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(vd) = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      if (window_row(k0 + key) >= 0) continue;
      const size_t src = ((size_t)(k0 + key) * nk + kh) * d + (size_t)c * 8;
      cp_async16(kd, kc + src);
      cp_async16(vd, vc + src);
    }
    // keys of the window's rows from the q|k|v rows (k roped at the key's position)
    for (int u = 0; u < T; ++u) {
      const int j = wpos[u];
      if (j < k0 || j >= k0 + nkeys || window_row(j) != u) continue;
      const uint16_t* urow = qkv + (size_t)u * q_ld;
      const uint16_t* krow = urow + (size_t)(nq + kh) * d;
      const uint16_t* vrow = urow + (size_t)(nq + nk + kh) * d;
      for (int p = tid; p < half; p += AD_THREADS) {
        uint16_t r0, r1;
        rope_pair(krow, p, half, j, log2_theta, r0, r1);
        ks[(size_t)(j - k0) * kld + p] = r0;
        ks[(size_t)(j - k0) * kld + p + half] = r1;
        vs[(size_t)(j - k0) * kld + p] = vrow[p];
        vs[(size_t)(j - k0) * kld + p + half] = vrow[p + half];
      }
    }
    // row t's g query heads roped at its position (bf16 rows 0..g-1 of qb; rows
    // g..15 zero): the half angles once, then every head (the same arithmetic
    // as rope_pair)
    for (int p = tid; p < half; p += AD_THREADS) {
      const float inv_freq = exp2f(-((float)p / (float)half) * log2_theta);
      float sn, cs;
      sincosf((float)pos * inv_freq, &sn, &cs);
      rot[p] = make_float2(cs, sn);
    }
    __syncthreads();
    for (int i = tid; i < 16 * half; i += AD_THREADS) {
      const int j = i / half, p = i % half;
      uint16_t r0 = 0, r1 = 0;
      if (j < g) {
        const uint16_t* x = row_t + (size_t)(kh * g + j) * d;
        const float2 cssn = rot[p];
        const float a = bf2f(x[p]), c2 = bf2f(x[p + half]);
        r0 = f2bf(a * cssn.x - c2 * cssn.y);
        r1 = f2bf(a * cssn.y + c2 * cssn.x);
      }
      qb[j * kld + p] = r0;
      qb[j * kld + p + half] = r1;
    }
    cp_async_wait_all();
    __syncthreads();
    // ---- S = Q K^T for the warp's 16 keys (two n8 tiles), fp32 ----
    const int r = lane >> 2, c = lane & 3;
    const int kb = warp * 16;  // the warp's first key in the chunk
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
    for (int k0e = 0; k0e < d; k0e += 16) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(qb + r * kld + k0e + 2 * c);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(qb + (r + 8) * kld + k0e + 2 * c);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(qb + r * kld + k0e + 8 + 2 * c);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(qb + (r + 8) * kld + k0e + 8 + 2 * c);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint16_t* krow = ks + (size_t)(kb + nt * 8 + r) * kld + k0e + 2 * c;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + 8);
        mma_bf16_16816(sc[nt], a0, a1, a2, a3, b0, b1);
      }
    }
    // lane: head rows r (d0, d1) and r + 8 (d2, d3), keys kb + 8 nt + 2 c, + 1
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int key = kb + nt * 8 + 2 * c + (q & 1);
        sc[nt][q] = key < nkeys ? sc[nt][q] * scale_log2 : -INFINITY;
        if (q < 2) mx0 = fmaxf(mx0, sc[nt][q]);
        else mx1 = fmaxf(mx1, sc[nt][q]);
      }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    if (c == 0) {
      red[warp][r] = mx0;
      red[warp][r + 8] = mx1;
    }
    __syncthreads();
    if (tid < 16) {
      float m = red[0][tid];
#pragma unroll
      for (int w = 1; w < AD_THREADS / 32; ++w) m = fmaxf(m, red[w][tid]);
      stat[tid] = m;  // finite: every chunk with keys has a valid key in some warp
    }
    __syncthreads();
    const float M0 = stat[r], M1 = stat[r + 8];
    float l0 = 0.0f, l1 = 0.0f;
    uint32_t pa[4];  // P as the A operand of the warp's one k16 step
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float p0 = exp2f(sc[nt][0] - M0), p1 = exp2f(sc[nt][1] - M0);
      const float p2 = exp2f(sc[nt][2] - M1), p3 = exp2f(sc[nt][3] - M1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pa[2 * nt] = pack_bf16(p0, p1);      // row r, keys 8 nt + 2 c, + 1
      pa[2 * nt + 1] = pack_bf16(p2, p3);  // row r + 8
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    __syncthreads();  // every warp has read stat from red's maxima
    if (c == 0) {
      red[warp][r] = l0;
      red[warp][r + 8] = l1;
    }
    // ---- O += P V over the warp's 16 keys: 8-column tiles of d, two per ldmatrix ----
    // A fragment order: a0 row r keys 0-7, a1 row r + 8 keys 0-7, a2 row r keys 8-15, a3 row r + 8 keys 8-15
    const uint32_t A0 = pa[0], A1 = pa[1], A2 = pa[2], A3 = pa[3];
    const int mi = lane >> 3, mr = lane & 7;  // the ldmatrix row this lane addresses
    for (int e0 = 0; e0 < d; e0 += 16) {
      // matrices: keys 0-7 / 8-15 of the warp x columns e0..e0+7 / e0+8..e0+15
      uint32_t v[4];
      ldsm_x4_trans(v, vs + (size_t)(kb + (mi & 1) * 8 + mr) * kld + e0 + (mi >> 1) * 8);
      float o0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, o1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      mma_bf16_16816(o0, A0, A1, A2, A3, v[0], v[1]);
      mma_bf16_16816(o1, A0, A1, A2, A3, v[2], v[3]);
      // rows r (o[0], o[1]) and r + 8 (o[2], o[3]), columns e + 2 c, + 1
      float* ow = ob + (size_t)warp * g * d;
      if (r < g) {
        *reinterpret_cast<float2*>(ow + r * d + e0 + 2 * c) = make_float2(o0[0], o0[1]);
        *reinterpret_cast<float2*>(ow + r * d + e0 + 8 + 2 * c) = make_float2(o1[0], o1[1]);
      }
      if (r + 8 < g) {
        *reinterpret_cast<float2*>(ow + (r + 8) * d + e0 + 2 * c) = make_float2(o0[2], o0[3]);
        *reinterpret_cast<float2*>(ow + (r + 8) * d + e0 + 8 + 2 * c) = make_float2(o1[2], o1[3]);
      }
    }
    __syncthreads();
    if (tid < g) {
      float l = 0.0f;
#pragma unroll
      for (int w = 0; w < AD_THREADS / 32; ++w) l += red[w][tid];
      pm[tid] = stat[tid];
      pm[g + tid] = l;
    }
    const int n4 = g * d / 4;
    for (int i = tid; i < n4; i += AD_THREADS) {
      float4 a = reinterpret_cast<const float4*>(ob)[i];
#pragma unroll
      for (int w = 1; w < AD_THREADS / 32; ++w) {
        const float4 b = reinterpret_cast<const float4*>(ob)[(size_t)w * n4 + i];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      reinterpret_cast<float4*>(pout)[i] = a;
    }
  }
  // the last CTA of (t, kh) merges the chunks holding keys (each thread's
  // partial stores fenced before the block's arrival is counted)
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&cnt[t * nk + kh], 1u);
    last_sm = prev == (unsigned)(n_chunks - 1);
    if (last_sm) cnt[t * nk + kh] = 0u;  // re-armed for the next call
  }
  __syncthreads();
  if (!last_sm) return;
  __threadfence();
  // merge: every chunk's max and sum staged at once, one weight per (head,
  // chunk), then each 4-value column of the outputs over the chunks with its
  // loads in flight together
  const int nc = pos / AD_CH + 1;  // chunks with keys
  const float* base = part + ((size_t)t * nk + kh) * n_chunks * (size_t)stride;
  float* cm = ob + (size_t)(AD_THREADS / 32) * g * d;  // [g][nc] maxima, [g][nc] sums, [g][nc] weights
  float* cl = cm + (size_t)g * n_chunks;
  float* cw = cl + (size_t)g * n_chunks;
  for (int i = tid; i < g * nc; i += AD_THREADS) {
    const int j = i / nc, c = i % nc;
    cm[i] = __ldcg(base + (size_t)c * stride + (size_t)g * d + j);
    cl[i] = __ldcg(base + (size_t)c * stride + (size_t)g * d + g + j);
  }
  __syncthreads();
  if (tid < g) {
    float M = -INFINITY;
    for (int c = 0; c < nc; ++c) M = fmaxf(M, cm[tid * nc + c]);
    float L = 0.0f;
    for (int c = 0; c < nc; ++c) L += exp2f(cm[tid * nc + c] - M) * cl[tid * nc + c];
    const float invL = 1.0f / L;
    for (int c = 0; c < nc; ++c) cw[tid * nc + c] = exp2f(cm[tid * nc + c] - M) * invL;
  }
  __syncthreads();
  // each thread's columns q and q + 128 (g * d / 4 <= 2 * AD_THREADS when
  // g * d <= 1024; more columns loop) with the loads of MB chunks of both in
  // flight together
  constexpr int MB = 8;
  const int ncol = g * d / 4;
  for (int q0 = tid; q0 < ncol; q0 += 2 * AD_THREADS) {
    const int q1 = q0 + AD_THREADS;
    const bool has1 = q1 < ncol;
    const int j0 = 4 * q0 / d, j1 = has1 ? 4 * q1 / d : j0;
    float4 a0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), a1 = a0;
    for (int c0 = 0; c0 < nc; c0 += MB) {
      float4 v0[MB], v1[MB];
#pragma unroll
      for (int u = 0; u < MB; ++u) {
        const bool in = c0 + u < nc;
        const float4* src = reinterpret_cast<const float4*>(base + (size_t)(c0 + u) * stride);
        v0[u] = in ? __ldcg(src + q0) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        v1[u] = in && has1 ? __ldcg(src + q1) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < MB; ++u) {
        const bool in = c0 + u < nc;
        const float w0 = in ? cw[j0 * nc + c0 + u] : 0.0f, w1 = in ? cw[j1 * nc + c0 + u] : 0.0f;
        a0.x = fmaf(w0, v0[u].x, a0.x);
        a0.y = fmaf(w0, v0[u].y, a0.y);
        a0.z = fmaf(w0, v0[u].z, a0.z);
        a0.w = fmaf(w0, v0[u].w, a0.w);
        a1.x = fmaf(w1, v1[u].x, a1.x);
        a1.y = fmaf(w1, v1[u].y, a1.y);
        a1.z = fmaf(w1, v1[u].z, a1.z);
        a1.w = fmaf(w1, v1[u].w, a1.w);
      }
    }
    uint16_t* ob0 = out + (size_t)t * nq * d + (size_t)kh * g * d + 4 * q0;
    *reinterpret_cast<uint2*>(ob0) = make_uint2(pack_bf16(a0.x, a0.y), pack_bf16(a0.z, a0.w));
    if (has1) {
      uint16_t* ob1 = out + (size_t)t * nq * d + (size_t)kh * g * d + 4 * q1;
      *reinterpret_cast<uint2*>(ob1) = make_uint2(pack_bf16(a1.x, a1.y), pack_bf16(a1.z, a1.w));
    }
  }
}

// ---- the same attention as one thread-block cluster per (row, kv head) -------------
// For head_dim 128: the AC_CL CTAs of a cluster share a kv head and row t; CTA
// rank r takes chunks r, r + AC_CL, ... of AC_CH keys (a 2-buffer cp.async
// ring), and each warp keeps an online softmax over its 16 keys of every chunk
// (running max, sum and P V accumulators in registers; the same tensor-core
// arithmetic as attn_decode_kernel). The eight warps are merged in shared
// memory, then the cluster's CTAs exchange their (max, sum, partial) through
// distributed shared memory and each writes a slice of the output: no global
// partials, fences or arrival counters.
constexpr int AC_CL = 8;         // CTAs per cluster
constexpr int AC_NB = 2;         // chunk buffers of the ring
constexpr int AC_D = 128;
constexpr int AC_CH = 128;       // keys per chunk: one 16-key slice per warp
constexpr int AC_THREADS = 256;  // eight warps

__host__ __device__ inline size_t ac_smem_bytes(int g) {
  const int kld = AC_D + 8;
  return (size_t)AC_NB * 2 * AC_CH * kld * 2 + (size_t)16 * kld * 2 + (size_t)(AC_THREADS / 32) * g * AC_D * 4 +
         (size_t)g * AC_D * 4;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ float ld_dsmem(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(AC_THREADS)
    attn_cluster_kernel(const uint16_t* __restrict__ qkv, int q_ld, int T, const int32_t* __restrict__ positions,
                        int nq, int nk, float log2_theta, uint16_t* __restrict__ kc, uint16_t* __restrict__ vc,
                        int window, float scale_log2, uint16_t* __restrict__ out, int* err) {
  constexpr int D = AC_D, KLD = D + 8, HALF = D / 2, VPR = D / 8;
  extern __shared__ __align__(16) unsigned char acs_[];
  uint16_t* kbuf = reinterpret_cast<uint16_t*>(acs_);      // [AC_NB][AC_CH][KLD]
  uint16_t* vbuf = kbuf + (size_t)AC_NB * AC_CH * KLD;       // [AC_NB][AC_CH][KLD]
  uint16_t* qb = vbuf + (size_t)AC_NB * AC_CH * KLD;         // [16][KLD]
  float* wo = reinterpret_cast<float*>(qb + (size_t)16 * KLD);  // [warp][g][D] warp partials
  const int g = nq / nk;
  float* co = wo + (size_t)(AC_THREADS / 32) * g * D;          // [g][D] the CTA's partial
  __shared__ float wm[AC_THREADS / 32][16], wl[AC_THREADS / 32][16];
  __shared__ float cm[16], cl[16];
  __shared__ float2 rot[HALF];
  __shared__ int wpos[AD_MAXT];
  const uint32_t rank = cluster_rank();
  const int kh = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_enter();
  if (tid < T) wpos[tid] = positions[tid];
  __syncthreads();
  int pos = wpos[t];
  const bool bad = pos < 0 || pos >= window;
  if (bad) {  // outside the cache window: recorded, attends row 0 only, appends nothing
    if (kh == 0 && rank == 0 && tid == 0) record_error(err, B2Q_EINVAL);
    pos = 0;
  }
  const uint16_t* row_t = qkv + (size_t)t * q_ld;
  // the g query heads' rows (contiguous g * D bf16, at most two 16-byte pieces
  // per thread) are requested now and stored to shared memory after the
  // cache append and the first copies, whose latency they share
  const uint4* qsrc = reinterpret_cast<const uint4*>(row_t + (size_t)kh * g * D);
  const int nq16 = g * D / 8;
  uint4 qv0 = make_uint4(0u, 0u, 0u, 0u), qv1 = qv0;
  if (tid < nq16) qv0 = __ldg(qsrc + tid);
  if (tid + AC_THREADS < nq16) qv1 = __ldg(qsrc + tid + AC_THREADS);
  auto window_row = [&](int j) {
    int w = -1;
    for (int u = 0; u < T; ++u)
      if (wpos[u] == j) w = u;
    return w;
  };
  // row t's k / v of head kh into the cache, by the CTA whose chunks hold its position
  if (!bad && (pos / AC_CH) % AC_CL == (int)rank) {
    const uint16_t* krow = row_t + (size_t)(nq + kh) * D;
    const uint16_t* vrow = row_t + (size_t)(nq + nk + kh) * D;
    uint16_t* kdst = kc + ((size_t)pos * nk + kh) * D;
    uint16_t* vdst = vc + ((size_t)pos * nk + kh) * D;
    for (int p = tid; p < HALF; p += AC_THREADS) {
      uint16_t r0, r1;
      rope_pair(krow, p, HALF, pos, log2_theta, r0, r1);
      kdst[p] = r0;
      kdst[p + HALF] = r1;
      vdst[p] = vrow[p];
      vdst[p + HALF] = vrow[p + HALF];
    }
  }
  const int nc = pos / AC_CH + 1;  // chunks with keys
  const int mc = (int)rank < nc ? (nc - 1 - (int)rank) / AC_CL + 1 : 0;  // this CTA's chunks
  // stage chunk i of this CTA into buffer b: cache keys by cp.async, the
  // window's own keys from q|k|v (roped), rows past the position zeroed
  auto issue = [&](int i, int b) {
    const int k0 = ((int)rank + i * AC_CL) * AC_CH;
    const int nkeys = min(AC_CH, pos + 1 - k0);
    uint16_t* ks = kbuf + (size_t)b * AC_CH * KLD;
    uint16_t* vs = vbuf + (size_t)b * AC_CH * KLD;
    for (int q = tid; q < AC_CH * VPR; q += AC_THREADS) {
      const int key = q / VPR, c = q % VPR;
      uint16_t* kd = ks + (size_t)key * KLD + c * 8;
      uint16_t* vd = vs + (size_t)key * KLD + c * 8;
      if (key >= nkeys) {
        *reinterpret_cast<uint4*>(kd) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(vd) = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      if (window_row(k0 + key) >= 0) continue;
      const size_t src = ((size_t)(k0 + key) * nk + kh) * D + (size_t)c * 8;
      cp_async16(kd, kc + src);
      cp_async16(vd, vc + src);
    }
    for (int u = 0; u < T; ++u) {
      const int j = wpos[u];
      if (j < k0 || j >= k0 + nkeys || window_row(j) != u) continue;
      const uint16_t* urow = qkv + (size_t)u * q_ld;
      const uint16_t* krow = urow + (size_t)(nq + kh) * D;
      const uint16_t* vrow = urow + (size_t)(nq + nk + kh) * D;
      for (int p = tid; p < HALF; p += AC_THREADS) {
        uint16_t r0, r1;
        rope_pair(krow, p, HALF, j, log2_theta, r0, r1);
        ks[(size_t)(j - k0) * KLD + p] = r0;
        ks[(size_t)(j - k0) * KLD + p + HALF] = r1;
        vs[(size_t)(j - k0) * KLD + p] = vrow[p];
        vs[(size_t)(j - k0) * KLD + p + HALF] = vrow[p + HALF];
      }
    }
  };
#pragma unroll
  for (int i = 0; i < AC_NB - 1; ++i) {
    if (i < mc) issue(i, i);
    cp_async_commit();
  }
  // q rows roped at row t's position: the g heads' rows (contiguous, g * D
  // bf16) staged with one 16-byte load per thread, the angles once, then every
  // head from shared memory
  uint16_t* qraw = reinterpret_cast<uint16_t*>(co);  // free until the CTA merge
  if (tid < nq16) reinterpret_cast<uint4*>(qraw)[tid] = qv0;
  if (tid + AC_THREADS < nq16) reinterpret_cast<uint4*>(qraw)[tid + AC_THREADS] = qv1;
  for (int p = tid; p < HALF; p += AC_THREADS) {
    const float inv_freq = exp2f(-((float)p / (float)HALF) * log2_theta);
    float sn, cs;
    sincosf((float)pos * inv_freq, &sn, &cs);
    rot[p] = make_float2(cs, sn);
  }
  __syncthreads();
  for (int q = tid; q < 16 * HALF; q += AC_THREADS) {
    const int j = q / HALF, p = q % HALF;
    uint16_t r0 = 0, r1 = 0;
    if (j < g) {
      const uint16_t* x = qraw + (size_t)j * D;
      const float2 cssn = rot[p];
      const float a = bf2f(x[p]), c2 = bf2f(x[p + HALF]);
      r0 = f2bf(a * cssn.x - c2 * cssn.y);
      r1 = f2bf(a * cssn.y + c2 * cssn.x);
    }
    qb[j * KLD + p] = r0;
    qb[j * KLD + p + HALF] = r1;
  }
  // ---- online softmax over this CTA's chunks; warp w: keys [16 w, 16 w + 16) ----
  const int r = lane >> 2, c = lane & 3;
  const int kb = warp * 16;
  const int mi = lane >> 3, mr = lane & 7;  // the ldmatrix row this lane addresses
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows r, r + 8
  float o[D / 8][4];  // n8 tiles of d: rows r (0, 1) and r + 8 (2, 3), columns 8 nt + 2 c, + 1
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
  for (int i = 0; i < mc; ++i) {
    if (i + AC_NB - 1 < mc) issue(i + AC_NB - 1, (i + AC_NB - 1) % AC_NB);
    cp_async_commit();
    cp_async_wait_group<AC_NB - 1>();
    __syncthreads();
    const int b = i % AC_NB;
    const int k0 = ((int)rank + i * AC_CL) * AC_CH;
    const int nkeys = min(AC_CH, pos + 1 - k0);
    const uint16_t* ks = kbuf + (size_t)b * AC_CH * KLD;
    const uint16_t* vs = vbuf + (size_t)b * AC_CH * KLD;
    if (kb < nkeys) {  // warp-uniform: a warp whose keys are all past the position adds nothing
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
      for (int k0e = 0; k0e < D; k0e += 16) {
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(qb + r * KLD + k0e + 2 * c);
        const uint32_t a1 = *reinterpret_cast<const uint32_t*>(qb + (r + 8) * KLD + k0e + 2 * c);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(qb + r * KLD + k0e + 8 + 2 * c);
        const uint32_t a3 = *reinterpret_cast<const uint32_t*>(qb + (r + 8) * KLD + k0e + 8 + 2 * c);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint16_t* krow = ks + (size_t)(kb + nt * 8 + r) * KLD + k0e + 2 * c;
          mma_bf16_16816(sc[nt], a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(krow),
                         *reinterpret_cast<const uint32_t*>(krow + 8));
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int key = kb + nt * 8 + 2 * c + (q & 1);
          sc[nt][q] = key < nkeys ? sc[nt][q] * scale_log2 : -INFINITY;
          if (q < 2) mx0 = fmaxf(mx0, sc[nt][q]);
          else mx1 = fmaxf(mx1, sc[nt][q]);
        }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      // key kb (the warp's first) is valid, so the new maxima are finite
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
      const float s0 = exp2f(m0 - n0), s1 = exp2f(m1 - n1);  // 0 on the first chunk (m = -inf)
      m0 = n0;
      m1 = n1;
      uint32_t pa[4];
      float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float p0 = exp2f(sc[nt][0] - n0), p1 = exp2f(sc[nt][1] - n0);
        const float p2 = exp2f(sc[nt][2] - n1), p3 = exp2f(sc[nt][3] - n1);
        ps0 += p0 + p1;
        ps1 += p2 + p3;
        pa[2 * nt] = pack_bf16(p0, p1);
        pa[2 * nt + 1] = pack_bf16(p2, p3);
      }
      l0 = l0 * s0 + ps0;  // lane partial (the quad's sum is taken at the end)
      l1 = l1 * s1 + ps1;
#pragma unroll
      for (int nt = 0; nt < D / 8; ++nt) {
        o[nt][0] *= s0;
        o[nt][1] *= s0;
        o[nt][2] *= s1;
        o[nt][3] *= s1;
      }
#pragma unroll
      for (int e0 = 0; e0 < D; e0 += 16) {
        uint32_t v[4];
        ldsm_x4_trans(v, vs + (size_t)(kb + (mi & 1) * 8 + mr) * KLD + e0 + (mi >> 1) * 8);
        mma_bf16_16816(o[e0 / 8], pa[0], pa[1], pa[2], pa[3], v[0], v[1]);
        mma_bf16_16816(o[e0 / 8 + 1], pa[0], pa[1], pa[2], pa[3], v[2], v[3]);
      }
    }
    __syncthreads();  // buffer b is refilled by the next iteration's issue
  }
  cp_async_wait_group<0>();
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  // ---- the four warps into the CTA's partial ----
  if (c == 0) {
    wm[warp][r] = m0;
    wm[warp][r + 8] = m1;
    wl[warp][r] = l0;
    wl[warp][r + 8] = l1;
  }
  {
    float* ow = wo + (size_t)warp * g * D;
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) {
      if (r < g) *reinterpret_cast<float2*>(ow + r * D + nt * 8 + 2 * c) = make_float2(o[nt][0], o[nt][1]);
      if (r + 8 < g) *reinterpret_cast<float2*>(ow + (r + 8) * D + nt * 8 + 2 * c) = make_float2(o[nt][2], o[nt][3]);
    }
  }
  __syncthreads();
  if (tid < g) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AC_THREADS / 32; ++w) M = fmaxf(M, wm[w][tid]);
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < AC_THREADS / 32; ++w) {
      const float a = M == -INFINITY ? 0.0f : exp2f(wm[w][tid] - M);
      wm[w][tid] = a;  // the warp's weight in the CTA's partial
      L += a * wl[w][tid];
    }
    cm[tid] = M;
    cl[tid] = L;
  }
  __syncthreads();
  for (int q = tid; q < g * D; q += AC_THREADS) {
    const int j = q / D;
    float a = 0.0f;
#pragma unroll
    for (int w = 0; w < AC_THREADS / 32; ++w) a = fmaf(wm[w][j], wo[(size_t)w * g * D + q], a);
    co[q] = a;
  }
  // ---- the cluster's CTAs through distributed shared memory ----
  cluster_sync_all();
  const int per = (g * D + AC_CL - 1) / AC_CL;
  for (int q = (int)rank * per + tid; q < min(g * D, ((int)rank + 1) * per); q += AC_THREADS) {
    const int j = q / D;
    float M = -INFINITY, mv[AC_CL];
#pragma unroll
    for (int cr = 0; cr < AC_CL; ++cr) {
      mv[cr] = ld_dsmem(dsmem_addr(&cm[j], cr));
      M = fmaxf(M, mv[cr]);  // finite: rank 0 holds chunk 0, whose first key is valid
    }
    float L = 0.0f, a = 0.0f;
#pragma unroll
    for (int cr = 0; cr < AC_CL; ++cr) {
      const float w = exp2f(mv[cr] - M);
      L = fmaf(w, ld_dsmem(dsmem_addr(&cl[j], cr)), L);
      a = fmaf(w, ld_dsmem(dsmem_addr(co + q, cr)), a);
    }
    out[(size_t)t * nq * D + (size_t)kh * g * D + q] = f2bf(a / L);
  }
  cluster_sync_all();  // every CTA's shared memory stays until the cluster has read it
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
  B2Q_TRY_CUDA(launch_pdl(add_rms_norm_kernel, dim3(T), dim3(NORM_THREADS), 0, static_cast<cudaStream_t>(stream), h,
                          delta, weight, h_out, out, H, eps));
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

extern "C" {

size_t b2q_attn_decode_workspace_size(int T, int nq, int nk, int head_dim, int window) {
  if (T < 1 || T > AD_MAXT || nq < 1 || nk < 1 || nq % nk || head_dim < 1 || window < 1) return 0;
  const size_t chunks = (size_t)(window + AD_CH - 1) / AD_CH;
  const size_t part = sizeof(float) * (size_t)T * nk * chunks * (size_t)ad_stride(nq / nk, head_dim);
  return ((size_t)AD_MAXT * nk * 4 + 255) / 256 * 256 + part;
}

int b2q_attn_decode(const uint16_t* qkv, int q_ld, const int32_t* positions, uint16_t* k_cache, uint16_t* v_cache,
                    uint16_t* out, int T, int nq, int nk, int head_dim, float theta, int window, int* status,
                    void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (T < 0 || T > AD_MAXT || nq < 1 || nk < 1 || nq % nk || nq / nk > ATT_MAXG || head_dim < 16 || head_dim % 16 ||
      head_dim > ATT_MAXD || window < 1 || q_ld < (nq + 2 * nk) * head_dim || q_ld % 8 || !(theta > 1.0f))
    return set_error(B2Q_EINVAL, "attn_decode: bad shape (T=%d nq=%d nk=%d head_dim=%d window=%d)", T, nq, nk,
                     head_dim, window);
  if (T == 0) return B2Q_OK;
  if (!qkv || !positions || !k_cache || !v_cache || !out || !workspace)
    return set_error(B2Q_EINVAL, "attn_decode: null pointer");
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(qkv) || (reinterpret_cast<uintptr_t>(out) & 7) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(B2Q_EINVAL,
                     "attn_decode: qkv, k_cache, v_cache 16-byte, out 8-byte and workspace 256-byte aligned");
  const size_t need = b2q_attn_decode_workspace_size(T, nq, nk, head_dim, window);
  if (workspace_bytes < need) return set_error(B2Q_EINVAL, "attn_decode: workspace of %zu bytes needed", need);
  const int g = nq / nk;
  const int chunks = (window + AD_CH - 1) / AD_CH;
  if (chunks > 65535) return set_error(B2Q_EINVAL, "attn_decode: window %d", window);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == AC_D) {
    // one cluster of AC_CL CTAs per (row, kv head), merged in distributed shared memory
    const size_t smem = ac_smem_bytes(g);
    static bool attr_set[64] = {};
    DeviceInfo di;
    int rc = device_info(&di);
    if (rc) return rc;
    if (smem + 2048 > (size_t)di.smem_optin)
      return set_error(B2Q_EUNSUPPORTED, "attn_decode: %zu bytes of shared memory", smem);
    if (!attr_set[di.device & 63]) {  // the largest g's need, once per device
      B2Q_TRY_CUDA(cudaFuncSetAttribute(attn_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)ac_smem_bytes(ATT_MAXG)));
      attr_set[di.device & 63] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(AC_CL, nk, T);
    cfg.blockDim = dim3(AC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = AC_CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
    B2Q_TRY_CUDA(cudaLaunchKernelEx(&cfg, attn_cluster_kernel, qkv, q_ld, T, positions, nq, nk, log2f(theta), k_cache,
                                    v_cache, window, scale_log2, out, status));
    return B2Q_OK;
  }
  // counters first (at the same place whatever T), then the chunk partials
  unsigned* cnt = static_cast<unsigned*>(workspace);
  float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + ((size_t)AD_MAXT * nk * 4 + 255) / 256 * 256);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  const size_t smem = ad_smem_bytes(g, head_dim, chunks);
  static size_t attr_bytes[64] = {};  // dynamic shared memory allowed so far, per device
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (smem + 1024 > (size_t)di.smem_optin)  // the kernel's static shared memory is under 1 KB
    return set_error(B2Q_EUNSUPPORTED, "attn_decode: %zu bytes of shared memory (window %d)", smem, window);
  if (smem > attr_bytes[di.device & 63]) {
    B2Q_TRY_CUDA(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_bytes[di.device & 63] = smem;
  }
  B2Q_TRY_CUDA(launch_pdl(attn_decode_kernel, dim3(nk, chunks, T), dim3(AD_THREADS), smem, st, qkv, q_ld, T,
                          positions, nq, nk, head_dim, log2f(theta), k_cache, v_cache, window, chunks, scale_log2,
                          part, cnt, out, status));
  B2Q_TRY_CUDA(cudaGetLastError());
  return B2Q_OK;
}

}  // extern "C"
