/* b2q_oracle.c -- CPU restatement of the reference arithmetic (TEST
 * INFRASTRUCTURE ONLY; see b2q_oracle.h for who may load it).
 *
 * Every function names the reference lines it restates. Paths are relative to
 * the reference project; MLXC = Vendor/mlx-swift/Source/Cmlx/mlx/mlx,
 * QH = MLXC/backend/metal/kernels/quantized.h, CQ = MLXC/backend/cpu/quantized.cpp,
 * MOE = Runner/FastModel/TrackFastMoE.swift.
 *
 * Compiled with -ffp-contract=off so every fp32 operation rounds as written. */
#include "b2q_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_EINVAL (-1)
#define ORC_EUNSUPPORTED (-2)
#define ORC_ENOMEM (-3)

/* ---- bf16 <-> f32, MLXC/types/bf16.h:39-69 (RNE, NaN -> 0x7FC0) ---------- */
typedef union {
  uint32_t u;
  float f;
} fbits;

float orc_bf2f(uint16_t h) {
  fbits v;
  v.u = (uint32_t)h << 16;
  return v.f;
}

uint16_t orc_f2bf(float f) {
  fbits v;
  if (isnan(f)) return 0x7FC0;
  v.f = f;
  v.u += ((v.u >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)(v.u >> 16);
}

static inline float rb(float f) { return orc_bf2f(orc_f2bf(f)); } /* round through bf16 */

static int bits_ok(int bits) { return bits == 2 || bits == 4 || bits == 8; }
static int gs_ok(int gs) { return gs == 32 || gs == 64 || gs == 128; }

static inline uint32_t qval(const uint32_t* wrow, int k, int bits) {
  const int per = 32 / bits;
  return (wrow[k / per] >> ((k % per) * bits)) & ((1u << bits) - 1u);
}

/* ---- quantize: CQ:1158-1236 (power-of-2 bits branch) ---------------------- */
int orc_quantize(const uint16_t* w, int64_t n_el, int group_size, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  if (!bits_ok(bits) || !gs_ok(group_size) || n_el % group_size) return ORC_EINVAL;
  const float n_bins = (float)((1 << bits) - 1);
  const float eps = 1e-7f;
  const int el_per_int = 32 / bits;
  const int int_per_group = group_size / el_per_int;
  const int64_t n_groups = n_el / group_size;
  for (int64_t i = 0; i < n_groups; ++i) {
    const int64_t w_idx = i * group_size;
    float w_min = INFINITY, w_max = -INFINITY;
    for (int j = 0; j < group_size; ++j) {
      const float v = orc_bf2f(w[w_idx + j]);
      w_max = (w_max < v) ? v : w_max; /* std::max(a, b) = (a < b) ? b : a */
      w_min = (v < w_min) ? v : w_min; /* std::min(a, b) = (b < a) ? b : a */
    }
    const int mask = fabsf(w_min) > fabsf(w_max);
    float scale = (w_max - w_min) / n_bins;
    scale = (scale < eps) ? eps : scale;
    scale = mask ? scale : -scale;
    const float edge = mask ? w_min : w_max;
    const float q0 = rintf(edge / scale);
    float bias = 0.0f;
    if (q0 != 0.0f) {
      scale = edge / q0;
      bias = edge;
    }
    for (int j = 0; j < int_per_group; ++j) {
      uint64_t out_el = 0;
      for (int kk = 0; kk < el_per_int; ++kk) {
        float w_el = orc_bf2f(w[w_idx + j * el_per_int + kk]);
        w_el = rintf((w_el - bias) / scale);
        w_el = (w_el < 0.0f) ? 0.0f : w_el;
        w_el = (n_bins < w_el) ? n_bins : w_el;
        out_el |= (uint64_t)w_el << (kk * bits);
      }
      wq[i * int_per_group + j] = (uint32_t)out_el;
    }
    scales[i] = orc_f2bf(scale);
    biases[i] = orc_f2bf(bias);
  }
  return ORC_OK;
}

/* ---- dequantize ------------------------------------------------------------ */
/* (ii) QH:485-530 (bits 4: sc = {s, s/16}; w_local = U(sc*(w & mask) + b)) and
 * the affine_dequantize kernel QH:3314-3373. s*q is exact in fp32, so this is
 * one fp32 rounding of the add followed by the bf16 rounding. */
int orc_dequantize_metal(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                         uint16_t* out, int64_t rows, int K, int group_size, int bits) {
  if (!bits_ok(bits) || !gs_ok(group_size) || K % group_size) return ORC_EINVAL;
  const int wpr = K * bits / 32, G = K / group_size;
  for (int64_t r = 0; r < rows; ++r)
    for (int k = 0; k < K; ++k) {
      const float sc = orc_bf2f(s[r * G + k / group_size]);
      const float bi = orc_bf2f(b[r * G + k / group_size]);
      const float q = (float)qval(w + r * wpr, k, bits);
      out[r * (int64_t)K + k] = orc_f2bf(sc * q + bi);
    }
  return ORC_OK;
}

/* (i) MLXC/ops.cpp:5290-5327: the unpacked uint32 tensor is multiplied by the
 * bf16 scales (promotes to bf16: one rounding) and the bf16 biases are added
 * (another rounding). */
int orc_dequantize_cpu(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                       uint16_t* out, int64_t rows, int K, int group_size, int bits) {
  if (!bits_ok(bits) || !gs_ok(group_size) || K % group_size) return ORC_EINVAL;
  const int wpr = K * bits / 32, G = K / group_size;
  for (int64_t r = 0; r < rows; ++r)
    for (int k = 0; k < K; ++k) {
      const float sc = orc_bf2f(s[r * G + k / group_size]);
      const float bi = orc_bf2f(b[r * G + k / group_size]);
      const float q = (float)qval(w + r * wpr, k, bits);
      out[r * (int64_t)K + k] = orc_f2bf(rb(q * sc) + bi);
    }
  return ORC_OK;
}

/* ---- Metal qmv lane association (bits = 4) --------------------------------- */
/* One output row. vpt = 16 (qmv_fast_impl, QH:757-822) or 8 (qmv_impl,
 * QH:824-987). Lane l owns x[blk + l*vpt, +vpt); load_vector (QH:28-105)
 * pre-divides x by 16^j and sums x in fours; qdot (QH:191-290) multiplies by
 * the masked 16-bit halves and returns s*accum + sum*b; simd_sum is taken as
 * an xor butterfly (16, 8, 4, 2, 1). */
static float qmv_row_metal(const uint16_t* x, const uint32_t* wrow, const uint16_t* srow,
                           const uint16_t* brow, int K, int gs) {
  const int vpt = (K % 512 == 0) ? 16 : 8;
  const int block = vpt * 32;
  const uint8_t* wb = (const uint8_t*)wrow;
  float lane_res[32];
  for (int lane = 0; lane < 32; ++lane) {
    float result = 0.0f;
    int k = 0;
    /* qmv_fast: k < K over whole blocks; qmv_impl: whole blocks while
     * k < K - block, then one guarded tail. */
    const int full_end = (vpt == 16) ? K : K - block;
    for (; (vpt == 16) ? (k < full_end) : (k < full_end); k += block) {
      const int k0 = k + lane * vpt;
      float xt[16];
      float sum = 0.0f;
      for (int i = 0; i < vpt; i += 4) {
        const float a = orc_bf2f(x[k0 + i]), bq = orc_bf2f(x[k0 + i + 1]);
        const float c = orc_bf2f(x[k0 + i + 2]), d = orc_bf2f(x[k0 + i + 3]);
        sum += ((a + bq) + c) + d;
        xt[i] = a;
        xt[i + 1] = bq / 16.0f;
        xt[i + 2] = c / 256.0f;
        xt[i + 3] = d / 4096.0f;
      }
      const float sc = orc_bf2f(srow[k0 / gs]), bi = orc_bf2f(brow[k0 / gs]);
      float accum = 0.0f;
      for (int i = 0; i < vpt / 4; ++i) {
        const uint16_t ws = (uint16_t)(wb[k0 / 2 + 2 * i] | (wb[k0 / 2 + 2 * i + 1] << 8));
        accum += ((xt[4 * i] * (float)(ws & 0x000f) + xt[4 * i + 1] * (float)(ws & 0x00f0)) +
                  xt[4 * i + 2] * (float)(ws & 0x0f00)) +
                 xt[4 * i + 3] * (float)(ws & 0xf000);
      }
      result += sc * accum + sum * bi;
    }
    if (vpt == 8) {
      int remaining = K - k - lane * vpt;
      remaining = remaining < 0 ? 0 : (remaining > vpt ? vpt : remaining);
      if (remaining > 0) {
        const int k0 = k + lane * vpt;
        float xt[8] = {0};
        float sum = 0.0f;
        for (int i = 0; i < remaining; i += 4) {
          const float a = orc_bf2f(x[k0 + i]), bq = orc_bf2f(x[k0 + i + 1]);
          const float c = orc_bf2f(x[k0 + i + 2]), d = orc_bf2f(x[k0 + i + 3]);
          sum += ((a + bq) + c) + d;
          xt[i] = a;
          xt[i + 1] = bq / 16.0f;
          xt[i + 2] = c / 256.0f;
          xt[i + 3] = d / 4096.0f;
        }
        const float sc = orc_bf2f(srow[k0 / gs]), bi = orc_bf2f(brow[k0 / gs]);
        float accum = 0.0f;
        for (int i = 0; i < remaining / 4; ++i) {
          const uint16_t ws = (uint16_t)(wb[k0 / 2 + 2 * i] | (wb[k0 / 2 + 2 * i + 1] << 8));
          accum += ((xt[4 * i] * (float)(ws & 0x000f) + xt[4 * i + 1] * (float)(ws & 0x00f0)) +
                    xt[4 * i + 2] * (float)(ws & 0x0f00)) +
                   xt[4 * i + 3] * (float)(ws & 0xf000);
        }
        result += sc * accum + sum * bi;
      }
    }
    lane_res[lane] = result;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float t[32];
    for (int l = 0; l < 32; ++l) t[l] = lane_res[l] + lane_res[l ^ off];
    memcpy(lane_res, t, sizeof(t));
  }
  return lane_res[0];
}

int orc_qmv_metal_f32(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                      const uint16_t* b, float* y, int M, int N, int K,
                      int group_size, int bits) {
  if (bits != 4) return ORC_EUNSUPPORTED;
  if (!gs_ok(group_size) || K % group_size || K % 32 || M < 0 || N < 0) return ORC_EINVAL;
  const int wpr = K / 8, G = K / group_size;
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n)
      y[(int64_t)m * N + n] = qmv_row_metal(x + (int64_t)m * K, w + (int64_t)n * wpr,
                                            s + (int64_t)n * G, b + (int64_t)n * G, K, group_size);
  return ORC_OK;
}

int orc_qmv_metal(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                  const uint16_t* b, uint16_t* y, int M, int N, int K,
                  int group_size, int bits) {
  if (bits != 4) return ORC_EUNSUPPORTED;
  if (!gs_ok(group_size) || K % group_size || K % 32 || M < 0 || N < 0) return ORC_EINVAL;
  const int wpr = K / 8, G = K / group_size;
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n)
      y[(int64_t)m * N + n] = orc_f2bf(qmv_row_metal(x + (int64_t)m * K, w + (int64_t)n * wpr,
                                                     s + (int64_t)n * G, b + (int64_t)n * G, K,
                                                     group_size));
  return ORC_OK;
}

/* ---- MLX CPU _qmm_t, CQ:155-210 with T = bfloat16 ---------------------------
 * sum += x * (scale * T(q) + bias): T(q) exact, then bf16 *, +, *, += each
 * computed in float and rounded to bf16 (MLXC/types/bf16.h:72-130). */
int orc_qmm_mlx_cpu(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                    const uint16_t* b, uint16_t* y, int M, int N, int K,
                    int group_size, int bits) {
  if (!bits_ok(bits) || !gs_ok(group_size) || K % group_size) return ORC_EINVAL;
  const int wpr = K * bits / 32, G = K / group_size;
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      float sum = 0.0f; /* a bf16 value held as float */
      const uint32_t* wrow = w + (int64_t)n * wpr;
      for (int k = 0; k < K; ++k) {
        const float sc = orc_bf2f(s[(int64_t)n * G + k / group_size]);
        const float bi = orc_bf2f(b[(int64_t)n * G + k / group_size]);
        const float q = (float)qval(wrow, k, bits);
        const float wd = rb(rb(sc * q) + bi);
        const float p = rb(orc_bf2f(x[(int64_t)m * K + k]) * wd);
        sum = rb(sum + p);
      }
      y[(int64_t)m * N + n] = orc_f2bf(sum);
    }
  return ORC_OK;
}

/* ---- tile-loader product (prefill) ------------------------------------------ */
int orc_qmm_tile(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                 const uint16_t* b, float* y, int M, int N, int K,
                 int group_size, int bits) {
  if (!bits_ok(bits) || !gs_ok(group_size) || K % group_size) return ORC_EINVAL;
  const int wpr = K * bits / 32, G = K / group_size;
  float* wrow = (float*)malloc(sizeof(float) * (size_t)K);
  if (!wrow) return ORC_ENOMEM;
  for (int n = 0; n < N; ++n) {
    for (int k = 0; k < K; ++k) {
      const float sc = orc_bf2f(s[(int64_t)n * G + k / group_size]);
      const float bi = orc_bf2f(b[(int64_t)n * G + k / group_size]);
      wrow[k] = rb(sc * (float)qval(w + (int64_t)n * wpr, k, bits) + bi);
    }
    for (int m = 0; m < M; ++m) {
      float acc = 0.0f;
      const uint16_t* xr = x + (int64_t)m * K;
      for (int k = 0; k < K; ++k) acc += orc_bf2f(xr[k]) * wrow[k];
      y[(int64_t)m * N + n] = acc;
    }
  }
  free(wrow);
  return ORC_OK;
}

/* ---- router ------------------------------------------------------------------ */
int orc_router_logits(const uint16_t* x, const uint16_t* wr, float* logits,
                      int T, int E, int H) {
  for (int t = 0; t < T; ++t)
    for (int e = 0; e < E; ++e) {
      float acc = 0.0f;
      for (int h = 0; h < H; ++h)
        acc += orc_bf2f(x[(int64_t)t * H + h]) * orc_bf2f(wr[(int64_t)e * H + h]);
      logits[(int64_t)t * E + e] = acc;
    }
  return ORC_OK;
}

/* MOE:767-911. Selection: k rounds, each takes the largest untaken value with
 * the lowest index on ties (lane-strided ownership + simd_max/simd_min).
 * Softmax: N_READS = 4 per lane in slot order, lane partial sums in order,
 * butterfly sum of the lane partials, w = e * (1 / sum). */
int orc_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k) {
  if (k < 1 || k > 32 || k > E) return ORC_EINVAL;
  unsigned char* taken = (unsigned char*)malloc((size_t)E);
  if (!taken) return ORC_ENOMEM;
  for (int t = 0; t < T; ++t) {
    const float* lr = logits + (int64_t)t * E;
    memset(taken, 0, (size_t)E);
    float vals[32];
    for (int j = 0; j < k; ++j) {
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (!taken[e] && (best < 0 || lr[e] > lr[best])) best = e;
      taken[best] = 1;
      idx[(int64_t)t * k + j] = (uint32_t)best;
      vals[j] = lr[best];
    }
    float mx = -INFINITY;
    for (int j = 0; j < k; ++j) mx = (mx < vals[j]) ? vals[j] : mx;
    float ex[32];
    float part[32];
    for (int l = 0; l < 32; ++l) part[l] = 0.0f;
    for (int j = 0; j < k; ++j) {
      ex[j] = expf(vals[j] - mx);
      part[j / 4] += ex[j];
    }
    for (int off = 16; off >= 1; off >>= 1) {
      float tmp[32];
      for (int l = 0; l < 32; ++l) tmp[l] = part[l] + part[l ^ off];
      memcpy(part, tmp, sizeof(tmp));
    }
    const float inv = 1.0f / part[0];
    for (int j = 0; j < k; ++j) w[(int64_t)t * k + j] = ex[j] * inv;
  }
  free(taken);
  return ORC_OK;
}

/* ---- bf16 elementwise, Runner/FastModel/TrackFastKernels2.swift:22-47 --------- */
uint16_t orc_sigmoid_bf16(uint16_t xb) {
  const float x = orc_bf2f(xb);
  const float e = rb(expf(rb(fabsf(x))));
  const float y = rb(1.0f / rb(1.0f + e));
  return orc_f2bf((x < 0.0f) ? y : rb(1.0f - y));
}
uint16_t orc_silu_bf16(uint16_t xb) {
  return orc_f2bf(orc_bf2f(xb) * orc_bf2f(orc_sigmoid_bf16(xb)));
}
uint16_t orc_swiglu_bf16(uint16_t g, uint16_t u) {
  return orc_f2bf(orc_bf2f(orc_silu_bf16(g)) * orc_bf2f(u));
}
/* mlx_colsum_small_f32<K>: TY = min(8, K) chains fold rows y, y+TY, ... into
 * 0 as r + acc, then total = t[0]; total = t[j] + total for j = 1.. */
float orc_colsum_small(const float* r, int K) {
  if (K <= 0) return 0.0f;
  const int TY = K < 8 ? K : 8;
  float t[8] = {0};
  for (int y = 0; y < TY; ++y) {
    float acc = 0.0f;
    for (int rr = y; rr < K; rr += TY) acc = r[rr] + acc;
    t[y] = acc;
  }
  float total = t[0];
  for (int j = 1; j < TY; ++j) total = t[j] + total;
  return total;
}

/* ---- decode MoE ----------------------------------------------------------------- */
static int expert_chain_decode(const uint16_t* xt, const uint32_t* idx, const float* wts,
                               const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                               const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                               const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                               int H, int F, int k, int gs, uint16_t* act_out, uint16_t* out) {
  const int64_t gu_w = (int64_t)F * (H / 8), gu_g = (int64_t)F * (H / gs);
  const int64_t d_w = (int64_t)H * (F / 8), d_g = (int64_t)H * (F / gs);
  float* g = (float*)malloc(sizeof(float) * (size_t)F);
  float* u = (float*)malloc(sizeof(float) * (size_t)F);
  uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)F * k);
  float* y = (float*)malloc(sizeof(float) * (size_t)H * k);
  int rc = ORC_OK;
  if (!g || !u || !act || !y) { rc = ORC_ENOMEM; goto done; }
  for (int j = 0; j < k; ++j) {
    const int64_t e = idx[j];
    rc = orc_qmv_metal_f32(xt, wg + e * gu_w, sg + e * gu_g, bg + e * gu_g, g, 1, F, H, gs, 4);
    if (rc) goto done;
    rc = orc_qmv_metal_f32(xt, wu + e * gu_w, su + e * gu_g, bu + e * gu_g, u, 1, F, H, gs, 4);
    if (rc) goto done;
    for (int f = 0; f < F; ++f) act[(int64_t)j * F + f] = orc_swiglu_bf16(orc_f2bf(g[f]), orc_f2bf(u[f]));
    rc = orc_qmv_metal_f32(act + (int64_t)j * F, wd + e * d_w, sd + e * d_g, bd + e * d_g,
                           y + (int64_t)j * H, 1, H, F, gs, 4);
    if (rc) goto done;
  }
  if (act_out) memcpy(act_out, act, sizeof(uint16_t) * (size_t)F * k);
  for (int h = 0; h < H; ++h) {
    float prod[64];
    for (int j = 0; j < k; ++j) prod[j] = rb(y[(int64_t)j * H + h]) * wts[j];
    out[h] = orc_f2bf(orc_colsum_small(prod, k));
  }
done:
  free(g); free(u); free(act); free(y);
  return rc;
}

int orc_moe_experts_decode(const uint16_t* x, const uint32_t* idx, const float* wts,
                           const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                           const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                           const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                           int H, int E, int F, int k, int group_size,
                           const int32_t* rows, int n_sel, uint16_t* out) {
  (void)E;
  if (k < 1 || k > 64) return ORC_EINVAL;
  for (int i = 0; i < n_sel; ++i) {
    const int t = rows ? rows[i] : i;
    int rc = expert_chain_decode(x + (int64_t)t * H, idx + (int64_t)t * k, wts + (int64_t)t * k,
                                 wg, sg, bg, wu, su, bu, wd, sd, bd, H, F, k, group_size, NULL,
                                 out + (int64_t)i * H);
    if (rc) return rc;
  }
  return ORC_OK;
}

int orc_moe_decode(const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   int S, int H, int E, int F, int k, int group_size,
                   float* logits, uint32_t* idx, float* wts, uint16_t* act,
                   uint16_t* out) {
  if (S < 1 || k < 1 || k > 32 || k > E) return ORC_EINVAL;
  float* lg = (float*)malloc(sizeof(float) * (size_t)S * E);
  uint32_t* ix = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)S * k);
  float* ww = (float*)malloc(sizeof(float) * (size_t)S * k);
  uint16_t* o = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)H);
  int rc = ORC_OK;
  if (!lg || !ix || !ww || !o) { rc = ORC_ENOMEM; goto done; }
  orc_router_logits(x, wr, lg, S, E, H);
  rc = orc_route(lg, ix, ww, S, E, k);
  if (rc) goto done;
  for (int t = 0; t < S; ++t) {
    rc = expert_chain_decode(x + (int64_t)t * H, ix + (int64_t)t * k, ww + (int64_t)t * k,
                             wg, sg, bg, wu, su, bu, wd, sd, bd, H, F, k, group_size,
                             act ? act + (int64_t)t * k * F : NULL, o);
    if (rc) goto done;
    if (out) memcpy(out + (int64_t)t * H, o, sizeof(uint16_t) * (size_t)H);
  }
  if (logits) memcpy(logits, lg, sizeof(float) * (size_t)S * E);
  if (idx) memcpy(idx, ix, sizeof(uint32_t) * (size_t)S * k);
  if (wts) memcpy(wts, ww, sizeof(float) * (size_t)S * k);
done:
  free(lg); free(ix); free(ww); free(o);
  return rc;
}

/* ---- stable counting sort, Runner/FastModel/TrackPrefillSort.swift:17-44 ----- */
int orc_sort_by_expert(const uint32_t* ids, int R, int E, int k,
                       uint32_t* sorted_ids, uint32_t* token_rows,
                       uint32_t* inverse, uint32_t* offsets) {
  if (R < 0 || E < 1 || k < 1) return ORC_EINVAL;
  uint32_t* cnt = (uint32_t*)calloc((size_t)E + 1, sizeof(uint32_t));
  if (!cnt) return ORC_ENOMEM;
  for (int i = 0; i < R; ++i) {
    if (ids[i] >= (uint32_t)E) { free(cnt); return ORC_EINVAL; }
    cnt[ids[i] + 1]++;
  }
  for (int e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
  if (offsets) memcpy(offsets, cnt, sizeof(uint32_t) * ((size_t)E + 1));
  for (int i = 0; i < R; ++i) {
    const uint32_t p = cnt[ids[i]]++;
    if (sorted_ids) sorted_ids[p] = ids[i];
    if (token_rows) token_rows[p] = (uint32_t)(i / k);
    if (inverse) inverse[i] = p;
  }
  free(cnt);
  return ORC_OK;
}

/* ---- prefill MoE experts ----------------------------------------------------------- */
int orc_moe_experts_prefill(const uint16_t* x, const uint32_t* idx, const float* wts,
                            const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                            const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                            const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                            int H, int E, int F, int k, int group_size,
                            const int32_t* rows, int n_sel, uint16_t* out) {
  (void)E;
  if (k < 1 || k > 64) return ORC_EINVAL;
  const int64_t gu_w = (int64_t)F * (H / 8), gu_g = (int64_t)F * (H / group_size);
  const int64_t d_w = (int64_t)H * (F / 8), d_g = (int64_t)H * (F / group_size);
  float* g = (float*)malloc(sizeof(float) * (size_t)F);
  float* u = (float*)malloc(sizeof(float) * (size_t)F);
  uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)F);
  float* y = (float*)malloc(sizeof(float) * (size_t)H * k);
  int rc = ORC_OK;
  if (!g || !u || !act || !y) { rc = ORC_ENOMEM; goto done; }
  for (int i = 0; i < n_sel; ++i) {
    const int t = rows ? rows[i] : i;
    const uint16_t* xt = x + (int64_t)t * H;
    for (int j = 0; j < k; ++j) {
      const int64_t e = idx[(int64_t)t * k + j];
      rc = orc_qmm_tile(xt, wg + e * gu_w, sg + e * gu_g, bg + e * gu_g, g, 1, F, H, group_size, 4);
      if (rc) goto done;
      rc = orc_qmm_tile(xt, wu + e * gu_w, su + e * gu_g, bu + e * gu_g, u, 1, F, H, group_size, 4);
      if (rc) goto done;
      for (int f = 0; f < F; ++f) act[f] = orc_swiglu_bf16(orc_f2bf(g[f]), orc_f2bf(u[f]));
      rc = orc_qmm_tile(act, wd + e * d_w, sd + e * d_g, bd + e * d_g, y + (int64_t)j * H, 1, H, F,
                        group_size, 4);
      if (rc) goto done;
    }
    for (int h = 0; h < H; ++h) {
      float prod[64];
      for (int j = 0; j < k; ++j) prod[j] = rb(y[(int64_t)j * H + h]) * wts[(int64_t)t * k + j];
      out[(int64_t)i * H + h] = orc_f2bf(orc_colsum_small(prod, k));
    }
  }
done:
  free(g); free(u); free(act); free(y);
  return rc;
}
