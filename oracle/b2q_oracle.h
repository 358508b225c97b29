/* b2q_oracle.h -- CPU restatement of the reference arithmetic for the affine
 * 4-bit weight-product path (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, bench.py's cpu_baseline / --impl reference legs and
 * __graft_entry__.smoke() may load this library, and only as the checker or
 * the timed CPU baseline. The product path (the C-ABI library in the package)
 * never links or calls it.
 *
 * Conventions: bf16 values are raw uint16 bit patterns; packed weights are
 * uint32 words holding 8 nibbles, element 8*i+j in bits [4j, 4j+4) of word i
 * (backend/cpu/quantized.cpp:215-233 of the vendored MLX); scales/biases are
 * bf16 [rows, K/group_size]. Every function returns 0 on success.
 *
 * Pinning: quantize and the MLX-CPU bf16 matmul restatements are compared
 * bit-for-bit with the reference's own MLX CPU kernels compiled from the
 * reference tree (oracle/_ref/libmlxref.so) and with the committed golden
 * fixtures in tests/golden/. */
#ifndef B2Q_ORACLE_H
#define B2Q_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

float orc_bf2f(uint16_t h);
uint16_t orc_f2bf(float f);

/* MLX affine quantize, backend/cpu/quantized.cpp:1158-1236 (power-of-2 bits). */
int orc_quantize(const uint16_t* w, int64_t n_el, int group_size, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases);

/* Dequantize, variant (ii): bf16(fp32(s)*q + fp32(b)), one rounding to bf16
 * after the fp32 add -- the Metal tile loader (quantized.h:485-530) and the
 * affine_dequantize kernel. */
int orc_dequantize_metal(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                         uint16_t* out, int64_t rows, int K, int group_size, int bits);
/* Dequantize, variant (i): bf16(bf16(q*s) + b), the CPU op fallback of
 * ops.cpp:5290-5327 (two bf16-rounding MLX ops). */
int orc_dequantize_cpu(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                       uint16_t* out, int64_t rows, int K, int group_size, int bits);

/* y[M,N] = x[M,K] . dequant(w)^T with the Metal qmv lane association:
 * qmv_fast_impl (quantized.h:757-822) when K % 512 == 0, else qmv_impl
 * (quantized.h:824-987); per-lane qdot factorisation s*sum(x*q) + b*sum(x)
 * (quantized.h:191-290), fp32 throughout, xor-butterfly simd_sum, one bf16
 * rounding of the result. */
int orc_qmv_metal(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                  const uint16_t* b, uint16_t* y, int M, int N, int K,
                  int group_size, int bits);
/* Same, but the fp32 result is returned unrounded (for the MoE epilogues). */
int orc_qmv_metal_f32(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                      const uint16_t* b, float* y, int M, int N, int K,
                      int group_size, int bits);

/* MLX CPU scalar _qmm_t with a bf16 running sum (backend/cpu/quantized.cpp:155-210
 * on x86, where simd::max_size == 1): every *, + rounds to bf16. */
int orc_qmm_mlx_cpu(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                    const uint16_t* b, uint16_t* y, int M, int N, int K,
                    int group_size, int bits);

/* Prefill-style dense product: y = bf16( sum_k f32(x) * f32(dequant_ii(w)) ),
 * fp32 accumulation in k order (the tile loader feeds bf16 operands to the
 * matrix units, quantized.h:485-530 + 1547-1673). */
int orc_qmm_tile(const uint16_t* x, const uint32_t* w, const uint16_t* s,
                 const uint16_t* b, float* y, int M, int N, int K,
                 int group_size, int bits);

/* Router logits f32 [T,E] = f32(x) . f32(Wr)^T, fp32 k-order accumulation
 * (TrackFastModel.swift:884-903). */
int orc_router_logits(const uint16_t* x, const uint16_t* wr, float* logits,
                      int T, int E, int H);

/* Top-k + softmax over the selected logits (TrackFastMoE.swift:767-911):
 * largest value first, ties to the lower index; max-subtract, exp, per-lane
 * partial sums of 4 values, butterfly sum, multiply by 1/sum. */
int orc_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k);

/* bf16 elementwise helpers of TrackFastKernels2.swift:22-47. */
uint16_t orc_sigmoid_bf16(uint16_t x);
uint16_t orc_silu_bf16(uint16_t x);
uint16_t orc_swiglu_bf16(uint16_t g, uint16_t u);
float orc_colsum_small(const float* r, int K);

/* Decode MoE layer for S tokens (S <= 8), the fused Runner path:
 * router -> route -> per slot gate|up qmv (fp32) -> bf16 -> SwiGLU (bf16)
 * -> down qmv -> bf16 -> f32 * w -> colsum association -> bf16.
 * TrackFastModel.swift:867-955, TrackFastMoE.swift:1192-1590.
 * Outputs (any may be NULL): logits [S,E], idx/wts [S,k], act [S*k,F], out [S,H]. */
int orc_moe_decode(const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   int S, int H, int E, int F, int k, int group_size,
                   float* logits, uint32_t* idx, float* wts, uint16_t* act,
                   uint16_t* out);

/* Same expert chain with routing given (idx/wts), tokens restricted to the
 * `n_sel` rows listed in `rows` (NULL = all S). Used for large-S checks. */
int orc_moe_experts_decode(const uint16_t* x, const uint32_t* idx, const float* wts,
                           const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                           const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                           const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                           int H, int E, int F, int k, int group_size,
                           const int32_t* rows, int n_sel, uint16_t* out);

/* Stable counting sort of R = T*k expert ids (TrackPrefillSort.swift:17-44):
 * sorted_ids[p], token_rows[p] = order[p]/k, inverse[order[p]] = p, and
 * per-expert offsets [E+1]. */
int orc_sort_by_expert(const uint32_t* ids, int R, int E, int k,
                       uint32_t* sorted_ids, uint32_t* token_rows,
                       uint32_t* inverse, uint32_t* offsets);

/* Prefill MoE experts for selected tokens with routing given: per assignment
 * gate/up = bf16(fp32 sum of x * dequant_ii), act = SwiGLU in bf16,
 * down = bf16(fp32 sum act * dequant_ii), out = bf16(colsum_k f32(down)*w)
 * (TrackP12Prefill.swift:180-237, TrackPrefillIndirectMetal.swift). */
int orc_moe_experts_prefill(const uint16_t* x, const uint32_t* idx, const float* wts,
                            const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                            const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                            const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                            int H, int E, int F, int k, int group_size,
                            const int32_t* rows, int n_sel, uint16_t* out);

#ifdef __cplusplus
}
#endif
#endif
