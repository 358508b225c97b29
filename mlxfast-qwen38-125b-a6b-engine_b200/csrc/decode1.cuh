// decode1.cuh -- single-column streaming products (qmv M = 1, fused one-token MoE decode).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

enum { D1_QMV = 0, D1_FUSED = 1, D1_FUSED_EP = 2 };

struct alignas(64) D1Params {
  CUtensorMap map[9];  // qmv: W, S, B; fused: gate W/S/B, up W/S/B, down W/S/B
  int gs;
  int K1;  // reduction length of the first family (qmv K, or H)
  int N;   // qmv rows
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* wr;
  uint16_t* out;
  uint32_t* idx_out;
  float* w_out;
  float* logits_out;
  int H, E, F, k;
  int* err;
  unsigned* counters;
  unsigned* sched;  // [2] dynamic unit counters (fused)
  float* ws_logits;
  uint16_t* ws_act;
  long long timeout_ns;
  int e_lo, e_local;  // expert parallel: this rank holds experts [e_lo, e_lo + e_local) (e_local 0: all)
  float* out_f32;     // expert parallel: fp32 partial output instead of bf16 `out`
  int off_slots, off_x, off_xs, off_act, off_acts, off_red, off_misc, smem_bytes;
  int XS1, XS2;
};

bool d1_qmv_eligible(int N, int K, int gs, const void* x, const void* w, const void* s, const void* b);
int d1_qmv(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b, uint16_t* y, int N, int K,
           int gs, cudaStream_t st);
bool d1_moe_eligible(int H, int E, int F, int k, int gs);
int d1_moe_decode(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                  const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd, const uint16_t* sd,
                  const uint16_t* bd, uint16_t* out, uint32_t* idx, float* w, float* logits, int H, int E, int F,
                  int k, int gs, int* err, unsigned* counters, unsigned* sched, float* ws_logits,
                  uint16_t* ws_act, cudaStream_t st, int e_lo = 0, int e_local = 0, float* out_f32 = nullptr);

}  // namespace b2q
