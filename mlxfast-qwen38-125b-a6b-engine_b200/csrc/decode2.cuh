// decode2.cuh -- single-column products on a unit queue: qmv for one row of x
// (M = 1) and the fused one-token MoE decode layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

enum { D2_QMV = 0, D2_FUSED = 1, D2_FUSED_EP = 2, D2_QMV_LUT = 3 };

// Grid words of the fused kernel (the last CTA out re-arms them):
//   [2] CTAs exited, [3] tag of the last call,
//   [4, 4 + 8) gate|up units finished per routed slot,
//   [512, 512 + 2 E) router logits, each 64-bit word (call tag << 32 | fp32 bits).
// A zeroed block is a valid state (tag 0); it stays valid call to call.
constexpr int D2_CTR_TAG = 3;
constexpr int D2_CTR_LOGITS = 512;

// Exchange buffer of the peer-memory expert-parallel decode (one per rank):
// bytes [0, 256) a header whose word 0 is the rank's call epoch; [256, 512)
// flags[2][D2_XMAX] (u32: the epoch whose partial source s left in slot e);
// from byte 512 data[2][D2_XMAX][H] fp32 partials.
constexpr int D2_XMAX = 8;
constexpr int D2_XFLAGS = 64;   // u32 index of flags[0][0]
constexpr int D2_XDATA = 128;   // float index of data[0][0][0]
inline size_t d2_xbuf_bytes(int H) { return 512 + sizeof(float) * 2 * D2_XMAX * (size_t)H; }

struct alignas(64) D2Params {
  CUtensorMap map[9];  // qmv: W, S, B; fused: gate W/S/B, up W/S/B, down W/S/B
  int gs;
  int K1;  // reduction length of the gate|up / qmv family (H, or the qmv K)
  int N;   // qmv rows
  int H, E, F, k;
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* wr;
  uint16_t* out;
  uint32_t* idx_out;
  float* w_out;
  float* logits_out;
  int* err;
  unsigned* ctr;
  float* ws_logits;   // [E]
  uint16_t* ws_act;   // [k][F] SwiGLU activations as int8 pieces (16 bytes per word of 8 values)
  float2* ws_asc;     // [k][F / 16] per block of 16 activations: (2^(E - 14), sum)
  long long timeout_ns;
  int e_lo, e_local;  // expert parallel: this rank holds experts [e_lo, e_lo + e_local) (e_local 0: all)
  float* out_f32;     // expert parallel: fp32 partial output instead of bf16 `out`
  // residual add + RMSNorm fused into the pass over x (nw != nullptr): x is
  // h, the call multiplies bf16(bf16(h + ndelta) * r * nw) with
  // r = rsqrt(mean(bf16(h + ndelta)^2) + neps); CTA 0 writes bf16(h + ndelta)
  // to nh_out (ndelta nullptr: no add, nh_out unused)
  const uint16_t* nw;
  const uint16_t* ndelta;
  uint16_t* nh_out;
  float neps;
  // expert parallel over peer memory (npeer > 0): every rank's exchange
  // buffer (this rank's at xpeer[prank]) mapped into this process; the
  // kernel stores its fp32 block partials into all of them, publishes a
  // per-call epoch, waits for every rank's and writes the summed bf16 `out`
  float* xpeer[D2_XMAX];
  int npeer, prank;
  const uint32_t* lut;  // qmv through the metadata pair table: scale_bits | bias_bits << 16 per entry
  int lut_words;        // table entries copied into shared memory (a multiple of 4)
  int off_lut;          // shared-memory offset of the table copy
  // launch plan (host)
  int nstage, stage_bytes, smem_bytes;
  int off_xs, off_ysm, off_red, off_misc;
  int mb1, mb2;             // metadata row bytes: first family, down
  int sw1, sw2;             // metadata blocks in the 128-byte swizzle
  int st_meta1, st_mstep1;  // first family: metadata blocks inside a stage
  int st_meta2, st_mstep2, st_act, st_asc;  // down units
};

bool d2_qmv_eligible(int N, int K, int gs, const void* x, const void* w, const void* s, const void* b);
// The residual add + RMSNorm of the product's input, fused into its pass over x.
struct D2Norm {
  const uint16_t* weight = nullptr;  // nullptr: x is used as given
  const uint16_t* delta = nullptr;
  uint16_t* h_out = nullptr;
  float eps = 0.0f;
};
int d2_qmv(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b, uint16_t* y, int N, int K,
           int gs, cudaStream_t st, const D2Norm& norm = D2Norm());
// the fused norm needs one 8-value chunk of the reduction per thread
bool d2_norm_ok(int K);
// qmv with the group metadata read through a pair table (index u16 [N, K/gs],
// table of `count` entries, 16-byte aligned, readable up to round_up(count, 4)).
bool d2_qmv_lut_eligible(int N, int K, int gs, int count, const void* x, const void* w, const void* index,
                         const void* table);
int d2_qmv_lut(const uint16_t* x, const uint32_t* w, const uint16_t* index, const uint32_t* table, int count,
               uint16_t* y, int N, int K, int gs, cudaStream_t st);
bool d2_moe_eligible(int H, int E, int F, int k, int gs);
// Device scratch of one fused call (all caller-owned; ctr zeroed once: the
// grid words and tagged router logits, 4096 bytes).
struct D2Scratch {
  int* err;
  unsigned* ctr;      // d2_counter_words(H)
  float* logits;      // [E]
  uint16_t* act;      // [k][F]
  float2* asc;        // [k][F / 16]
};
int d2_moe_decode(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                  const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd, const uint16_t* sd,
                  const uint16_t* bd, uint16_t* out, uint32_t* idx, float* w, float* logits, int H, int E, int F,
                  int k, int gs, const D2Scratch& scr, cudaStream_t st, int e_lo = 0, int e_local = 0,
                  float* out_f32 = nullptr, const D2Norm& norm = D2Norm(), float* const* xpeer = nullptr,
                  int npeer = 0, int prank = 0);

}  // namespace b2q
