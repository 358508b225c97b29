// engine.cuh -- the streaming (decode) product engine: shared declarations.
//
// One persistent CTA per SM. Warp 8 is the producer: its lane 0 walks the
// CTA's static list of units and, per pass, issues 1-D bulk copies (TMA) of 16
// weight rows (two 8-row blocks P and Q) plus their scale/bias rows into a
// 4-stage shared-memory ring, completion counted on an mbarrier. Warps 0-7 are
// consumers: each takes an equal share of the pass's quantization groups,
// decodes nibbles to bf16 pairs and runs m16n8k16 MMAs whose A operand is the
// 16 weight rows and whose B operand is up to 8 activation columns (tokens or
// routed slots); the per-group affine epilogue s*D + (b - 128 s)*sum(x) is
// applied in fp32. A unit's warp partials are reduced in a fixed order in
// shared memory and finished by a mode-specific epilogue (bf16 store, SwiGLU,
// or the weighted expert combine).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {
namespace eng {

constexpr int NC_WARPS = 8;
constexpr int NCT = NC_WARPS * 32;
constexpr int NTHREADS = NCT + 32;
constexpr int NSTAGE = 4;
constexpr int MAX_COLS = 8;
constexpr int STAGE_MAX = 40 * 1024;

enum Mode : int { MODE_QMV = 0, MODE_GU = 1, MODE_DOWN = 2, MODE_FUSED = 3 };

// Geometry of one product family (reduction length K).
struct Geo {
  int K;    // reduction length
  int G;    // groups per row (K / gs)
  int KC;   // reduction chunk per pass
  int nkc;  // passes per row block
  int RS;   // shared-memory weight-row stride (bytes)
  int MS;   // shared-memory meta-row stride (bytes)
  int XS;   // shared-memory activation-column stride (bytes)
};

struct Params {
  int mode;
  int gs;
  int wpt;  // packed words per lane per group = gs / 32
  // QMV / gather
  const uint16_t* x;
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  const uint32_t* lhs;
  const uint32_t* rhs;
  uint16_t* y;
  int batch, M, N, n_x, n_w;
  // MoE
  const uint16_t* wr;
  const uint32_t *wg, *wu, *wd;
  const uint16_t *sg, *bg, *su, *bu, *sd, *bd;
  const uint32_t* idx_in;
  const uint32_t* xrow_in;
  const float* w_in;
  const uint16_t* act_in;
  uint16_t* act_out;
  uint16_t* out;
  uint32_t* idx_out;
  float* w_out;
  float* logits_out;
  int S, H, E, F, k, n_slots;
  // workspace (FUSED)
  int* err;
  unsigned* counters;  // [0] router rows done, [1] gate|up units done, [2] CTAs exited
  float* ws_logits;
  uint16_t* ws_act;
  // geometry
  Geo g1;  // QMV: K; GU / FUSED gate|up: K = H
  Geo g2;  // DOWN / FUSED down: K = F
  int stage_bytes;
  int off_x, off_xs, off_act, off_acts, off_red, off_misc, smem_bytes;
  int xcols;  // activation columns staged at off_x
  long long timeout_ns;
};

// Host side: fill geometry / shared-memory plan; returns B2Q_OK or an error.
int plan(Params& p);
int launch(const Params& p, void* stream, bool cooperative);

int launch_router_logits(const uint16_t* x, const uint16_t* wr, float* logits, int T, int E, int H,
                         cudaStream_t s);
int launch_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k, cudaStream_t s);

}  // namespace eng
}  // namespace b2q
