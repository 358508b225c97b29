// engine.cuh -- the streaming (decode) product engine: shared declarations.
//
// One persistent CTA per SM. Warp NC_WARPS is the producer: its lane 0 walks
// the CTA's static list of units and, per pass, issues six TMA tensor copies
// (an 8-row weight block P, an 8-row weight block Q, and their scale / bias
// blocks) into a 4-stage shared-memory ring; completion is counted on an
// mbarrier per stage. Warps 0..NC_WARPS-1 are consumers: each takes an equal
// share of the pass's quantization groups (in pairs), decodes nibbles to bf16
// pairs and runs m16n8k16 MMAs whose A operand is the 16 weight rows (P rows
// 0-7, Q rows 8-15) and whose B operand is up to 8 activation columns (tokens
// or routed slots); the per-group affine epilogue s*D + (b - 128 s)*sum(x) is
// applied in fp32. A unit's warp partials are reduced in a fixed order in
// shared memory and finished by a mode-specific epilogue (bf16 store, SwiGLU,
// or the weighted expert combine).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {
namespace eng {

constexpr int NC_WARPS = 8;
constexpr int NCT = NC_WARPS * 32;
constexpr int NTHREADS = NCT + 64;  // + producer warp + finisher warp
constexpr int NSTAGE_MAX = 8;  // stage ring size is planned per call from free shared memory
constexpr int NRED = 4;  // ring of per-unit partial-sum slots handed to the finisher
constexpr int MAX_COLS = 8;
constexpr int STAGE_MAX = 40 * 1024;

enum Mode : int { MODE_QMV = 0, MODE_GU = 1, MODE_DOWN = 2, MODE_FUSED = 3 };
// tensor-map slots
enum Map : int { M_W = 0, M_S = 1, M_B = 2, M_WG = 0, M_SG = 1, M_BG = 2, M_WU = 3, M_SU = 4, M_BU = 5, M_WD = 6,
                 M_SD = 7, M_BD = 8, N_MAPS = 9 };

// Geometry of one product family (reduction length K).
struct Geo {
  int K;      // reduction length
  int G;      // groups per row (K / gs)
  int KC;     // reduction chunk per pass (elements, a multiple of 256)
  int nkc;    // passes per row block
  int GC;     // groups per full pass (KC / gs)
  int blkw;   // bytes of an 8-row weight block of a full pass (8 * KC / 2, 1024-aligned)
  int blkm;   // bytes reserved per 8-row scale (or bias) block
  int mswz;   // 1: meta blocks use the 128-byte swizzled layout, 0: plain [row][GC]
  int mrow;   // plain meta: bytes per row in shared memory (GC * 2)
  int XS;     // shared-memory activation-column stride (bytes)
};

struct alignas(64) Params {
  CUtensorMap map[N_MAPS];
  int mode;
  int gs;
  int wpt;  // packed words per lane per group = gs / 32
  // QMV / gather
  const uint16_t* x;
  uint16_t* y;
  const uint32_t* lhs;
  const uint32_t* rhs;
  int batch, M, N, n_x, n_w;
  // MoE
  const uint16_t* wr;
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
  int nstage;  // stages in the ring (2..NSTAGE_MAX)
  int off_x, off_xs, off_act, off_acts, off_red, off_misc, smem_bytes;
  int xcols;  // activation columns staged at off_x
  long long timeout_ns;
};

// Host side: geometry / shared-memory plan and tensor maps; launch.
int plan(Params& p);
int set_maps_qmv(Params& p, const uint32_t* w, const uint16_t* s, const uint16_t* b);
int set_maps_gu(Params& p, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg, const uint32_t* wu,
                const uint16_t* su, const uint16_t* bu);
int set_maps_down(Params& p, const uint32_t* wd, const uint16_t* sd, const uint16_t* bd);
int launch(const Params& p, void* stream, bool cooperative);

int launch_router_logits(const uint16_t* x, const uint16_t* wr, float* logits, int T, int E, int H,
                         cudaStream_t s);
int launch_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k, cudaStream_t s);
// Long windows with fp32 scratch of at least 8 * T * E floats: the split-K
// router GEMM (falls back to launch_router_logits otherwise).
int launch_router_logits_sk(const uint16_t* x, const uint16_t* wr, float* logits, float* scratch,
                            size_t scratch_bytes, int T, int E, int H, cudaStream_t s);

}  // namespace eng
}  // namespace b2q
