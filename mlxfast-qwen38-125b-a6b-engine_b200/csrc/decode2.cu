// decode2.cu -- single-column streaming products: qmv for one row of x
// (M = 1) and the fused one-token MoE decode layer.
//
// Reference operators (paths relative to the reference project):
//   qmv_fast_impl / qdot       Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/metal/kernels/quantized.h:28-105,191-290,757-822
//   gateUpAct / downCombine    Runner/FastModel/TrackFastMoE.swift:1192-1590
//   route (top-k + softmax)    Runner/FastModel/TrackFastMoE.swift:767-911
//   combine association        Runner/FastModel/TrackFastKernels2.swift:36-47
//
// Organisation: one CTA per SM: 16 consumer warps, a producer warp and an
// epilogue warp.
//  * The work of a call is a sequence of units, each one TMA fill of a stage:
//      gate|up unit  16 outputs of one routed expert: its 16 gate rows and 16
//                    up rows over the whole hidden size (two copies of 16 rows
//                    x the whole row) plus their 4 scale / bias blocks;
//      down unit     one 16-row block of the output for 4 routed slots: each
//                    slot's 16 down rows over the whole expert width, their
//                    scales / biases, and the slot's activations;
//      qmv unit      32 rows of the matrix over the whole reduction.
//    Units are assigned statically: qmv unit u to CTA u mod grid; gate|up
//    unit u to CTA grid - 1 - u mod grid; down block j to CTA j mod grid,
//    which streams the block's rows of every routed slot and folds the slots
//    itself. A down unit waits only for its slots' activations to be final
//    (a per-slot count of finished gate|up units): no grid-wide barrier
//    between the phases. The static order keeps global round trips out of
//    the producer's loop: at full bandwidth a round trip waits behind the
//    CTA's copies in flight for microseconds.
//  * Large copies (32 KB boxes of whole rows) keep the per-copy issue cost of
//    the TMA small against the bytes moved.
//  * The producer fills a ring of stages (full / empty mbarrier per stage) with
//    whole-row TMA boxes in the 128-byte swizzle (16-byte unit u of row r at
//    position u ^ (r % 8)); the consumer warps split the unit's reduction (or
//    its slots and reduction) between them and post their row partials to
//    shared memory; the epilogue warp sums them, releases the stage and does
//    the unit's global work: bf16 store (qmv), SwiGLU activations (gate|up)
//    or the block's slot table, whose last unit folds the k slots in the
//    reference's combine order (down).
//  * Dot products: integer MMAs (mma.sync m16n8k32 u8 x s8 -> s32) on the
//    raw weight nibbles and an int8 split of the activation (see dot_i8):
//    per group of x a 16-bit fixed point, per block of 16 SwiGLU outputs
//    (made by the epilogue) the same with its own scale (see dot_i8_act).
//  * Launches use programmatic dependent launch: barrier set-up, tensor-map
//    prefetch and L2 prefetches (router rows; the first qmv units) run while
//    the previous kernel in the stream finishes; nothing is read into the CTA
//    before griddepcontrol.wait.
// All waits are bounded; a wait that runs out records B2Q_ETIMEOUT and raises
// an abort flag that ends every loop; the producer lets its copies land
// before the CTA exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "decode2.cuh"
#include "host.hpp"
#include "tc.cuh"
#include "tmap.hpp"

namespace b2q {
namespace d2 {

constexpr int NCW = 16;              // consumer warps
constexpr int NEPI = 2;              // epilogue warps (unit n: warp n % NEPI)
constexpr int NWARP = NCW + 1 + NEPI; // + the producer warp and the epilogue warps
constexpr int NTH = NWARP * 32;
constexpr int MAXK = 8;              // routed slots
constexpr int MAXST = 6;             // stages at most
constexpr int ROWS_QMV = 32;         // rows of a qmv unit (two 16-row MMA blocks)
constexpr int ROWS_GU = 16;          // outputs of a gate|up unit (16 gate + 16 up rows)
constexpr int ROWS_D = 16;           // rows of a down block (output rows h)
constexpr int SLOTS_D = 4;           // routed slots of a down unit
constexpr int MAXBLK = 16;           // down blocks of one CTA at most
constexpr int MISC_BYTES = 1024;

enum : int { U_END = -1, U_GU = 0, U_DOWN = 1, U_QMV = 2 };
enum : int { MW = 0, MS = 1, MB = 2, MWG = 0, MSG = 1, MBG = 2, MWU = 3, MSU = 4, MBU = 5, MWD = 6, MSD = 7, MBD = 8 };

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar,
                                     uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// system-scope release store / acquire load (the exchange flags between GPUs)
__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float lbf(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hbf(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Byte offset of metadata (row, group) in a block whose rows are `mb` bytes,
// stored plain or in the 128-byte swizzle (then mb == 128).
__device__ __forceinline__ int moff(int row, int g, int mb, bool sw) {
  const int b = 2 * g;
  return sw ? row * 128 + ((((b >> 4) ^ row) & 7) << 4) + (b & 15) : row * mb + b;
}

// ---------------------------------------------------------------------------
// Consumer warp arithmetic. A warp multiplies 16-row blocks (P: 8 rows, Q: 8
// rows; lane (r = lane / 4, c = lane % 4) owns P row r and Q row r) by the
// activation over a range of chunk columns; a chunk column is 32 reduction
// values, 16 bytes of every row. Word w of 16-byte unit u of a row sits at
// piece * (rows * 128) + row * 128 + ((u ^ (row % 8)) << 4) + 4 w  (the TMA
// 128-byte swizzle over boxes of `rows` rows).
// ---------------------------------------------------------------------------
struct Meta {
  const uint8_t *sP, *bP, *sQ, *bQ;
  int rowP, rowQ, mb;
  bool sw;
};

// ---------------------------------------------------------------------------
// Units whose activation is the call's x (gate|up, qmv): integer MMAs.
// x is held per group g as 16-bit fixed point X = round(x * 2^(14 - E_g))
// (E_g: exponent of the group's max |x|; exact for every value within 2^7 of
// the max, |X| <= 32640), split into int8 pieces hi = (X + 128) >> 8 and
// lo = X - 256 hi. The pieces reach 256 hi + lo <= 32639: the one positive
// value above it, 32640 (a max of mantissa 0x7f), is held as 32639, an error
// of 2^-15 of the group's max. Weights go in as raw u8 nibbles (two masks per word), so
// mma.sync m16n8k32 u8 x s8 -> s32 sums q * hi and q * lo exactly.
// A "slot" is min(gs, 64) reduction values; in one MMA lane c of a quad
// carries a word of slot 4t + c (rotated so the four lanes of a 16-byte unit
// read different banks), and the B operand is zero except in columns 2c (hi
// pieces) and 2c + 1 (lo pieces) at lane c's k-slots, so D[row][2c] and
// D[row][2c + 1] -- registers d0, d1 of lane c -- are slot 4t + c's sums.
// Per group: q.x = 2^(E_g - 14) * (256 * hi_sum + lo_sum), then
// s * q.x + b * sum(x).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void imma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int XB = 16;  // activation piece registers per lane (8 MMA steps x 2)

// word of slot `slot` a lane c reads at step j (rotated inside each 4-word chunk)
template <int WS>
__device__ __forceinline__ int slot_word(int j, int c) {
  return (j & ~3) + ((j + c) & 3);
}

// Staged activation pieces in shared memory: 16 bytes per word of 8 values,
// [hi of values 0,2,4,6][hi of 1,3,5,7][lo of 0,2,4,6][lo of 1,3,5,7].
// Builds this lane's B registers for the warp's slice of chunk columns
// [cc0, cc0 + ncc): nonzero only in the two lanes of each quad column pair.
template <int SLOT>
__device__ __forceinline__ void load_pieces(const uint8_t* pieces, int cc0, int ncc, uint32_t (&xb)[XB]) {
  constexpr int WS = SLOT / 8, CPS = SLOT / 32;
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const int nslot = ncc / CPS;
#pragma unroll
  for (int i = 0; i < XB; ++i) xb[i] = 0u;
  if ((r >> 1) != c) return;
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < WS; ++j) {
      const int st = t * WS + j;
      const int slot = 4 * t + c;
      if (st >= XB / 2 || slot >= nslot) continue;
      const int w = slot_word<WS>(j, c);
      const int wi = (cc0 + slot * CPS) * 4 + w;  // word of x
      const uint2 v = *reinterpret_cast<const uint2*>(pieces + wi * 16 + (r & 1) * 8);
      xb[2 * st] = v.x;
      xb[2 * st + 1] = v.y;
    }
}

// Byte offset, inside a stage, of the word lane (r, c) reads at each step, for
// P row r of row block 0 (boxes of `rows` rows: piece stride rows * 128).
template <int SLOT>
__device__ __forceinline__ void word_offsets(int cc0, int rows, uint32_t (&woff)[XB / 2]) {
  constexpr int WS = SLOT / 8, CPS = SLOT / 32;
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < WS; ++j) {
      const int st = t * WS + j;
      if (st >= XB / 2) continue;
      const int slot = 4 * t + c;
      const int w = slot_word<WS>(j, c);
      const int cc = cc0 + slot * CPS + (w >> 2);
      woff[st] = (uint32_t)((cc >> 3) * rows * 128 + r * 128 + (((cc & 7) ^ r) << 4) + 4 * (w & 3));
    }
}

// Row block b's P rows start at b * bstride, its Q rows qoff further.
// LUT: the metadata blocks hold u16 pair indices (sP / sQ) into `lut`, a
// shared-memory copy of the pair table (scale bits | bias bits << 16): the same
// bf16 bits reach the same arithmetic as with the scale / bias blocks.
template <int SLOT, int NRB, bool LUT = false>
__device__ __forceinline__ void dot_i8(const uint8_t* st_base, const uint32_t (&woff)[XB / 2], int bstride, int qoff,
                                       int slot0, int nslot, int gs, const uint32_t (&xb)[XB], const float2* gsc,
                                       const Meta (&m)[NRB], float (&accP)[NRB], float (&accQ)[NRB],
                                       const uint32_t* lut = nullptr) {
  constexpr int WS = SLOT / 8;
  const int c = threadIdx.x & 3;
  const int spg = gs / SLOT;  // slots per group (1 or 2)
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    if (4 * t < nslot) {
      const int slot = 4 * t + c;
      const bool live = slot < nslot;
      int D[NRB][2][4];
#pragma unroll
      for (int b = 0; b < NRB; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h) D[b][h][0] = D[b][h][1] = D[b][h][2] = D[b][h][3] = 0;
#pragma unroll
      for (int j = 0; j < WS; ++j) {
        const int st = t * WS + j;
        if (st < XB / 2) {
          const uint8_t* wp = st_base + woff[st];
#pragma unroll
          for (int b = 0; b < NRB; ++b) {
            const uint32_t W0 = live ? *reinterpret_cast<const uint32_t*>(wp + b * bstride) : 0u;
            const uint32_t W8 = live ? *reinterpret_cast<const uint32_t*>(wp + b * bstride + qoff) : 0u;
            imma_u8s8(D[b][j & 1], W0 & 0x0F0F0F0Fu, W8 & 0x0F0F0F0Fu, (W0 >> 4) & 0x0F0F0F0Fu,
                      (W8 >> 4) & 0x0F0F0F0Fu, xb[2 * st], xb[2 * st + 1]);
          }
        }
      }
      // lane c: slot 4t + c of P row r (d0 hi, d1 lo) and Q row r (d2, d3)
      const int g = (slot0 + slot) / spg;
#pragma unroll
      for (int b = 0; b < NRB; ++b) {
        const int vP = 256 * (D[b][0][0] + D[b][1][0]) + (D[b][0][1] + D[b][1][1]);
        const int vQ = 256 * (D[b][0][2] + D[b][1][2]) + (D[b][0][3] + D[b][1][3]);
        // each lane scales its slot; with two slots per group (spg 2) the bias
        // term b * sum(x) goes with the group's first slot, and the quad sum at
        // the end adds the slots
        if (live) {
          const float2 sc = gsc[g];
          const float xg = (spg == 1 || (c & 1) == 0) ? sc.y : 0.0f;
          float sP, bP, sQ, bQ;
          if (LUT) {
            const uint32_t pP = lut[*reinterpret_cast<const uint16_t*>(m[b].sP + moff(m[b].rowP, g, m[b].mb, m[b].sw))];
            const uint32_t pQ = lut[*reinterpret_cast<const uint16_t*>(m[b].sQ + moff(m[b].rowQ, g, m[b].mb, m[b].sw))];
            sP = lbf(pP);
            bP = hbf(pP);
            sQ = lbf(pQ);
            bQ = hbf(pQ);
          } else {
            sP = bf2f(*reinterpret_cast<const uint16_t*>(m[b].sP + moff(m[b].rowP, g, m[b].mb, m[b].sw)));
            bP = bf2f(*reinterpret_cast<const uint16_t*>(m[b].bP + moff(m[b].rowP, g, m[b].mb, m[b].sw)));
            sQ = bf2f(*reinterpret_cast<const uint16_t*>(m[b].sQ + moff(m[b].rowQ, g, m[b].mb, m[b].sw)));
            bQ = bf2f(*reinterpret_cast<const uint16_t*>(m[b].bQ + moff(m[b].rowQ, g, m[b].mb, m[b].sw)));
          }
          accP[b] = fmaf(sP, (float)vP * sc.x, fmaf(bP, xg, accP[b]));
          accQ[b] = fmaf(sQ, (float)vQ * sc.x, fmaf(bQ, xg, accQ[b]));
        }
      }
    }
  }
}

// Down units: the activations are int8 pieces too, made by the epilogue from
// the bf16 SwiGLU outputs of each gate|up unit with one scale per block of 16
// values (the unit's outputs), 16 bytes per word like x's pieces; asc holds
// (2^(E_b - 14), sum of the block's values) per block. One 32-value chunk per
// lane slot; at step j lane c takes word j ^ c of its chunk (the four lanes of
// a quad read four different words: no bank conflict), so steps 0, 1 cover
// words c, c ^ 1 (block c / 2) and steps 2, 3 the chunk's other block: two
// accumulators, one scale each.
template <int U>
__device__ __forceinline__ void dot_i8_act(const uint8_t* wbox, const uint8_t* pcs, const float2* asc, int cc0,
                                           int nslot, int gs, const Meta& m, float& accP, float& accQ) {
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const bool diag = (r >> 1) == c;  // B lanes of lane c's column pair
  const int spg = gs / 32;          // chunks per group
  // U rounds of 4 chunks per pass, unrolled so that the loads and MMAs of a
  // round overlap the epilogue of the one before (nslot is a multiple of 4 U
  // for U > 1)
  for (int t0 = 0; 4 * t0 < nslot; t0 += U) {
    int A[U][4], B[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int cc = cc0 + 4 * (t0 + u) + c;
      const bool live = U > 1 || 4 * (t0 + u) + c < nslot;
      const uint8_t* wr = wbox + (cc >> 3) * (ROWS_D * 128) + r * 128 + (((cc & 7) ^ r) << 4);
      const uint8_t* xp = pcs + (size_t)cc * 64 + (r & 1) * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) A[u][i] = B[u][i] = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int w = j ^ c;
        const uint32_t W0 = live ? *reinterpret_cast<const uint32_t*>(wr + 4 * w) : 0u;
        const uint32_t W8 = live ? *reinterpret_cast<const uint32_t*>(wr + 4 * w + 8 * 128) : 0u;
        uint2 xv = make_uint2(0u, 0u);
        if (live && diag) xv = *reinterpret_cast<const uint2*>(xp + w * 16);
        if (j < 2)
          imma_u8s8(A[u], W0 & 0x0F0F0F0Fu, W8 & 0x0F0F0F0Fu, (W0 >> 4) & 0x0F0F0F0Fu, (W8 >> 4) & 0x0F0F0F0Fu,
                    xv.x, xv.y);
        else
          imma_u8s8(B[u], W0 & 0x0F0F0F0Fu, W8 & 0x0F0F0F0Fu, (W0 >> 4) & 0x0F0F0F0Fu, (W8 >> 4) & 0x0F0F0F0Fu,
                    xv.x, xv.y);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      // lane c: chunk cc of P row r (d0 hi, d1 lo) and Q row r (d2, d3)
      const int cc = cc0 + 4 * (t0 + u) + c;
      const bool live = U > 1 || 4 * (t0 + u) + c < nslot;
      float fP = 0.0f, fQ = 0.0f, xs = 0.0f;
      if (live) {
        const float2 sa = asc[2 * cc + (c >> 1)], sb = asc[2 * cc + ((c >> 1) ^ 1)];
        fP = (float)(256 * A[u][0] + A[u][1]) * sa.x + (float)(256 * B[u][0] + B[u][1]) * sb.x;
        fQ = (float)(256 * A[u][2] + A[u][3]) * sa.x + (float)(256 * B[u][2] + B[u][3]) * sb.x;
        xs = sa.y + sb.y;
      }
      // each lane scales its chunk by its group's scale / bias; the quad sum at
      // the end adds the chunks of a group (spg > 1) with the rest
      if (live) {
        const int g = cc / spg;
        const float sP = bf2f(*reinterpret_cast<const uint16_t*>(m.sP + moff(m.rowP, g, m.mb, m.sw)));
        const float bP = bf2f(*reinterpret_cast<const uint16_t*>(m.bP + moff(m.rowP, g, m.mb, m.sw)));
        const float sQ = bf2f(*reinterpret_cast<const uint16_t*>(m.sQ + moff(m.rowQ, g, m.mb, m.sw)));
        const float bQ = bf2f(*reinterpret_cast<const uint16_t*>(m.bQ + moff(m.rowQ, g, m.mb, m.sw)));
        accP = fmaf(sP, fP, fmaf(bP, xs, accP));
        accQ = fmaf(sQ, fQ, fmaf(bQ, xs, accQ));
      }
    }
  }
}

// softmax over the k selected logits held by lanes 0..k-1 (slot order): max,
// exp, per-lane partial sums of 4 then a butterfly, as the reference's softmax
// over its k values (Runner/FastModel/TrackFastMoE.swift:846-880)
__device__ void softmax_k(float selv, int k, float* sw) {
  const int lane = threadIdx.x & 31;
  float mx = (lane < k) ? selv : -INFINITY;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float ex = (lane < k) ? expf(selv - mx) : 0.0f;
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float t = __shfl_sync(0xffffffffu, ex, (4 * lane + i) & 31);
    part += (lane < 8) ? t : 0.0f;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  const float inv = 1.0f / part;
  if (lane < k) sw[lane] = ex * inv;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int CPG, int MODE>
__global__ void __launch_bounds__(NTH, 1) d2_kernel(const __grid_constant__ D2Params p) {
  constexpr int SLOT = CPG == 1 ? 32 : 64;  // reduction values per column slot of the integer MMAs
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // aligned by pointer arithmetic on the shared array (an integer round trip
  // would hide the address space and turn every shared access generic)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr bool FUSED = MODE == D2_FUSED || MODE == D2_FUSED_EP;
  constexpr bool EP = MODE == D2_FUSED_EP;
  constexpr bool LUT = MODE == D2_QMV_LUT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.nstage;

  uint8_t* misc = smem + p.off_misc;
  uint64_t* full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty = full + MAXST;
  uint64_t* rfull = empty + MAXST;                               // [MAXST] consumer partials of a unit posted
  int4* info = reinterpret_cast<int4*>(rfull + MAXST);          // [MAXST] unit of each stage fill
  volatile int* abort_flag = reinterpret_cast<volatile int*>(info + MAXST);
  int* nloc_sm = const_cast<int*>(abort_flag) + 1;
  uint32_t* sidx = reinterpret_cast<uint32_t*>(nloc_sm + 3);     // [MAXK] selected experts, slot order
  float* sw = reinterpret_cast<float*>(sidx + MAXK);             // [MAXK] their weights
  int* lslot = reinterpret_cast<int*>(sw + MAXK);                // [MAXK] routed slots held here (EP)
  float* rsum = reinterpret_cast<float*>(lslot + MAXK);          // [NWARP]
  int* lastf_sm = reinterpret_cast<int*>(rsum + NWARP);          // [MAXST] producer bookkeeping
  unsigned* ycnt = reinterpret_cast<unsigned*>(lastf_sm + MAXST); // [MAXBLK] down units finished per block
  uint64_t* lutbar = reinterpret_cast<uint64_t*>(misc + 640);   // the pair table's copy landed (LUT)
  uint32_t* lut_sm = reinterpret_cast<uint32_t*>(smem + p.off_lut);
  float* ysm = reinterpret_cast<float*>(smem + p.off_ysm);       // [MAXBLK][MAXK][ROWS_D] slot products
  float* red = reinterpret_cast<float*>(smem + p.off_red);       // [nstage][NCW][32]
  float2* gsc = reinterpret_cast<float2*>(smem + p.off_xs);     // per group: 2^(E_g - 14), sum(x)
  unsigned* done = p.ctr + 4;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&rfull[i], NCW);
    }
    for (int i = 0; i < MAXBLK; ++i) ycnt[i] = 0u;
    if (LUT) mbar_init(lutbar, 1);
    *abort_flag = 0;
    nloc_sm[1] = 0;  // routed slots selected so far (the producer's early start)
    fence_barrier_init();
  }
  if (warp == NCW && lane == 0) {
    for (int i = 0; i < (FUSED ? 9 : 3); ++i)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.map[i])) : "memory");
    if (FUSED)
      for (int e = blockIdx.x; e < p.E; e += gridDim.x) prefetch_l2(p.wr + (size_t)e * p.H, (uint32_t)p.H * 2u);
    if (!FUSED) {
      // the first units' weight rows go to L2 only: a prefetch reads nothing
      // into the CTA, and the stage loads after the wait see whatever the
      // previous kernel wrote (L2 is the point of coherence)
      for (int i = 0; i < NS; ++i) {
        const unsigned u = blockIdx.x + (unsigned)i * gridDim.x;
        if (u >= (unsigned)((p.N + ROWS_QMV - 1) / ROWS_QMV)) break;
        asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                         reinterpret_cast<uint64_t>(&p.map[MW])),
                     "r"(0), "r"((int)u * ROWS_QMV), "r"(0)
                     : "memory");
      }
    }
  }
  // everything below may read what the previous kernel in the stream wrote
  griddep_wait();
  griddep_launch();
  const uint64_t deadline = globaltimer() + (uint64_t)p.timeout_ns;
  // the call's tag: router logits carry it, so a value read is complete and
  // of this call with no separate count (the last CTA out advances it)
  const unsigned tag = FUSED ? __ldcg(p.ctr + D2_CTR_TAG) + 1u : 0u;
  unsigned long long* tlg = reinterpret_cast<unsigned long long*>(p.ctr + D2_CTR_LOGITS);
  // peer exchange: this call's epoch (the last CTA of the previous call
  // advanced the rank's counter) and its slot of the double buffer
  const bool XP = EP && p.npeer > 0;
  const unsigned xep = XP ? __ldcg(reinterpret_cast<const unsigned*>(p.xpeer[p.prank])) + 1u : 0u;
  const int xslot = (int)(xep & 1u);
  __syncthreads();
  // qmv: the weights do not depend on x, so the producer issues the copies of
  // its first units (stages 0 .. NS - 2; the last stage holds the staged x
  // pieces) before the pass over x, which they overlap
  int npre = 0;
  if (!FUSED && warp == NCW && lane == 0) {
    const int uq = (p.N + ROWS_QMV - 1) / ROWS_QMV;
    npre = min(NS - 1, max((uq - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x, 0));
    const uint64_t pol = policy_evict_first();
    for (int i = 0; i < npre; ++i) {
      const int u = (int)blockIdx.x + i * (int)gridDim.x, row = u * ROWS_QMV;
      uint8_t* st = smem + (size_t)i * p.stage_bytes;
      info[i] = make_int4(U_QMV, 0, u, 0);
      mbar_arrive_expect_tx(&full[i], (uint32_t)(ROWS_QMV * p.K1 / 2 + (LUT ? 1 : 2) * ROWS_QMV * p.mb1));
      tma3(st, &p.map[MW], 0, row, 0, &full[i], pol);
      tc::tma_load_2d(st + p.st_meta1, &p.map[MS], 0, row, &full[i], pol);
      if (!LUT) tc::tma_load_2d(st + p.st_meta1 + p.st_mstep1, &p.map[MB], 0, row, &full[i], pol);
    }
  }
  if (LUT && warp == NCW && lane == 0) {
    // the pair table, one bulk copy; the consumers wait for it before their
    // first unit's scaling (after the pass over x)
    mbar_arrive_expect_tx(lutbar, (uint32_t)p.lut_words * 4u);
    bulk_g2s(lut_sm, p.lut, (uint32_t)p.lut_words * 4u, lutbar, policy_evict_last());
  }

  const int K1 = p.K1;
  constexpr int CPC = CPG * 4;  // 8-value chunks per group
  // ---- one pass over x: this CTA's router rows (fused), and per group of x
  // the fixed-point scale 2^(E_g - 14), sum(x) and the int8 pieces of every
  // word (staged at the end of the stage ring, which the producer does not
  // fill before the block barrier after routing) ----
  uint8_t* pieces = smem + (size_t)NS * p.stage_bytes - (size_t)K1 * 2;
  // fused residual add + RMSNorm (one chunk of 8 values per thread, checked on
  // the host): h' = bf16(h + delta) (CTA 0 stores it), the block's sum of h'^2
  // in warp order, then x = bf16(h' * r * w), as the separate norm kernel
  uint4 xn = make_uint4(0u, 0u, 0u, 0u);
  if (p.nw) {
    const bool live = tid < K1 / 8;
    float ss = 0.0f;
    uint32_t u[4] = {0u, 0u, 0u, 0u};
    if (live) {
      const uint4 hv = __ldg(reinterpret_cast<const uint4*>(p.x) + tid);
      u[0] = hv.x;
      u[1] = hv.y;
      u[2] = hv.z;
      u[3] = hv.w;
      if (p.ndelta) {
        const uint4 dq = __ldg(reinterpret_cast<const uint4*>(p.ndelta) + tid);
        const uint32_t du[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = lbf(u[j]) + lbf(du[j]), c = hbf(u[j]) + hbf(du[j]);
          u[j] = (uint32_t)f2bf(a) | ((uint32_t)f2bf(c) << 16);
        }
        if (blockIdx.x == 0) reinterpret_cast<uint4*>(p.nh_out)[tid] = make_uint4(u[0], u[1], u[2], u[3]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = lbf(u[j]), c = hbf(u[j]);
        ss = fmaf(a, a, ss);
        ss = fmaf(c, c, ss);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) rsum[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < NWARP; ++w) tot += rsum[w];
    __syncthreads();  // rsum is the router's scratch below
    const float rr = rsqrtf(tot / (float)K1 + p.neps);
    if (live) {
      const uint4 g = __ldg(reinterpret_cast<const uint4*>(p.nw) + tid);
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = (uint32_t)f2bf(lbf(u[j]) * rr * lbf(gw[j])) | ((uint32_t)f2bf(hbf(u[j]) * rr * hbf(gw[j])) << 16);
      xn = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  {
    const int nch = K1 / 8;
    for (int q0 = 0; q0 < nch; q0 += NTH) {
      const int q = q0 + tid;
      const bool live = q < nch;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (live) v = p.nw ? xn : __ldg(reinterpret_cast<const uint4*>(p.x) + q);
      if (FUSED && q0 == 0 && nch <= NTH) {
        // router rows e = blockIdx.x + i * grid (x word q of each)
        for (int e = blockIdx.x; e < p.E; e += gridDim.x) {
          float part = 0.0f;
          if (live) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(p.wr + (size_t)e * p.H) + q);
            part = lbf(v.x) * lbf(wv.x) + hbf(v.x) * hbf(wv.x);
            part += lbf(v.y) * lbf(wv.y) + hbf(v.y) * hbf(wv.y);
            part += lbf(v.z) * lbf(wv.z) + hbf(v.z) * hbf(wv.z);
            part += lbf(v.w) * lbf(wv.w) + hbf(v.w) * hbf(wv.w);
          }
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
          if (lane == 0) rsum[warp] = part;
          __syncthreads();
          if (tid == 0) {
            float lg = 0.0f;
            for (int w = 0; w < NWARP; ++w) lg += rsum[w];
            st_relaxed_u64(tlg + e, ((unsigned long long)tag << 32) | __float_as_uint(lg));
          }
          __syncthreads();
        }
      }
      float s = ((lbf(v.x) + hbf(v.x)) + (lbf(v.y) + hbf(v.y))) + ((lbf(v.z) + hbf(v.z)) + (lbf(v.w) + hbf(v.w)));
      // bf16 bits of the chunk's max |x| (per-halfword maxima, then the two halves)
      unsigned mx = __vmaxu2(__vmaxu2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu), __vmaxu2(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu));
      mx = max(mx & 0xffffu, mx >> 16);
#pragma unroll
      for (int off = 1; off < CPC; off <<= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, off);
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      }
      // exponent of the group's max; zero, infinite or NaN maxima take 0 (values
      // then saturate: no defined result for non-finite inputs)
      int e = (int)((mx >> 7) & 0xffu) - 127;
      if (mx == 0u || mx >= 0x7f80u) e = 0;
      e = max(-110, min(120, e));
      if (live && (q % CPC) == 0) gsc[q / CPC] = make_float2(__int_as_float((127 + e - 14) << 23), s);
      if (live) {
        const float f = __int_as_float((127 + 14 - e) << 23);  // 2^(14 - E_g)
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
        uint32_t he = 0u, ho = 0u, le = 0u, lo = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t h = (i & 1) ? (vw[i >> 1] & 0xffff0000u) : (vw[i >> 1] << 16);
          const int X = min(__float2int_rn(__uint_as_float(h) * f), 32639);
          const int hi = (X + 128) >> 8;
          const uint32_t hb = (uint32_t)hi & 0xffu, lb = (uint32_t)(X - (hi << 8)) & 0xffu;
          const int sh = 8 * (i >> 1);
          if (i & 1) {
            ho |= hb << sh;
            lo |= lb << sh;
          } else {
            he |= hb << sh;
            le |= lb << sh;
          }
        }
        *reinterpret_cast<uint4*>(pieces + (size_t)q * 16) = make_uint4(he, ho, le, lo);
      }
    }
  }
  __syncthreads();
  // ---- the consumer lane's activation pieces (B operands) and word offsets ----
  uint32_t xb[XB], woff[XB / 2];
  const int ncc1 = K1 / 32 / NCW, cc01 = (warp < NCW ? warp : 0) * ncc1;
  load_pieces<SLOT>(pieces, cc01, warp < NCW ? ncc1 : 0, xb);
  word_offsets<SLOT>(cc01, FUSED ? ROWS_GU : ROWS_QMV, woff);
  const int nslot1 = ncc1 / (SLOT / 32), slot01 = cc01 / (SLOT / 32);
  // A fused call without expert parallelism lets the producer start on each
  // unit as soon as top-k has chosen its slot's expert (a slot count in shared
  // memory) instead of after the whole routing; it fills the stage that holds
  // the staged pieces only after every consumer has its share in registers.
  constexpr bool early = FUSED && !EP;
  volatile int* topk_ready = nloc_sm + 1;
  if (early) {
    if (warp < NCW)
      named_bar_arrive(2, (NCW + 1) * 32);
    else if (warp == NCW)
      named_bar_sync(2, (NCW + 1) * 32);
  }
  // ---- routing (fused): every CTA selects the same top-k in warp 0 ----
  if (FUSED && warp == 0) {
    // lane l holds experts l, l + 32, ...: poll until every logit carries this
    // call's tag (one read of the values, no separate count)
    constexpr int EPL = 8;  // experts per lane at most (E <= 256)
    uint32_t key[EPL];
    bool ok = true;
    for (int poll = 0;; ++poll) {
      bool all = true;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        key[i] = 0u;
        if (e < p.E) {
          const unsigned long long v = ld_relaxed_u64(tlg + e);
          all = all && (unsigned)(v >> 32) == tag;
          key[i] = (uint32_t)v;
        }
      }
      if (__all_sync(0xffffffffu, all)) break;
      if ((poll & 7) == 7 && __shfl_sync(0xffffffffu, (globaltimer() > deadline || *abort_flag) ? 1 : 0, 0)) {
        ok = false;
        break;
      }
    }
    if (!ok) {
      if (lane == 0) record_error(p.err, B2Q_ETIMEOUT);
      *abort_flag = 1;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (!ok) key[i] = 0u;  // routing on zero logits after a timeout (the call reports it)
      if (blockIdx.x == 0 && p.logits_out && e < p.E) p.logits_out[e] = __uint_as_float(key[i]);
      // order-preserving keys, NaN as -inf; 0 marks no expert (or one taken)
      uint32_t u = key[i];
      if ((u & 0x7fffffffu) > 0x7f800000u) u = 0xff800000u;
      key[i] = e < p.E ? ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) : 0u;
    }
    // k rounds of a warp arg-max: larger key first, ties to the lower index
    // (the reference's stable selection)
    float selv = -INFINITY;
    for (int slot = 0; slot < p.k; ++slot) {
      uint32_t bk = 0u;
      unsigned be = 0xffffffffu;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (key[i] > bk) {
          bk = key[i];
          be = (unsigned)(lane + 32 * i);
        }
      const uint32_t m = __reduce_max_sync(0xffffffffu, bk);
      const int e = (int)__reduce_min_sync(0xffffffffu, bk == m ? be : 0xffffffffu);
      if (lane == slot) selv = __uint_as_float((m & 0x80000000u) ? (m & 0x7fffffffu) : ~m);
      if (lane == 0) {
        sidx[slot] = (uint32_t)e;
        __threadfence_block();
        *topk_ready = slot + 1;
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (e == lane + 32 * i) key[i] = 0u;
    }
    softmax_k(selv, p.k, sw);
    __syncwarp();
    if (blockIdx.x == 0 && lane < p.k) {
      if (p.idx_out) p.idx_out[lane] = sidx[lane];
      if (p.w_out) p.w_out[lane] = sw[lane];
    }
    if (lane == 0) {
      int n = 0;
      for (int s2 = 0; s2 < p.k; ++s2) {
        const int e = (int)sidx[s2];
        if (!EP || (e >= p.e_lo && e < p.e_lo + p.e_local)) lslot[n++] = s2;
      }
      *nloc_sm = n;
    }
  }
  if (early) {
    if (warp != NCW) named_bar_sync(1, (NWARP - 1) * 32);
  } else {
    __syncthreads();
  }

  // every routed slot is local without expert parallelism
  const int nloc = !FUSED ? 0 : (EP ? *nloc_sm : p.k);
  const int F = p.F, H = p.H;
  // Static schedule. qmv: unit u to CTA u mod grid. Fused: gate|up unit u to
  // CTA grid - 1 - (u mod grid); 16-row down block j to CTA j mod grid, each
  // CTA streaming its blocks' rows of every routed slot (units of 4 slots,
  // slots 0-3 of all its blocks first) and folding the slots locally; the
  // CTAs with a block fewer take the extra gate|up units.
  const int G = (int)gridDim.x, bx = (int)blockIdx.x;
  const int U1 = FUSED ? nloc * (F / ROWS_GU) : (p.N + ROWS_QMV - 1) / ROWS_QMV;
  const int nq = (nloc + SLOTS_D - 1) / SLOTS_D;     // down units per block
  const int nblk = FUSED ? (H / ROWS_D + G - 1 - bx) / G : 0;
  const int ngu = FUSED ? (U1 + bx) / G : (U1 - bx + G - 1) / G;  // first-family units of this CTA
  const int UT = ngu + nblk * nq;

  if (warp == NCW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      int* lastf = lastf_sm;  // parity of each stage's latest fill, -1 before the first
      for (int i = 0; i < MAXST; ++i) lastf[i] = -1;
      int s = -1;
      uint32_t eph = 1u;  // parity of the empty phase the next reuse of stage s waits for
      uint32_t ready = 0u;  // slots whose activations this CTA has seen final
      // top-k has chosen slot z's expert (bounded wait on the slot count)
      auto slot_chosen = [&](int z) -> bool {
        for (uint32_t n = 0; *topk_ready <= z; ++n) {
          if (*abort_flag || ((n & 63u) == 63u && globaltimer() > deadline)) {
            if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
            *abort_flag = 1;
            return false;
          }
        }
        __threadfence_block();  // the slot's expert id is read after the count
        return true;
      };
      for (int it = 0;; ++it) {
        if (++s == NS) {
          s = 0;
          eph ^= 1u;
        }
        if (it < npre) {  // qmv units issued before the pass over x (it < NS - 1: no reuse yet)
          lastf[s] = (int)(eph ^ 1u);
          continue;
        }
        if (it >= NS && !tc::wait(&empty[s], eph, deadline, abort_flag)) {
          if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
          *abort_flag = 1;
        }
        if (it >= UT || *abort_flag) {
          info[s] = make_int4(U_END, 0, 0, 0);
          mbar_arrive(&full[s]);
          lastf[s] = (int)(eph ^ 1u);
          break;
        }
        uint8_t* st = smem + (size_t)s * p.stage_bytes;
        if (!FUSED) {
          const int u = bx + it * G;
          const int row = u * ROWS_QMV;
          info[s] = make_int4(U_QMV, 0, u, 0);
          // LUT: one block of pair indices in place of the scale and bias blocks
          mbar_arrive_expect_tx(&full[s], (uint32_t)(ROWS_QMV * K1 / 2 + (LUT ? 1 : 2) * ROWS_QMV * p.mb1));
          tma3(st, &p.map[MW], 0, row, 0, &full[s], pol);
          tc::tma_load_2d(st + p.st_meta1, &p.map[MS], 0, row, &full[s], pol);
          if (!LUT) tc::tma_load_2d(st + p.st_meta1 + p.st_mstep1, &p.map[MB], 0, row, &full[s], pol);
        } else if (it < ngu) {
          const int u = G - 1 - bx + it * G;
          const int z = u / (F / ROWS_GU), rb = u % (F / ROWS_GU);
          if (early && !slot_chosen(z)) {
            info[s] = make_int4(U_END, 0, 0, 0);
            mbar_arrive(&full[s]);
            lastf[s] = (int)(eph ^ 1u);
            break;
          }
          const uint32_t e = EP ? sidx[lslot[z]] - (uint32_t)p.e_lo : sidx[z];
          const int row = (int)(e * (uint32_t)F) + rb * ROWS_GU;
          info[s] = make_int4(U_GU, z, rb, 0);
          mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * ROWS_GU * K1 / 2 + 4 * ROWS_GU * p.mb1));
          tma3(st, &p.map[MWG], 0, row, 0, &full[s], pol);
          tma3(st + ROWS_GU * K1 / 2, &p.map[MWU], 0, row, 0, &full[s], pol);
          uint8_t* m = st + p.st_meta1;
          tc::tma_load_2d(m, &p.map[MSG], 0, row, &full[s], pol);
          tc::tma_load_2d(m + p.st_mstep1, &p.map[MBG], 0, row, &full[s], pol);
          tc::tma_load_2d(m + 2 * p.st_mstep1, &p.map[MSU], 0, row, &full[s], pol);
          tc::tma_load_2d(m + 3 * p.st_mstep1, &p.map[MBU], 0, row, &full[s], pol);
        } else {
          const int d = it - ngu, nbk = max(nblk, 1), quad = d / nbk, lb = d % nbk, blk = bx + lb * G;
          const int z0 = quad * SLOTS_D, nsl = min(SLOTS_D, nloc - z0);
          if (early && !slot_chosen(z0 + nsl - 1)) {
            info[s] = make_int4(U_END, 0, 0, 0);
            mbar_arrive(&full[s]);
            lastf[s] = (int)(eph ^ 1u);
            break;
          }
          // the weights and their scales / biases do not depend on the gate|up
          // units: they are requested before the wait for the slots
          info[s] = make_int4(U_DOWN, quad, blk, lb | (nsl << 8));
          const int wb = ROWS_D * F / 2;  // one slot's weight box
          mbar_arrive_expect_tx(&full[s], (uint32_t)(nsl * (wb + 2 * ROWS_D * p.mb2 + F * 2 + F / 2)));
          for (int i = 0; i < nsl; ++i) {
            const int z = z0 + i;
            const uint32_t e = EP ? sidx[lslot[z]] - (uint32_t)p.e_lo : sidx[z];
            const int row = (int)(e * (uint32_t)H) + blk * ROWS_D;
            uint8_t* m = st + p.st_meta2 + i * 2 * p.st_mstep2;
            tma3(st + i * wb, &p.map[MWD], 0, row, 0, &full[s], pol);
            tc::tma_load_2d(m, &p.map[MSD], 0, row, &full[s], pol);
            tc::tma_load_2d(m + p.st_mstep2, &p.map[MBD], 0, row, &full[s], pol);
          }
          // the slots' activations must be final: every gate|up unit of them
          // finished. The counts of the unit's slots not yet seen final are
          // read together (one round trip per poll, not one per slot).
          bool ok = true;
          const uint32_t need = (((1u << nsl) - 1u) << z0) & ~ready;
          if (need) {
            for (uint32_t n = 0;; ++n) {
              uint32_t seen = 0u;
#pragma unroll
              for (int i = 0; i < SLOTS_D; ++i) {
                const int z = z0 + i;
                if ((need >> z) & 1u)
                  seen |= (ld_relaxed_u32(&done[z]) >= (unsigned)(F / ROWS_GU) ? 1u : 0u) << z;
              }
              if (seen == need) break;
              if (*abort_flag || ((n & 15u) == 15u && globaltimer() > deadline)) {
                ok = false;
                break;
              }
              __nanosleep(32);
            }
            // relaxed reads that saw the counts, then one fence: the acquire
            // side of the epilogues' release counts
            fence_acq_rel_gpu();
            ready |= need;
          }
          if (!ok) {
            if (!*abort_flag) record_error(p.err, B2Q_ETIMEOUT);
            *abort_flag = 1;
          }
          fence_proxy_async_global();  // the copies below read what generic stores wrote
          // the unit's slots are consecutive: their activations and block
          // scales (written by the epilogues, in L2) are one copy each; issued
          // after a failed wait too, so the stage completes before the abort
          bulk_g2s(st + p.st_act, p.ws_act + (size_t)z0 * F, (uint32_t)(nsl * F * 2), &full[s], pol_keep);
          bulk_g2s(st + p.st_asc, p.ws_asc + (size_t)z0 * (F / 16), (uint32_t)(nsl * F / 2), &full[s], pol_keep);
          if (!ok) {
            lastf[s] = (int)(eph ^ 1u);
            break;
          }
        }
        lastf[s] = (int)(eph ^ 1u);
      }
      // let every copy issued land before the CTA exits (after an abort some
      // fills may never have been consumed): wait for the latest phase of
      // every stage used, end markers included (lastf: that fill's parity)
      const uint64_t dl = globaltimer() + 200000000ull;
      for (int i = 0; i < NS; ++i)
        if (lastf[i] >= 0) tc::wait_until(&full[i], (uint32_t)lastf[i], dl);
    }
    __syncwarp();
  } else if (warp > NCW) {
    // ------------------------------ epilogue ------------------------------
    // Epilogue warp e finishes units e, e + NEPI, ... once the consumers
    // posted their partials: it releases the stage, then does the unit's
    // global work (bf16 store, SwiGLU activations, or the down block's slot
    // table and fold). A finished gate|up unit is published at once (fence,
    // then the slot's count): the fence waits for this warp's stores to be
    // acknowledged, which at full bandwidth takes about as long as a unit
    // streams, so the units alternate between warps and no compute warp waits.
    const int ew = warp - NCW - 1;
    for (int n = ew; n < UT; n += NEPI) {
      const int s = n % NS;
      const uint32_t ph = (uint32_t)(n / NS) & 1u;
      if (!__all_sync(0xffffffffu, tc::wait(&rfull[s], ph, deadline, abort_flag))) {
        if (!*abort_flag && lane == 0) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        break;
      }
      const int4 inf = info[s];
      const float* rb = red + (size_t)s * NCW * 32;
      float t0 = 0.0f, t1 = 0.0f;
      if (FUSED && inf.x == U_DOWN) {
        // rows lane and lane + 32 of the unit: row i is slot block i / 16, partial row i % 16
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int i = lane + 32 * h2, b = i >> 4, j = i & 15;
          const float y2 = (rb[(4 * b) * 32 + j] + rb[(4 * b + 1) * 32 + j]) +
                           (rb[(4 * b + 2) * 32 + j] + rb[(4 * b + 3) * 32 + j]);
          if (h2 == 0) t0 = y2; else t1 = y2;
        }
      } else {
        // lane l: total of partial row l over the warps (pairwise)
        float v[NCW];
#pragma unroll
        for (int w = 0; w < NCW; ++w) v[w] = rb[w * 32 + lane];
#pragma unroll
        for (int h = NCW / 2; h >= 1; h >>= 1)
#pragma unroll
          for (int w = 0; w < h; ++w) v[w] += v[w + h];
        t0 = v[0];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (FUSED && inf.x == U_GU) {
        // t0 at lane l: row l of [gate 0..7][up 0..7][gate 8..15][up 8..15]
        const int z = inf.y, blk = inf.z;
        const int f = lane & 15;  // output f of the unit (lanes 16..31 repeat lanes 0..15)
        const float g = __shfl_sync(0xffffffffu, t0, 16 * (f >> 3) + (f & 7));
        const float up = __shfl_sync(0xffffffffu, t0, 16 * (f >> 3) + 8 + (f & 7));
        const uint16_t a = swiglu_bf16_cvt(f2bf(g), f2bf(up));
        // the block of 16 as int8 pieces: scale 2^(14 - E) from the max |a|,
        // X = round(a * 2^(14 - E)) <= 32639 (as for x), hi = byte 1 of
        // X + 128, lo = byte 0 of X (lanes 16..31 repeat lanes 0..15)
        const unsigned mx = __reduce_max_sync(0xffffffffu, a & 0x7fffu);
        float sm = lane < 16 ? bf2f(a) : 0.0f;
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
        int e = (int)((mx >> 7) & 0xffu) - 127;
        if (mx == 0u || mx >= 0x7f80u) e = 0;
        e = max(-110, min(120, e));
        const int X = min(__float2int_rn(bf2f(a) * __int_as_float((127 + 14 - e) << 23)), 32639);
        const uint32_t hb = ((uint32_t)(X + 128) >> 8) & 0xffu, lb = (uint32_t)X & 0xffu;
        // lane l < 8 builds 32-bit piece q = l % 4 of word l / 4: byte i is value
        // 2 i (+1 for odd q) of the word, hi pieces for q < 2, lo for q >= 2
        const int wq = (lane >> 2) & 1, q = lane & 3;
        uint32_t pw = 0u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int src = 8 * wq + 2 * i + (q & 1);
          const uint32_t hv = __shfl_sync(0xffffffffu, hb, src), lv = __shfl_sync(0xffffffffu, lb, src);
          pw |= ((q & 2) ? lv : hv) << (8 * i);
        }
        if (lane < 8) reinterpret_cast<uint32_t*>(p.ws_act + (size_t)z * F + blk * ROWS_GU)[lane] = pw;
        if (lane == 0) p.ws_asc[(size_t)z * (F / 16) + blk] = make_float2(__int_as_float((127 + e - 14) << 23), sm);
        // warp barrier, then one release count by lane 0 (cumulative over the
        // lanes' stores)
        __syncwarp();
        if (lane == 0) red_release_add_u32(&done[z], 1u);
      } else if (FUSED) {
        // rows lane, lane + 32: slot quad * 4 + row / 16, block row row % 16;
        // the bf16 products go to the block's slot table, and the block's last
        // unit folds its slots in the reference's combine order
        const int quad = inf.y, blk = inf.z, lb = inf.w & 0xff, nsl = inf.w >> 8;
        float* yb = ysm + (size_t)lb * MAXK * ROWS_D;
        if ((lane >> 4) < nsl) yb[(quad * SLOTS_D + (lane >> 4)) * ROWS_D + (lane & 15)] = bf2f(f2bf(t0));
        if ((lane >> 4) + 2 < nsl) yb[(quad * SLOTS_D + 2 + (lane >> 4)) * ROWS_D + (lane & 15)] = bf2f(f2bf(t1));
        // the block's units go to both epilogue warps: the one that finishes
        // the block's last unit folds
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) {
          __threadfence_block();
          prev = atomicAdd(&ycnt[lb], 1u);
        }
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == (unsigned)(nq - 1)) {
          __threadfence_block();
          if (lane < ROWS_D) {
            // y_j = bf16 product, prod_j = y_j * w_j: with nloc <= 8 slots the
            // colsum association has one product per chain (chain q = 0 +
            // prod_q) and folds the chains in slot order
            float total = 0.0f;
#pragma unroll
            for (int q = 0; q < MAXK; ++q) {
              if (q < nloc) {
                const float a2 = yb[q * ROWS_D + lane] * sw[EP ? lslot[q] : q] + 0.0f;
                total = (q == 0) ? a2 : a2 + total;
              }
            }
            const int h = blk * ROWS_D + lane;
            if (XP) {
              // the rank's partial of row h into every rank's exchange slot
              for (int r2 = 0; r2 < p.npeer; ++r2)
                p.xpeer[r2][D2_XDATA + ((size_t)(xslot * D2_XMAX + p.prank)) * H + h] = total;
            } else if (EP) {
              p.out_f32[h] = total;
            } else {
              p.out[h] = f2bf(total);
            }
          }
        }
      } else {
        // row lane of the unit: partial slot lane ([P 0..7][Q 8..15][P 16..23][Q 24..31])
        const int row = inf.z * ROWS_QMV + lane;
        if (row < p.N) p.y[row] = f2bf(t0);
      }
    }
  } else {
    // ------------------------------ consumers ------------------------------
    // A CTA's units are all its gate|up units, then its down units, so the
    // consumers run two phases: units whose activation is in registers
    // (gate|up, qmv), then down units (their activation is in the stage).
    const int r = lane >> 2, c = lane & 3;
    // stage and phase of the consumers' current unit
    int cs = 0;
    uint32_t cph = 0u;
    auto advance = [&]() {
      if (++cs == NS) {
        cs = 0;
        cph ^= 1u;
      }
    };
    auto wait_full = [&]() -> bool {
      const int s = cs;
      if (!__all_sync(0xffffffffu, tc::wait(&full[s], cph, deadline, abort_flag))) {
        if (!*abort_flag && lane == 0) record_error(p.err, B2Q_ETIMEOUT);
        *abort_flag = 1;
        return false;
      }
      return true;
    };
    // the warp's partials are in `red`: post them to the epilogue warp
    auto post = [&](int s) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[s]);
    };

    int4 inf = make_int4(U_END, 0, 0, 0);
    bool live = true;
    if (LUT && !__all_sync(0xffffffffu, tc::wait(lutbar, 0u, deadline, abort_flag))) {
      if (!*abort_flag && lane == 0) record_error(p.err, B2Q_ETIMEOUT);
      *abort_flag = 1;
    }
    // ---- phase 1: gate|up (fused) or qmv units ----
    for (;; advance()) {
      if (!wait_full()) {
        live = false;
        break;
      }
      const int s = cs;
      inf = info[s];
      if (inf.x == U_END || inf.x == U_DOWN) break;
      const uint8_t* st = smem + (size_t)s * p.stage_bytes;
      float* rp = red + ((size_t)s * NCW + warp) * 32;
      const uint8_t* mb = st + p.st_meta1;
      if (FUSED) {
        // both row blocks of the 16 outputs, the warp's slice of the reduction
        const Meta m[2] = {
            {mb, mb + p.st_mstep1, mb + 2 * p.st_mstep1, mb + 3 * p.st_mstep1, r, r, p.mb1, p.sw1 != 0},
            {mb, mb + p.st_mstep1, mb + 2 * p.st_mstep1, mb + 3 * p.st_mstep1, 8 + r, 8 + r, p.mb1, p.sw1 != 0}};
        const int ub = ROWS_GU * K1 / 2;  // the up rows' box
        float accP[2] = {0.0f, 0.0f}, accQ[2] = {0.0f, 0.0f};
        dot_i8<SLOT, 2>(st, woff, 1024, ub, slot01, nslot1, p.gs, xb, gsc, m, accP, accQ);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          accP[b] += __shfl_xor_sync(0xffffffffu, accP[b], 1);
          accQ[b] += __shfl_xor_sync(0xffffffffu, accQ[b], 1);
          accP[b] += __shfl_xor_sync(0xffffffffu, accP[b], 2);
          accQ[b] += __shfl_xor_sync(0xffffffffu, accQ[b], 2);
          if (c == 0) {
            rp[16 * b + r] = accP[b];
            rp[16 * b + 8 + r] = accQ[b];
          }
        }
      } else {
        // two row blocks of 16 rows (P: rows 16b..16b+7, Q: rows 16b+8..16b+15)
        const Meta m[2] = {{mb, mb + p.st_mstep1, mb, mb + p.st_mstep1, r, 8 + r, p.mb1, p.sw1 != 0},
                           {mb, mb + p.st_mstep1, mb, mb + p.st_mstep1, 16 + r, 24 + r, p.mb1, p.sw1 != 0}};
        float accP[2] = {0.0f, 0.0f}, accQ[2] = {0.0f, 0.0f};
        dot_i8<SLOT, 2, LUT>(st, woff, 2048, 1024, slot01, nslot1, p.gs, xb, gsc, m, accP, accQ, lut_sm);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          accP[b] += __shfl_xor_sync(0xffffffffu, accP[b], 1);
          accQ[b] += __shfl_xor_sync(0xffffffffu, accQ[b], 1);
          accP[b] += __shfl_xor_sync(0xffffffffu, accP[b], 2);
          accQ[b] += __shfl_xor_sync(0xffffffffu, accQ[b], 2);
          if (c == 0) {
            rp[16 * b + r] = accP[b];
            rp[16 * b + 8 + r] = accQ[b];
          }
        }
      }
      post(s);
    }
    // ---- phase 2 (fused): down units; the current unit has already been waited for ----
    if (FUSED && live) {
      for (;;) {
        const int s = cs;
        if (inf.x != U_DOWN) break;
        const uint8_t* st = smem + (size_t)s * p.stage_bytes;
        float* rp = red + ((size_t)s * NCW + warp) * 32;
        // 4 slots (16 rows each) x 4 reduction quarters
        const int b = warp >> 2, qw = warp & 3, nsl = inf.w >> 8;
        float accP = 0.0f, accQ = 0.0f;
        if (b < nsl) {
          const uint8_t* mb = st + p.st_meta2 + b * 2 * p.st_mstep2;
          const Meta m{mb, mb + p.st_mstep2, mb, mb + p.st_mstep2, r, 8 + r, p.mb2, p.sw2 != 0};
          const uint8_t* wbx = st + b * (ROWS_D * F / 2);
          const uint8_t* pcs = st + p.st_act + b * F * 2;
          const float2* asc = reinterpret_cast<const float2*>(st + p.st_asc + b * (F / 2));
          const int ns = F / 128;  // chunks of the warp's quarter
          if (ns % 12 == 0)
            dot_i8_act<3>(wbx, pcs, asc, qw * ns, ns, p.gs, m, accP, accQ);
          else if (ns % 8 == 0)
            dot_i8_act<2>(wbx, pcs, asc, qw * ns, ns, p.gs, m, accP, accQ);
          else
            dot_i8_act<1>(wbx, pcs, asc, qw * ns, ns, p.gs, m, accP, accQ);
        }
        accP += __shfl_xor_sync(0xffffffffu, accP, 1);
        accQ += __shfl_xor_sync(0xffffffffu, accQ, 1);
        accP += __shfl_xor_sync(0xffffffffu, accP, 2);
        accQ += __shfl_xor_sync(0xffffffffu, accQ, 2);
        if (c == 0) {
          rp[r] = accP;
          rp[r + 8] = accQ;
        }
        post(s);
        advance();
        if (!wait_full()) break;
        inf = info[cs];
      }
    }
  }

  // expert parallel with no routed slot here: the partial is zero
  if (EP && nloc == 0) {
    for (int h = blockIdx.x * NTH + tid; h < H; h += gridDim.x * NTH) {
      if (XP) {
        for (int r2 = 0; r2 < p.npeer; ++r2)
          p.xpeer[r2][D2_XDATA + ((size_t)(xslot * D2_XMAX + p.prank)) * H + h] = 0.0f;
      } else {
        p.out_f32[h] = 0.0f;
      }
    }
  }
  // every thread's stores into other GPUs' exchange buffers are visible there
  // before this CTA is counted
  if (XP) __threadfence_system();

  // ---- exit: the last CTA out re-arms the grid words for the next call ----
  __syncthreads();
  if (FUSED && tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&p.ctr[2], 1u);
    if (prev == gridDim.x - 1) {
      p.ctr[2] = 0u;
      p.ctr[D2_CTR_TAG] = tag;
      for (int i = 0; i < MAXK; ++i) done[i] = 0u;
      __threadfence();
      if (XP) {
        // the rank's whole partial is in every exchange buffer: advance the
        // rank's epoch and publish this call's flag to every rank
        __threadfence_system();
        *reinterpret_cast<volatile unsigned*>(p.xpeer[p.prank]) = xep;
        for (int r2 = 0; r2 < p.npeer; ++r2)
          st_release_sys_u32(reinterpret_cast<unsigned*>(p.xpeer[r2]) + D2_XFLAGS + xslot * D2_XMAX + p.prank, xep);
      }
    }
  }
  if (XP) {
    // every rank's partial of this call (bounded wait on the local flags), then
    // the rows of this CTA's down blocks summed in rank order
    if (tid == 0) {
      const unsigned* fl = reinterpret_cast<const unsigned*>(p.xpeer[p.prank]) + D2_XFLAGS + xslot * D2_XMAX;
      bool ok = !*abort_flag;
      for (int r2 = 0; r2 < p.npeer && ok; ++r2) {
        for (uint32_t n = 0; (int)(ld_acquire_sys_u32(fl + r2) - xep) < 0; ++n) {
          if ((n & 63u) == 63u && globaltimer() > deadline) {
            record_error(p.err, B2Q_ETIMEOUT);
            ok = false;
            break;
          }
        }
      }
      if (!ok) *abort_flag = 1;
    }
    __syncthreads();
    if (!*abort_flag) {
      const float* xd = p.xpeer[p.prank] + D2_XDATA + (size_t)xslot * D2_XMAX * H;
      for (int i = tid; i < nblk * ROWS_D; i += NTH) {
        const int h = ((int)blockIdx.x + (i / ROWS_D) * (int)gridDim.x) * ROWS_D + (i % ROWS_D);
        float sum = 0.0f;
        for (int r2 = 0; r2 < p.npeer; ++r2) sum += __ldcg(xd + (size_t)r2 * H + h);
        p.out[h] = f2bf(sum);
      }
    }
  }
}

}  // namespace d2
}  // namespace b2q

namespace b2q {
namespace d2 {

static int round_up(int v, int a) { return (v + a - 1) / a * a; }

static int plan(D2Params& p, int mode) {
  const int K1 = p.K1;
  p.mb1 = K1 / p.gs * 2;
  p.sw1 = p.mb1 == 128;
  int st;
  const bool qmv = mode == D2_QMV || mode == D2_QMV_LUT;
  if (qmv) {
    p.st_meta1 = ROWS_QMV * K1 / 2;
    p.st_mstep1 = round_up(ROWS_QMV * p.mb1, p.sw1 ? 1024 : 128);
    // scale and bias blocks, or (LUT) one block of pair indices of the same layout
    st = p.st_meta1 + (mode == D2_QMV_LUT ? 1 : 2) * p.st_mstep1;
    p.mb2 = p.sw2 = p.st_meta2 = p.st_mstep2 = p.st_act = p.st_asc = 0;
  } else {
    p.st_meta1 = 2 * ROWS_GU * K1 / 2;
    p.st_mstep1 = round_up(ROWS_GU * p.mb1, p.sw1 ? 1024 : 128);
    const int gu = p.st_meta1 + 4 * p.st_mstep1;
    p.mb2 = p.F / p.gs * 2;
    p.sw2 = p.mb2 == 128;
    // down unit: 4 slots' 16-row weight boxes, their scale / bias tiles, activations, chunk sums
    p.st_meta2 = SLOTS_D * ROWS_D * p.F / 2;
    p.st_mstep2 = round_up(ROWS_D * p.mb2, p.sw2 ? 1024 : 128);
    p.st_act = p.st_meta2 + SLOTS_D * 2 * p.st_mstep2;
    p.st_asc = p.st_act + SLOTS_D * p.F * 2;
    const int dn = p.st_asc + SLOTS_D * p.F / 2;
    st = std::max(gu, dn);
  }
  p.stage_bytes = round_up(st, 1024);
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  // stages first (1024-aligned), then the group sums of x, the warp partials
  // of every stage and the barriers / routing state
  const int xs_bytes = round_up(K1 / p.gs * 8, 128);
  // down blocks' slot tables (fused)
  const int ys_bytes = qmv ? 0 : (p.H / ROWS_D + di.sm_count - 1) / di.sm_count * MAXK * ROWS_D * 4;
  // the shared-memory copy of the pair table (LUT)
  const int lut_bytes = mode == D2_QMV_LUT ? round_up(p.lut_words * 4, 128) : 0;
  int ns = MAXST;
  for (; ns >= 2; --ns) {
    const int total = ns * p.stage_bytes + xs_bytes + ys_bytes + ns * NCW * 32 * 4 + MISC_BYTES + lut_bytes + 1024;
    if (total <= di.smem_optin) break;
  }
  if (ns < 2) return set_error(B2Q_EUNSUPPORTED, "decode kernel: stages of %d bytes do not fit", p.stage_bytes);
  p.nstage = ns;
  int off = ns * p.stage_bytes;
  p.off_xs = off;
  off += xs_bytes;
  p.off_ysm = off;
  off += ys_bytes;
  p.off_red = off;
  off += ns * NCW * 32 * 4;
  p.off_misc = off;
  off += MISC_BYTES;
  p.off_lut = off;
  off += lut_bytes;
  p.smem_bytes = off + 1024;
  return B2Q_OK;
}

template <int CPG, int MODE>
static int launch_t(const D2Params& p, cudaStream_t st, int grid) {
  static bool attr_done[64] = {};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (!attr_done[di.device & 63]) {
    B2Q_TRY_CUDA(cudaFuncSetAttribute(d2_kernel<CPG, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      di.smem_optin));
    attr_done[di.device & 63] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTH);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = st;
  // one CTA per SM, all resident at once (the fused kernel's CTAs wait on
  // each other's counts): a cooperative launch guarantees it or fails
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  B2Q_TRY_CUDA(cudaLaunchKernelEx(&cfg, d2_kernel<CPG, MODE>, p));
  return B2Q_OK;
}

static int launch(const D2Params& p, int mode, cudaStream_t st) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int grid = di.sm_count;
  const int cpg = p.gs / 32;
  switch (cpg * 4 + mode) {
    case 1 * 4 + D2_QMV: return launch_t<1, D2_QMV>(p, st, grid);
    case 2 * 4 + D2_QMV: return launch_t<2, D2_QMV>(p, st, grid);
    case 4 * 4 + D2_QMV: return launch_t<4, D2_QMV>(p, st, grid);
    case 1 * 4 + D2_QMV_LUT: return launch_t<1, D2_QMV_LUT>(p, st, grid);
    case 2 * 4 + D2_QMV_LUT: return launch_t<2, D2_QMV_LUT>(p, st, grid);
    case 4 * 4 + D2_QMV_LUT: return launch_t<4, D2_QMV_LUT>(p, st, grid);
    case 1 * 4 + D2_FUSED: return launch_t<1, D2_FUSED>(p, st, grid);
    case 2 * 4 + D2_FUSED: return launch_t<2, D2_FUSED>(p, st, grid);
    case 4 * 4 + D2_FUSED: return launch_t<4, D2_FUSED>(p, st, grid);
    case 1 * 4 + D2_FUSED_EP: return launch_t<1, D2_FUSED_EP>(p, st, grid);
    case 2 * 4 + D2_FUSED_EP: return launch_t<2, D2_FUSED_EP>(p, st, grid);
    case 4 * 4 + D2_FUSED_EP: return launch_t<4, D2_FUSED_EP>(p, st, grid);
    default: return set_error(B2Q_EUNSUPPORTED, "decode kernel: group size %d", p.gs);
  }
}

// Tensor maps of recently used weight sets. Encoding the (up to nine) maps of
// a call costs microseconds of host time, while a model calls the same layers
// over and over; maps depend only on addresses, shapes and boxes, so an entry
// keyed by those stays valid whatever the buffers hold. Least recently used
// entries are replaced.
struct MapKey {
  const void* ptr[9];
  int device, mode, a, b, c, gs;
};
struct MapEntry {
  MapKey key;
  CUtensorMap map[9];
  uint64_t stamp;
};
constexpr int MAP_CACHE = 128;
static std::mutex g_map_mu;
static MapEntry g_maps[MAP_CACHE];
static uint64_t g_map_clock = 0;

static MapKey map_key(int mode, const void* const* ptrs, int n, int a, int b, int c, int gs) {
  MapKey k;
  std::memset(&k, 0, sizeof(k));  // padding included: keys compare bytewise
  for (int i = 0; i < n; ++i) k.ptr[i] = ptrs[i];
  cudaGetDevice(&k.device);
  k.mode = mode;
  k.a = a;
  k.b = b;
  k.c = c;
  k.gs = gs;
  return k;
}
static bool find_maps(const MapKey& k, CUtensorMap* out, int n) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (MapEntry& e : g_maps) {
    if (e.stamp && std::memcmp(&e.key, &k, sizeof(k)) == 0) {
      std::memcpy(out, e.map, sizeof(CUtensorMap) * n);
      e.stamp = ++g_map_clock;
      return true;
    }
  }
  return false;
}
static void put_maps(const MapKey& k, const CUtensorMap* m, int n) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  MapEntry* victim = &g_maps[0];
  for (MapEntry& e : g_maps)
    if (e.stamp < victim->stamp) victim = &e;
  victim->key = k;
  std::memcpy(victim->map, m, sizeof(CUtensorMap) * n);
  victim->stamp = ++g_map_clock;
}

// weights: 3-D swizzled map, box of `box_rows` rows x the whole row;
// scales / biases: 2-D map, box of `box_rows` rows x the whole metadata row
static int set_family(D2Params& p, int mw, int ms, int mb, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                      uint64_t rows, int K, int box_rows) {
  int rc = make_row_tile_map(&p.map[mw], w, rows, (uint64_t)K / 2, (uint32_t)box_rows);
  if (rc) return rc;
  const int mrow = K / p.gs * 2;
  const int swz = mrow == 128 ? 128 : 0;
  rc = make_2d_map(&p.map[ms], s, rows, (uint64_t)mrow, (uint32_t)mrow, (uint32_t)box_rows, swz);
  if (rc) return rc;
  return make_2d_map(&p.map[mb], b, rows, (uint64_t)mrow, (uint32_t)mrow, (uint32_t)box_rows, swz);
}

static bool gs_ok(int gs) { return gs == 32 || gs == 64 || gs == 128; }

// The gate|up / qmv reduction splits into NCW equal slices of whole groups of
// at most XR chunk columns each (a chunk column is 32 values).
static bool xreg_split_ok(int K, int gs) {
  const int ncc = K / (32 * NCW);  // chunk columns per consumer warp
  const int cps = gs == 32 ? 1 : 2;  // chunk columns per column slot
  // whole groups per warp, at most two batches of four slots, at most XB / 2 MMA steps
  const int nslot = ncc / cps, steps = ((nslot + 3) / 4) * (cps * 4);
  return K > 0 && K % (32 * NCW) == 0 && K % (8 * gs) == 0 && ncc % (gs / 32) == 0 && ncc % cps == 0 &&
         nslot <= 8 && steps <= XB / 2;
}

}  // namespace d2

using namespace d2;

bool d2_qmv_eligible(int N, int K, int gs, const void* x, const void* w, const void* s, const void* b) {
  return gs_ok(gs) && N >= ROWS_QMV && N % 16 == 0 && xreg_split_ok(K, gs) && aligned16(x) && aligned16(w) &&
         aligned16(s) && aligned16(b);
}

bool d2_norm_ok(int K) { return K > 0 && K % 8 == 0 && K / 8 <= NTH; }

int d2_qmv(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b, uint16_t* y, int N, int K,
           int gs, cudaStream_t st, const D2Norm& norm) {
  D2Params p;
  std::memset(&p, 0, sizeof(p));
  p.nw = norm.weight;
  p.ndelta = norm.delta;
  p.nh_out = norm.h_out;
  p.neps = norm.eps;
  p.gs = gs;
  p.K1 = K;
  p.N = N;
  p.x = x;
  p.y = y;
  p.timeout_ns = 2000000000ll;
  int rc = plan(p, D2_QMV);
  if (rc) return rc;
  const void* ptrs[3] = {w, s, b};
  const MapKey key = map_key(D2_QMV, ptrs, 3, N, K, 0, gs);
  if (!find_maps(key, p.map, 3)) {
    rc = set_family(p, MW, MS, MB, w, s, b, (uint64_t)N, K, ROWS_QMV);
    if (rc) return rc;
    put_maps(key, p.map, 3);
  }
  return launch(p, D2_QMV, st);
}

// Largest pair table the kernel copies into shared memory: 16,384 entries
// (64 KB) leave room for a ring of two 68 KB stages at K = 4096.
constexpr int LUT_MAX_WORDS = 16384;

bool d2_qmv_lut_eligible(int N, int K, int gs, int count, const void* x, const void* w, const void* index,
                         const void* table) {
  if (!(gs_ok(gs) && N >= ROWS_QMV && N % 16 == 0 && xreg_split_ok(K, gs) && count >= 1 &&
        round_up(count, 4) <= LUT_MAX_WORDS && aligned16(x) && aligned16(w) && aligned16(index) &&
        aligned16(table)))
    return false;
  D2Params p;
  std::memset(&p, 0, sizeof(p));
  p.gs = gs;
  p.K1 = K;
  p.lut_words = round_up(count, 4);
  const bool fits = plan(p, D2_QMV_LUT) == B2Q_OK;
  clear_error();
  return fits;
}

int d2_qmv_lut(const uint16_t* x, const uint32_t* w, const uint16_t* index, const uint32_t* table, int count,
               uint16_t* y, int N, int K, int gs, cudaStream_t st) {
  D2Params p;
  std::memset(&p, 0, sizeof(p));
  p.gs = gs;
  p.K1 = K;
  p.N = N;
  p.x = x;
  p.y = y;
  p.lut = table;
  p.lut_words = round_up(count, 4);
  p.timeout_ns = 2000000000ll;
  int rc = plan(p, D2_QMV_LUT);
  if (rc) return rc;
  const void* ptrs[3] = {w, index, nullptr};
  const MapKey key = map_key(D2_QMV_LUT, ptrs, 3, N, K, 0, gs);
  if (!find_maps(key, p.map, 3)) {
    // the index has the layout of the scales ([N, K/gs] 16-bit): the same maps
    rc = set_family(p, MW, MS, MB, w, index, index, (uint64_t)N, K, ROWS_QMV);
    if (rc) return rc;
    put_maps(key, p.map, 3);
  }
  return launch(p, D2_QMV_LUT, st);
}

bool d2_moe_eligible(int H, int E, int F, int k, int gs) {
  if (!(gs_ok(gs) && H > 0 && F > 0 && xreg_split_ok(H, gs) && F % (8 * gs) == 0 && F % 256 == 0 &&
        (F / 128) % (gs / 32) == 0 && F % ROWS_GU == 0 && H % ROWS_D == 0 && F / gs * 2 <= 512 &&
        k >= 1 && k <= MAXK && E >= k && E <= 256 && H / 8 <= NTH))
    return false;
  DeviceInfo di;
  if (device_info(&di) || H / ROWS_D > MAXBLK * di.sm_count) {
    clear_error();
    return false;
  }
  D2Params p;
  std::memset(&p, 0, sizeof(p));
  p.gs = gs;
  p.K1 = H;
  p.H = H;
  p.F = F;
  const bool fits = plan(p, D2_FUSED) == B2Q_OK;
  clear_error();
  return fits;
}

int d2_moe_decode(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                  const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd, const uint16_t* sd,
                  const uint16_t* bd, uint16_t* out, uint32_t* idx, float* w, float* logits, int H, int E, int F,
                  int k, int gs, const D2Scratch& scr, cudaStream_t st, int e_lo, int e_local, float* out_f32,
                  const D2Norm& norm, float* const* xpeer, int npeer, int prank) {
  D2Params p;
  std::memset(&p, 0, sizeof(p));
  if (npeer > 0) {
    if (npeer > D2_XMAX || !out_f32 || !out)
      return set_error(B2Q_EINVAL, "decode kernel: peer exchange needs the expert-parallel mode and bf16 out");
    for (int r = 0; r < npeer; ++r) p.xpeer[r] = xpeer[r];
    p.npeer = npeer;
    p.prank = prank;
  }
  p.nw = norm.weight;
  p.ndelta = norm.delta;
  p.nh_out = norm.h_out;
  p.neps = norm.eps;
  p.gs = gs;
  p.K1 = H;
  p.x = x;
  p.wr = wr;
  p.out = out;
  p.idx_out = idx;
  p.w_out = w;
  p.logits_out = logits;
  p.H = H;
  p.E = E;
  p.F = F;
  p.k = k;
  p.err = scr.err;
  p.ctr = scr.ctr;
  p.ws_logits = scr.logits;
  p.ws_act = scr.act;
  p.ws_asc = scr.asc;
  p.e_lo = e_lo;
  p.e_local = e_local;
  p.out_f32 = out_f32;
  p.timeout_ns = 2000000000ll;
  const int mode = out_f32 ? D2_FUSED_EP : D2_FUSED;
  int rc = plan(p, mode);
  if (rc) return rc;
  const void* ptrs[9] = {wg, sg, bg, wu, su, bu, wd, sd, bd};
  const int Eh = e_local > 0 ? e_local : E;  // experts in the stacks this call reads
  const MapKey key = map_key(D2_FUSED, ptrs, 9, H, Eh, F, gs);
  if (!find_maps(key, p.map, 9)) {
    const uint64_t rgu = (uint64_t)Eh * F, rd = (uint64_t)Eh * H;
    rc = set_family(p, MWG, MSG, MBG, wg, sg, bg, rgu, H, ROWS_GU);
    if (rc) return rc;
    rc = set_family(p, MWU, MSU, MBU, wu, su, bu, rgu, H, ROWS_GU);
    if (rc) return rc;
    rc = set_family(p, MWD, MSD, MBD, wd, sd, bd, rd, F, ROWS_D);
    if (rc) return rc;
    put_maps(key, p.map, 9);
  }
  return launch(p, mode, st);
}

}  // namespace b2q
