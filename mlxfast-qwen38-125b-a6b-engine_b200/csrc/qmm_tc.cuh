// qmm_tc.cuh -- grouped 4-bit affine GEMM on tcgen05 tensor cores (host side).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

enum { TC_GLU = 0, TC_PLAIN = 1 };

struct alignas(64) TcParams {
  CUtensorMap map_w0;  // packed weights (gate, or the only matrix)
  CUtensorMap map_w1;  // packed up weights (GLU)
  CUtensorMap map_b;   // token rows, bf16 [R, K], K-permuted
  const uint16_t* s0;
  const uint16_t* b0;
  const uint16_t* s1;
  const uint16_t* b1;
  const uint32_t* offsets;   // [E + 1] row ranges per expert
  const uint32_t* prefix;    // [E + 1] unit ranges per expert
  uint16_t* out;
  const uint32_t* out_rows;  // PLAIN: output row of each sorted row (nullptr: same row)
  int E, K, Nw, gs, out_ld;
  int* err;
  long long timeout_ns;
};

// Shape conditions of the kernel (Nw rows per expert, K reduction length).
bool tc_shape_ok(int Nw, int K, int gs, int mode);
size_t tc_smem_bytes();
// Unit ranges for two products sharing the expert row ranges (prefix1 may be null).
int tc_unit_tables(const uint32_t* offsets, int E, int mt0, int mt1, uint32_t* prefix0, uint32_t* prefix1,
                   cudaStream_t st);
inline int tc_m_tiles(int Nw, int mode) { return mode == TC_GLU ? Nw / 64 : Nw / 128; }
// xs[i] = x[rows[i]] (rows may be null: identity) with the 8-block K reorder; rows >= n_src give zeros.
int tc_gather_rows(const uint16_t* x, const uint32_t* rows, uint16_t* xs, int R, int K, int n_src, cudaStream_t st);
// The same for the rows [offsets[0], offsets[n_groups]) only (device-side bounds).
int tc_gather_rows_range(const uint16_t* x, const uint32_t* rows, uint16_t* xs, int R, int K, int n_src,
                         const uint32_t* offsets, int n_groups, cudaStream_t st);
// Tensor maps for the weights (w1 only for GLU) and the token rows xs [R, K].
int tc_setup(TcParams& p, int mode, const uint16_t* xs, int R, const uint32_t* w0, const uint32_t* w1);
int tc_launch(const TcParams& p, int mode, cudaStream_t st);

}  // namespace b2q
