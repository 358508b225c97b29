// ep.cuh -- pieces shared by the two expert-parallel translation units
// (ep.cu: all-reduce layers; ep_a2a.cu: all-to-all token exchange).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

// ---- the NCCL entry points the library uses, resolved with dlsym ------------
struct NcclUid {
  char internal[128];
};
typedef void* NcclComm;
typedef int (*FnGetUniqueId)(NcclUid*);
typedef int (*FnCommInitRank)(NcclComm*, int, NcclUid, int);
typedef int (*FnCommDestroy)(NcclComm);
typedef int (*FnAllReduce)(const void*, void*, size_t, int, int, NcclComm, cudaStream_t);
typedef int (*FnAllGather)(const void*, void*, size_t, int, NcclComm, cudaStream_t);
typedef int (*FnSend)(const void*, size_t, int, int, NcclComm, cudaStream_t);
typedef int (*FnRecv)(void*, size_t, int, int, NcclComm, cudaStream_t);
typedef int (*FnGroup)();
typedef const char* (*FnGetErrorString)(int);
constexpr int kNcclUint8 = 1;    // ncclUint8
constexpr int kNcclInt32 = 2;    // ncclInt32 / ncclInt
constexpr int kNcclFloat32 = 7;  // ncclFloat32 / ncclFloat
constexpr int kNcclSum = 0;      // ncclSum

struct Nccl {
  FnGetUniqueId get_unique_id = nullptr;
  FnCommInitRank comm_init_rank = nullptr;
  FnCommDestroy comm_destroy = nullptr;
  FnAllReduce all_reduce = nullptr;
  FnAllGather all_gather = nullptr;
  FnSend send = nullptr;
  FnRecv recv = nullptr;
  FnGroup group_start = nullptr;
  FnGroup group_end = nullptr;
  FnGetErrorString error_string = nullptr;
  bool ok = false;      // communicator + all-reduce
  bool p2p_ok = false;  // all-gather + grouped send / recv (all-to-all exchange)
};

const Nccl& nccl();
int nccl_check(int r, const char* what);

struct EpComm {
  NcclComm comm;
  int nranks, rank;
  // peer-memory exchange of the one-token decode (b2q_ep_peer_setup / _open):
  // this rank's buffer, every rank's mapped here (xbuf[rank] == local), hidden size
  float* xlocal = nullptr;
  float* xbuf[8] = {};
  int xH = 0;
  bool xready = false;
};

// Expert ownership: rank r holds the contiguous block [e_lo, e_lo + e_local),
// the first E % nranks ranks one expert more than the others.
inline void ep_expert_block(int E, int nranks, int rank, int* e_lo, int* e_local) {
  const int base = E / nranks, extra = E % nranks;
  *e_lo = rank * base + (rank < extra ? rank : extra);
  *e_local = base + (rank < extra ? 1 : 0);
}

// Argument checks shared by the expert-parallel entry points.
int ep_check_common(const char* fn, int T, int H, int E, int F, int k, int e_lo, int e_local, int gs, int bits);

// partial[t, h] = colsum_j (p = inverse[t*k+j] in [offsets[e_lo], offsets[e_lo+e_local])
//                           ? rb(y[p, h]) * w[t*k+j] : 0), the association of
// mlx_colsum_small_f32 (Runner/FastModel/TrackFastKernels2.swift:36-47).
int launch_ep_sorted_combine(const uint16_t* y, const uint32_t* inverse, const float* w, const uint32_t* offsets,
                             int e_lo, int e_local, float* partial, int T, int H, int k, cudaStream_t st);

}  // namespace b2q
