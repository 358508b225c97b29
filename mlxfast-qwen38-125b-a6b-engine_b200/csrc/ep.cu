// ep.cu -- expert-parallel MoE layers: experts sharded over ranks, one NCCL
// all-reduce of the fp32 layer partial per call.
//
// Every rank holds the replicated router and the experts [e_lo, e_lo + e_local)
// (stacked tensors of the local experts only). The routing is computed in
// full on every rank (same inputs, same kernels, same result); each rank then
// multiplies only the selected experts it holds and adds their weighted
// outputs into an fp32 partial [T, H]; the sum over ranks (NCCL all-reduce on
// the caller's stream) is the layer output, rounded to bf16 once.
//
// Reference: the expert-parallel configuration of the engine's MoE layer
// (moeForwardShared, Runner/FastModel/TrackFastModel.swift:867-1009, with the
// expert stacks bound per layer at :470-540). The combine association differs
// from the single-GPU kernel (per-rank partial sums, then the sum over ranks),
// so the result matches it to rounding, not bit for bit.
//
// Decode (T <= 8): gate / up / down are gathered products over the k slots in
// which the slots holding a non-local expert are invalid items: they load no
// weights and produce zeros. Prefill: the tensor-core grouped GEMMs run over
// the contiguous sorted-row range of the local experts only.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2), so the library has no
// link-time dependency on it; a process that already loaded NCCL (through
// PyTorch, for instance) shares that copy.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "decode2.cuh"
#include "decode_ws.hpp"
#include "engine.cuh"
#include "ep.cuh"
#include "host.hpp"
#include "prefill.cuh"
#include "qmm_tc.cuh"

namespace b2q {

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.get_unique_id = reinterpret_cast<FnGetUniqueId>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<FnCommInitRank>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<FnCommDestroy>(dlsym(h, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<FnAllReduce>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<FnAllGather>(dlsym(h, "ncclAllGather"));
    n.send = reinterpret_cast<FnSend>(dlsym(h, "ncclSend"));
    n.recv = reinterpret_cast<FnRecv>(dlsym(h, "ncclRecv"));
    n.group_start = reinterpret_cast<FnGroup>(dlsym(h, "ncclGroupStart"));
    n.group_end = reinterpret_cast<FnGroup>(dlsym(h, "ncclGroupEnd"));
    n.error_string = reinterpret_cast<FnGetErrorString>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.error_string;
    n.p2p_ok = n.ok && n.all_gather && n.send && n.recv && n.group_start && n.group_end;
  });
  return n;
}

int nccl_check(int r, const char* what) {
  if (r == 0) return B2Q_OK;
  const Nccl& n = nccl();
  return set_error(B2Q_ENCCL, "%s: %s (%d)", what, n.error_string ? n.error_string(r) : "NCCL error", r);
}

namespace {

size_t a256(size_t v) { return (v + 255) / 256 * 256; }

// ---- decode -----------------------------------------------------------------
struct EpDecodeWs {
  int* err;
  float* logits;
  uint32_t* idx;
  float* w;
  uint32_t* rhs;  // local expert of each slot, 0xFFFFFFFF when not held here
  uint32_t* tok;  // token of each slot
  uint16_t *g, *u, *act, *y;
  float2* asc;    // one-token fused kernel: per block of 16 activations (scale, sum)
  unsigned* ctr;  // one-token fused kernel: grid counters (fixed offset)
  size_t bytes;
};

EpDecodeWs ep_decode_layout(void* base, int S, int H, int E, int F, int k) {
  EpDecodeWs d{};
  char* b = static_cast<char*>(base);
  const size_t R = (size_t)S * k;
  size_t off = 0;
  d.err = reinterpret_cast<int*>(b);
  off = 256;
  d.ctr = reinterpret_cast<unsigned*>(b + off);  // fixed offset, as in decode_ws_layout
  off += D2_CTR_BYTES;
  d.logits = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * (size_t)S * E);
  d.idx = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.w = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * R);
  d.rhs = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.tok = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + 4 * R);
  d.g = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * F);
  d.u = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * F);
  d.act = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * F);
  d.y = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * H);
  d.asc = reinterpret_cast<float2*>(b + off);
  off = a256(off + 8 * R * (F / 16));
  d.bytes = off;
  return d;
}

__global__ void ep_slots_kernel(const uint32_t* __restrict__ idx, uint32_t* __restrict__ rhs,
                                uint32_t* __restrict__ tok, int R, int k, int e_lo, int e_local) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R) return;
  const uint32_t le = idx[i] - (uint32_t)e_lo;  // wraps for experts below e_lo
  rhs[i] = le < (uint32_t)e_local ? le : 0xFFFFFFFFu;
  tok[i] = (uint32_t)(i / k);
}

// partial[t, h] = colsum_j (rb(y[t*k + j, h]) * w[t, j]) over this rank's slots
// (the others are zero), the association of mlx_colsum_small_f32
// (Runner/FastModel/TrackFastKernels2.swift:36-47).
__global__ void ep_combine_kernel(const uint16_t* __restrict__ y, const uint32_t* __restrict__ rhs,
                                  const float* __restrict__ w, float* __restrict__ partial, int T, int H, int k) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  const int t = blockIdx.y;
  if (h >= H || t >= T) return;
  float prod[32];
  for (int j = 0; j < k; ++j) {
    const int sl = t * k + j;
    prod[j] = (rhs[sl] != 0xFFFFFFFFu) ? bf2f(y[(size_t)sl * H + h]) * w[sl] : 0.0f;
  }
  const int TY = k < 8 ? k : 8;
  float tt[8];
  for (int q = 0; q < TY; ++q) {
    float a = 0.0f;
    for (int r = q; r < k; r += TY) a = prod[r] + a;
    tt[q] = a;
  }
  float total = tt[0];
  for (int q = 1; q < TY; ++q) total = tt[q] + total;
  partial[(size_t)t * H + h] = total;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, uint16_t* __restrict__ out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f2bf(in[i]);
}

// ---- prefill: combine over the local sorted-row range -------------------------
// partial[t, h] = colsum_j (p = inverse[t*k+j] in [offsets[e_lo], offsets[e_lo+e_local])
//                          ? rb(y[p, h]) * w[t, j] : 0)
__global__ void ep_sorted_combine_kernel(const uint16_t* __restrict__ y, const uint32_t* __restrict__ inverse,
                                         const float* __restrict__ w, const uint32_t* __restrict__ offsets,
                                         int e_lo, int e_local, float* __restrict__ partial, int T, int H, int k) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  const int t = blockIdx.y;
  if (h >= H || t >= T) return;
  const uint32_t lo = offsets[e_lo], hi = offsets[e_lo + e_local];
  float prod[32];
  for (int j = 0; j < k; ++j) {
    const uint32_t pj = inverse[(size_t)t * k + j];
    prod[j] = (pj >= lo && pj < hi) ? bf2f(y[(size_t)pj * H + h]) * w[(size_t)t * k + j] : 0.0f;
  }
  const int TY = k < 8 ? k : 8;
  float tt[8];
  for (int q = 0; q < TY; ++q) {
    float a = 0.0f;
    for (int r = q; r < k; r += TY) a = prod[r] + a;
    tt[q] = a;
  }
  float total = tt[0];
  for (int q = 1; q < TY; ++q) total = tt[q] + total;
  partial[(size_t)t * H + h] = total;
}

struct EpPrefillWs {
  int* err;
  float* logits;
  uint32_t *idx, *sorted_ids, *token_rows, *inverse, *offsets, *prefix_gu, *prefix_dn;
  float* w;
  uint16_t *xs, *act, *y;
  size_t bytes;
};

EpPrefillWs ep_prefill_layout(void* base, int T, int H, int E, int F, int k) {
  EpPrefillWs d{};
  char* b = static_cast<char*>(base);
  const size_t R = (size_t)T * k;
  size_t off = 0;
  d.err = reinterpret_cast<int*>(b);
  off = 256;
  d.logits = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * (size_t)T * E);
  uint32_t** u32s[] = {&d.idx, &d.sorted_ids, &d.token_rows, &d.inverse};
  for (uint32_t** q : u32s) {
    *q = reinterpret_cast<uint32_t*>(b + off);
    off = a256(off + 4 * R);
  }
  d.w = reinterpret_cast<float*>(b + off);
  off = a256(off + 4 * R);
  uint32_t** per_e[] = {&d.offsets, &d.prefix_gu, &d.prefix_dn};
  for (uint32_t** q : per_e) {
    *q = reinterpret_cast<uint32_t*>(b + off);
    off = a256(off + 4 * ((size_t)E + 1));
  }
  d.xs = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * H);
  d.act = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * F);
  d.y = reinterpret_cast<uint16_t*>(b + off);
  off = a256(off + 2 * R * H);
  d.bytes = off;
  return d;
}

int ep_finish(EpComm* c, float* partial, uint16_t* out, size_t n, cudaStream_t st) {
  if (c && c->nranks > 1) {
    int rc = nccl_check(nccl().all_reduce(partial, partial, n, kNcclFloat32, kNcclSum, c->comm, st),
                        "ep: ncclAllReduce");
    if (rc) return rc;
  }
  if (out) {
    f32_to_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(partial, out, n);
    B2Q_TRY_CUDA(cudaGetLastError());
  }
  return B2Q_OK;
}

}  // namespace

int ep_check_common(const char* fn, int T, int H, int E, int F, int k, int e_lo, int e_local, int gs, int bits) {
  if (bits != 4) return set_error(B2Q_EUNSUPPORTED, "%s: bits=%d", fn, bits);
  if (!(gs == 32 || gs == 64 || gs == 128)) return set_error(B2Q_EUNSUPPORTED, "%s: group_size=%d", fn, gs);
  if (T < 0 || H <= 0 || E < 1 || E > 1024 || F <= 0 || k < 1 || k > 32 || k > E || e_lo < 0 || e_local < 1 ||
      e_lo + e_local > E || H % gs || F % gs || H % 8 || F % 8)
    return set_error(B2Q_EINVAL, "%s: bad shape or expert range [%d, %d) of %d", fn, e_lo, e_lo + e_local, E);
  return B2Q_OK;
}

int launch_ep_sorted_combine(const uint16_t* y, const uint32_t* inverse, const float* w, const uint32_t* offsets,
                             int e_lo, int e_local, float* partial, int T, int H, int k, cudaStream_t st) {
  // rows in chunks of at most 65535 (the grid's y limit)
  for (int t0 = 0; t0 < T; t0 += 65535) {
    const int n = T - t0 < 65535 ? T - t0 : 65535;
    dim3 grid((H + 255) / 256, n);
    ep_sorted_combine_kernel<<<grid, 256, 0, st>>>(y, inverse + (size_t)t0 * k, w + (size_t)t0 * k, offsets, e_lo,
                                                   e_local, partial + (size_t)t0 * H, n, H, k);
    B2Q_TRY_CUDA(cudaGetLastError());
  }
  return B2Q_OK;
}

}  // namespace b2q

using namespace b2q;

extern "C" {

int b2q_ep_unique_id(void* id_out, size_t id_bytes) {
  clear_error();
  if (!id_out || id_bytes < sizeof(NcclUid)) return set_error(B2Q_EINVAL, "ep_unique_id: need %zu bytes", sizeof(NcclUid));
  if (!nccl().ok) return set_error(B2Q_ENCCL, "ep_unique_id: libnccl.so.2 could not be loaded");
  NcclUid id;
  int rc = nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
  if (rc) return rc;
  std::memcpy(id_out, &id, sizeof(id));
  return B2Q_OK;
}

int b2q_ep_comm_init(void** comm_out, int nranks, int rank, const void* id, size_t id_bytes) {
  clear_error();
  if (!comm_out || nranks < 1 || rank < 0 || rank >= nranks || (nranks > 1 && (!id || id_bytes < sizeof(NcclUid))))
    return set_error(B2Q_EINVAL, "ep_comm_init: bad arguments");
  EpComm* c = new EpComm{};
  c->nranks = nranks;
  c->rank = rank;
  if (nranks > 1) {
    if (!nccl().ok) {
      delete c;
      return set_error(B2Q_ENCCL, "ep_comm_init: libnccl.so.2 could not be loaded");
    }
    NcclUid uid;
    std::memcpy(&uid, id, sizeof(uid));
    int rc = nccl_check(nccl().comm_init_rank(&c->comm, nranks, uid, rank), "ncclCommInitRank");
    if (rc) {
      delete c;
      return rc;
    }
  }
  *comm_out = c;
  return B2Q_OK;
}

int b2q_ep_comm_destroy(void* comm) {
  clear_error();
  if (!comm) return B2Q_OK;
  EpComm* c = static_cast<EpComm*>(comm);
  int rc = B2Q_OK;
  if (c->comm) rc = nccl_check(nccl().comm_destroy(c->comm), "ncclCommDestroy");
  for (int r = 0; r < c->nranks && r < 8; ++r)
    if (c->xbuf[r] && r != c->rank) cudaIpcCloseMemHandle(c->xbuf[r]);
  if (c->xlocal) cudaFree(c->xlocal);
  delete c;
  return rc;
}

size_t b2q_ep_peer_buffer_bytes(int H) { return H > 0 ? d2_xbuf_bytes(H) : 0; }

int b2q_ep_peer_setup(void* comm, int H, void* handle_out, size_t handle_bytes) {
  clear_error();
  EpComm* c = static_cast<EpComm*>(comm);
  if (!c || H <= 0 || H % 16 || !handle_out || handle_bytes < sizeof(cudaIpcMemHandle_t))
    return set_error(B2Q_EINVAL, "ep_peer_setup: bad arguments (handle needs %zu bytes)", sizeof(cudaIpcMemHandle_t));
  if (c->nranks < 2) return set_error(B2Q_EINVAL, "ep_peer_setup: one rank has nothing to exchange");
  if (c->nranks > D2_XMAX) return set_error(B2Q_EUNSUPPORTED, "ep_peer_setup: at most %d ranks", D2_XMAX);
  if (c->xlocal) return set_error(B2Q_EINVAL, "ep_peer_setup: already set up");
  const size_t bytes = d2_xbuf_bytes(H);
  B2Q_TRY_CUDA(cudaMalloc(reinterpret_cast<void**>(&c->xlocal), bytes));
  B2Q_TRY_CUDA(cudaMemset(c->xlocal, 0, bytes));  // epoch 0, flags 0
  B2Q_TRY_CUDA(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  B2Q_TRY_CUDA(cudaIpcGetMemHandle(&h, c->xlocal));
  std::memcpy(handle_out, &h, sizeof(h));
  c->xH = H;
  return B2Q_OK;
}

int b2q_ep_peer_open(void* comm, const void* handles, size_t handle_bytes) {
  clear_error();
  EpComm* c = static_cast<EpComm*>(comm);
  if (!c || !c->xlocal || !handles || handle_bytes < sizeof(cudaIpcMemHandle_t))
    return set_error(B2Q_EINVAL, "ep_peer_open: call b2q_ep_peer_setup first; handles of every rank needed");
  if (c->xready) return set_error(B2Q_EINVAL, "ep_peer_open: already open");
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < c->nranks; ++r) {
    if (r == c->rank) {
      c->xbuf[r] = c->xlocal;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + (size_t)r * handle_bytes, sizeof(h));
    void* ptr = nullptr;
    B2Q_TRY_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    c->xbuf[r] = static_cast<float*>(ptr);
  }
  c->xready = true;
  return B2Q_OK;
}

size_t b2q_ep_moe_decode_workspace_size(int S, int H, int E, int F, int k) {
  if (S < 1 || H < 1 || E < 1 || F < 1 || k < 1) return 0;
  return ep_decode_layout(nullptr, S, H, E, F, k).bytes;
}

int b2q_ep_moe_decode(void* comm, const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg,
                      const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                      const uint32_t* wd, const uint16_t* sd, const uint16_t* bd, float* partial, uint16_t* out,
                      uint32_t* idx, float* w, int S, int H, int E, int F, int k, int e_lo, int e_local,
                      int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = ep_check_common("ep_moe_decode", S, H, E, F, k, e_lo, e_local, group_size, bits);
  if (rc) return rc;
  if (S < 1 || S > 8) return set_error(B2Q_EUNSUPPORTED, "ep_moe_decode: S=%d (1..8)", S);
  if (!x || !wr || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !partial)
    return set_error(B2Q_EINVAL, "ep_moe_decode: null pointer");
  const EpDecodeWs ws = ep_decode_layout(workspace, S, H, E, F, k);
  if (!workspace || workspace_bytes < ws.bytes || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "ep_moe_decode: workspace of %zu bytes needed", ws.bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int R = S * k;
  if (S == 1) {
    // one token: the fused single-column kernel over the local slots only,
    // writing this rank's fp32 partial (the workspace header doubles as its
    // error word and grid counters)
    const void* ptrs[] = {x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, partial};
    bool all_aligned = true;
    for (const void* q : ptrs) all_aligned = all_aligned && aligned16(q);
    if (all_aligned && d2_moe_eligible(H, E, F, k, group_size)) {
      const D2Scratch scr{ws.err, ws.ctr, ws.logits, ws.act, ws.asc};
      EpComm* c = static_cast<EpComm*>(comm);
      if (c && c->nranks > 1 && c->xready && c->xH == H && out) {
        // the reduction inside the kernel over peer memory: no collective call
        return d2_moe_decode(x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, out, idx, w, nullptr, H, E, F, k,
                             group_size, scr, st, e_lo, e_local, partial, D2Norm(), c->xbuf, c->nranks, c->rank);
      }
      rc = d2_moe_decode(x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, nullptr, idx, w, nullptr, H, E, F, k, group_size,
                         scr, st, e_lo, e_local, partial);
      if (rc) return rc;
      return ep_finish(c, partial, out, (size_t)S * H, st);
    }
  }
  uint32_t* ix = idx ? idx : ws.idx;
  float* ww = w ? w : ws.w;
  rc = eng::launch_router_logits(x, wr, ws.logits, S, E, H, st);
  if (rc) return rc;
  rc = eng::launch_route(ws.logits, ix, ww, S, E, k, st);
  if (rc) return rc;
  ep_slots_kernel<<<(R + 127) / 128, 128, 0, st>>>(ix, ws.rhs, ws.tok, R, k, e_lo, e_local);
  B2Q_TRY_CUDA(cudaGetLastError());
  // gate and up: item i = slot i, x row tok[i], local expert rhs[i] (invalid: no loads, zeros)
  rc = b2q_gather_qmm(x, wg, sg, bg, ws.tok, ws.rhs, ws.g, R, 1, F, H, S, e_local, group_size, bits, 1, 0, stream);
  if (rc) return rc;
  rc = b2q_gather_qmm(x, wu, su, bu, ws.tok, ws.rhs, ws.u, R, 1, F, H, S, e_local, group_size, bits, 1, 0, stream);
  if (rc) return rc;
  rc = b2q_swiglu(ws.g, ws.u, ws.act, (int64_t)R * F, stream);
  if (rc) return rc;
  rc = b2q_gather_qmm(ws.act, wd, sd, bd, nullptr, ws.rhs, ws.y, R, 1, H, F, R, e_local, group_size, bits, 1, 0,
                      stream);
  if (rc) return rc;
  dim3 grid((H + 255) / 256, S);
  ep_combine_kernel<<<grid, 256, 0, st>>>(ws.y, ws.rhs, ww, partial, S, H, k);
  B2Q_TRY_CUDA(cudaGetLastError());
  return ep_finish(static_cast<EpComm*>(comm), partial, out, (size_t)S * H, st);
}

size_t b2q_ep_moe_prefill_workspace_size(int T, int H, int E, int F, int k) {
  if (T < 1 || H < 1 || E < 1 || F < 1 || k < 1) return 0;
  return ep_prefill_layout(nullptr, T, H, E, F, k).bytes;
}

int b2q_ep_moe_prefill(void* comm, const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg,
                       const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                       const uint32_t* wd, const uint16_t* sd, const uint16_t* bd, float* partial, uint16_t* out,
                       uint32_t* idx, float* w, int T, int H, int E, int F, int k, int e_lo, int e_local,
                       int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = ep_check_common("ep_moe_prefill", T, H, E, F, k, e_lo, e_local, group_size, bits);
  if (rc) return rc;
  if (T == 0) return B2Q_OK;
  if (!x || !wr || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !partial)
    return set_error(B2Q_EINVAL, "ep_moe_prefill: null pointer");
  if (!tc_shape_ok(F, H, group_size, TC_GLU) || !tc_shape_ok(H, F, group_size, TC_PLAIN))
    return set_error(B2Q_EUNSUPPORTED, "ep_moe_prefill: H %% 128, F %% 64 and K %% (8 * group_size) are required");
  const void* wptrs[] = {x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, partial};
  for (const void* q : wptrs)
    if (!aligned16(q)) return set_error(B2Q_EINVAL, "ep_moe_prefill: tensors must be 16-byte aligned");
  const EpPrefillWs ws = ep_prefill_layout(workspace, T, H, E, F, k);
  if (!workspace || workspace_bytes < ws.bytes || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "ep_moe_prefill: workspace of %zu bytes needed", ws.bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int R = T * k;
  uint32_t* ix = idx ? idx : ws.idx;
  float* ww = w ? w : ws.w;
  rc = eng::launch_router_logits(x, wr, ws.logits, T, E, H, st);
  if (rc) return rc;
  rc = eng::launch_route(ws.logits, ix, ww, T, E, k, st);
  if (rc) return rc;
  rc = launch_expert_sort(ix, ws.sorted_ids, ws.token_rows, ws.inverse, ws.offsets, R, E, k, ws.err, st);
  if (rc) return rc;
  // the local experts own the contiguous sorted rows [offsets[e_lo], offsets[e_lo + e_local])
  const uint32_t* loff = ws.offsets + e_lo;
  rc = tc_unit_tables(loff, e_local, tc_m_tiles(F, TC_GLU), tc_m_tiles(H, TC_PLAIN), ws.prefix_gu, ws.prefix_dn, st);
  if (rc) return rc;
  rc = tc_gather_rows_range(x, ws.token_rows, ws.xs, R, H, T, loff, e_local, st);
  if (rc) return rc;
  TcParams pg{};
  pg.E = e_local;
  pg.K = H;
  pg.Nw = F;
  pg.gs = group_size;
  pg.s0 = sg;
  pg.b0 = bg;
  pg.s1 = su;
  pg.b1 = bu;
  pg.offsets = loff;
  pg.prefix = ws.prefix_gu;
  pg.out = ws.act;
  pg.out_ld = F;
  pg.err = ws.err;
  pg.timeout_ns = 2000000000ll;
  rc = tc_setup(pg, TC_GLU, ws.xs, R, wg, wu);
  if (rc) return rc;
  rc = tc_launch(pg, TC_GLU, st);
  if (rc) return rc;
  TcParams pd{};
  pd.E = e_local;
  pd.K = F;
  pd.Nw = H;
  pd.gs = group_size;
  pd.s0 = sd;
  pd.b0 = bd;
  pd.offsets = loff;
  pd.prefix = ws.prefix_dn;
  pd.out = ws.y;
  pd.out_ld = H;
  pd.err = ws.err;
  pd.timeout_ns = 2000000000ll;
  rc = tc_setup(pd, TC_PLAIN, ws.act, R, wd, nullptr);
  if (rc) return rc;
  rc = tc_launch(pd, TC_PLAIN, st);
  if (rc) return rc;
  rc = launch_ep_sorted_combine(ws.y, ws.inverse, ww, ws.offsets, e_lo, e_local, partial, T, H, k, st);
  if (rc) return rc;
  return ep_finish(static_cast<EpComm*>(comm), partial, out, (size_t)T * H, st);
}

}  // extern "C"
