// host_loop.cpp -- a caller's one-token decode loop through the C ABI, as a
// native host (the reference's Swift runner, a C++ server) would run it. It
// exists to measure the API path end to end: every step copies its token row
// in from pinned host memory, runs b2q_moe_decode, and copies the output row
// back. No counterpart in the reference.
//
// Copies run on a second stream with two device buffers per direction: step
// i + 1's input copy and step i's output copy overlap the kernels, the kernels
// follow one another on the caller's stream, and every step still moves its
// own input in and its own output out. The timed segment starts from an empty
// pipeline: its first input copy is inside the timed region.
#include <cuda_runtime.h>

#include "../../include/b2q.h"
#include "host.hpp"

using namespace b2q;

namespace {

struct Loop {
  const uint16_t* host_x;
  int n_tokens;
  uint16_t* host_out;
  const uint16_t* const* wr;
  const void* const* w9;
  int n_layers, H, E, F, k, gs, bits;
  uint16_t* dx2;
  uint16_t* dy2;
  void* ws;
  size_t ws_bytes;
  cudaStream_t cs;              // copy stream
  cudaEvent_t in_ready[2], kdone[2], out_free[2], join;
};

// Enqueues steps [first, first + count) on `st` (kernels) and the copy stream:
// step i reads token i % n_tokens and runs layer i % n_layers; the device
// buffers alternate with the step's place in this segment. The copy stream
// starts after what `st` holds, and `st` ends after the segment's last copy.
int enqueue_steps(Loop& L, cudaStream_t st, int first, int count) {
  int rc = B2Q_OK;
  auto cu = [&](cudaError_t e) {
    if (e != cudaSuccess && rc == B2Q_OK) rc = set_error(B2Q_ECUDA, "moe_decode_host_loop: %s", cudaGetErrorString(e));
    return rc == B2Q_OK;
  };
  const size_t row = (size_t)L.H * sizeof(uint16_t);
  (void)(cu(cudaEventRecord(L.kdone[0], st)) && cu(cudaStreamWaitEvent(L.cs, L.kdone[0], 0)) &&
         cu(cudaMemcpyAsync(L.dx2, L.host_x + (size_t)(first % L.n_tokens) * L.H, row, cudaMemcpyHostToDevice,
                            L.cs)) &&
         cu(cudaEventRecord(L.in_ready[0], L.cs)));
  for (int j = 0; j < count && rc == B2Q_OK; ++j) {
    const int i = first + j, s = j & 1, n = (j + 1) & 1, l = i % L.n_layers;
    // next step's input, once the kernel that last read that buffer is done
    if (j + 1 < count) {
      if (j >= 1) cu(cudaStreamWaitEvent(L.cs, L.kdone[n], 0));
      cu(cudaMemcpyAsync(L.dx2 + (size_t)n * L.H, L.host_x + (size_t)((i + 1) % L.n_tokens) * L.H, row,
                         cudaMemcpyHostToDevice, L.cs));
      cu(cudaEventRecord(L.in_ready[n], L.cs));
    }
    // this step: its input landed, and the output buffer's previous copy out is done
    cu(cudaStreamWaitEvent(st, L.in_ready[s], 0));
    if (j >= 2) cu(cudaStreamWaitEvent(st, L.out_free[s], 0));
    if (rc != B2Q_OK) break;
    const void* const* w = L.w9 + 9 * (size_t)l;
    const int r = b2q_moe_decode(L.dx2 + (size_t)s * L.H, L.wr[l], static_cast<const uint32_t*>(w[0]),
                                 static_cast<const uint16_t*>(w[1]), static_cast<const uint16_t*>(w[2]),
                                 static_cast<const uint32_t*>(w[3]), static_cast<const uint16_t*>(w[4]),
                                 static_cast<const uint16_t*>(w[5]), static_cast<const uint32_t*>(w[6]),
                                 static_cast<const uint16_t*>(w[7]), static_cast<const uint16_t*>(w[8]),
                                 L.dy2 + (size_t)s * L.H, nullptr, nullptr, nullptr, 1, L.H, L.E, L.F, L.k, L.gs,
                                 L.bits, L.ws, L.ws_bytes, st);
    if (r != B2Q_OK) return r;
    cu(cudaEventRecord(L.kdone[s], st));
    // this step's output back to the host
    cu(cudaStreamWaitEvent(L.cs, L.kdone[s], 0));
    cu(cudaMemcpyAsync(L.host_out, L.dy2 + (size_t)s * L.H, row, cudaMemcpyDeviceToHost, L.cs));
    cu(cudaEventRecord(L.out_free[s], L.cs));
  }
  if (rc == B2Q_OK) (void)(cu(cudaEventRecord(L.join, L.cs)) && cu(cudaStreamWaitEvent(st, L.join, 0)));
  return rc;
}

int host_loop(const uint16_t* host_x, int n_tokens, uint16_t* host_out, const uint16_t* const* wr,
              const void* const* w9, int n_layers, int H, int E, int F, int k, int group_size, int bits,
              uint16_t* dev_x2, uint16_t* dev_out2, void* workspace, size_t workspace_bytes, int warmup, int steps,
              void* stream, float* ms_per_step) {
  if (!host_x || !host_out || !wr || !w9 || !dev_x2 || !dev_out2 || !ms_per_step || n_tokens <= 0 ||
      n_layers <= 0 || warmup < 0 || steps <= 0 || H <= 0)
    return set_error(B2Q_EINVAL, "moe_decode_host_loop: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Loop L{host_x, n_tokens, host_out, wr, w9, n_layers, H, E, F, k, group_size, bits, dev_x2, dev_out2, workspace,
         workspace_bytes, nullptr, {}, {}, {}, nullptr};
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  int rc = B2Q_OK;
  auto cu = [&](cudaError_t e) {
    if (e != cudaSuccess && rc == B2Q_OK) rc = set_error(B2Q_ECUDA, "moe_decode_host_loop: %s", cudaGetErrorString(e));
    return rc == B2Q_OK;
  };
  cu(cudaStreamCreateWithFlags(&L.cs, cudaStreamNonBlocking));
  cudaEvent_t* evs[7] = {&L.in_ready[0], &L.in_ready[1], &L.kdone[0], &L.kdone[1], &L.out_free[0], &L.out_free[1],
                         &L.join};
  for (cudaEvent_t* e : evs)
    if (rc == B2Q_OK) cu(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  if (rc == B2Q_OK) cu(cudaEventCreate(&t0));
  if (rc == B2Q_OK) cu(cudaEventCreate(&t1));
  if (rc == B2Q_OK && warmup > 0) rc = enqueue_steps(L, st, 0, warmup);
  if (rc == B2Q_OK) {
    cu(cudaEventRecord(t0, st));
    if (rc == B2Q_OK) rc = enqueue_steps(L, st, warmup, steps);
    if (rc == B2Q_OK) cu(cudaEventRecord(t1, st));
  }
  if (rc == B2Q_OK) cu(cudaEventSynchronize(t1));
  float ms = 0.0f;
  if (rc == B2Q_OK && cu(cudaEventElapsedTime(&ms, t0, t1))) *ms_per_step = ms / (float)steps;
  // nothing of the loop is left in flight when it returns
  cudaStreamSynchronize(st);
  if (L.cs) {
    cudaStreamSynchronize(L.cs);
    cudaStreamDestroy(L.cs);
  }
  for (cudaEvent_t* e : evs)
    if (*e) cudaEventDestroy(*e);
  if (t0) cudaEventDestroy(t0);
  if (t1) cudaEventDestroy(t1);
  return rc;
}

}  // namespace

extern "C" {

B2Q_API int b2q_moe_decode_host_loop(const uint16_t* host_x, int n_tokens, uint16_t* host_out,
                                     const uint16_t* const* wr, const void* const* w9, int n_layers, int H, int E,
                                     int F, int k, int group_size, int bits, uint16_t* dev_x2, uint16_t* dev_out2,
                                     void* workspace, size_t workspace_bytes, int warmup, int steps, void* stream,
                                     float* ms_per_step) {
  return host_loop(host_x, n_tokens, host_out, wr, w9, n_layers, H, E, F, k, group_size, bits, dev_x2, dev_out2,
                   workspace, workspace_bytes, warmup, steps, stream, ms_per_step);
}

}  // extern "C"
