// host_loop.cpp -- a caller's one-token decode loop through the C ABI, as a
// native host (the reference's Swift runner, a C++ server) would run it. It
// exists to measure the API path end to end: every step copies its token row
// in from pinned host memory, runs b2q_moe_decode, and copies the output row
// back. No counterpart in the reference.
//
// Copies run on a second stream with two device buffers per direction: step
// i + 1's input copy and step i's output copy overlap the kernels, the kernels
// follow one another on the caller's stream, and every step still moves its
// own input in and its own output out.
#include <cuda_runtime.h>

#include "../../include/b2q.h"
#include "host.hpp"

using namespace b2q;

extern "C" B2Q_API int b2q_moe_decode_host_loop(const uint16_t* host_x, int n_tokens, uint16_t* host_out,
                                                const uint16_t* const* wr, const void* const* w9, int n_layers,
                                                int H, int E, int F, int k, int group_size, int bits,
                                                uint16_t* dev_x2, uint16_t* dev_out2, void* workspace,
                                                size_t workspace_bytes, int warmup, int steps, void* stream,
                                                float* ms_per_step) {
  if (!host_x || !host_out || !wr || !w9 || !dev_x2 || !dev_out2 || !ms_per_step || n_tokens <= 0 ||
      n_layers <= 0 || warmup < 0 || steps <= 0 || H <= 0)
    return set_error(B2Q_EINVAL, "moe_decode_host_loop: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStream_t cs = nullptr;
  cudaEvent_t ev[8] = {};  // in_ready[2], kdone[2], out_free[2], t0, t1
  int rc = B2Q_OK;
  auto cu = [&](cudaError_t e) {
    if (e != cudaSuccess && rc == B2Q_OK) rc = set_error(B2Q_ECUDA, "moe_decode_host_loop: %s", cudaGetErrorString(e));
    return e == cudaSuccess;
  };
  cu(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
  for (int i = 0; i < 6 && rc == B2Q_OK; ++i) cu(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
  if (rc == B2Q_OK) cu(cudaEventCreate(&ev[6]));
  if (rc == B2Q_OK) cu(cudaEventCreate(&ev[7]));
  cudaEvent_t* in_ready = ev;
  cudaEvent_t* kdone = ev + 2;
  cudaEvent_t* out_free = ev + 4;
  const size_t row = (size_t)H * sizeof(uint16_t);
  const int total = warmup + steps;
  // the copy stream starts after what the caller queued on its stream
  if (rc == B2Q_OK && cu(cudaEventRecord(kdone[0], st))) cu(cudaStreamWaitEvent(cs, kdone[0], 0));
  if (rc == B2Q_OK) cu(cudaMemcpyAsync(dev_x2, host_x, row, cudaMemcpyHostToDevice, cs));
  if (rc == B2Q_OK) cu(cudaEventRecord(in_ready[0], cs));
  for (int i = 0; i < total && rc == B2Q_OK; ++i) {
    const int s = i & 1, n = (i + 1) & 1, l = i % n_layers;
    if (i == warmup) cu(cudaEventRecord(ev[6], st));
    // next step's input, once the kernel that last read that buffer is done
    if (i + 1 < total) {
      if (i >= 1) cu(cudaStreamWaitEvent(cs, kdone[n], 0));
      cu(cudaMemcpyAsync(dev_x2 + (size_t)n * H, host_x + (size_t)((i + 1) % n_tokens) * H, row,
                         cudaMemcpyHostToDevice, cs));
      cu(cudaEventRecord(in_ready[n], cs));
    }
    // this step: its input landed, and the output buffer's previous copy out is done
    cu(cudaStreamWaitEvent(st, in_ready[s], 0));
    if (i >= 2) cu(cudaStreamWaitEvent(st, out_free[s], 0));
    if (rc != B2Q_OK) break;
    const void* const* w = w9 + 9 * (size_t)l;
    const int r = b2q_moe_decode(dev_x2 + (size_t)s * H, wr[l], static_cast<const uint32_t*>(w[0]),
                                 static_cast<const uint16_t*>(w[1]), static_cast<const uint16_t*>(w[2]),
                                 static_cast<const uint32_t*>(w[3]), static_cast<const uint16_t*>(w[4]),
                                 static_cast<const uint16_t*>(w[5]), static_cast<const uint32_t*>(w[6]),
                                 static_cast<const uint16_t*>(w[7]), static_cast<const uint16_t*>(w[8]),
                                 dev_out2 + (size_t)s * H, nullptr, nullptr, nullptr, 1, H, E, F, k, group_size, bits,
                                 workspace, workspace_bytes, stream);
    if (r != B2Q_OK) {
      rc = r;
      break;
    }
    cu(cudaEventRecord(kdone[s], st));
    // this step's output back to the host
    cu(cudaStreamWaitEvent(cs, kdone[s], 0));
    cu(cudaMemcpyAsync(host_out, dev_out2 + (size_t)s * H, row, cudaMemcpyDeviceToHost, cs));
    cu(cudaEventRecord(out_free[s], cs));
  }
  if (rc == B2Q_OK) cu(cudaEventRecord(ev[7], cs));
  if (rc == B2Q_OK) cu(cudaEventSynchronize(ev[7]));
  float ms = 0.0f;
  if (rc == B2Q_OK && cu(cudaEventElapsedTime(&ms, ev[6], ev[7]))) *ms_per_step = ms / (float)steps;
  // the caller's stream continues after the loop's last copy
  if (cs) {
    cudaStreamSynchronize(cs);
    cudaStreamDestroy(cs);
  }
  for (cudaEvent_t e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}
