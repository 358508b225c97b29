// capi.cpp -- C-ABI plumbing of libb2q: per-thread error messages, version,
// device info, workspace helpers and the failure-path self test.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "host.hpp"

namespace b2q {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int device_info(DeviceInfo* out) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  B2Q_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(B2Q_ECUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].device != dev) {
    DeviceInfo d;
    d.device = dev;
    B2Q_TRY_CUDA(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
    B2Q_TRY_CUDA(cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    cache[dev] = d;
  }
  *out = cache[dev];
  return B2Q_OK;
}

}  // namespace b2q

extern "C" {

const char* b2q_last_error(void) { return b2q::g_last_error.c_str(); }

int b2q_version(void) { return 100; /* 0.1.0 */ }

int b2q_device_sm_count(void) {
  b2q::DeviceInfo d;
  int rc = b2q::device_info(&d);
  return rc ? rc : d.sm_count;
}

int b2q_workspace_reset(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes == 0) return b2q::set_error(B2Q_EINVAL, "workspace_reset: empty workspace");
  B2Q_TRY_CUDA(cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)));
  return B2Q_OK;
}

}  // extern "C"
