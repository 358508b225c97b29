// host.hpp -- host-side helpers shared by the C-ABI translation units:
// per-thread error message, CUDA error mapping, device properties cache.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/b2q.h"

namespace b2q {

// Sets the calling thread's message and returns `code` (mirrors mlx-c's
// status + error-handler convention, MLXCAPI/ops.cpp:1505-1508).
int set_error(int code, const char* fmt, ...);
void clear_error();

inline int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B2Q_OK;
  return set_error(B2Q_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// SM count and opt-in shared memory of the current device (cached per device).
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int smem_optin = 0;
};
int device_info(DeviceInfo* out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace b2q

#define B2Q_TRY_CUDA(expr)                                 \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return ::b2q::cuda_check(_e, #expr); \
  } while (0)
