// noalloc.cu -- the one-token fused MoE decode without a caller workspace.
//
// Some callers cannot allocate device memory at the point where they decode:
// a host whose device memory is owned by another allocator (a framework's
// caching allocator or a fixed arena, so a raw cudaMalloc fails or fragments
// it), a plugin that is handed only input and output buffers, or code that
// must not make allocating CUDA calls while it runs. b2q_moe_decode needs a
// workspace for its router logits, selected experts, SwiGLU activations and
// grid counters; this form takes that scratch from one file-scope device array
// instead, so the call allocates nothing.
//
// Costs and rules of the shared array:
//  * every GPU that loads the library holds B2Q_NOALLOC_SCRATCH_BYTES of it
//    until the process exits;
//  * the first call on a device looks up the array's address there
//    (cudaGetSymbolAddress); make that first call before any stream capture
//    on that device;
//  * all calls on a device share the array and it keeps the last call's
//    contents; each call clears what must start at zero (the error word and
//    the grid counters) with an asynchronous memset on its own stream before
//    the kernel, so calls in stream order are independent, but calls whose
//    kernels overlap on the GPU (two streams, two threads) race on the
//    counters and the activations and give wrong results.
// The kernel is the one b2q_moe_decode runs for the same shape (the
// single-column fused kernel where its shape rules hold, else the streaming
// engine's fused mode).
#include <cuda_runtime.h>

#include <mutex>

#include "decode2.cuh"
#include "decode_ws.hpp"
#include "engine.cuh"
#include "host.hpp"

static_assert(B2Q_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size is a multiple of 256 bytes");

// The scratch of every call on a device (header, logits, experts, weights,
// activations in the decode workspace layout).
static __device__ __align__(256) unsigned char g_decode_scratch[B2Q_NOALLOC_SCRATCH_BYTES];

namespace b2q {
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Address of the scratch array on the current device; the first request per
// device resolves it.
int scratch_on_current_device(void** out) {
  int dev = -1;
  B2Q_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(B2Q_EUNSUPPORTED, "moe_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess || !ptr)
      return set_error(B2Q_ECUDA, "moe_decode_noalloc: cudaGetSymbolAddress of the scratch array: %s",
                       cudaGetErrorString(e));
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return B2Q_OK;
}

}  // namespace
}  // namespace b2q

using namespace b2q;

extern "C" int b2q_moe_decode_noalloc(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg,
                                      const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                                      const uint32_t* wd, const uint16_t* sd, const uint16_t* bd, uint16_t* out,
                                      uint32_t* idx, float* w, float* logits, int H, int E, int F, int k,
                                      int group_size, int bits, int* status, void* stream) {
  clear_error();
  int rc = check_bits_gs("moe_decode_noalloc", bits, group_size);
  if (rc) return rc;
  if (k < 1 || k > eng::MAX_COLS || E < k || E > 1024 || F % 8 || H % 8 || !engine_k_ok(H, group_size) ||
      !engine_k_ok(F, group_size))
    return set_error(B2Q_EUNSUPPORTED,
                     "moe_decode_noalloc: shape outside the kernel (k<=8, E<=1024, H,F multiples of 8*group_size)");
  const size_t need = decode_ws_layout(nullptr, 1, H, E, F, k).bytes;
  if (need > (size_t)B2Q_NOALLOC_SCRATCH_BYTES)
    return set_error(B2Q_EINVAL,
                     "moe_decode_noalloc: E=%d, k=%d, F=%d need %zu bytes of scratch, above the fixed %d "
                     "(use b2q_moe_decode with a workspace)",
                     E, k, F, need, B2Q_NOALLOC_SCRATCH_BYTES);
  if (!x || !wr || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !out)
    return set_error(B2Q_EINVAL, "moe_decode_noalloc: null pointer");
  void* scratch = nullptr;
  rc = scratch_on_current_device(&scratch);
  if (rc) return rc;
  const DecodeWs ws = decode_ws_layout(scratch, 1, H, E, F, k);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // what must start at zero: the error word and the grid counters (header and
  // the counter block that follows it)
  B2Q_TRY_CUDA(cudaMemsetAsync(ws.hdr, 0, sizeof(WsHeader) + D2_CTR_BYTES, st));
  if (status) B2Q_TRY_CUDA(cudaMemsetAsync(status, 0, sizeof(int), st));
  const void* ptrs[] = {x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd};
  bool all_aligned = true;
  for (const void* q : ptrs) all_aligned = all_aligned && aligned16(q);
  if (all_aligned && d2_moe_eligible(H, E, F, k, group_size)) {
    const D2Scratch scr{status ? status : &ws.hdr->error, ws.ctr, ws.logits, ws.act, ws.asc};
    return d2_moe_decode(x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, out, idx, w, logits, H, E, F, k, group_size, scr,
                         st);
  }
  eng::Params p;
  base_params(p, eng::MODE_FUSED, group_size);
  p.x = x;
  p.wr = wr;
  p.out = out;
  p.idx_out = idx;
  p.w_out = w;
  p.logits_out = logits;
  p.S = 1;
  p.H = H;
  p.E = E;
  p.F = F;
  p.k = k;
  p.n_slots = k;
  p.err = status ? status : &ws.hdr->error;
  p.counters = ws.hdr->counters;
  p.ws_logits = ws.logits;
  p.ws_act = ws.act;
  rc = eng::plan(p);
  if (rc) return rc;
  rc = eng::set_maps_gu(p, wg, sg, bg, wu, su, bu);
  if (rc) return rc;
  rc = eng::set_maps_down(p, wd, sd, bd);
  if (rc) return rc;
  return eng::launch(p, stream, true);
}
