// api_decode.cu -- extern "C" entry points for packing, the products and the
// decode MoE operators (argument checks, routing policy, workspace layout).
//
// Routing policy mirrors QuantizedMatmul::eval_gpu / GatherQMM::eval_gpu
// (Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/metal/quantized.cpp:1982-2205):
// few rows per weight matrix -> the streaming qmv engine, many rows -> the
// tensor-core qmm kernel; shapes outside a kernel's fast path take the
// shape-general kernel instead of failing.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "decode2.cuh"
#include "decode_ws.hpp"
#include "engine.cuh"
#include "host.hpp"
#include "misc.cuh"
#include "prefill.cuh"

using namespace b2q;

extern "C" {

int b2q_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, uint16_t* out, int64_t rows,
                   int K, int group_size, int bits, void* stream) {
  clear_error();
  int rc = check_bits_gs("dequantize", bits, group_size);
  if (rc) return rc;
  if (rows < 0 || K <= 0 || K % group_size || K % 8) return set_error(B2Q_EINVAL, "dequantize: bad shape");
  if (rows == 0) return B2Q_OK;
  if (!w || !scales || !biases || !out) return set_error(B2Q_EINVAL, "dequantize: null pointer");
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(w) & 3))
    return set_error(B2Q_EINVAL, "dequantize: out must be 16-byte and w 4-byte aligned");
  return launch_dequantize(w, scales, biases, out, rows, K, group_size, static_cast<cudaStream_t>(stream));
}

int b2q_quantize(const uint16_t* w, uint32_t* w_q, uint16_t* scales, uint16_t* biases, int64_t rows, int K,
                 int group_size, int bits, void* stream) {
  clear_error();
  int rc = check_bits_gs("quantize", bits, group_size);
  if (rc) return rc;
  if (rows < 0 || K <= 0 || K % group_size) return set_error(B2Q_EINVAL, "quantize: bad shape");
  if (rows == 0) return B2Q_OK;
  if (!w || !w_q || !scales || !biases) return set_error(B2Q_EINVAL, "quantize: null pointer");
  return launch_quantize(w, w_q, scales, biases, rows, K, group_size, static_cast<cudaStream_t>(stream));
}

static int gather_impl(const char* fn, const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                       const uint32_t* lhs, const uint32_t* rhs, uint16_t* y, int batch, int M, int N, int K,
                       int n_x, int n_w, int gs, int bits, int transpose, int sorted, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = check_bits_gs(fn, bits, gs);
  if (rc) return rc;
  if (!transpose) return set_error(B2Q_EUNSUPPORTED, "%s: transpose=false is not implemented", fn);
  if (batch < 0 || M < 0 || N < 0 || K <= 0 || K % gs || K % 8 || n_x < 0 || n_w < 0)
    return set_error(B2Q_EINVAL, "%s: bad shape", fn);
  if (batch == 0 || M == 0 || N == 0) return B2Q_OK;
  if (!x || !w || !s || !b || !y) return set_error(B2Q_EINVAL, "%s: null pointer", fn);
  if (!aligned16(x)) return set_error(B2Q_EINVAL, "%s: x must be 16-byte aligned", fn);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // one row of x times one weight matrix: the single-column streaming kernel
  if (M == 1 && batch == 1 && !lhs && !rhs && n_x >= 1 && n_w >= 1 && aligned16(y)) {
    if (d2_qmv_eligible(N, K, gs, x, w, s, b)) return d2_qmv(x, w, s, b, y, N, K, gs, st);
  }
  const bool engine_ok = M <= eng::MAX_COLS && engine_k_ok(K, gs) && aligned16(w) && aligned16(s) &&
                         aligned16(b);
  if (engine_ok) {
    eng::Params p;
    base_params(p, eng::MODE_QMV, gs);
    p.x = x;
    p.lhs = lhs;
    p.rhs = rhs;
    p.y = y;
    p.batch = batch;
    p.M = M;
    p.N = N;
    p.n_x = n_x;
    p.n_w = n_w;
    p.g1.K = K;
    rc = eng::plan(p);
    if (rc == B2Q_OK) rc = eng::set_maps_qmv(p, w, s, b);
    if (rc == B2Q_OK) return eng::launch(p, stream, false);
    if (rc != B2Q_EUNSUPPORTED) return rc;
  }
  if (M > eng::MAX_COLS && prefill_qmm_eligible(batch, M, N, K, gs, x, w, s, b, y)) {
    return launch_prefill_gather_qmm(x, w, s, b, lhs, rhs, y, batch, M, N, K, n_x, n_w, gs, sorted, workspace,
                                     workspace_bytes, st);
  }
  GenericArgs a{x, w, s, b, lhs, rhs, y, batch, M, N, K, n_x, n_w, gs};
  return launch_generic_qmv(a, st);
}

int b2q_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* scales, const uint16_t* biases, uint16_t* y, int M,
            int N, int K, int group_size, int bits, int transpose, void* stream) {
  clear_error();
  return gather_impl("quantized_matmul", x, w, scales, biases, nullptr, nullptr, y, 1, M, N, K, 1, 1, group_size,
                     bits, transpose, 0, nullptr, 0, stream);
}

int b2q_gather_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   const uint32_t* lhs_indices, const uint32_t* rhs_indices, uint16_t* y, int batch, int M, int N,
                   int K, int n_x, int n_w, int group_size, int bits, int transpose, int sorted_indices,
                   void* stream) {
  clear_error();
  return gather_impl("gather_qmm", x, w, scales, biases, lhs_indices, rhs_indices, y, batch, M, N, K, n_x, n_w,
                     group_size, bits, transpose, sorted_indices, nullptr, 0, stream);
}

size_t b2q_gather_qmm_workspace_size(int batch, int M, int N, int K, int n_w) {
  (void)N;
  if (M <= eng::MAX_COLS) return 256;  // the streaming kernels take no workspace
  return prefill_gather_qmm_ws_bytes(batch, M, K, n_w);
}

int b2q_qmm_ws(const uint16_t* x, const uint32_t* w, const uint16_t* scales, const uint16_t* biases, uint16_t* y,
               int M, int N, int K, int group_size, int bits, int transpose, void* workspace,
               size_t workspace_bytes, void* stream) {
  clear_error();
  if (!workspace) return set_error(B2Q_EINVAL, "quantized_matmul_ws: null workspace");
  return gather_impl("quantized_matmul_ws", x, w, scales, biases, nullptr, nullptr, y, 1, M, N, K, 1, 1,
                     group_size, bits, transpose, 0, workspace, workspace_bytes, stream);
}

int b2q_gather_qmm_ws(const uint16_t* x, const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                      const uint32_t* lhs_indices, const uint32_t* rhs_indices, uint16_t* y, int batch, int M, int N,
                      int K, int n_x, int n_w, int group_size, int bits, int transpose, int sorted_indices,
                      void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!workspace) return set_error(B2Q_EINVAL, "gather_qmm_ws: null workspace");
  return gather_impl("gather_qmm_ws", x, w, scales, biases, lhs_indices, rhs_indices, y, batch, M, N, K, n_x, n_w,
                     group_size, bits, transpose, sorted_indices, workspace, workspace_bytes, stream);
}

int b2q_moe_router_logits(const uint16_t* x, const uint16_t* wr, float* logits, int T, int E, int H, void* stream) {
  clear_error();
  if (T < 0 || E <= 0 || H <= 0 || H % 8) return set_error(B2Q_EINVAL, "router_logits: bad shape");
  if (T == 0) return B2Q_OK;
  if (!x || !wr || !logits || !aligned16(x) || !aligned16(wr))
    return set_error(B2Q_EINVAL, "router_logits: null or unaligned pointer");
  return eng::launch_router_logits(x, wr, logits, T, E, H, static_cast<cudaStream_t>(stream));
}

int b2q_moe_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k, void* stream) {
  clear_error();
  if (T < 0 || E <= 0 || E > 1024 || k < 1 || k > 32 || k > E) return set_error(B2Q_EINVAL, "route: bad shape");
  if (T == 0) return B2Q_OK;
  if (!logits || !idx || !w) return set_error(B2Q_EINVAL, "route: null pointer");
  return eng::launch_route(logits, idx, w, T, E, k, static_cast<cudaStream_t>(stream));
}

static int gate_up_impl(const uint16_t* x, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                        const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* idx,
                        const uint32_t* xrow, int tok_div, uint16_t* act, int n_slots, int S, int H, int E, int F,
                        int gs, int bits, void* stream) {
  int rc = check_bits_gs("moe_gate_up_act", bits, gs);
  if (rc) return rc;
  if (n_slots < 0 || S < 1 || S > eng::MAX_COLS || E < 1 || F <= 0 || F % 8 || !engine_k_ok(H, gs))
    return set_error(B2Q_EUNSUPPORTED, "moe_gate_up_act: shape outside the kernel (S<=8, F%%8==0, H%%(8*gs)==0)");
  if (n_slots == 0) return B2Q_OK;
  if (!x || !wg || !sg || !bg || !wu || !su || !bu || !idx || !act) return set_error(B2Q_EINVAL, "moe_gate_up_act: null pointer");
  if (!aligned16(x) || !aligned16(wg) || !aligned16(wu) || !aligned16(sg) || !aligned16(bg) || !aligned16(su) ||
      !aligned16(bu))
    return set_error(B2Q_EINVAL, "moe_gate_up_act: tensors must be 16-byte aligned");
  eng::Params p;
  base_params(p, eng::MODE_GU, gs);
  p.x = x;
  p.idx_in = idx;
  p.xrow_in = xrow;
  p.k = tok_div;
  p.act_out = act;
  p.n_slots = n_slots;
  p.S = S;
  p.H = H;
  p.E = E;
  p.F = F;
  rc = eng::plan(p);
  if (rc) return rc;
  rc = eng::set_maps_gu(p, wg, sg, bg, wu, su, bu);
  if (rc) return rc;
  return eng::launch(p, stream, false);
}

int b2q_moe_gate_up_act(const uint16_t* x, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                        const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* idx,
                        const uint32_t* xrow, uint16_t* act, int n_slots, int S, int H, int E, int F, int group_size,
                        int bits, void* stream) {
  clear_error();
  return gate_up_impl(x, wg, sg, bg, wu, su, bu, idx, xrow, 0, act, n_slots, S, H, E, F, group_size, bits, stream);
}

int b2q_moe_down_combine(const uint16_t* act, const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                         const uint32_t* idx, const float* w, uint16_t* out, int S, int H, int E, int F, int k,
                         int group_size, int bits, void* stream) {
  clear_error();
  int rc = check_bits_gs("moe_down_combine", bits, group_size);
  if (rc) return rc;
  if (S < 0 || k < 1 || k > eng::MAX_COLS || E < 1 || H <= 0 || H % 8 || !engine_k_ok(F, group_size))
    return set_error(B2Q_EUNSUPPORTED, "moe_down_combine: shape outside the kernel (k<=8, H%%8==0, F%%(8*gs)==0)");
  if (S == 0) return B2Q_OK;
  if (!act || !wd || !sd || !bd || !idx || !w || !out) return set_error(B2Q_EINVAL, "moe_down_combine: null pointer");
  if (!aligned16(act) || !aligned16(wd) || !aligned16(sd) || !aligned16(bd))
    return set_error(B2Q_EINVAL, "moe_down_combine: tensors must be 16-byte aligned");
  eng::Params p;
  base_params(p, eng::MODE_DOWN, group_size);
  p.act_in = act;
  p.idx_in = idx;
  p.w_in = w;
  p.out = out;
  p.S = S;
  p.H = H;
  p.E = E;
  p.F = F;
  p.k = k;
  rc = eng::plan(p);
  if (rc) return rc;
  rc = eng::set_maps_down(p, wd, sd, bd);
  if (rc) return rc;
  return eng::launch(p, stream, false);
}

size_t b2q_moe_decode_workspace_size(int S, int H, int E, int F, int k) {
  (void)H;
  if (S < 1 || E < 1 || F < 1 || k < 1) return 0;
  return decode_ws_layout(nullptr, S, H, E, F, k).bytes;
}

int b2q_moe_decode(const uint16_t* x, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd, const uint16_t* sd,
                   const uint16_t* bd, uint16_t* out, uint32_t* idx, float* w, float* logits, int S, int H, int E,
                   int F, int k, int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = check_bits_gs("moe_decode", bits, group_size);
  if (rc) return rc;
  if (S < 1 || S > eng::MAX_COLS || k < 1 || k > eng::MAX_COLS || E < k || E > 1024 || F % 8 || H % 8 ||
      !engine_k_ok(H, group_size) || !engine_k_ok(F, group_size))
    return set_error(B2Q_EUNSUPPORTED,
                     "moe_decode: shape outside the kernel (S<=8, k<=8, E<=1024, H,F multiples of 8*group_size)");
  if (!x || !wr || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !out)
    return set_error(B2Q_EINVAL, "moe_decode: null pointer");
  const DecodeWs ws = decode_ws_layout(workspace, S, H, E, F, k);
  if (!workspace || workspace_bytes < ws.bytes || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "moe_decode: workspace of %zu bytes needed", ws.bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const void* ptrs[] = {x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd};
  bool all_aligned = true;
  for (const void* q : ptrs) all_aligned = all_aligned && aligned16(q);
  if (S == 1 && all_aligned && d2_moe_eligible(H, E, F, k, group_size)) {
    const D2Scratch scr{&ws.hdr->error, ws.ctr, ws.logits, ws.act, ws.asc};
    return d2_moe_decode(x, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, out, idx, w, logits, H, E, F, k, group_size, scr,
                         st);
  }
  if (S == 1) {
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
    p.err = &ws.hdr->error;
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
  // S > 1: the four operators in sequence
  float* lg = logits ? logits : ws.logits;
  uint32_t* ix = idx ? idx : ws.idx;
  float* ww = w ? w : ws.w;
  rc = eng::launch_router_logits(x, wr, lg, S, E, H, st);
  if (rc) return rc;
  rc = eng::launch_route(lg, ix, ww, S, E, k, st);
  if (rc) return rc;
  rc = gate_up_impl(x, wg, sg, bg, wu, su, bu, ix, nullptr, k, ws.act, S * k, S, H, E, F, group_size, bits, stream);
  if (rc) return rc;
  return b2q_moe_down_combine(ws.act, wd, sd, bd, ix, ww, out, S, H, E, F, k, group_size, bits, stream);
}

// ---- the residual add + RMSNorm fused into the one-token products ----------
static int norm_args_ok(const char* fn, const uint16_t* h, const uint16_t* delta, const uint16_t* nw, float eps,
                        const uint16_t* h_out, int K) {
  if (!h || !nw) return set_error(B2Q_EINVAL, "%s: null pointer", fn);
  if (delta && !h_out) return set_error(B2Q_EINVAL, "%s: h_out is needed with delta", fn);
  if (delta && (h_out == h || h_out == delta))
    return set_error(B2Q_EINVAL, "%s: h_out must not alias h or delta (every CTA reads them)", fn);
  if (!(eps >= 0.0f)) return set_error(B2Q_EINVAL, "%s: eps", fn);
  if (!aligned16(h) || !aligned16(nw) || (delta && (!aligned16(delta) || !aligned16(h_out))))
    return set_error(B2Q_EINVAL, "%s: h, delta, h_out and the norm weight must be 16-byte aligned", fn);
  if (!d2_norm_ok(K)) return set_error(B2Q_EUNSUPPORTED, "%s: K=%d outside the fused norm", fn, K);
  return B2Q_OK;
}

int b2q_qmv_norm(const uint16_t* h, const uint16_t* delta, const uint16_t* norm_weight, float eps, uint16_t* h_out,
                 const uint32_t* w, const uint16_t* scales, const uint16_t* biases, uint16_t* y, int N, int K,
                 int group_size, int bits, void* stream) {
  clear_error();
  int rc = check_bits_gs("qmv_norm", bits, group_size);
  if (rc) return rc;
  if (N <= 0 || K <= 0 || K % group_size) return set_error(B2Q_EINVAL, "qmv_norm: bad shape");
  rc = norm_args_ok("qmv_norm", h, delta, norm_weight, eps, h_out, K);
  if (rc) return rc;
  if (!w || !scales || !biases || !y) return set_error(B2Q_EINVAL, "qmv_norm: null pointer");
  if (!aligned16(y) || !d2_qmv_eligible(N, K, group_size, h, w, scales, biases))
    return set_error(B2Q_EUNSUPPORTED, "qmv_norm: shape outside the single-column kernel");
  D2Norm nm;
  nm.weight = norm_weight;
  nm.delta = delta;
  nm.h_out = h_out;
  nm.eps = eps;
  return d2_qmv(h, w, scales, biases, y, N, K, group_size, static_cast<cudaStream_t>(stream), nm);
}

int b2q_moe_decode_norm(const uint16_t* h, const uint16_t* delta, const uint16_t* norm_weight, float eps,
                        uint16_t* h_out, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                        const uint32_t* wu, const uint16_t* su, const uint16_t* bu, const uint32_t* wd,
                        const uint16_t* sd, const uint16_t* bd, uint16_t* out, uint32_t* idx, float* w, float* logits,
                        int H, int E, int F, int k, int group_size, int bits, void* workspace, size_t workspace_bytes,
                        void* stream) {
  clear_error();
  int rc = check_bits_gs("moe_decode_norm", bits, group_size);
  if (rc) return rc;
  rc = norm_args_ok("moe_decode_norm", h, delta, norm_weight, eps, h_out, H);
  if (rc) return rc;
  if (!wr || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !out)
    return set_error(B2Q_EINVAL, "moe_decode_norm: null pointer");
  const void* ptrs[] = {wr, wg, sg, bg, wu, su, bu, wd, sd, bd};
  bool all_aligned = true;
  for (const void* q : ptrs) all_aligned = all_aligned && aligned16(q);
  if (!all_aligned || k < 1 || E < k || !d2_moe_eligible(H, E, F, k, group_size))
    return set_error(B2Q_EUNSUPPORTED, "moe_decode_norm: shape outside the single-column kernel");
  const DecodeWs ws = decode_ws_layout(workspace, 1, H, E, F, k);
  if (!workspace || workspace_bytes < ws.bytes || !aligned16(workspace))
    return set_error(B2Q_EINVAL, "moe_decode_norm: workspace of %zu bytes needed", ws.bytes);
  const D2Scratch scr{&ws.hdr->error, ws.ctr, ws.logits, ws.act, ws.asc};
  D2Norm nm;
  nm.weight = norm_weight;
  nm.delta = delta;
  nm.h_out = h_out;
  nm.eps = eps;
  return d2_moe_decode(h, wr, wg, sg, bg, wu, su, bu, wd, sd, bd, out, idx, w, logits, H, E, F, k, group_size, scr,
                       static_cast<cudaStream_t>(stream), 0, 0, nullptr, nm);
}

int b2q_workspace_status(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < sizeof(WsHeader)) return set_error(B2Q_EINVAL, "workspace_status: no workspace");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int code = 0;
  B2Q_TRY_CUDA(cudaMemcpyAsync(&code, workspace, sizeof(int), cudaMemcpyDeviceToHost, st));
  B2Q_TRY_CUDA(cudaStreamSynchronize(st));
  if (code != 0) {
    B2Q_TRY_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), st));
    B2Q_TRY_CUDA(cudaStreamSynchronize(st));
    return set_error(code, "a kernel recorded device-side error %d", code);
  }
  return B2Q_OK;
}

}  // extern "C"

namespace b2q {
// Waits on a flag nothing sets, bounded by timeout_ns, then records the timeout.
__global__ void selftest_wait_kernel(WsHeader* h, long long timeout_ns) {
  if (threadIdx.x != 0) return;
  const uint64_t deadline = globaltimer() + (uint64_t)timeout_ns;
  if (!wait_counter_geq(&h->flag, 1u, deadline, nullptr)) record_error(&h->error, B2Q_ETIMEOUT);
}
}  // namespace b2q

extern "C" int b2q_selftest_wait_timeout(void* workspace, size_t workspace_bytes, long long timeout_ns, void* stream) {
  clear_error();
  if (!workspace || workspace_bytes < sizeof(WsHeader)) return set_error(B2Q_EINVAL, "selftest: no workspace");
  if (timeout_ns <= 0 || timeout_ns > 10000000000ll) return set_error(B2Q_EINVAL, "selftest: timeout out of range");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  selftest_wait_kernel<<<1, 32, 0, st>>>(static_cast<WsHeader*>(workspace), timeout_ns);
  B2Q_TRY_CUDA(cudaGetLastError());
  return b2q_workspace_status(workspace, workspace_bytes, stream);
}
