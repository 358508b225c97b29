// common.cuh -- shared device helpers for the sm_100a kernels of libb2q.
//
// bf16 rounding, the nibble -> bf16 pair decode used by every product kernel,
// inline-PTX wrappers for mbarriers, 1-D bulk (TMA) copies, the legacy
// m16n8k16 bf16 MMA used by the streaming (decode) kernels, and bounded waits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b2q.h"

namespace b2q {

// ---- error word -------------------------------------------------------------
// Device kernels report failures (a bounded wait that ran out, an index out of
// range) by writing a B2Q_E* code into a caller-owned int; the first code wins.
__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- bf16 helpers -----------------------------------------------------------
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }
// Round-to-nearest-even (NaN -> 0x7FC0) exactly as MLX's float -> bf16
// conversion (MLXC/types/bf16.h:39-58): written out so it does not depend on
// the library intrinsic's NaN payload.
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7FC0;
  u += ((u >> 16) & 1u) + 0x7FFFu;
  return uint16_t(u >> 16);
}
__device__ __forceinline__ float rb(float f) { return bf2f(f2bf(f)); }

// MLX Sigmoid functor in bf16 (one rounding per op) and compiled silu, as the
// Runner's exact helpers (Runner/FastModel/TrackFastKernels2.swift:22-31).
__device__ __forceinline__ uint16_t sigmoid_bf16(uint16_t xb) {
  const float x = bf2f(xb);
  const float e = rb(expf(rb(fabsf(x))));
  const float y = rb(1.0f / rb(1.0f + e));
  return f2bf(x < 0.0f ? y : rb(1.0f - y));
}
__device__ __forceinline__ uint16_t silu_bf16(uint16_t xb) {
  return f2bf(bf2f(xb) * bf2f(sigmoid_bf16(xb)));
}
__device__ __forceinline__ uint16_t swiglu_bf16(uint16_t g, uint16_t u) {
  return f2bf(bf2f(silu_bf16(g)) * bf2f(u));
}
// The same SwiGLU with the conversion instruction for every rounding (equal to
// f2bf except for NaN payloads) and the correctly rounded reciprocal (equal to
// 1 / x): a shorter dependent chain, identical finite results.
__device__ __forceinline__ float rb_cvt(float f) {
  uint16_t h;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return bf2f(h);
}
__device__ __forceinline__ uint16_t swiglu_bf16_cvt(uint16_t gb, uint16_t ub) {
  const float x = bf2f(gb);
  const float e = rb_cvt(expf(rb_cvt(fabsf(x))));
  const float y = rb_cvt(__frcp_rn(rb_cvt(1.0f + e)));
  const float sg = x < 0.0f ? y : rb_cvt(1.0f - y);
  const float si = rb_cvt(x * sg);
  uint16_t h;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(si * bf2f(ub)));
  return h;
}

// ---- nibble decode ------------------------------------------------------------
// A packed word W holds values e0..e7 (e_j in bits [4j, 4j+4)). OR-ing a nibble
// into the mantissa of bf16 128.0 (0x4300) gives exactly 128 + e (bf16 has unit
// spacing on [128, 256)). The four pairs (e0,e4) (e1,e5) (e2,e6) (e3,e7) come
// out of one mask per shift; the caller pairs x the same way, so the MMA's k
// slots see matching (x, q) elements. The +128 offset is removed in the group
// epilogue: s*(D - 128*sum(x)) + b*sum(x).
__device__ __forceinline__ uint32_t lop_or_and(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t d;
  // d = (a & mask) | magic
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(magic));
  return d;
}
__device__ __forceinline__ void decode_word(uint32_t W, uint32_t& p0, uint32_t& p1, uint32_t& p2,
                                            uint32_t& p3) {
  const uint32_t m = 0x000F000Fu, mg = 0x43004300u;
  p0 = lop_or_and(W, m, mg);
  p1 = lop_or_and(W >> 4, m, mg);
  p2 = lop_or_and(W >> 8, m, mg);
  p3 = lop_or_and(W >> 12, m, mg);
}

// fp16 variant: OR-ing into fp16 1024.0 (0x6400; unit spacing on [1024, 2048))
// holds a nibble in bits 0-3 as 1024 + q and one in bits 4-7 as 1024 + 16 q,
// so one shift serves the four pairs (e0,e4) (16e1,16e5) (e2,e6) (16e3,16e7);
// the activation side carries the matching 1/16 on the odd slots.
__device__ __forceinline__ void decode_word_h(uint32_t W, uint32_t& p0, uint32_t& p1, uint32_t& p2,
                                              uint32_t& p3) {
  const uint32_t mg = 0x64006400u;
  p0 = lop_or_and(W, 0x000F000Fu, mg);
  p1 = lop_or_and(W, 0x00F000F0u, mg);
  const uint32_t t = W >> 8;
  p2 = lop_or_and(t, 0x000F000Fu, mg);
  p3 = lop_or_and(t, 0x00F000F0u, mg);
}

// x chunk of 8 bf16 (x0..x7 as 4 packed pairs) -> (x0,x4) (x1,x5) (x2,x6) (x3,x7)
__device__ __forceinline__ uint4 perm_x8(uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
  o.y = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
  o.z = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
  o.w = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
  return o;
}

// ---- legacy MMA (decode streaming kernels) -------------------------------------
// D(16x8, f32) += A(16x16, bf16, row) * B(16x8, bf16, col).
// Not volatile: the MMA is a pure function of its registers, so the compiler
// may interleave independent accumulator chains.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8, f32) = A * B (accumulator starts at zero).
__device__ __forceinline__ void mma_bf16_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                    uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.0f;
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// fp16 operands, fp32 accumulation: D += A * B, and D = A * B.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                   uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.0f;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// ---- shared memory / mbarrier / bulk copy ----------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase with `parity` completed, false when the
// deadline (globaltimer ns) passed or *abort became non-zero first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline,
                                          volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if (globaltimer() > deadline) return false;
  }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (complete_tx).
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier among `nthreads` threads (multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Arrives at named barrier `id` without waiting (the waiting side uses bar.sync).
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- global-memory flags -----------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_u32(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Spin until *p >= target; false when the deadline passed or *abort was set.
__device__ __forceinline__ bool wait_counter_geq(const unsigned* p, unsigned target, uint64_t deadline,
                                                 volatile int* abort) {
  for (;;) {
    if (ld_acquire_u32(p) >= target) return true;
    if (abort && *abort) return false;
    if (globaltimer() > deadline) return false;
    __nanosleep(64);
  }
}

}  // namespace b2q
