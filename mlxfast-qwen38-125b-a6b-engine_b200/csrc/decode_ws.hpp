// decode_ws.hpp -- workspace header and layout of the decode MoE entry points,
// shared by the workspace-taking and the scratch-array (no allocation) forms.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

#include "decode2.cuh"
#include "engine.cuh"
#include "host.hpp"

namespace b2q {

// Every workspace starts with this 256-byte header.
struct WsHeader {
  int error;             // first device-side B2Q_E* code, 0 if none
  unsigned counters[3];  // grid counters of the fused decode kernels
  unsigned flag;         // self-test flag (never set)
  unsigned sched[2];     // single-column decode kernel: next gate|up unit, next down unit
  unsigned pad[57];
};
static_assert(sizeof(WsHeader) == 256, "workspace header is 256 bytes");

static inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

static inline bool gs_ok(int gs) { return gs == 32 || gs == 64 || gs == 128; }

static inline int check_bits_gs(const char* fn, int bits, int gs) {
  if (bits != 4) return set_error(B2Q_EUNSUPPORTED, "%s: bits=%d (only 4 is implemented)", fn, bits);
  if (!gs_ok(gs)) return set_error(B2Q_EUNSUPPORTED, "%s: group_size=%d (32, 64 or 128)", fn, gs);
  return B2Q_OK;
}

// Streaming-engine fast path: K a multiple of 8 groups (meta rows are whole
// 16-byte units), 16-byte aligned bases.
static inline bool engine_k_ok(int K, int gs) { return K > 0 && K % (8 * gs) == 0; }

struct DecodeWs {
  WsHeader* hdr;
  unsigned* ctr;  // one-token fused kernel: grid counters (d2_counter_words(H))
  float* logits;
  uint32_t* idx;
  float* w;
  uint16_t* act;
  float2* asc;    // one-token fused kernel: per block of 16 activations (scale, sum) [k][F / 16]
  size_t bytes;
};

// The one-token fused kernel's grid counters sit at a fixed offset right after
// the header, whatever the shapes: a workspace reused for another shape keeps
// them where the last call left them (zero).
constexpr size_t D2_CTR_BYTES = 4096;
static_assert(D2_CTR_LOGITS * 4 + 256 * 8 <= (int)D2_CTR_BYTES, "counter block");

static inline DecodeWs decode_ws_layout(void* base, int S, int H, int E, int F, int k) {
  (void)H;  // no region scales with the hidden size; kept for the size query's signature
  DecodeWs d{};
  size_t off = 0;
  char* b = static_cast<char*>(base);
  d.hdr = reinterpret_cast<WsHeader*>(b + off);
  off += sizeof(WsHeader);
  d.ctr = reinterpret_cast<unsigned*>(b + off);
  off += D2_CTR_BYTES;
  d.logits = reinterpret_cast<float*>(b + off);
  off = align256(off + sizeof(float) * (size_t)S * E);
  d.idx = reinterpret_cast<uint32_t*>(b + off);
  off = align256(off + sizeof(uint32_t) * (size_t)S * k);
  d.w = reinterpret_cast<float*>(b + off);
  off = align256(off + sizeof(float) * (size_t)S * k);
  d.act = reinterpret_cast<uint16_t*>(b + off);
  off = align256(off + sizeof(uint16_t) * (size_t)S * k * F);
  d.asc = reinterpret_cast<float2*>(b + off);
  off = align256(off + sizeof(float2) * (size_t)k * (F / 16));
  d.bytes = off;
  return d;
}

static inline void base_params(eng::Params& p, int mode, int gs) {
  std::memset(&p, 0, sizeof(p));
  p.mode = mode;
  p.gs = gs;
  p.wpt = gs / 32;
  p.timeout_ns = 2000000000ll;
}

}  // namespace b2q
