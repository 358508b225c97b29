/* b2q.h -- C ABI of the B200 affine 4-bit weight-product library (libb2q.so).
 *
 * The entry points replace the quantized-product surface of the reference
 * engine (Layr-Labs/mlxfast-qwen38-125b-a6b-engine). Each declaration names the
 * reference interface it stands in for; paths are relative to that project,
 * with MLXC = Vendor/mlx-swift/Source/Cmlx/mlx/mlx and
 * MLXCAPI = Vendor/mlx-swift/Source/Cmlx/mlx-c/mlx/c.
 *
 * Conventions (all entry points):
 *  - Plain pointers and sizes. Tensors are row-major and live in device memory
 *    unless a parameter says otherwise. bf16 values are 16-bit patterns
 *    (uint16_t). Packed weights are uint32 words holding 32/bits values, value
 *    8*i+j of a row in bits [4j, 4j+4) of word i (MLXC/backend/cpu/quantized.cpp:215-233);
 *    scales and biases are bf16 [rows, K/group_size].
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *    stream) and is stream-ordered; nothing blocks the host unless stated.
 *  - Return 0 on success, a negative B2Q_E* code on failure; no exception
 *    crosses the ABI. b2q_last_error() gives a message for the calling thread
 *    (mirrors mlx-c's status + error handler, MLXCAPI/ops.cpp:1505-1508).
 *  - Entry points that need scratch take a caller-owned `workspace` whose
 *    size comes from the matching *_workspace_size() call and allocate
 *    nothing; it must be zero-filled once before first use
 *    (b2q_workspace_reset) and is left zero-filled by every call that
 *    completes without a device-side error. Calls sharing one workspace must
 *    be ordered on one stream. b2q_qmm and b2q_gather_qmm keep mlx-c's
 *    workspace-free signatures: with more than 8 rows per item they take
 *    stream-ordered temporaries (cudaMallocAsync / cudaFreeAsync on `stream`);
 *    b2q_qmm_ws / b2q_gather_qmm_ws take a caller workspace instead.
 *  - Only bits == 4 is implemented on the device (the packed format of the
 *    path); group_size is 32, 64 or 128. Other values return B2Q_EUNSUPPORTED.
 */
#ifndef B2Q_H
#define B2Q_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2Q_API __attribute__((visibility("default")))
#else
#define B2Q_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B2Q_OK 0
#define B2Q_EINVAL (-1)       /* invalid shape, pointer or argument */
#define B2Q_EUNSUPPORTED (-2) /* valid for the reference, not implemented here */
#define B2Q_ECUDA (-3)        /* a CUDA runtime / launch error */
#define B2Q_ETIMEOUT (-4)     /* a bounded device-side wait ran out */
#define B2Q_ENCCL (-5)        /* an NCCL error (expert-parallel mode) */

/* Message of the last failing call on this thread ("" if none). */
B2Q_API const char* b2q_last_error(void);
/* ABI version: major*10000 + minor*100 + patch. */
B2Q_API int b2q_version(void);
/* Number of SMs of the current device (the persistent-grid size), or < 0. */
B2Q_API int b2q_device_sm_count(void);

/* ---- packing ------------------------------------------------------------ */

/* Replaces mlx_dequantize (MLXCAPI/ops.h:359-369) -> affine_dequantize
 * (MLXC/ops.cpp:5254-5346; Metal kernel MLXC/backend/metal/kernels/quantized.h:3314-3373).
 * out[r, k] = bf16(fp32(s)*q + fp32(b)) for r < rows, k < K (bit-exact with the
 * Metal dequantizer). */
B2Q_API int b2q_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   uint16_t* out, int64_t rows, int K, int group_size, int bits,
                   void* stream);

/* Replaces mlx_quantize (MLXCAPI/ops.h:801-808) -> quantize
 * (MLXC/ops.cpp:5214-5253; CPU kernel MLXC/backend/cpu/quantized.cpp:1158-1236).
 * w bf16 [rows, K] -> packed w_q [rows, K*bits/32], scales/biases [rows, K/gs]. */
B2Q_API int b2q_quantize(const uint16_t* w, uint32_t* w_q, uint16_t* scales, uint16_t* biases,
                 int64_t rows, int K, int group_size, int bits, void* stream);

/* ---- products ------------------------------------------------------------ */

/* Replaces mlx_quantized_matmul (MLXCAPI/ops.h:809-818, MLXCAPI/ops.cpp:2585-2616)
 * -> quantized_matmul (MLXC/ops.cpp:4784-4832), QuantizedMatmul::eval_gpu
 * (MLXC/backend/metal/quantized.cpp:1982-2075).
 * transpose != 0: y[M, N] = x[M, K] . dequant(w[N, K])^T (the only layout the
 * engine uses; transpose == 0 returns B2Q_EUNSUPPORTED).
 * Routing mirrors the reference's: M <= 8 -> the streaming qmv kernel
 * (decode), larger M -> the tensor-core qmm kernel (prefill). */
B2Q_API int b2q_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
            const uint16_t* biases, uint16_t* y, int M, int N, int K,
            int group_size, int bits, int transpose, void* stream);

/* Replaces mlx_gather_qmm (MLXCAPI/ops.h:475-488, MLXCAPI/ops.cpp:1471-1510)
 * -> gather_qmm (MLXC/ops.cpp:5559-5643), GatherQMM::eval_gpu
 * (MLXC/backend/metal/quantized.cpp:2089-2205).
 * For i < batch: y[i] (M x N) = x[lhs[i]] (M x K) . dequant(w[rhs[i]])^T, with
 * x [n_x, M, K], w [n_w, N, K*bits/32], scales/biases [n_w, N, K/gs],
 * y [batch, M, N]. lhs_indices/rhs_indices may be NULL (identity). Indices are
 * checked on the device: an item whose lhs >= n_x or rhs >= n_w is not read and
 * its y rows are written as zeros (the reference reads out of bounds instead).
 * sorted_indices is the reference's hint that rhs is non-decreasing. */
B2Q_API int b2q_gather_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                   const uint16_t* biases, const uint32_t* lhs_indices,
                   const uint32_t* rhs_indices, uint16_t* y, int batch, int M,
                   int N, int K, int n_x, int n_w, int group_size, int bits,
                   int transpose, int sorted_indices, void* stream);

/* Workspace-taking forms of b2q_qmm / b2q_gather_qmm (same reference functions:
 * MLXCAPI/ops.h:809-818 and :475-488). mlx-c's signatures carry no workspace,
 * so b2q_qmm / b2q_gather_qmm take a stream-ordered temporary for the M > 8
 * tensor-core path (sorted row tables and the grouped copy of x); these forms
 * use the caller's buffer instead and allocate nothing, for a runtime that
 * owns a fixed arena. workspace: 256-byte aligned, at least
 * b2q_gather_qmm_workspace_size(batch, M, N, K, n_w) bytes (M <= 8 needs none
 * beyond a non-null pointer); no contents carried between calls, so it needs no
 * clearing. Calls sharing one workspace must be ordered on one stream. */
B2Q_API size_t b2q_gather_qmm_workspace_size(int batch, int M, int N, int K, int n_w);
B2Q_API int b2q_qmm_ws(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                       const uint16_t* biases, uint16_t* y, int M, int N, int K,
                       int group_size, int bits, int transpose, void* workspace,
                       size_t workspace_bytes, void* stream);
B2Q_API int b2q_gather_qmm_ws(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                              const uint16_t* biases, const uint32_t* lhs_indices,
                              const uint32_t* rhs_indices, uint16_t* y, int batch, int M,
                              int N, int K, int n_x, int n_w, int group_size, int bits,
                              int transpose, int sorted_indices, void* workspace,
                              size_t workspace_bytes, void* stream);

/* ---- metadata pair index (load-time derived cache) ------------------------ */

/* Replaces TrackAffineLUT.build / buildOnDevice / verified
 * (Runner/FastModel/TrackAffineLUT.swift:58-110). For one tensor's bf16
 * scales / biases (n_groups groups, any shape), writes table (uint32, entry =
 * scale_bits | bias_bits << 16, 16-byte aligned, max_entries entries of room)
 * and index (uint16 per group, the scales' layout) and sets *count_out to the
 * number of distinct pairs. Table order: first occurrence when
 * n_groups < 2^20, ascending pair value otherwise (the reference's host loop
 * and device sort). *count_out = -1 (status B2Q_OK) when the tensor is not
 * indexed: more than max_entries distinct pairs (the reference's limit is
 * 32768), or a group whose round trip table[index[g]] does not give back its
 * exact bits. max_entries: 4..65536, a multiple of 4; table entries from the
 * count up to the next multiple of 4 are zeroed. Load-time call: it reads two
 * counts back to the host and synchronises the stream twice.
 * workspace: 256-byte aligned, b2q_affine_lut_workspace_size(max_entries). */
B2Q_API size_t b2q_affine_lut_workspace_size(int max_entries);
B2Q_API int b2q_affine_lut_build(const uint16_t* scales, const uint16_t* biases, int64_t n_groups,
                                 uint16_t* index, uint32_t* table, int max_entries, int* count_out,
                                 void* workspace, size_t workspace_bytes, void* stream);
/* Replaces TrackAffineLUT.lazyScales / lazyBiases (TrackAffineLUT.swift:46-53):
 * the bf16 scales and biases an index encodes, bit for bit. */
B2Q_API int b2q_affine_lut_expand(const uint16_t* index, const uint32_t* table, int64_t n_groups,
                                  uint16_t* scales, uint16_t* biases, void* stream);
/* Replaces TrackLUTGemv.apply (TrackAffineLUT.swift:330-368): one row,
 * y[1, N] = x[1, K] . dequant(w[N, K])^T with each group's scale / bias read
 * as table[index[n, g]]. The same single-column kernel as b2q_qmm at M = 1,
 * with a block of indices in place of the scale and bias blocks and the table
 * copied into shared memory: bit-identical to b2q_qmm on the scales / biases
 * the index encodes. B2Q_EUNSUPPORTED outside the kernel's shapes
 * (N % 16 == 0, N >= 32, K % 512 == 0, gs 32/64/128, 16-byte aligned tensors,
 * at most 16,384 table entries), where the reference also falls back. */
B2Q_API int b2q_qmv_lut(const uint16_t* x, const uint32_t* w, const uint16_t* index,
                        const uint32_t* table, int count, uint16_t* y, int N, int K,
                        int group_size, int bits, void* stream);

/* ---- MoE operators (the Runner's fused-operator surface) ------------------ */

/* Replaces TrackFastMoEKernels.routerGemv (Runner/FastModel/TrackFastMoE.swift:2246-2310)
 * and the generic matmul(x_f32, W_f32^T) (Runner/FastModel/TrackFastModel.swift:884-903):
 * logits f32 [T, E] = f32(x[T, H]) . f32(wr[E, H])^T. */
B2Q_API int b2q_moe_router_logits(const uint16_t* x, const uint16_t* wr, float* logits,
                          int T, int E, int H, void* stream);

/* Replaces TrackFastMoEKernels.route (Runner/FastModel/TrackFastMoE.swift:767-911):
 * top-k (largest first, ties to the lower index) + softmax over the k selected.
 * logits f32 [T, E] -> idx u32 [T, k], w f32 [T, k]. k <= 32, E <= 1024. */
B2Q_API int b2q_moe_route(const float* logits, uint32_t* idx, float* w, int T, int E, int k,
                  void* stream);

/* Replaces TrackFastMoEKernels.gateUpAct (Runner/FastModel/TrackFastMoE.swift:1192-1410)
 * for routed slots: for slot z < n_slots with expert idx[z] and token xrow[z]:
 * act[z, f] = silu(bf16(g)) * bf16(u) in bf16, g/u the gate/up qmv of x[xrow[z]].
 * x [S, H]; wg/wu [E, F, H/8]; act [n_slots, F]. xrow may be NULL (slot z -> token z / k
 * is then NOT assumed: NULL means token 0 for every slot). */
B2Q_API int b2q_moe_gate_up_act(const uint16_t* x, const uint32_t* wg, const uint16_t* sg,
                        const uint16_t* bg, const uint32_t* wu, const uint16_t* su,
                        const uint16_t* bu, const uint32_t* idx, const uint32_t* xrow,
                        uint16_t* act, int n_slots, int S, int H, int E, int F,
                        int group_size, int bits, void* stream);

/* Replaces TrackFastMoEKernels.downCombine (Runner/FastModel/TrackFastMoE.swift:1412-1590)
 * without the shared expert: out[t, h] = bf16(colsum_j f32(bf16(y_j[h])) * w[t, j]),
 * y_j = qmv(wd[idx[t*k+j]], act[t*k+j]). act [S*k, F], idx/w [S, k], out [S, H].
 * k <= 8. */
B2Q_API int b2q_moe_down_combine(const uint16_t* act, const uint32_t* wd, const uint16_t* sd,
                         const uint16_t* bd, const uint32_t* idx, const float* w,
                         uint16_t* out, int S, int H, int E, int F, int k,
                         int group_size, int bits, void* stream);

/* One decode MoE layer for S tokens (S <= 8): router logits, route,
 * gate|up + SwiGLU, down + weighted combine. S == 1 runs as ONE persistent
 * launch (grid barrier after the router, in-CTA combine); S > 1 chains the
 * four operators above. Replaces the
 * decode branch of moeForwardShared (Runner/FastModel/TrackFastModel.swift:867-955)
 * minus the shared expert. Outputs: out [S, H] bf16; idx/w [S, k] (may be
 * NULL); logits [S, E] f32 (may be NULL). k <= 8. The workspace holds the
 * grid barrier counters, the slot activations and the error word. */
B2Q_API size_t b2q_moe_decode_workspace_size(int S, int H, int E, int F, int k);
B2Q_API int b2q_moe_decode(const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   uint16_t* out, uint32_t* idx, float* w, float* logits,
                   int S, int H, int E, int F, int k, int group_size, int bits,
                   void* workspace, size_t workspace_bytes, void* stream);

/* b2q_moe_decode for one token (S == 1) that allocates nothing and takes no
 * workspace. No counterpart in the reference: it exists for callers that
 * cannot allocate device memory when they decode (device memory owned by
 * another allocator or a fixed arena, plugins handed only their input and
 * output buffers, code that must avoid allocating CUDA calls). Its scratch is
 * one file-scope device array of B2Q_NOALLOC_SCRATCH_BYTES per GPU that loads
 * the library, held until exit; shapes whose decode workspace
 * (b2q_moe_decode_workspace_size(1, H, E, F, k)) exceeds it are refused with
 * B2Q_EINVAL. The first call on a device resolves the array's address
 * (cudaGetSymbolAddress): make it before any stream capture. All calls on a
 * device share the array; each clears its error word and grid counters with
 * an asynchronous memset on `stream` first, so calls in stream order are
 * independent, but calls that overlap on the GPU race. It runs the same kernel
 * as b2q_moe_decode for the shape. `status` (device int, may be NULL)
 * receives the call's device-side status in stream order: 0, or B2Q_ETIMEOUT
 * if a bounded wait ran out. Other arguments as b2q_moe_decode. */
#define B2Q_NOALLOC_SCRATCH_BYTES 131072
B2Q_API int b2q_moe_decode_noalloc(const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   uint16_t* out, uint32_t* idx, float* w, float* logits,
                   int H, int E, int F, int k, int group_size, int bits,
                   int* status, void* stream);

/* A caller's one-token decode loop through this ABI, as a native host runs it
 * (no counterpart in the reference; it measures the API path end to end). For
 * step i of warmup + steps: the token row host_x + (i % n_tokens) * H (pinned
 * host memory) is copied in, b2q_moe_decode runs layer l = i % n_layers (wr[l]
 * and w9[9 l .. 9 l + 8] = gate w/s/b, up w/s/b, down w/s/b), and the output
 * row is copied back to host_out (pinned). The copies run on a second stream
 * with two device buffers each way (dev_x2, dev_out2: 2 * H bf16), so they
 * overlap the kernels. *ms_per_step receives the CUDA-event time of the last
 * `steps` steps, from their first input copy to their last output copy (the
 * timed steps start from an empty pipeline). Returns after the loop finished
 * (it synchronises). */
B2Q_API int b2q_moe_decode_host_loop(const uint16_t* host_x, int n_tokens, uint16_t* host_out,
                   const uint16_t* const* wr, const void* const* w9, int n_layers,
                   int H, int E, int F, int k, int group_size, int bits,
                   uint16_t* dev_x2, uint16_t* dev_out2, void* workspace, size_t workspace_bytes,
                   int warmup, int steps, void* stream, float* ms_per_step);
/* Expert parallelism (experts sharded over ranks; one NCCL all-reduce per layer).
 * The reference's expert-parallel configuration of its MoE layer
 * (moeForwardShared, Runner/FastModel/TrackFastModel.swift:867-1009) with
 * the expert stacks of each layer bound per rank (:470-540): every rank holds
 * the router and the experts [e_lo, e_lo + e_local) as stacked tensors of its
 * local experts only, computes the routing in full, multiplies the selected
 * experts it holds and adds their weighted outputs into the fp32 `partial`
 * [T, H]; the all-reduce (sum) runs on `stream`, then `out` (bf16, may be
 * NULL) receives the rounded layer output. With comm == NULL (or one rank)
 * there is no all-reduce and `partial` is this rank's share.
 * b2q_ep_unique_id fills a 128-byte NCCL id on one rank; the caller sends it
 * to the others (its own transport), then every rank calls b2q_ep_comm_init
 * with its device current. NCCL is loaded at run time (libnccl.so.2). */
B2Q_API int b2q_ep_unique_id(void* id_out, size_t id_bytes);
B2Q_API int b2q_ep_comm_init(void** comm_out, int nranks, int rank, const void* id, size_t id_bytes);
B2Q_API int b2q_ep_comm_destroy(void* comm);
/* Peer-memory reduction of the one-token layer (no reference counterpart:
 * the reference runs on one GPU). b2q_ep_peer_setup allocates this rank's
 * exchange buffer (b2q_ep_peer_buffer_bytes(H), zeroed; the communicator owns
 * it) and returns its CUDA IPC handle (64 bytes); the caller gathers every
 * rank's handle (its own transport, rank order) and every rank calls
 * b2q_ep_peer_open with the nranks handles of handle_bytes each. From then on
 * b2q_ep_moe_decode with S == 1, this H and a non-NULL `out` runs without a
 * collective call: each rank's kernel stores its fp32 partial rows into every
 * rank's buffer (plain stores over NVLink, double-buffered by a per-call
 * epoch), publishes the epoch, waits (bounded: B2Q_ETIMEOUT in the workspace)
 * for every rank's, and writes the summed bf16 `out` itself; `partial` is not
 * written on this path. Every rank must make the same sequence of such calls
 * on the communicator, one per stream order. 2 to 8 ranks; set-up and open
 * once per communicator (a repeat is refused with B2Q_EINVAL).
 * b2q_ep_comm_destroy releases the buffer and the peer mappings: call it after
 * this rank's last exchange call has completed on its stream (every peer's
 * stores into this rank's buffer precede the flags that call waited for). */
B2Q_API size_t b2q_ep_peer_buffer_bytes(int H);
B2Q_API int b2q_ep_peer_setup(void* comm, int H, void* handle_out, size_t handle_bytes);
B2Q_API int b2q_ep_peer_open(void* comm, const void* handles, size_t handle_bytes);
B2Q_API size_t b2q_ep_moe_decode_workspace_size(int S, int H, int E, int F, int k);
B2Q_API int b2q_ep_moe_decode(void* comm, const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   float* partial, uint16_t* out, uint32_t* idx, float* w,
                   int S, int H, int E, int F, int k, int e_lo, int e_local,
                   int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream);
B2Q_API size_t b2q_ep_moe_prefill_workspace_size(int T, int H, int E, int F, int k);
B2Q_API int b2q_ep_moe_prefill(void* comm, const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   float* partial, uint16_t* out, uint32_t* idx, float* w,
                   int T, int H, int E, int F, int k, int e_lo, int e_local,
                   int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream);

/* Expert-parallel prefill over an all-to-all token exchange (dispatch /
 * combine). No counterpart in the reference, which keeps all experts of a
 * layer on one Apple GPU: this is its MoE layer (moeForwardShared,
 * Runner/FastModel/TrackFastModel.swift:867-1009, sorted prefill
 * Runner/FastModel/TrackP12Prefill.swift:180-237) with tokens owned by ranks
 * and experts sharded by b2q_ep_expert_range (contiguous blocks, the first
 * E % nranks ranks one expert more). Up to B2Q_EP_MAX_RANKS ranks.
 *
 * b2q_ep_a2a_dispatch (token owner): routes its T tokens and, for every rank d
 *   holding one of a token's k experts, copies the token row once into block d
 *   of send_x [nranks, T, H] (bf16) and its k expert ids and k fp32 weight bits
 *   into send_meta [nranks, T, 2k] (u32); send_counts [nranks] (int32) = rows
 *   in each block, pos [T, nranks] (int32) = a token's row in block d or -1.
 *   idx / w (may be NULL) receive the routing [T, k].
 * b2q_ep_a2a_experts (expert rank): for R received rows (recv_x [R, H],
 *   recv_meta [R, 2k], blocks of all senders concatenated) multiplies the slots
 *   whose expert lies in [e_lo, e_lo + e_local) by the local stacks
 *   (tensor cores, gate|up + SwiGLU, down) and writes each row's weighted sum
 *   of its local slots to partial [R, H] (fp32).
 * b2q_ep_a2a_combine (token owner): ret [nranks, T, H] (fp32) holds in block d
 *   the partial rows rank d returned, in the order they were sent;
 *   out[t] = bf16(sum over d in rank order of ret[d, pos[t, d]]).
 * b2q_ep_moe_prefill_a2a chains the three over the library's communicator
 *   (comm == NULL: one rank): all-gather of the counts, grouped NCCL send /
 *   recv of the blocks, the experts, the partial rows back, the combine. Every
 *   rank calls it (T may be 0, T <= T_max); it reads the counts on the host
 *   (a copy to the host and a synchronisation of `stream`, once per call), so
 *   it returns after the dispatch has run, blocks the calling thread until
 *   then, and cannot be captured in a CUDA graph. The three phase entry
 *   points above are stream-ordered and asynchronous. */
#define B2Q_EP_MAX_RANKS 8
B2Q_API int b2q_ep_expert_range(int E, int nranks, int rank, int* e_lo, int* e_local);
B2Q_API size_t b2q_ep_a2a_dispatch_workspace_size(int T, int H, int E, int k, int nranks);
B2Q_API int b2q_ep_a2a_dispatch(const uint16_t* x, const uint16_t* wr, uint16_t* send_x, uint32_t* send_meta,
                   int32_t* send_counts, int32_t* pos, uint32_t* idx, float* w,
                   int T, int H, int E, int k, int nranks,
                   void* workspace, size_t workspace_bytes, void* stream);
B2Q_API size_t b2q_ep_a2a_experts_workspace_size(int R, int H, int E, int F, int k);
B2Q_API int b2q_ep_a2a_experts(const uint16_t* recv_x, const uint32_t* recv_meta,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   float* partial, int R, int H, int E, int F, int k, int e_lo, int e_local,
                   int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream);
B2Q_API int b2q_ep_a2a_combine(const float* ret, const int32_t* pos, uint16_t* out,
                   int T, int H, int nranks, void* stream);
B2Q_API size_t b2q_ep_moe_prefill_a2a_workspace_size(int T_max, int H, int E, int F, int k, int nranks);
B2Q_API int b2q_ep_moe_prefill_a2a(void* comm, const uint16_t* x, const uint16_t* wr,
                   const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                   const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                   uint16_t* out, uint32_t* idx, float* w,
                   int T, int T_max, int H, int E, int F, int k,
                   int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream);

/* ---- decoder around the path (configs with a full model) -------------------
 * b2q_embed_gather: out[t] (bf16 [T, K]) = dequantize(table row ids[t]) of a
 *   4-bit table w [V, K/8], scales / biases [V, K/gs] -- MLXNN
 *   QuantizedEmbedding.callAsFunction (Vendor/mlx-swift/Source/MLXNN/
 *   Quantized.swift:238-300) with the Metal dequantizer's arithmetic. An id
 *   outside [0, V) gives a zero row and B2Q_EINVAL in *status (may be NULL).
 * b2q_rms_norm: out [T, H] = bf16(weight * x * rsqrt(mean(x^2) + eps)), fp32
 *   inside (MLX fast::rms_norm, which the reference's norms call).
 * b2q_rope: x [T, heads, head_dim] in place, non-interleaved rotary embedding
 *   (MLX fast::rope, traditional = false, scale 1) at positions[t] or, when
 *   positions is NULL, pos0 + t. */
B2Q_API int b2q_embed_gather(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   const int32_t* ids, uint16_t* out, int T, int V, int K, int group_size, int bits,
                   int* status, void* stream);
B2Q_API int b2q_rms_norm(const uint16_t* x, const uint16_t* weight, uint16_t* out, int T, int H, float eps,
                   void* stream);
B2Q_API int b2q_rope(uint16_t* x, int T, int heads, int head_dim, const int32_t* positions, int pos0,
                   float theta, void* stream);
/* b2q_add_rms_norm: h_out = bf16(h + delta) (delta may be NULL: no add, h_out
 *   unused; h_out may be h), out = rms_norm(h_out) as b2q_rms_norm -- the
 *   residual add of one block fused into the next norm.
 * b2q_rope_kv: qkv [T, (nq + 2 nk) * head_dim] (a fused q|k|v product): rope
 *   on its q and k heads in place at positions[t], then the k and v heads
 *   written to k_cache / v_cache [max_seq, nk, head_dim] at row positions[t]
 *   (a position outside [0, max_seq) writes nothing and sets B2Q_EINVAL in
 *   *status).
 * b2q_gqa_decode: attention of T query rows (q row t at q + t * q_ld, nq heads)
 *   over cache rows [0, positions[t]] with nq / nk query heads per kv head,
 *   softmax(q.k / sqrt(d)) v in fp32, out [T, nq * head_dim] bf16. `window`
 *   bounds the positions (and must not exceed the cache rows); the workspace
 *   (b2q_gqa_decode_workspace_size) holds the per-chunk partial sums. For
 *   decode steps and short verify windows; prefill uses a causal attention
 *   kernel of the framework (off the path). */
B2Q_API int b2q_add_rms_norm(const uint16_t* h, const uint16_t* delta, const uint16_t* weight, uint16_t* h_out,
                   uint16_t* out, int T, int H, float eps, void* stream);
B2Q_API int b2q_rope_kv(uint16_t* qkv, int T, int nq, int nk, int head_dim, const int32_t* positions, float theta,
                   uint16_t* k_cache, uint16_t* v_cache, int max_seq, int* status, void* stream);
B2Q_API size_t b2q_gqa_decode_workspace_size(int T, int nq, int nk, int head_dim, int window);
B2Q_API int b2q_gqa_decode(const uint16_t* q, int q_ld, const uint16_t* k_cache, const uint16_t* v_cache,
                   const int32_t* positions, uint16_t* out, int T, int nq, int nk, int head_dim, int window,
                   int* status, void* workspace, size_t workspace_bytes, void* stream);
/* b2q_attn_decode: b2q_rope_kv followed by b2q_gqa_decode in one launch, for
 *   windows of at most 8 rows (qkv rows at qkv + t * q_ld are read, not
 *   modified): the k / v rows go to the caches at their positions exactly as
 *   b2q_rope_kv writes them, and each row attends cache rows [0, positions[t]]
 *   with the window's own rows taken from qkv. The workspace
 *   (b2q_attn_decode_workspace_size, 256-byte aligned; the size for 8 rows
 *   serves every T) holds one counter per row and kv head, then the chunk
 *   partials: zero it once before the first call; each call leaves the
 *   counters at zero. Calls sharing a workspace must be ordered on one stream.
 *   B2Q_EUNSUPPORTED when the window's merge buffers exceed shared memory
 *   (past ~125k positions at 8 query heads per kv head). */
/* b2q_qmv_norm / b2q_moe_decode_norm: b2q_add_rms_norm fused into the
 *   one-token product that consumes its output (the q|k|v product and the MoE
 *   layer of a decode step): every CTA of the single-column kernel computes
 *   x = rms_norm(bf16(h + delta)) * norm_weight itself during its pass over x
 *   (one launch instead of two; the block sum of squares is taken in another
 *   order than b2q_add_rms_norm's, so x can differ from it in the last bit),
 *   and CTA 0 writes h_out = bf16(h + delta) (delta NULL: x = rms_norm(h) and
 *   h_out is not written). h_out must not alias h or delta. The rest as
 *   b2q_qmm (M = 1) / b2q_moe_decode (S = 1). B2Q_EUNSUPPORTED outside the
 *   single-column kernel's shapes (H or K at most 4864): the caller then uses
 *   b2q_add_rms_norm and the plain call. */
B2Q_API int b2q_qmv_norm(const uint16_t* h, const uint16_t* delta, const uint16_t* norm_weight, float eps,
                   uint16_t* h_out, const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   uint16_t* y, int N, int K, int group_size, int bits, void* stream);
B2Q_API int b2q_moe_decode_norm(const uint16_t* h, const uint16_t* delta, const uint16_t* norm_weight, float eps,
                   uint16_t* h_out, const uint16_t* wr, const uint32_t* wg, const uint16_t* sg,
                   const uint16_t* bg, const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                   const uint32_t* wd, const uint16_t* sd, const uint16_t* bd, uint16_t* out,
                   uint32_t* idx, float* w, float* logits, int H, int E, int F, int k, int group_size,
                   int bits, void* workspace, size_t workspace_bytes, void* stream);
B2Q_API size_t b2q_attn_decode_workspace_size(int T, int nq, int nk, int head_dim, int window);
B2Q_API int b2q_attn_decode(const uint16_t* qkv, int q_ld, const int32_t* positions, uint16_t* k_cache,
                   uint16_t* v_cache, uint16_t* out, int T, int nq, int nk, int head_dim, float theta,
                   int window, int* status, void* workspace, size_t workspace_bytes, void* stream);

/* ---- checkpoint reading (per-layer packed-weight binding) ------------------ */

/* Replaces the reference's safetensors header reader
 * (Sources/MLXFastCore/Safetensors.swift:75-180) for binding a layer's
 * stacked expert tensors (Runner/FastModel/TrackFastModel.swift:470-540).
 * b2q_st_open maps the file read-only and checks the header (8-byte
 * little-endian length, at most 100,000,000 bytes, a JSON object of
 * {dtype, shape, data_offsets}, offsets ordered and inside the data section).
 * b2q_st_read copies a tensor's stored bytes to host memory (to_device == 0)
 * or to device memory (copy on `stream`, synchronised before returning). */
B2Q_API int b2q_st_open(const char* path, void** handle);
B2Q_API int b2q_st_close(void* handle);
B2Q_API int b2q_st_count(void* handle);
B2Q_API int b2q_st_name(void* handle, int i, char* buf, size_t buf_bytes);
B2Q_API int b2q_st_info(void* handle, const char* name, char* dtype, size_t dtype_bytes,
                int64_t* shape, int max_dims, int* ndim, uint64_t* nbytes);
B2Q_API int b2q_st_read(void* handle, const char* name, void* dst, size_t dst_bytes,
                int to_device, void* stream);

/* One prefill MoE layer over T tokens: router logits, route, stable sort of the
 * T*k assignments by expert (TrackPrefillSort.swift:84-201), gate|up + SwiGLU
 * gather GEMM and down gather GEMM on the tensor cores over expert-aligned row
 * tiles (TrackPrefillIndirect.swift:40-227), and the weighted combine through
 * the inverse permutation (TrackP12Prefill.swift:180-237).
 * out [T, H] bf16; idx/w [T, k] may be NULL. */
B2Q_API size_t b2q_moe_prefill_workspace_size(int T, int H, int E, int F, int k);
B2Q_API int b2q_moe_prefill(const uint16_t* x, const uint16_t* wr,
                    const uint32_t* wg, const uint16_t* sg, const uint16_t* bg,
                    const uint32_t* wu, const uint16_t* su, const uint16_t* bu,
                    const uint32_t* wd, const uint16_t* sd, const uint16_t* bd,
                    uint16_t* out, uint32_t* idx, float* w,
                    int T, int H, int E, int F, int k, int group_size, int bits,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Replaces TrackFastKernels.swiglu2 (Runner/FastModel/TrackFastKernels2.swift:575-600):
 * act[i] = silu(g[i]) * u[i] with the bf16 Sigmoid functor, n elements. */
B2Q_API int b2q_swiglu(const uint16_t* g, const uint16_t* u, uint16_t* act, int64_t n, void* stream);

/* Replaces track_p12_moe_sorted_combine (Runner/FastModel/TrackP12Prefill.swift:180-197)
 * without the shared expert: out[t, h] = bf16(colsum_j f32(y[inverse[t*k+j], h]) * w[t, j]),
 * y [T*k, H] in sorted-row order. k <= 32. */
B2Q_API int b2q_moe_sorted_combine(const uint16_t* y, const uint32_t* inverse, const float* w, uint16_t* out,
                           int T, int H, int k, void* stream);

/* Stable counting sort of R expert ids (the first stage of b2q_moe_prefill):
 * sorted_ids[p], token_rows[p] = order[p] / k, inverse[order[p]] = p,
 * offsets[E + 1]. Replaces TrackPrefillSort.apply (TrackPrefillSort.swift:84-105). */
B2Q_API size_t b2q_sort_workspace_size(int R, int E);
B2Q_API int b2q_moe_sort(const uint32_t* ids, uint32_t* sorted_ids, uint32_t* token_rows,
                 uint32_t* inverse, uint32_t* offsets, int R, int E, int k,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- workspace / status -------------------------------------------------- */

/* Zero-fills a workspace (cudaMemsetAsync on `stream`). */
B2Q_API int b2q_workspace_reset(void* workspace, size_t workspace_bytes, void* stream);
/* Reads (synchronously) and clears the device error word a workspace carries:
 * returns B2Q_OK or the B2Q_E* code a kernel recorded (e.g. B2Q_ETIMEOUT). */
B2Q_API int b2q_workspace_status(void* workspace, size_t workspace_bytes, void* stream);

/* Test hook for the failure path: launches one kernel that waits, with a
 * bound of timeout_ns, on a flag in `workspace` that nothing sets, and returns
 * (after a stream sync) B2Q_ETIMEOUT when the bound ran out as designed. */
B2Q_API int b2q_selftest_wait_timeout(void* workspace, size_t workspace_bytes,
                              long long timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B2Q_H */
