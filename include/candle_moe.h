/*
 * candle-moe-b200: C ABI of the Blackwell (sm_100a) fused-MoE library.
 *
 * The first two entry points are drop-in replacements for the two symbols that the reference
 * crate kozistr/candle-moe declares in src/ffi.rs and links from its static libmoe.a; its Rust
 * layer (src/lib.rs) can call them unchanged.  The remaining entry points extend the interface
 * with status returns, caller-owned workspace and the sort/align step on its own.
 *
 * Conventions (all entry points):
 *   - every pointer is a CUDA device pointer to contiguous row-major data; the caller owns all
 *     buffers;
 *   - work is enqueued on `stream` (a cudaStream_t / CUstream; NULL = the legacy default
 *     stream) and the call returns without synchronising;
 *   - dtype codes: 0 = f16, 1 = bf16, 2 = f32; activation codes: 0 = SiLU, 1 = GELU (tanh form),
 *     2 = ReLU (any other value = SiLU); moe_type: 0 = Qwen3 (gate/up/down), 1 = Nomic
 *     (fc1 -> act -> fc2, the second matrix applied transposed).
 */
#ifndef CANDLE_MOE_B200_H
#define CANDLE_MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes of the extended entry points (and of moe_last_status()). */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARG 1   /* bad size, code or null pointer */
#define MOE_ERR_UNSUPPORTED 2   /* valid request outside what the library implements */
#define MOE_ERR_CUDA 3          /* a CUDA call or kernel launch failed */
#define MOE_ERR_WORKSPACE 4     /* caller workspace smaller than moe_fused_workspace_size() */
#define MOE_ERR_NO_MEMORY 5     /* the library's workspace pool could not allocate */

/*
 * Fused softmax + top-k router.  Replaces kernels/topk_softmax.cu:331-353 (declared for Rust at
 * src/ffi.rs:15-24).
 *   gating_output        [num_tokens, num_experts] f32 router logits
 *   topk_weights         [num_tokens, topk] f32 out: softmax probability of each pick (not
 *                        renormalised, as in the reference)
 *   topk_indices         [num_tokens, topk] i32/u32 out: expert id of each pick, descending
 *                        probability, ties to the lower id
 *   token_expert_indices [num_tokens, topk] i32/u32 out: j*num_tokens + t
 *   num_experts          power of two, 1..256
 * num_tokens is int32_t here: the reference C definition says int64_t but its Rust caller passes
 * a c_int (src/ffi.rs:21 vs topk_softmax.cu:337); this declaration matches the caller.
 * Errors (unsupported num_experts, launch failure) are reported by moe_last_status().
 */
void topk_softmax(void* gating_output, void* topk_weights, void* topk_indices,
                  void* token_expert_indices, int32_t num_experts, int32_t num_tokens,
                  int32_t topk, void* stream);

/*
 * Fused MoE expert FFN.  Replaces kernels/moe.cu:451-773 (declared for Rust at
 * src/ffi.rs:45-62).
 *   input            [num_tokens, hidden_dim]                       dtype
 *   gate_weights     [num_experts, hidden_dim, intermediate_dim]     dtype
 *   up_weights       [num_experts, hidden_dim, intermediate_dim]     dtype
 *   down_weights     [num_experts, intermediate_dim, hidden_dim]     dtype (Qwen3), NULL (Nomic)
 *   routing_weights  [num_tokens, num_selected_experts]              f32
 *   expert_indices   [num_tokens, num_selected_experts]              u32 (ids >= num_experts are
 *                                                                    skipped)
 *   output           [num_tokens, hidden_dim]                        dtype, out
 * Qwen3: out[t] = sum_j w[t,j] * (act(x_t.G_e) * (x_t.U_e)).D_e ;  Nomic: out[t] = sum_j w[t,j] *
 * act(x_t.G_e).U_e^T, with e = expert_indices[t,j].  The reference required a zeroed output and
 * accumulated into it; this library overwrites it, which gives the same result for every input
 * the reference accepts.  Workspace comes from a library-owned stream-ordered pool.  Errors are
 * reported by moe_last_status().
 */
void fused_moe(void* input, void* gate_weights, void* up_weights, void* down_weights,
               void* routing_weights, void* expert_indices, void* output, int num_tokens,
               int hidden_dim, int intermediate_dim, int num_experts, int num_selected_experts,
               int activation_type, uint32_t moe_type, uint32_t dtype, void* stream);

/* Status of the last drop-in call (topk_softmax / fused_moe) made by this thread. */
int moe_last_status(void);

/* Human-readable name of a status code. */
const char* moe_status_string(int status);

/*
 * Router with a status return and optional renormalisation of the k weights (w / sum_j w, as
 * Qwen3's norm_topk_prob does; the reference has no such option).  Same semantics as
 * topk_softmax (kernels/topk_softmax.cu:331-353) otherwise.
 */
int moe_topk_softmax_v2(const float* gating_output, float* topk_weights, int32_t* topk_indices,
                        int32_t* token_expert_indices, int32_t num_experts, int64_t num_tokens,
                        int32_t topk, int32_t renormalize, void* stream);

/*
 * The router's gate projection fused with the softmax + top-k (no counterpart in the reference,
 * whose caller computes the logits with a Linear layer and passes them to topk_softmax,
 * README.md:67-73): logits = input . gate_proj^T on the tensor cores, then topk_softmax's picks
 * and weights (optionally renormalised as moe_topk_softmax_v2 does), without writing the
 * logits to memory.
 *   input          [num_tokens, hidden_dim] f16/bf16 (dtype 0/1), 16-byte aligned
 *   gate_proj      [num_experts, hidden_dim] same dtype (the Linear's weight), 16-byte aligned
 *   topk_weights, topk_indices, token_expert_indices: as topk_softmax
 *   logits         [num_tokens, num_experts] f32 out: the logits the picks were made from, or
 *                  NULL (for checking: topk_softmax on them gives the same picks and weights)
 * num_experts a power of two <= 256, topk <= min(num_experts, 16), hidden_dim a multiple of 64;
 * otherwise MOE_ERR_UNSUPPORTED.
 */
int moe_router_project_topk(const void* input, const void* gate_proj, int64_t num_tokens,
                            int32_t hidden_dim, int32_t num_experts, int32_t topk,
                            int32_t renormalize, uint32_t dtype, float* topk_weights,
                            int32_t* topk_indices, int32_t* token_expert_indices, float* logits,
                            void* stream);

/*
 * Sort / align step on its own.  Replaces launch_preprocessing (kernels/preprocessing.cuh:253-313),
 * which the reference runs inside fused_moe without exporting it.
 *   expert_offsets    [num_experts + 2] i32 out: exclusive prefix of per-expert row counts,
 *                     [num_experts] = routed rows, [num_experts + 1] = largest count
 *   sorted_token_ids  [num_tokens * topk] i32 out: token id of each routed row, grouped by expert
 *   sorted_weights    [num_tokens * topk] f32 out: routing weight of each routed row
 * Within an expert, rows are in ascending (token, slot) order (the reference's order there
 * depends on atomics).  Scratch memory, when needed, comes from the library's pool.
 */
int moe_route_prep(const uint32_t* expert_indices, const float* routing_weights,
                   int64_t num_tokens, int32_t topk, int32_t num_experts, int32_t* expert_offsets,
                   int32_t* sorted_token_ids, float* sorted_weights, void* stream);

/*
 * moe_route_prep that also returns, for every sorted row, its flat index t*topk + j
 * (sorted_flat, [num_tokens * topk] i32).  Any of sorted_token_ids, sorted_weights and
 * sorted_flat may be NULL.  Used to bucket (token, slot) rows by destination rank in the
 * expert-parallel layer (no counterpart in the reference, which has no multi-GPU path).
 */
int moe_route_prep_ex(const uint32_t* expert_indices, const float* routing_weights,
                      int64_t num_tokens, int32_t topk, int32_t num_experts,
                      int32_t* expert_offsets, int32_t* sorted_token_ids, float* sorted_weights,
                      int32_t* sorted_flat, void* stream);

/*
 * dst[r, :] = src[index[r], :] for r < rows; rows of hidden_dim elements of `dtype`.  The row
 * gather of the expert-parallel dispatch (no counterpart in the reference).
 */
int moe_gather_rows(const void* src, const int32_t* index, int64_t rows, int32_t hidden_dim,
                    uint32_t dtype, void* dst, void* stream);

/*
 * Slot-ordered combine of contributions that arrive in exchange order: with sorted_flat[r] the
 * flat index t*topk + j of row r of rows_buf (r < rows), output[t, :] = sum over j (in slot
 * order) of rows_buf[r(t,j), :], accumulated in f32 and rounded once to `dtype`; slots with no
 * row contribute nothing.  The expert-parallel counterpart of the reference's weighted
 * scatter-add into the output (qwen3_moe.cu:637-641).
 */
int moe_combine_rows(const void* rows_buf, const int32_t* sorted_flat, int64_t rows,
                     int64_t num_tokens, int32_t topk, int32_t hidden_dim, uint32_t dtype,
                     void* output, void* stream);

/*
 * Expert-parallel bookkeeping (no counterpart in the reference, which has no multi-GPU path).
 * With num_ranks ranks owning num_experts/num_ranks experts each:
 *
 * moe_ep_dest_groups: groups[t*num_ranks + d] = (t / tokens_per_chunk) * num_ranks + d when
 *   token t has one of its topk experts on rank d, else INT32_MAX (no group); route
 *   preparation over these groups buckets the (token, rank) pairs to send.  With
 *   assignment_counts (else NULL), also writes the number of (token, slot) assignments to
 *   experts of rank d among the tokens of chunk c to assignment_counts[c*num_ranks + d]
 *   (num_chunks * num_ranks <= 12288 counters; every token's chunk must be < num_chunks).
 * moe_ep_pack: for the num_pairs sorted pairs (pair_token[r] = t, pair_flat[r] = t*num_ranks + d)
 *   copy input row t to rows[r], write the pair's topk-slot metadata (meta[r*2*topk + j] = local
 *   expert id of slot j if its expert lives on rank d, else num_experts/num_ranks;
 *   meta[r*2*topk + topk + j] = that slot's routing weight bits, or 0) and slot_count[r] = the
 *   pair's slots.  With num_pairs_device (else NULL) the pair count is read from that device
 *   int32 when the kernel runs and num_pairs is only the capacity of the outputs, so the pack
 *   can be enqueued before the host has the count.
 * moe_ep_entry_flat: with pair_start the exclusive prefix of slot_count, write
 *   flat[pair_start[r] + i] = t*topk + j for the pair's i-th slot j (the token slot of each
 *   per-slot contribution returned for pair r).
 */
int moe_ep_dest_groups(const uint32_t* expert_indices, int64_t num_tokens, int32_t topk,
                       int32_t num_experts, int32_t num_ranks, int64_t tokens_per_chunk,
                       int32_t* groups, int32_t num_chunks, int64_t* assignment_counts,
                       void* stream);
int moe_ep_pack(const void* input, const int32_t* pair_token, const int32_t* pair_flat,
                int64_t num_pairs, const int32_t* num_pairs_device,
                const uint32_t* expert_indices, const float* routing_weights, int32_t topk,
                int32_t num_experts, int32_t num_ranks, int32_t hidden_dim, uint32_t dtype,
                void* rows, int32_t* meta, int32_t* slot_count, void* stream);
/*
 * output[r, :] = sum of rows_in[segment_start[r] .. segment_start[r+1]) in row order, f32
 * accumulation, one rounding to `dtype` (segment_start: num_segments + 1 int64 offsets).  The
 * remote half of the expert-parallel "partials" return: a pair's slot contributions, written
 * consecutively by moe_fused_scatter, become one partial row.
 */
int moe_segment_sum_rows(const void* rows_in, const int64_t* segment_start, int64_t num_segments,
                         int32_t hidden_dim, uint32_t dtype, void* output, void* stream);
int moe_ep_entry_flat(const int32_t* pair_token, const int32_t* pair_flat,
                      const int64_t* pair_start, int64_t num_pairs,
                      const uint32_t* expert_indices, int32_t topk, int32_t num_experts,
                      int32_t num_ranks, int32_t* flat, void* stream);

/* Bytes of caller workspace that moe_fused_v2 needs for these sizes (0 for num_tokens == 0). */
size_t moe_fused_workspace_size(int64_t num_tokens, int32_t hidden_dim, int32_t intermediate_dim,
                                int32_t num_experts, int32_t topk, uint32_t moe_type,
                                uint32_t dtype);

/*
 * fused_moe with a status return and optional caller-owned workspace (workspace == NULL: use the
 * library pool; else it must hold moe_fused_workspace_size() bytes, 256-byte aligned, and must
 * not be in use by another call still running on the GPU).  Same semantics as fused_moe
 * (kernels/moe.cu:451-773) otherwise.
 */
int moe_fused_v2(const void* input, const void* gate_weights, const void* up_weights,
                 const void* down_weights, const float* routing_weights,
                 const uint32_t* expert_indices, void* output, int64_t num_tokens,
                 int32_t hidden_dim, int32_t intermediate_dim, int32_t num_experts, int32_t topk,
                 int32_t activation_type, uint32_t moe_type, uint32_t dtype, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * The expert computation of fused_moe without the combine: the weighted contribution
 * w[t,j] * y_{e(t,j)}(x_t) of every routed (t, j) (ids >= num_experts skipped) is written,
 * rounded to `dtype`, to row out_row[t*topk + j] of `output` ([rows, hidden_dim]; the rows of
 * routed slots must be distinct; other rows are left untouched).  This is the remote half of the
 * expert-parallel layer, which writes contributions straight into the buffer it sends back (no
 * counterpart in the reference, which has no multi-GPU path).
 */
int moe_fused_scatter(const void* input, const void* gate_weights, const void* up_weights,
                      const void* down_weights, const float* routing_weights,
                      const uint32_t* expert_indices, const int32_t* out_row, void* output,
                      int64_t num_tokens, int32_t hidden_dim, int32_t intermediate_dim,
                      int32_t num_experts, int32_t topk, int32_t activation_type,
                      uint32_t moe_type, uint32_t dtype, void* stream);

/*
 * Error bits the tensor-core kernels raised on `device` (a bounded wait that ran out; see
 * DevErr in csrc/common.cuh).  Synchronises the device.  clear != 0 resets them.
 */
uint32_t moe_device_error_bits(int32_t device, int32_t clear);

/*
 * Kernel family selection for the f16/bf16 expert GEMMs: 0 = automatic (tensor cores where the
 * shape allows: calls of at most 32 tokens take the decode kernels, weight-streaming with the
 * combine fused; larger ones the grouped GEMMs, whose Qwen3 GEMM-2 in fused_moe / moe_fused_v2
 * runs on CTA pairs, cta_group::2 with M = 256, when the hidden size is a multiple of 256),
 * 1 = always the SIMT kernels, 2 = tensor cores only (unsupported shapes then return
 * MOE_ERR_UNSUPPORTED), 3 = as 0 but no CTA pairs, 4 = as 0 with the Qwen3 GEMM-1 on CTA pairs
 * too and no decode kernels (experimental: correct, slower), 5 = as 0 without the decode
 * kernels, 6 = as 0 with the decode kernels at any token count.  Process-wide; returns the
 * previous value (-1 for an unknown path).
 */
int32_t moe_set_gemm_path(int32_t path);

/*
 * Number of SMs the persistent tensor-core GEMMs leave unused (0 by default, at most 128), so
 * that kernels running concurrently on other streams -- the collectives of the expert-parallel
 * exchange -- keep SMs of their own.  Process-wide; returns the previous value.
 */
int32_t moe_set_sm_reserve(int32_t sms);

/* Which family served the last moe_fused_v2 / fused_moe call of this thread: 1 SIMT, 2 tensor-core
 * grouped GEMMs, 3 tensor-core decode kernels, 0 none. */
int32_t moe_last_gemm_path(void);

/*
 * Benchmark instrumentation (counterpart of the NVTX ranges the reference's profiling binary
 * puts around each forward, src/bin/profile_fused_moe.rs:109-127).
 *
 * moe_kernel_launches: kernels this library has launched so far in this process.
 * moe_phase_timing(1): from now on every moe_fused_v2 / fused_moe call records CUDA events on
 *   its stream around route preparation, GEMM-1, GEMM-2 and the combine (resets the totals);
 *   moe_phase_timing(0) stops recording.
 * moe_phase_times: waits for the recorded events and writes the summed milliseconds of the four
 *   phases to ms[0..3] and the number of recorded calls to *calls.
 */
int64_t moe_kernel_launches(void);
int moe_phase_timing(int32_t enable);
int moe_phase_times(double* ms, int64_t* calls);

/*
 * moe_route_prep without any allocation.  This entry point has no counterpart in the reference.
 * It exists for callers that cannot allocate device memory during the step (an allocator that
 * owns all of HBM, a plugin handed only its buffers, a graph being recorded): instead of the pool,
 * its scratch is a fixed 2 MiB device array built into the library, held by every GPU that loads
 * the library until the process exits.  Same arguments, outputs and statuses as moe_route_prep;
 * requests needing more scratch than the array holds (2 * ceil(num_tokens * topk / 4096) *
 * num_experts > 524288 ints, e.g. more than 8,388,608 routed rows at 128 experts) return
 * MOE_ERR_WORKSPACE without launching anything.  All calls share the array, so calls that overlap
 * on the GPU race: serialise them (one stream).  The first call on a device sets it up (resolves
 * the array's address with that device current); make it before any stream capture.
 */
int moe_route_prep_noalloc(const uint32_t* expert_indices, const float* routing_weights,
                           int64_t num_tokens, int32_t topk, int32_t num_experts,
                           int32_t* expert_offsets, int32_t* sorted_token_ids,
                           float* sorted_weights, void* stream);

/*
 * Peer-mapped buffers and arrival flags for the expert-parallel exchange over NVLink (no
 * counterpart in the reference, which has no multi-GPU path).  Rows move into a peer's landing
 * buffer either by SM stores fused with the kernels that produce them (moe_ep_push_pairs,
 * moe_segment_sum_push below: the default "push" transport of expert_parallel.py) or by copy
 * engine (moe_copy_async: the "copy" transport, no SM time).
 *
 * moe_peer_alloc: device memory on the current device that other processes can map, zero-filled;
 *   writes the pointer and a MOE_PEER_HANDLE_BYTES-byte handle to pass to the other ranks.
 * moe_peer_free: frees a moe_peer_alloc buffer (after every peer has closed its mapping).
 * moe_peer_open / moe_peer_close: map / unmap another process's buffer on the current device.
 * moe_copy_async: `bytes` from src to dst on `stream` (either side may be a peer mapping).
 * moe_peer_signal: after the work before it on `stream`, stores `value` with release semantics
 *   (system scope) to each of the `count` (<= 64) 32-bit flags flag_addrs[0..count).
 * moe_peer_wait: stream-ordered wait until every flags[i] (i < count <= 64) has reached `value`
 *   (flag - value >= 0 as int32); after timeout_ns it sets bit 64 of the device error word
 *   (moe_device_error_bits) and lets the stream continue.
 */
/*
 * The same exchange with the rows moved by SM stores over NVLink, fused with the kernels that
 * produce them (no staging buffer, no copy engine), for num_ranks <= 32:
 *
 * moe_ep_push_pairs: dispatch of chunk `chunk`, fused with moe_ep_pack: the pairs
 *   [pair_offsets[chunk*num_ranks], pair_offsets[(chunk+1)*num_ranks]) (moe_route_prep_ex
 *   offsets over the moe_ep_dest_groups groups, read on the device) are written to
 *   dst_rows[d] + i rows and dst_meta[d] + i metadata rows (2*topk int32: local expert ids, then
 *   weight bits, as moe_ep_pack) for the i-th pair of destination d; slot_count (optional) as
 *   moe_ep_pack.  dst_rows / dst_meta: num_ranks device addresses, 16-byte aligned, usually in
 *   peers' moe_peer_alloc buffers.
 * moe_segment_sum_push: moe_segment_sum_rows whose output row r goes to
 *   dst[s] + (r - first_row[s]) rows for first_row[s] <= r < first_row[s+1]
 *   (first_row: num_ranks + 1 ascending offsets from 0 to num_segments); f16/bf16 only,
 *   hidden_dim a multiple of 8.
 * Both end with a system-scope fence, so a moe_peer_signal enqueued after them on the same
 * stream publishes their rows.  blocks = 0: one 128-thread block per SM (each fits beside a
 * persistent GEMM block).
 */
int moe_ep_push_pairs(const void* input, const int32_t* pair_token, const int32_t* pair_flat,
                      const int32_t* pair_offsets, int32_t chunk, const uint32_t* expert_indices,
                      const float* routing_weights, int32_t topk, int32_t num_experts,
                      int32_t num_ranks, int32_t hidden_dim, uint32_t dtype,
                      void* const* dst_rows, void* const* dst_meta, int32_t* slot_count,
                      int32_t blocks, void* stream);
int moe_segment_sum_push(const void* rows_in, const int64_t* segment_start, int64_t num_segments,
                         int32_t hidden_dim, uint32_t dtype, int32_t num_ranks,
                         void* const* dst, const int64_t* first_row, int32_t blocks,
                         void* stream);

#define MOE_PEER_HANDLE_BYTES 64
int moe_peer_alloc(size_t bytes, void** ptr, uint8_t* handle);
int moe_peer_free(void* ptr);
int moe_peer_open(const uint8_t* handle, void** ptr);
int moe_peer_close(void* ptr);
int moe_copy_async(void* dst, const void* src, size_t bytes, void* stream);
int moe_peer_signal(uint32_t* const* flag_addrs, int32_t count, uint32_t value, void* stream);
int moe_peer_wait(const uint32_t* flags, int32_t count, uint32_t value, int64_t timeout_ns,
                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CANDLE_MOE_B200_H */
