// Internal interface between the C-ABI layer (capi.cu) and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cmoe {

// ---- capi.cu ---------------------------------------------------------------------------------
// Adds n to the count moe_kernel_launches() reports (for entry points outside capi.cu).
void add_launches(int64_t n);

// ---- router.cu -------------------------------------------------------------------------------
int launch_router(const float* logits, float* w, int32_t* idx, int32_t* src, int num_experts,
                  int num_tokens, int k, int renorm, int num_sms, cudaStream_t stream);

// ---- router_proj.cu (R0: gate projection fused with the softmax + top-k) ---------------------
struct RouterProjParams {
  float* out_w;          // [T, k]
  int32_t* out_idx;      // [T, k]
  int32_t* out_src;      // [T, k] = j*T + t
  float* logits;         // [T, E] f32 copy of the logits, or null
  uint32_t* err;         // device error word
  int num_tokens, H, k, renorm;
};
int router_project_max_k();
bool router_project_set_attributes();
int launch_router_project(int dtype, int E, const CUtensorMap& x, const CUtensorMap& w,
                          const RouterProjParams& p, int grid, cudaStream_t s);

// ---- route_prep.cu ---------------------------------------------------------------------------
size_t route_prep_scratch_bytes(int64_t rows, int E);
int route_prep_max_experts();
bool route_prep_set_attributes();
// zero / zero_n: words cleared before the tables are complete (the decode kernels' counters).
int launch_route_prep(const uint32_t* idx, const float* wts, int64_t num_tokens, int k, int E,
                      int bm, int32_t* offsets, int32_t* tile_prefix, int32_t* s_token,
                      float* s_weight, int32_t* s_flat, void* scratch, cudaStream_t stream,
                      uint32_t* zero = nullptr, int64_t zero_n = 0);

// ---- moe_simt.cu -----------------------------------------------------------------------------
struct SimtParams {
  const void* a;                // GEMM-1: x [T, K]; GEMM-2: intermediate [rows, K]
  const void* b0;               // GEMM-1: gate [E, K, N]; GEMM-2: down [E, K, N] or up [E, N, K]
  const void* b1;               // GEMM-1 Qwen3: up [E, K, N]
  const int32_t* offsets;       // [E+2]
  const int32_t* tile_prefix;   // [E+1], tile height simt_tile_m()
  const int32_t* sorted_token;  // [rows]
  const int32_t* sorted_flat;   // [rows]
  const float* sorted_w;        // [rows]
  void* out;                    // GEMM-1: intermediate [rows, N]; GEMM-2: slot [T*k, N] / out [T, N]
  const int32_t* out_row;       // GEMM-2 only: output row of flat index t*k+j (null: the flat index)
  int N, K, E, act;
};
int simt_tile_m();
int launch_simt_gemm(int dtype, int mode, const SimtParams& p, int64_t mtile_bound,
                     cudaStream_t s);
int launch_combine(int dtype, const void* slot, const uint32_t* idx, int64_t num_tokens, int k,
                   int H, int E, void* out, int num_sms, cudaStream_t s);
int launch_gather_rows(int dtype, const void* src, const int32_t* index, int64_t rows, int H,
                       void* dst, int num_sms, cudaStream_t s);
int launch_combine_indirect(int dtype, const void* rows_buf, const int32_t* flat, int64_t rows,
                            int64_t num_tokens, int k, int H, int32_t* inv, void* out,
                            int num_sms, cudaStream_t s);

// ---- moe_sm100.cu ----------------------------------------------------------------------------
// GEMM modes shared by both grouped-GEMM families
enum GemmMode : int {
  kModeG1Dual = 0,    // Qwen3 GEMM-1: act(x.G) * (x.U)
  kModeG1Single = 1,  // Nomic GEMM-1: act(x.G)
  kModeG2MN = 2,      // Qwen3 GEMM-2: h.D (D_e [I,H], N contiguous) * w
  kModeG2K = 3,       // Nomic GEMM-2: h.U^T (U_e [H,I], K contiguous) * w
};

struct Sm100Params {
  const void* a_rows;           // GEMM-1: x [T, K] (rows gathered by sorted_token); else unused
  const int32_t* offsets;       // [E+2]
  const int32_t* tile_prefix;   // [E+1], tile height sm100_tile_m()
  const int32_t* sorted_token;  // [rows]
  const int32_t* sorted_flat;   // [rows]
  const float* sorted_w;        // [rows]
  void* out;                    // GEMM-1: intermediate [rows, N]; GEMM-2: slot [T*k, N] / out [T, N]
  const int32_t* out_row;       // GEMM-2 only: output row of flat index t*k+j (null: the flat index)
  int N;                        // output columns (I for GEMM-1, H for GEMM-2)
  int K;                        // reduction length (H for GEMM-1, I for GEMM-2)
  int E;
  int act;
  int n_tiles;                  // N / output columns per tile
  uint32_t* tile_counter;       // zeroed before the launch: next unclaimed tile
  uint32_t* err;                // device error word
};
int sm100_tile_m();
int sm100_tile_k();
size_t sm100_smem_bytes(int num_experts);
int sm100_max_experts();
bool sm100_set_attributes();
// Output columns covered by one tile of `mode` with B tile width bn (128 or 256).
int sm100_out_cols(int mode, int bn);
int launch_sm100_gemm(int dtype, int mode, int bn, const CUtensorMap& a, const CUtensorMap& b0,
                      const CUtensorMap& b1, const Sm100Params& p, int grid, cudaStream_t s);

// ---- moe_tf32.cu (G1/G2 for f32 operands: three TF32 products on the tensor cores) ----------
bool tf32x3_set_attributes();
// Output columns of one tile of `mode` when the GEMM has N output columns.
int tf32x3_out_cols(int mode, int N);
int launch_tf32x3_gemm(int mode, int bn, const CUtensorMap& a, const CUtensorMap& b0,
                       const CUtensorMap& b1, const Sm100Params& p, int grid, cudaStream_t s);

// ---- moe_decode.cu (D1: decode-sized calls, weights as the MMA's A operand, stream-K) -------
struct DecodeParams {
  const void* b_src;            // GEMM-1: x [T, K]; GEMM-2: intermediate [rows, K]
  const int32_t* offsets;       // [E+2] route preparation offsets
  const int32_t* chunk_prefix;  // [E+1] route preparation tile prefix, tile height = chunk rows
  const int32_t* sorted_token;  // [rows]
  const int32_t* sorted_flat;   // [rows]
  const float* sorted_w;        // [rows]
  const uint32_t* idx;          // [T*k] expert ids (GEMM-2's fused combine)
  void* out;                    // GEMM-1: intermediate [rows, M]; GEMM-2: slot rows [T*k, M]
  void* final_out;              // GEMM-2: output [T, M]
  float* partials;              // decode_partial_bytes(): stream-K partial sums
  uint32_t* unit_counter;       // [4 * units], zeroed before the launch
  uint32_t* tile_counter;       // [4 * M/128], zeroed before the launch (GEMM-2)
  uint32_t* err;                // device error word
  int M;                        // weight output columns (I for GEMM-1, H for GEMM-2)
  int K;                        // reduction length (H for GEMM-1, I for GEMM-2)
  int E, act, k, num_tokens;
};
int decode_max_experts();
int decode_max_grid();
// Rows of one expert per MMA (the B operand's N) for a call of num_tokens tokens.
int decode_chunk_rows(int64_t num_tokens);
size_t decode_partial_bytes(int n, int grid);
bool decode_set_attributes();
int launch_decode_ffn(int dtype, int mode, int n, const CUtensorMap& a0, const CUtensorMap& a1,
                      const DecodeParams& p, int grid, cudaStream_t s);

// ---- ep_kernels.cu -------------------------------------------------------------------------
constexpr int kMaxEpBins = 12288;  // (chunk, rank) counters of ep_dest_groups (48 KB smem)
int launch_ep_dest_groups(const uint32_t* idx, int64_t T, int k, int E, int G,
                          int64_t tokens_per_chunk, int32_t* groups, int64_t* asg, int chunks,
                          int num_sms, cudaStream_t s);
int launch_ep_pack(int dtype, const void* x, const int32_t* pair_token, const int32_t* pair_flat,
                   int64_t U, const int32_t* n_dev, const uint32_t* idx, const float* w, int k,
                   int E, int G, int H, void* rows, int32_t* meta, int32_t* count, int num_sms,
                   cudaStream_t s);
int launch_segment_sum_rows(int dtype, const void* in, const int64_t* start, int64_t R, int H,
                            void* out, int num_sms, cudaStream_t s);
int launch_ep_entry_flat(const int32_t* pair_token, const int32_t* pair_flat,
                         const int64_t* start, int64_t U, const uint32_t* idx, int k, int E,
                         int G, int32_t* flat, int num_sms, cudaStream_t s);

// fused exchange kernels (ep_kernels.cu): destinations in peer-mapped landing buffers
constexpr int kMaxEpRanks = 32;
struct EpPeerRows {
  char* rows[kMaxEpRanks];  // per destination: first row of this rank's block
  char* meta[kMaxEpRanks];
};
struct EpPeerReturn {
  char* dst[kMaxEpRanks];             // per origin: first row of this rank's block
  int64_t first[kMaxEpRanks + 1];     // output rows [first[s], first[s+1]) go to origin s
};
int launch_ep_push_pairs(int dtype, const void* x, const int32_t* pair_token,
                         const int32_t* pair_flat, const int32_t* off, int c,
                         const uint32_t* idx, const float* w, int k, int E, int G, int H,
                         const EpPeerRows& tab, int32_t* count, int blocks, cudaStream_t s);
int launch_segment_sum_push(int dtype, const void* in, const int64_t* start, int64_t R, int H,
                            int G, const EpPeerReturn& tab, int blocks, cudaStream_t s);

// GEMM-2 (Qwen3 down projection) on CTA pairs, cta_group::2 (moe_sm100_pair.cu)
size_t sm100_pair_smem_bytes(int num_experts);
bool sm100_pair_set_attributes();
int sm100_pair_max_clusters();
int launch_sm100_gemm2_pair(int dtype, const CUtensorMap& a, const CUtensorMap& b,
                            const Sm100Params& p, int pairs, cudaStream_t s);
int launch_sm100_gemm1_pair(int dtype, const CUtensorMap& g, const CUtensorMap& u,
                            const Sm100Params& p, int pairs, cudaStream_t s);

// arrival flags of the expert-parallel exchange (peer.cu)
constexpr int kMaxPeerFlags = 64;
struct PeerFlagPtrs {
  uint32_t* p[kMaxPeerFlags];
};
int launch_peer_signal(const PeerFlagPtrs& targets, int count, uint32_t value, cudaStream_t s);
int launch_peer_wait(const uint32_t* flags, int count, uint32_t value,
                     unsigned long long timeout_ns, uint32_t* err, cudaStream_t s);

}  // namespace cmoe
