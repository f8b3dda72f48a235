// src/ffi.rs for the candle-moe crate linked against libcandle_moe_b200.so.
//
// The first two declarations are the symbols the crate's src/lib.rs calls (src/ffi.rs:15-24 and
// :45-62 of the reference crate), with the same argument order, types and meaning; lib.rs keeps
// calling them unchanged.  num_tokens of topk_softmax stays c_int: the library's header declares
// int32_t, matching this caller (the reference's C definition said int64_t).  The remaining
// declarations are the library's extensions (include/candle_moe.h): the per-thread status of the
// two drop-in calls, which the reference never reported, and status-returning variants.
//
// Not compiled in the image this library was built in (no cargo there): unverified.
use core::ffi::{c_char, c_int, c_void};

unsafe extern "C" {
    // ---- drop-in symbols (called by src/lib.rs) -------------------------------------------

    /// Softmax over the experts of each token's router logits, then the top-k picks.
    /// gating_output [num_tokens, num_experts] f32; topk_weight [num_tokens, topk] f32 out;
    /// topk_indices, token_expert_indices [num_tokens, topk] u32 out.  num_experts: a power of
    /// two <= 256.  Failures are reported by moe_last_status().
    pub(crate) fn topk_softmax(
        gating_output: *const c_void,
        topk_weight: *mut c_void,
        topk_indices: *const c_void,
        token_expert_indices: *const c_void,
        num_experts: c_int,
        num_tokens: c_int,
        topk: c_int,
        stream: *mut c_void,
    );

    /// The expert FFN of the routed tokens, weighted by the routing weights and summed per token
    /// into output [num_tokens, hidden_dim].  The output is overwritten (the zeroed output the
    /// crate passes, src/lib.rs:296, gives the same result).  dtype: 0 f16, 1 bf16, 2 f32;
    /// moe_type: 0 Qwen3 (gate/up/down), 1 Nomic (down_weights null).  Failures are reported by
    /// moe_last_status().
    pub(crate) fn fused_moe(
        input: *const c_void,
        gate_weights: *const c_void,
        up_weights: *const c_void,
        down_weights: *const c_void,
        routing_weights: *const c_void,
        expert_indices: *const c_void,
        output: *mut c_void,
        num_tokens: c_int,
        hidden_dim: c_int,
        intermediate_dim: c_int,
        num_experts: c_int,
        num_selected_experts: c_int,
        activation_type: c_int,
        moe_type: u32,
        dtype: u32,
        stream: *mut c_void,
    );

    // ---- status of the drop-in calls -------------------------------------------------------

    /// 0 when the last topk_softmax / fused_moe call of this thread succeeded.
    pub(crate) fn moe_last_status() -> c_int;
    /// A static, NUL-terminated description of a status code.
    pub(crate) fn moe_status_string(status: c_int) -> *const c_char;

    // ---- extensions --------------------------------------------------------------------------

    /// topk_softmax with a status return and optional renormalisation of the k weights.
    pub(crate) fn moe_topk_softmax_v2(
        gating_output: *const f32,
        topk_weights: *mut f32,
        topk_indices: *mut i32,
        token_expert_indices: *mut i32,
        num_experts: i32,
        num_tokens: i64,
        topk: i32,
        renormalize: i32,
        stream: *mut c_void,
    ) -> c_int;

    /// The router's Linear fused with topk_softmax: logits = input . gate_proj^T (f16/bf16),
    /// softmax, top-k; logits (f32 [num_tokens, num_experts]) may be null.
    pub(crate) fn moe_router_project_topk(
        input: *const c_void,
        gate_proj: *const c_void,
        num_tokens: i64,
        hidden_dim: i32,
        num_experts: i32,
        topk: i32,
        renormalize: i32,
        dtype: u32,
        topk_weights: *mut f32,
        topk_indices: *mut i32,
        token_expert_indices: *mut i32,
        logits: *mut f32,
        stream: *mut c_void,
    ) -> c_int;

    /// Bytes of workspace moe_fused_v2 needs for a call of these sizes.
    pub(crate) fn moe_fused_workspace_size(
        num_tokens: i64,
        hidden_dim: i32,
        intermediate_dim: i32,
        num_experts: i32,
        topk: i32,
        moe_type: u32,
        dtype: u32,
    ) -> usize;

    /// fused_moe with a status return and an optional caller-owned workspace (null: the
    /// library's stream-ordered pool).
    pub(crate) fn moe_fused_v2(
        input: *const c_void,
        gate_weights: *const c_void,
        up_weights: *const c_void,
        down_weights: *const c_void,
        routing_weights: *const f32,
        expert_indices: *const u32,
        output: *mut c_void,
        num_tokens: i64,
        hidden_dim: i32,
        intermediate_dim: i32,
        num_experts: i32,
        topk: i32,
        activation_type: i32,
        moe_type: u32,
        dtype: u32,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: *mut c_void,
    ) -> c_int;
}
