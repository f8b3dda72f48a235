// Test-only shim compiled together with the reference's own kernel sources (see build_ref.sh).
// The reference runs its sort/align step (kernels/preprocessing.cuh:253-313) only inside
// fused_moe and exports no entry point for it; this shim includes that header inside its own
// namespace (so its kernels do not collide with the copies compiled into moe.cu) and exports one
// C entry point, plus a reader of the CUDA runtime's sticky launch error so that callers can
// tell which reference launches failed.
#include "common.cuh"
namespace refshim {
#include "preprocessing.cuh"
}

extern "C" __attribute__((visibility("default"))) void ref_preprocessing(
    const uint32_t* expert_indices, const float* routing_weights, int* expert_offsets,
    int* sorted_token_ids, float* sorted_weights, int num_tokens, int num_experts, int top_k,
    void* stream) {
  refshim::launch_preprocessing(expert_indices, routing_weights, expert_offsets, sorted_token_ids,
                                sorted_weights, num_tokens, num_experts, top_k,
                                reinterpret_cast<cudaStream_t>(stream));
}

extern "C" __attribute__((visibility("default"))) int ref_get_last_error(void) {
  return static_cast<int>(cudaGetLastError());
}
