// Arrival flags of the expert-parallel exchange over peer-mapped memory.
//
// Rows travel between GPUs into a peer's IPC-mapped landing buffer either by SM stores fused
// with the kernels that produce them (the default "push" transport: moe_ep_push_pairs and
// moe_segment_sum_push in ep_kernels.cu, which share the SMs with the grouped GEMMs) or by copy
// engine (the "copy" transport: cudaMemcpyAsync, no SM time).  Either way the arrival signal is
// this file's kernel: after a rank's rows to every peer are written (stream-ordered behind
// them), one thread per peer release-stores an epoch number into that peer's flag array, and the
// receiving rank's compute stream runs a bounded acquire-load wait on its own flags before the
// kernels that read the rows.  The reference has no multi-GPU path.
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// flag i of the targets <- value (each target is a slot in some peer's flag array)
__global__ void peer_signal_kernel(PeerFlagPtrs targets, int count, uint32_t value) {
  const int i = threadIdx.x;
  if (i < count) st_release_sys(targets.p[i], value);
}

// Wait until every flags[i] (i < count) has reached `value` (wrap-safe comparison; a peer may
// already be at a later epoch).  Gives up after timeout_ns, sets kErrPeerWait and returns, so a
// peer that never signals ends in an error status instead of a hung stream.
__global__ void peer_wait_kernel(const uint32_t* flags, int count, uint32_t value,
                                 unsigned long long timeout_ns, uint32_t* err) {
  const int i = threadIdx.x;
  if (i >= count) return;
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (static_cast<int32_t>(ld_acquire_sys(flags + i) - value) >= 0) return;
    if (global_ns() - t0 > timeout_ns) {
      atomicOr(err, kErrPeerWait);
      return;
    }
    __nanosleep(128);
  }
}

int launch_peer_signal(const PeerFlagPtrs& targets, int count, uint32_t value, cudaStream_t s) {
  if (count < 0 || count > kMaxPeerFlags) return 1;
  if (count == 0) return 0;
  peer_signal_kernel<<<1, 32 * ((count + 31) / 32), 0, s>>>(targets, count, value);
  return 0;
}

int launch_peer_wait(const uint32_t* flags, int count, uint32_t value,
                     unsigned long long timeout_ns, uint32_t* err, cudaStream_t s) {
  if (count < 0 || count > kMaxPeerFlags) return 1;
  if (count == 0) return 0;
  peer_wait_kernel<<<1, 32 * ((count + 31) / 32), 0, s>>>(flags, count, value, timeout_ns, err);
  return 0;
}

}  // namespace cmoe
