// P1: token -> expert route preparation (replaces kernels/preprocessing.cuh:5-313).
//
// Outputs, for the (token, slot) rows of a [T,k] index matrix:
//   offsets[E+2]      exclusive prefix of per-expert row counts, offsets[E] = routed rows,
//                     offsets[E+1] = largest count (preprocessing.cuh:35-46)
//   tile_prefix[E+1]  exclusive prefix of ceil(count_e / bm): the m-tile schedule of the grouped
//                     GEMM that follows (bm = its tile height)
//   sorted_token[r]   token id of sorted row r (preprocessing.cuh:55-57)
//   sorted_weight[r]  routing weight of sorted row r
//   sorted_flat[r]    flat index t*k + j of sorted row r
// Rows whose expert id is >= E are skipped, as in preprocessing.cuh:29.  Unlike the reference
// (atomic slot claims, so the order within an expert varies run to run) the order within an
// expert is ascending flat index, i.e. a stable counting sort; counts and offsets are identical.
//
// Large inputs use three kernels: per-block histograms (shared-memory atomics), one scan block
// (warp scans over experts and over blocks), and a stable scatter in which each warp ranks its
// rows with __match_any_sync and warps are ordered through a small per-warp count table.  Inputs
// of at most kPrepRows rows run all three phases in one CTA.
#include <stdint.h>

#include <atomic>
#include <climits>
#include <mutex>

#include "../../include/candle_moe.h"
#include "common.cuh"
#include "kernels.h"

namespace cmoe {

constexpr int kPrepRows = 4096;   // rows per block
constexpr int kPrepThreads = 512;  // 16 warps
constexpr int kPrepWarps = kPrepThreads / 32;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Histogram of block b's rows into s_cnt (shared, E entries, zeroed by the caller).
__device__ __forceinline__ void prep_histogram(const uint32_t* __restrict__ idx, int64_t lo,
                                               int64_t hi, int E, int* s_cnt) {
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const uint32_t e = __ldg(idx + i);
    if (e < static_cast<uint32_t>(E)) atomicAdd(&s_cnt[e], 1);
  }
}

// Stable scatter of rows [lo, hi) given each expert's first output position in s_run (shared,
// advanced in place).  s_wc is a kPrepWarps x E table of epoch-stamped per-warp counts.
__device__ __forceinline__ void prep_scatter_rows(const uint32_t* __restrict__ idx,
                                                  const float* __restrict__ wts, int64_t lo,
                                                  int64_t hi, int k, int E, int* s_run,
                                                  uint32_t* s_wc, int32_t* __restrict__ s_token,
                                                  float* __restrict__ s_weight,
                                                  int32_t* __restrict__ s_flat) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t epoch = 0;
  for (int64_t b0 = lo; b0 < hi; b0 += kPrepThreads) {
    ++epoch;
    const int64_t i = b0 + threadIdx.x;
    uint32_t e = static_cast<uint32_t>(E);
    if (i < hi) {
      e = __ldg(idx + i);
      if (e > static_cast<uint32_t>(E)) e = static_cast<uint32_t>(E);
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lanemask_lt());
    const bool leader = (__ffs(peers) - 1) == lane;
    const int wcount = __popc(peers);
    if (leader && e < static_cast<uint32_t>(E)) s_wc[warp * E + e] = (epoch << 8) | static_cast<uint32_t>(wcount);
    __syncthreads();
    if (e < static_cast<uint32_t>(E)) {
      int pos = s_run[e] + rank;
      for (int w2 = 0; w2 < warp; ++w2) {
        const uint32_t c = s_wc[w2 * E + e];
        if ((c >> 8) == epoch) pos += static_cast<int>(c & 0xffu);
      }
      if (s_token) s_token[pos] = static_cast<int32_t>(i / k);
      if (s_weight) s_weight[pos] = __ldg(wts + i);
      if (s_flat) s_flat[pos] = static_cast<int32_t>(i);
    }
    __syncthreads();
    if (leader && e < static_cast<uint32_t>(E)) atomicAdd(&s_run[e], wcount);
    __syncthreads();
  }
}

// Exclusive scan over experts by warp 0: writes offsets[0..E+1] and tile_prefix[0..E].
// s_cnt holds the per-expert counts; s_run receives the exclusive offsets.
__device__ __forceinline__ void prep_scan_experts(const int* s_cnt, int E, int bm, int* s_run,
                                                  int32_t* __restrict__ offsets,
                                                  int32_t* __restrict__ tile_prefix) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  int run = 0, trun = 0, mx = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int c = e < E ? s_cnt[e] : 0;
    const int t = (c + bm - 1) / bm;
    const int ic = warp_incl_scan(c);
    const int it = warp_incl_scan(t);
    if (e < E) {
      offsets[e] = run + ic - c;
      s_run[e] = run + ic - c;
      if (tile_prefix) tile_prefix[e] = trun + it - t;
    }
    int m = c;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    mx = max(mx, m);
    run += __shfl_sync(0xffffffffu, ic, 31);
    trun += __shfl_sync(0xffffffffu, it, 31);
  }
  if (lane == 0) {
    offsets[E] = run;
    offsets[E + 1] = mx;
    if (tile_prefix) tile_prefix[E] = trun;
  }
}

// ---- small inputs: everything in one CTA --------------------------------------------------
// Launched as a programmatic dependent: it waits for the previous kernel (the router, whose
// picks it reads) and at once lets the next one launch, which waits in turn for this kernel's
// completion before it reads the tables.  `zero` / `zero_n`: words to clear for the next kernels
// (the decode kernels' counters), in place of a separate memset.
__global__ void __launch_bounds__(kPrepThreads) route_prep_single_kernel(
    const uint32_t* __restrict__ idx, const float* __restrict__ wts, int64_t rows, int k, int E,
    int bm, int32_t* __restrict__ offsets, int32_t* __restrict__ tile_prefix,
    int32_t* __restrict__ s_token, float* __restrict__ s_weight, int32_t* __restrict__ s_flat,
    uint32_t* __restrict__ zero, int64_t zero_n) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int64_t i = threadIdx.x; i < zero_n; i += blockDim.x) zero[i] = 0u;
  extern __shared__ int smem_i[];
  int* s_cnt = smem_i;
  int* s_run = smem_i + E;
  uint32_t* s_wc = reinterpret_cast<uint32_t*>(smem_i + 2 * E);
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  for (int e = threadIdx.x; e < kPrepWarps * E; e += blockDim.x) s_wc[e] = 0;
  __syncthreads();
  prep_histogram(idx, 0, rows, E, s_cnt);
  __syncthreads();
  prep_scan_experts(s_cnt, E, bm, s_run, offsets, tile_prefix);
  __syncthreads();
  prep_scatter_rows(idx, wts, 0, rows, k, E, s_run, s_wc, s_token, s_weight, s_flat);
}

// ---- large inputs: histogram / scan / scatter ----------------------------------------------
__global__ void __launch_bounds__(kPrepThreads) route_prep_count_kernel(
    const uint32_t* __restrict__ idx, int64_t rows, int E, int nb, int32_t* __restrict__ counts) {
  extern __shared__ int smem_i[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) smem_i[e] = 0;
  __syncthreads();
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kPrepRows;
  const int64_t hi = lo + kPrepRows < rows ? lo + kPrepRows : rows;
  prep_histogram(idx, lo, hi, E, smem_i);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[static_cast<int64_t>(e) * nb + blockIdx.x] = smem_i[e];
}

__global__ void __launch_bounds__(1024) route_prep_scan_kernel(
    const int32_t* __restrict__ counts, int E, int nb, int bm, int32_t* __restrict__ offsets,
    int32_t* __restrict__ tile_prefix, int32_t* __restrict__ base) {
  extern __shared__ int smem_i[];
  int* s_cnt = smem_i;
  int* s_run = smem_i + E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int e = warp; e < E; e += nwarps) {
    int s = 0;
    for (int b = lane; b < nb; b += 32) s += counts[static_cast<int64_t>(e) * nb + b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) s_cnt[e] = s;
  }
  __syncthreads();
  prep_scan_experts(s_cnt, E, bm, s_run, offsets, tile_prefix);
  __syncthreads();
  for (int e = warp; e < E; e += nwarps) {
    int run = s_run[e];
    for (int b0 = 0; b0 < nb; b0 += 32) {
      const int b = b0 + lane;
      const int c = b < nb ? counts[static_cast<int64_t>(e) * nb + b] : 0;
      const int ic = warp_incl_scan(c);
      if (b < nb) base[static_cast<int64_t>(e) * nb + b] = run + ic - c;
      run += __shfl_sync(0xffffffffu, ic, 31);
    }
  }
}

__global__ void __launch_bounds__(kPrepThreads) route_prep_scatter_kernel(
    const uint32_t* __restrict__ idx, const float* __restrict__ wts, int64_t rows, int k, int E,
    int nb, const int32_t* __restrict__ base, int32_t* __restrict__ s_token,
    float* __restrict__ s_weight, int32_t* __restrict__ s_flat) {
  extern __shared__ int smem_i[];
  int* s_run = smem_i;
  uint32_t* s_wc = reinterpret_cast<uint32_t*>(smem_i + E);
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_run[e] = base[static_cast<int64_t>(e) * nb + blockIdx.x];
  for (int e = threadIdx.x; e < kPrepWarps * E; e += blockDim.x) s_wc[e] = 0;
  __syncthreads();
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kPrepRows;
  const int64_t hi = lo + kPrepRows < rows ? lo + kPrepRows : rows;
  prep_scatter_rows(idx, wts, lo, hi, k, E, s_run, s_wc, s_token, s_weight, s_flat);
}

size_t route_prep_scratch_bytes(int64_t rows, int E) {
  const int64_t nb = (rows + kPrepRows - 1) / kPrepRows;
  return nb <= 1 ? 0 : static_cast<size_t>(2 * nb * E) * sizeof(int32_t);
}

int route_prep_max_experts() { return 2048; }

// Once per device: allow the shared-memory sizes that large expert counts need.
bool route_prep_set_attributes() {
  bool ok = cudaFuncSetAttribute(route_prep_single_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(2 * 2048 + kPrepWarps * 2048) * 4) == cudaSuccess;
  ok &= cudaFuncSetAttribute(route_prep_scatter_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(2048 + kPrepWarps * 2048) * 4) == cudaSuccess;
  return ok;
}

// scratch: route_prep_scratch_bytes() bytes (may be null when that is 0).
int launch_route_prep(const uint32_t* idx, const float* wts, int64_t num_tokens, int k, int E,
                      int bm, int32_t* offsets, int32_t* tile_prefix, int32_t* s_token,
                      float* s_weight, int32_t* s_flat, void* scratch, cudaStream_t stream,
                      uint32_t* zero, int64_t zero_n) {
  if (E < 1 || E > route_prep_max_experts() || k < 1 || bm < 1) return 1;
  const int64_t rows = num_tokens * k;
  const int64_t nb = (rows + kPrepRows - 1) / kPrepRows;
  if (nb <= 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kPrepThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(2 * E + kPrepWarps * E) * sizeof(int);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, route_prep_single_kernel, idx, wts, rows, k, E, bm, offsets,
                              tile_prefix, s_token, s_weight, s_flat, zero, zero_n) == cudaSuccess
               ? 0
               : 1;
  }
  if (zero_n > 0 && cudaMemsetAsync(zero, 0, sizeof(uint32_t) * zero_n, stream) != cudaSuccess)
    return 1;
  if (nb > 0x7fffffff / E) return 1;
  int32_t* counts = static_cast<int32_t*>(scratch);
  int32_t* base = counts + nb * E;
  route_prep_count_kernel<<<static_cast<unsigned>(nb), kPrepThreads, E * sizeof(int), stream>>>(
      idx, rows, E, static_cast<int>(nb), counts);
  route_prep_scan_kernel<<<1, 1024, 2 * E * sizeof(int), stream>>>(
      counts, E, static_cast<int>(nb), bm, offsets, tile_prefix, base);
  route_prep_scatter_kernel<<<static_cast<unsigned>(nb), kPrepThreads,
                              (E + kPrepWarps * E) * sizeof(int), stream>>>(
      idx, wts, rows, k, E, static_cast<int>(nb), base, s_token, s_weight, s_flat);
  return 0;
}


// ---- route preparation without allocation ---------------------------------------------------
//
// Some callers cannot allocate device memory while they run this step: a serving loop whose
// allocator owns every byte of HBM and forbids side allocations, a framework plugin that is
// handed its buffers and must not call cudaMalloc, or code that records the step into a CUDA
// graph.  moe_route_prep_noalloc serves them: its scratch (the per-block histograms and block
// bases of the multi-block path, 2 * ceil(T*k / 4096) * E ints) lives in the fixed device array
// below, which every GPU that loads this library holds until the process exits.  Requests whose
// scratch would not fit are rejected with MOE_ERR_WORKSPACE before anything is launched.
//
// All calls share the one array.  Each call overwrites every scratch entry it later reads (the
// count kernel writes all histograms, the scan all bases), so nothing has to start at zero, but
// two calls that overlap on the GPU (different streams, or host threads racing on one device)
// race on the array: serialise them, e.g. on one stream.
//
// The first call on each device performs the set-up (it resolves the array's device address with
// cudaGetSymbolAddress and sets the kernels' shared-memory attributes, with that device current);
// make that first call before any stream capture begins.

constexpr int kNoAllocScratchInts = 1 << 19;  // 2 MiB
static __device__ __align__(256) int32_t g_route_prep_noalloc_scratch[kNoAllocScratchInts];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::atomic<int32_t*> g_noalloc_ptr[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device (set up on first use).
int32_t* noalloc_scratch_current_device(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    cudaGetLastError();
    *status = MOE_ERR_CUDA;
    return nullptr;
  }
  int32_t* p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (p) return p;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  p = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
  if (!p) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_route_prep_noalloc_scratch);
    if (e != cudaSuccess || addr == nullptr) {
      cudaGetLastError();
      *status = MOE_ERR_CUDA;
      return nullptr;
    }
    if (!route_prep_set_attributes()) {
      cudaGetLastError();
      *status = MOE_ERR_CUDA;
      return nullptr;
    }
    p = static_cast<int32_t*>(addr);
    g_noalloc_ptr[dev].store(p, std::memory_order_release);
  }
  return p;
}
}  // namespace

}  // namespace cmoe

extern "C" __attribute__((visibility("default"))) int moe_route_prep_noalloc(
    const uint32_t* expert_indices, const float* routing_weights, int64_t num_tokens,
    int32_t topk, int32_t num_experts, int32_t* expert_offsets, int32_t* sorted_token_ids,
    float* sorted_weights, void* stream) {
  using namespace cmoe;
  if (num_tokens < 0 || topk <= 0 || num_experts <= 0) return MOE_ERR_INVALID_ARG;
  // an empty request reads nothing: only the offsets (all zero) are written
  if ((num_tokens > 0 && (!expert_indices || !routing_weights)) || !expert_offsets)
    return MOE_ERR_INVALID_ARG;
  if (num_experts > route_prep_max_experts() || num_tokens * topk > INT32_MAX)
    return MOE_ERR_UNSUPPORTED;
  const size_t need = route_prep_scratch_bytes(num_tokens * topk, num_experts);
  if (need > sizeof(int32_t) * static_cast<size_t>(kNoAllocScratchInts)) return MOE_ERR_WORKSPACE;
  int status = MOE_OK;
  int32_t* scratch = noalloc_scratch_current_device(&status);
  if (!scratch) return status;
  if (launch_route_prep(expert_indices, routing_weights, num_tokens, topk, num_experts, 1,
                        expert_offsets, nullptr, sorted_token_ids, sorted_weights, nullptr,
                        scratch, static_cast<cudaStream_t>(stream)) != 0)
    return MOE_ERR_UNSUPPORTED;
  if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
  add_launches(need ? 3 : 1);
  return MOE_OK;
}
