// Bookkeeping kernels of the expert-parallel exchange (candle-moe_b200/expert_parallel.py).
//
// The reference has no multi-GPU path.  With G ranks owning E/G experts each, a token is sent
// once to every rank that owns at least one of its k experts.  These kernels turn the router's
// [T,k] expert ids into (token, rank) pairs, pack the pairs' rows and slot metadata for the
// all-to-all, and map the contributions that come back to the token slots they belong to.
#include <stdint.h>
#include <climits>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {

// groups[t*G + d] = (t / tokens_per_chunk) * G + d when token t has an expert on rank d, else
// INT32_MAX (above any group count, so route preparation ignores it).  Ids >= E (skipped
// everywhere) select no rank.
// With `asg` (nbins = chunks * G counters, zeroed by the caller), also counts the (token, slot)
// assignments per (chunk, rank): per-block shared-memory histogram, one global add per bin.
__global__ void __launch_bounds__(256) ep_dest_groups_kernel(const uint32_t* __restrict__ idx,
                                                             int64_t T, int k, int E, int El,
                                                             int G, int64_t tokens_per_chunk,
                                                             int32_t* __restrict__ groups,
                                                             unsigned long long* asg, int nbins) {
  extern __shared__ int s_hist[];
  if (asg) {
    for (int i = threadIdx.x; i < nbins; i += blockDim.x) s_hist[i] = 0;
    __syncthreads();
  }
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < T;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t mask = 0;  // G <= 32
    const int32_t chunk = static_cast<int32_t>(t / tokens_per_chunk);
    for (int j = 0; j < k; ++j) {
      const uint32_t e = __ldg(idx + t * k + j);
      if (e < static_cast<uint32_t>(E)) {
        mask |= 1u << (e / El);
        if (asg) atomicAdd(&s_hist[chunk * G + static_cast<int>(e / El)], 1);
      }
    }
    for (int d = 0; d < G; ++d)
      groups[t * G + d] = (mask >> d) & 1u ? chunk * G + d : INT32_MAX;
  }
  if (asg) {
    __syncthreads();
    for (int i = threadIdx.x; i < nbins; i += blockDim.x)
      if (s_hist[i]) atomicAdd(asg + i, static_cast<unsigned long long>(s_hist[i]));
  }
}

// For the U sorted (token, rank) pairs (pair_token[r], pair_flat[r] = t*G + d): copy x[t] to
// rows[r] (one warp per pair, 16-byte lanes) and write the pair's slot metadata: meta[r*2k + j] =
// local expert id of slot j if that slot's expert lives on rank d, else El; meta[r*2k + k + j] =
// the slot's routing weight bits (0 for foreign slots).  count[r] = slots of the pair.
// With n_dev, the pair count is read from device memory (at most U, the capacity), so the pack
// can be enqueued before the host knows the count.
template <typename V>
__global__ void __launch_bounds__(256) ep_pack_kernel(
    const V* __restrict__ x, const int32_t* __restrict__ pair_token,
    const int32_t* __restrict__ pair_flat, int64_t U, const int32_t* __restrict__ n_dev,
    const uint32_t* __restrict__ idx, const float* __restrict__ w, int k, int E, int El, int G,
    int vec_per_row, V* __restrict__ rows, int32_t* __restrict__ meta,
    int32_t* __restrict__ count) {
  if (n_dev) U = min(U, static_cast<int64_t>(max(__ldg(n_dev), 0)));
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp0; r < U; r += nwarps) {
    const int64_t t = __ldg(pair_token + r);
    const int d = __ldg(pair_flat + r) % G;
    const V* src = x + t * vec_per_row;
    V* dst = rows + r * vec_per_row;
    for (int c = lane; c < vec_per_row; c += 32) dst[c] = __ldg(src + c);
    if (lane < k) {
      const uint32_t e = __ldg(idx + t * k + lane);
      const bool mine = e < static_cast<uint32_t>(E) && static_cast<int>(e / El) == d;
      meta[r * 2 * k + lane] = mine ? static_cast<int32_t>(e % El) : El;
      meta[r * 2 * k + k + lane] = mine ? __float_as_int(__ldg(w + t * k + lane)) : 0;
      const uint32_t ballot = __ballot_sync(0xffffffffu >> (32 - k), mine);
      if (lane == 0) count[r] = __popc(ballot);
    }
  }
}

// Exact mode: the contributions of pair r come back as count[r] consecutive rows starting at
// start[r] (exclusive prefix of count), one per slot of the pair in slot order; record the token
// slot each row belongs to: flat[start[r] + i] = t*k + j for the pair's i-th slot j.
__global__ void __launch_bounds__(256) ep_entry_flat_kernel(
    const int32_t* __restrict__ pair_token, const int32_t* __restrict__ pair_flat,
    const int64_t* __restrict__ start, int64_t U, const uint32_t* __restrict__ idx, int k, int E,
    int El, int G, int32_t* __restrict__ flat) {
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < U;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = __ldg(pair_token + r);
    const int d = __ldg(pair_flat + r) % G;
    int64_t pos = __ldg(start + r);
    for (int j = 0; j < k; ++j) {
      const uint32_t e = __ldg(idx + t * k + j);
      if (e < static_cast<uint32_t>(E) && static_cast<int>(e / El) == d)
        flat[pos++] = static_cast<int32_t>(t * k + j);
    }
  }
}

// out[r, :] = sum of rows_in[start[r] .. start[r+1]) in order, f32 accumulation, one rounding:
// the per-rank partial of a (token, rank) pair from its slot contributions, which the scatter
// GEMM wrote consecutively in slot order.  Up to KC rows of a segment are loaded at once.
template <typename T, int V, int KC>
__global__ void __launch_bounds__(256) segment_sum_rows_kernel(const T* __restrict__ rows_in,
                                                               const int64_t* __restrict__ start,
                                                               int64_t R, int H,
                                                               T* __restrict__ out) {
  const int vec_per_row = H / V;
  const int64_t total = R * vec_per_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = v / vec_per_row;
    const int c = static_cast<int>(v - r * vec_per_row) * V;
    const int64_t s0 = __ldg(start + r), s1 = __ldg(start + r + 1);
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int64_t b = s0; b < s1; b += KC) {
      uint4 q[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const T* src = rows_in + (b + j < s1 ? b + j : s0) * H + c;
        if (V * sizeof(T) == 16) {
          q[j] = b + j < s1 ? __ldcs(reinterpret_cast<const uint4*>(src)) : make_uint4(0, 0, 0, 0);
        } else {
          T* qe = reinterpret_cast<T*>(&q[j]);
#pragma unroll
          for (int i = 0; i < V; ++i) qe[i] = b + j < s1 ? src[i] : Elem<T>::from_f(0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        if (b + j >= s1) continue;
        const T* qe = reinterpret_cast<const T*>(&q[j]);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += Elem<T>::to_f(qe[i]);
      }
    }
    T* dst = out + r * H + c;
    if (V * sizeof(T) == 16) {
      uint4 qo;
      T* qe = reinterpret_cast<T*>(&qo);
#pragma unroll
      for (int i = 0; i < V; ++i) qe[i] = Elem<T>::from_f(acc[i]);
      *reinterpret_cast<uint4*>(dst) = qo;
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) dst[i] = Elem<T>::from_f(acc[i]);
    }
  }
}

// ---- fused exchange kernels: SM stores over NVLink into peer-mapped landing buffers ---------

// Dispatch of chunk c, fused with the pack: pair r in [off[c*G], off[c*G+G]) (sorted by
// destination d, then token) goes to row (r - off[c*G + d]) of the block that this rank owns in
// d's landing buffer, tab.rows[d] (row bytes) and tab.meta[d] (2k ints).  One warp per pair;
// count[r] = slots of the pair (exact mode's bookkeeping).  Ends with a system-scope fence so
// the arrival flag stored after this kernel orders behind the rows.
// 128 threads x at most 48 registers (launch bounds for 10 blocks): one block fits beside a
// persistent GEMM CTA on every SM, so these kernels run while the GEMMs of another chunk do.
template <typename V>
__global__ void __launch_bounds__(128, 10) ep_push_pairs_kernel(
    const V* __restrict__ x, const int32_t* __restrict__ pair_token,
    const int32_t* __restrict__ pair_flat, const int32_t* __restrict__ off, int c,
    const uint32_t* __restrict__ idx, const float* __restrict__ w, int k, int E, int El, int G,
    int vec_per_row, const EpPeerRows tab, int32_t* __restrict__ count) {
  const int lane = threadIdx.x & 31;
  const int64_t p0 = __ldg(off + c * G), p1 = __ldg(off + c * G + G);
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  constexpr int kU = 4;  // 16-byte units in flight per lane
  for (int64_t r = p0 + warp0; r < p1; r += nwarps) {
    const int64_t t = __ldg(pair_token + r);
    const int d = __ldg(pair_flat + r) % G;
    const int64_t pos = r - __ldg(off + c * G + d);
    const V* src = x + t * vec_per_row;
    V* dst = reinterpret_cast<V*>(tab.rows[d]) + pos * vec_per_row;
    for (int c0 = 0; c0 < vec_per_row; c0 += 32 * kU) {
      V q[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int cc = c0 + u * 32 + lane;
        if (cc < vec_per_row) q[u] = __ldg(src + cc);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int cc = c0 + u * 32 + lane;
        if (cc < vec_per_row) dst[cc] = q[u];
      }
    }
    if (lane < k) {
      const uint32_t e = __ldg(idx + t * k + lane);
      const bool mine = e < static_cast<uint32_t>(E) && static_cast<int>(e / El) == d;
      int32_t* m = reinterpret_cast<int32_t*>(tab.meta[d]) + pos * 2 * k;
      m[lane] = mine ? static_cast<int32_t>(e % El) : El;
      m[k + lane] = mine ? __float_as_int(__ldg(w + t * k + lane)) : 0;
      const uint32_t ballot = __ballot_sync(0xffffffffu >> (32 - k), mine);
      if (lane == 0 && count) count[r] = __popc(ballot);
    }
  }
  __threadfence_system();
}

// Return of chunk c, fused with the slot sum: output row r (received-row order, grouped by
// origin s: rows [tab.first[s], tab.first[s+1])) = sum of rows_in[start[r] .. start[r+1]) in
// order, f32 accumulation, one rounding, stored to tab.dst[s] + (r - tab.first[s]) rows.  One warp
// per row, KC rows of a segment loaded at once.  Ends with a system-scope fence.
template <typename T, int KC>
__global__ void __launch_bounds__(128, 10) segment_sum_push_kernel(
    const T* __restrict__ rows_in, const int64_t* __restrict__ start, int64_t R, int H, int G,
    const EpPeerReturn tab) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int units = H / V;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp0; r < R; r += nwarps) {
    const int s = __popc(__ballot_sync(0xffffffffu, lane < G && tab.first[lane] <= r)) - 1;
    T* dst = reinterpret_cast<T*>(tab.dst[s]) + (r - tab.first[s]) * H;
    const int64_t s0 = __ldg(start + r), s1 = __ldg(start + r + 1);
    for (int u = lane; u < units; u += 32) {
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      for (int64_t b = s0; b < s1; b += KC) {
        uint4 q[KC];
#pragma unroll
        for (int j = 0; j < KC; ++j)
          q[j] = b + j < s1 ? __ldcs(reinterpret_cast<const uint4*>(rows_in + (b + j) * H) + u)
                            : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < KC; ++j) {
          if (b + j >= s1) continue;
          const T* qe = reinterpret_cast<const T*>(&q[j]);
#pragma unroll
          for (int i = 0; i < V; ++i) acc[i] += Elem<T>::to_f(qe[i]);
        }
      }
      uint4 qo;
      T* qe = reinterpret_cast<T*>(&qo);
#pragma unroll
      for (int i = 0; i < V; ++i) qe[i] = Elem<T>::from_f(acc[i]);
      reinterpret_cast<uint4*>(dst)[u] = qo;
    }
  }
  __threadfence_system();
}

static unsigned ep_grid(int64_t work, int num_sms) {
  int64_t b = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}

int launch_ep_dest_groups(const uint32_t* idx, int64_t T, int k, int E, int G,
                          int64_t tokens_per_chunk, int32_t* groups, int64_t* asg, int chunks,
                          int num_sms, cudaStream_t s) {
  if (G < 1 || G > 32 || E % G != 0 || tokens_per_chunk < 1) return 1;
  const int nbins = asg ? chunks * G : 0;
  if (asg && (chunks < 1 || nbins > kMaxEpBins || (T + tokens_per_chunk - 1) / tokens_per_chunk > chunks))
    return 1;
  if (asg && cudaMemsetAsync(asg, 0, sizeof(int64_t) * nbins, s) != cudaSuccess) return 1;
  if (T <= 0) return 0;
  ep_dest_groups_kernel<<<ep_grid(T, num_sms), 256, nbins * sizeof(int), s>>>(
      idx, T, k, E, E / G, G, tokens_per_chunk, groups,
      reinterpret_cast<unsigned long long*>(asg), nbins);
  return 0;
}

int launch_ep_pack(int dtype, const void* x, const int32_t* pair_token, const int32_t* pair_flat,
                   int64_t U, const int32_t* n_dev, const uint32_t* idx, const float* w, int k,
                   int E, int G, int H, void* rows, int32_t* meta, int32_t* count, int num_sms,
                   cudaStream_t s) {
  if (G < 1 || G > 32 || E % G != 0 || k > 32) return 1;
  if (U <= 0) return 0;
  const size_t row_bytes = static_cast<size_t>(H) * (dtype == kF32 ? 4 : 2);
  const unsigned grid = ep_grid(U * 32, num_sms);
  if (row_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(rows) % 16 == 0)
    ep_pack_kernel<uint4><<<grid, 256, 0, s>>>(
        static_cast<const uint4*>(x), pair_token, pair_flat, U, n_dev, idx, w, k, E, E / G, G,
        static_cast<int>(row_bytes / 16), static_cast<uint4*>(rows), meta, count);
  else
    ep_pack_kernel<uint16_t><<<grid, 256, 0, s>>>(
        static_cast<const uint16_t*>(x), pair_token, pair_flat, U, n_dev, idx, w, k, E, E / G, G,
        static_cast<int>(row_bytes / 2), static_cast<uint16_t*>(rows), meta, count);
  return 0;
}

int launch_ep_entry_flat(const int32_t* pair_token, const int32_t* pair_flat,
                         const int64_t* start, int64_t U, const uint32_t* idx, int k, int E,
                         int G, int32_t* flat, int num_sms, cudaStream_t s) {
  if (G < 1 || G > 32 || E % G != 0) return 1;
  if (U <= 0) return 0;
  ep_entry_flat_kernel<<<ep_grid(U, num_sms), 256, 0, s>>>(pair_token, pair_flat, start, U, idx,
                                                           k, E, E / G, G, flat);
  return 0;
}

template <typename T>
static void segment_sum_t(const void* in, const int64_t* start, int64_t R, int H, void* out,
                          int num_sms, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = (H % V) == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  if (vec)
    segment_sum_rows_kernel<T, V, 8><<<ep_grid(R * (H / V), num_sms), 256, 0, s>>>(
        static_cast<const T*>(in), start, R, H, static_cast<T*>(out));
  else
    segment_sum_rows_kernel<T, 1, 4><<<ep_grid(R * H, num_sms), 256, 0, s>>>(
        static_cast<const T*>(in), start, R, H, static_cast<T*>(out));
}

int launch_ep_push_pairs(int dtype, const void* x, const int32_t* pair_token,
                         const int32_t* pair_flat, const int32_t* off, int c,
                         const uint32_t* idx, const float* w, int k, int E, int G, int H,
                         const EpPeerRows& tab, int32_t* count, int blocks, cudaStream_t s) {
  const size_t row_bytes = static_cast<size_t>(H) * (dtype == kF32 ? 4 : 2);
  if (G < 1 || G > kMaxEpRanks || E % G != 0 || k > 32 || row_bytes % 16 != 0 ||
      reinterpret_cast<uintptr_t>(x) % 16 != 0 || blocks < 1)
    return 1;
  for (int d = 0; d < G; ++d)
    if (reinterpret_cast<uintptr_t>(tab.rows[d]) % 16 != 0) return 1;
  ep_push_pairs_kernel<uint4><<<blocks, 128, 0, s>>>(
      static_cast<const uint4*>(x), pair_token, pair_flat, off, c, idx, w, k, E, E / G, G,
      static_cast<int>(row_bytes / 16), tab, count);
  return 0;
}

int launch_segment_sum_push(int dtype, const void* in, const int64_t* start, int64_t R, int H,
                            int G, const EpPeerReturn& tab, int blocks, cudaStream_t s) {
  if (R <= 0) return 0;
  if (dtype == kF32 || H % 8 != 0 || G < 1 || G > kMaxEpRanks || blocks < 1 ||
      reinterpret_cast<uintptr_t>(in) % 16 != 0)
    return 1;
  for (int d = 0; d < G; ++d)
    if (reinterpret_cast<uintptr_t>(tab.dst[d]) % 16 != 0) return 1;
  if (dtype == kBF16)
    segment_sum_push_kernel<__nv_bfloat16, 4><<<blocks, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(in), start, R, H, G, tab);
  else
    segment_sum_push_kernel<__half, 4><<<blocks, 128, 0, s>>>(static_cast<const __half*>(in),
                                                             start, R, H, G, tab);
  return 0;
}

int launch_segment_sum_rows(int dtype, const void* in, const int64_t* start, int64_t R, int H,
                            void* out, int num_sms, cudaStream_t s) {
  if (R <= 0) return 0;
  if (dtype == kF32) segment_sum_t<float>(in, start, R, H, out, num_sms, s);
  else if (dtype == kBF16) segment_sum_t<__nv_bfloat16>(in, start, R, H, out, num_sms, s);
  else segment_sum_t<__half>(in, start, R, H, out, num_sms, s);
  return 0;
}

}  // namespace cmoe
