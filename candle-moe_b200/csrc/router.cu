// R1: fused softmax + top-k router (replaces kernels/topk_softmax.cu:136-353).
//
// One row (token) is owned by a group of TPR lanes; each lane loads its VPT logits with 128-bit
// loads, the group reduces max / sum with xor shuffles, then runs k rounds of a shuffle argmax
// (ties go to the lower expert, topk_softmax.cu:240) and clears the winner to -10000
// (topk_softmax.cu:256-264).  The lane grouping and the order in which a lane sums its values
// are those of the reference launcher (topk_softmax.cu:268-295), and this file is compiled with
// --use_fast_math like the reference build (build.rs:59), so the weights come out bit-identical
// to the reference kernel's.  Differences from the reference: a grid-stride loop sized to the
// SM count instead of one CTA per 4 warps of rows, picks made with two warp reductions per round
// when a warp owns the row (same picks; see below), an optional renormalisation of the k
// weights (Qwen3 norm_topk_prob), and a status return for unsupported expert counts.
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {

template <int E>
struct RouterGeom {
  static constexpr int kBytes = (4 * E < 16) ? 4 * E : 16;
  static constexpr int kElts = kBytes / 4;  // floats per vector load
  static constexpr int kVecs = (E / (kElts * 32)) > 1 ? (E / (kElts * 32)) : 1;
  static constexpr int kVpt = kVecs * kElts;  // values per lane
  static constexpr int kTpr = E / kVpt;       // lanes per row
  static constexpr int kRpw = 32 / kTpr;      // rows per warp
};

template <int N> struct alignas(4 * N) FVec { float v[N]; };

// Order-preserving map of non-NaN floats to 32-bit unsigned keys (a < b  <=>  key(a) < key(b))
// and its inverse; equal floats other than +-0 have equal bits.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// KC > 0: k is the compile-time KC (rounds unrolled, pick bookkeeping folded); KC = 0: any k.
template <int E, int KC>
__global__ void __launch_bounds__(256) router_topk_softmax_kernel(
    const float* __restrict__ logits, float* __restrict__ out_w, int32_t* __restrict__ out_idx,
    int32_t* __restrict__ out_src, int num_tokens, int k_arg, int renorm) {
  // a kernel launched after this one as its programmatic dependent (the route preparation) may
  // start now; it waits for this kernel's completion before it reads the picks
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int k = KC > 0 ? KC : k_arg;
  using G = RouterGeom<E>;
  constexpr int kElts = G::kElts, kVpt = G::kVpt, kTpr = G::kTpr, kVecs = G::kVecs;
  const int lane = threadIdx.x & 31;
  const int g = lane % kTpr;    // position of this lane in its row group
  const int sub = lane / kTpr;  // row of the group within the warp
  const int warps_per_block = blockDim.x >> 5;
  const int64_t warp0 = static_cast<int64_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * warps_per_block;

  // this lane's logits of `row` (zeros past the last row)
  auto load_row = [&](int64_t row, float (&dst)[kVpt]) {
    if (row < num_tokens) {
      const float* rp = logits + row * E + g * kElts;
#pragma unroll
      for (int l = 0; l < kVecs; ++l) {
        const FVec<kElts> q = *reinterpret_cast<const FVec<kElts>*>(rp + l * kElts * kTpr);
#pragma unroll
        for (int i = 0; i < kElts; ++i) dst[l * kElts + i] = q.v[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < kVpt; ++i) dst[i] = 0.f;
    }
  };
  const int64_t row_stride = warp_stride * G::kRpw;
  float vn[kVpt];
  load_row(warp0 * G::kRpw + sub, vn);
  for (int64_t wbase = warp0 * G::kRpw; wbase < num_tokens; wbase += row_stride) {
    const int64_t row = wbase + sub;
    const bool active = row < num_tokens;
    float v[kVpt];
#pragma unroll
    for (int i = 0; i < kVpt; ++i) v[i] = vn[i];
    load_row(row + row_stride, vn);  // the next row's loads overlap this row's work
    // softmax (max subtracted), same operation order as the reference
    float m = v[0];
#pragma unroll
    for (int i = 1; i < kVpt; ++i) m = max(m, v[i]);
#pragma unroll
    for (int mask = kTpr / 2; mask > 0; mask /= 2) m = max(m, __shfl_xor_sync(0xffffffffu, m, mask, kTpr));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kVpt; ++i) {
      v[i] = expf(v[i] - m);
      s += v[i];
    }
#pragma unroll
    for (int mask = kTpr / 2; mask > 0; mask /= 2) s += __shfl_xor_sync(0xffffffffu, s, mask, kTpr);
    const float rs = 1.f / s;
#pragma unroll
    for (int i = 0; i < kVpt; ++i) v[i] = v[i] * rs;

    // k rounds of group argmax.  Pick j is kept by lane j % TPR of the group (slot j / TPR) so
    // that the k results leave in one coalesced store per output array; rows with more picks
    // than the group has slots fall back to the group leader writing each pick as it is made.
    constexpr int kSlots = 4;
    const bool staged = k <= kSlots * kTpr;
    const int col0 = g * kElts;
    float wsum = 0.f;
    float pw[kSlots];
    int pe[kSlots];
#pragma unroll
    for (int s2 = 0; s2 < kSlots; ++s2) {
      pw[s2] = 0.f;
      pe[s2] = 0;
    }
    // Records pick j: kept for the coalesced store, or written at once when not staged.
    auto record = [&](int j, float best, int be) {
      wsum += best;
      if (staged) {
        if (j % kTpr == g) {
#pragma unroll
          for (int s2 = 0; s2 < kSlots; ++s2)
            if (s2 == j / kTpr) {
              pw[s2] = best;
              pe[s2] = be;
            }
        }
      } else if (active && g == 0) {
        const int64_t o = row * k + j;
        out_w[o] = best;
        out_idx[o] = be;
        out_src[o] = static_cast<int32_t>(static_cast<int64_t>(j) * num_tokens + row);
      }
    };
    // When one warp owns the row, its probabilities are numbers and k <= E, the picks -- largest
    // value first, ties to the lower expert -- come from each lane's values sorted once by
    // (value desc, expert asc): a round is one warp max over the lanes' heads (as
    // order-preserving 32-bit keys), one warp min over the experts of the lanes at that max, and
    // the winning lane pops its head.  Same picks as the shuffle argmax below, which the other
    // rows keep (with NaN its picks depend on the lane order, as in the reference; with k > E it
    // re-picks cleared experts at -10000, as the reference does).
    const bool redux = kTpr == 32 && k <= E && (__float_as_uint(s) & 0x7fffffffu) <= 0x7f800000u;
    if (redux) {
      uint32_t key[kVpt];
      int id[kVpt];
#pragma unroll
      for (int i = 0; i < kVpt; ++i) {
        key[i] = order_key(v[i]);
        id[i] = col0 + (i / kElts) * kElts * kTpr + i % kElts;
      }
      // odd-even transposition sort, kVpt rounds (a lane holds 4 or 8 values)
#pragma unroll
      for (int r = 0; r < kVpt; ++r) {
#pragma unroll
        for (int a = r & 1; a + 1 < kVpt; a += 2) {
          const bool sw = key[a + 1] > key[a] || (key[a + 1] == key[a] && id[a + 1] < id[a]);
          const uint32_t ka = key[a], kb = key[a + 1];
          const int ia = id[a], ib = id[a + 1];
          key[a] = sw ? kb : ka;
          key[a + 1] = sw ? ka : kb;
          id[a] = sw ? ib : ia;
          id[a + 1] = sw ? ia : ib;
        }
      }
#pragma unroll
      for (int j = 0; j < (KC > 0 ? KC : k); ++j) {
        const uint32_t km = __reduce_max_sync(0xffffffffu, key[0]);
        const int be = static_cast<int>(
            __reduce_min_sync(0xffffffffu, key[0] == km ? static_cast<uint32_t>(id[0]) : 0xffffffffu));
        if (id[0] == be) {  // this lane held the pick: pop it (0 sorts below every value)
#pragma unroll
          for (int i = 0; i + 1 < kVpt; ++i) {
            key[i] = key[i + 1];
            id[i] = id[i + 1];
          }
          key[kVpt - 1] = 0u;
          id[kVpt - 1] = 0x7fffffff;
        }
        record(j, from_order_key(km), be);
      }
    } else {
      for (int j = 0; j < k; ++j) {
        float best = v[0];
        int be = col0;
#pragma unroll
        for (int l = 0; l < kVecs; ++l) {
#pragma unroll
          for (int i = 0; i < kElts; ++i) {
            const float x = v[l * kElts + i];
            if (x > best) {
              best = x;
              be = col0 + l * kElts * kTpr + i;
            }
          }
        }
#pragma unroll
        for (int mask = kTpr / 2; mask > 0; mask /= 2) {
          const float ob = __shfl_xor_sync(0xffffffffu, best, mask, kTpr);
          const int oe = __shfl_xor_sync(0xffffffffu, be, mask, kTpr);
          if (ob > best || (ob == best && oe < be)) {
            best = ob;
            be = oe;
          }
        }
        record(j, best, be);
        // the owning lane clears the winner
        if (g == (be / kElts) % kTpr) {
          const int l = be / (kElts * kTpr);
          const int i = be % kElts;
#pragma unroll
          for (int ll = 0; ll < kVecs; ++ll)
#pragma unroll
            for (int ii = 0; ii < kElts; ++ii)
              if (ll == l && ii == i) v[ll * kElts + ii] = -10000.f;
        }
      }
    }
    if (staged) {
      if (active) {
#pragma unroll
        for (int s2 = 0; s2 < kSlots; ++s2) {
          const int j = s2 * kTpr + g;
          if (j < k) {
            const int64_t o = row * k + j;
            out_w[o] = renorm ? pw[s2] / wsum : pw[s2];
            out_idx[o] = pe[s2];
            out_src[o] = static_cast<int32_t>(static_cast<int64_t>(j) * num_tokens + row);
          }
        }
      }
    } else if (renorm && active && g == 0) {
      for (int j = 0; j < k; ++j) out_w[row * k + j] = out_w[row * k + j] / wsum;
    }
  }
}

// Returns 0 on success, 1 for an unsupported expert count.
int launch_router(const float* logits, float* w, int32_t* idx, int32_t* src, int num_experts,
                  int num_tokens, int k, int renorm, int num_sms, cudaStream_t stream) {
  if (num_tokens <= 0) return 0;
  const int threads = 256;
  // one wave: as many blocks as fit on the SMs at once (the grid-stride loop prefetches rows)
  auto grid_for = [&](int rows_per_warp, int resident_per_sm) {
    const int64_t warps = (static_cast<int64_t>(num_tokens) + rows_per_warp - 1) / rows_per_warp;
    int64_t blocks = (warps + 7) / 8;
    const int64_t cap = static_cast<int64_t>(num_sms) * resident_per_sm;
    return static_cast<int>(blocks < cap ? blocks : cap);
  };
#define CMOE_ROUTER_LAUNCH(EE, KK)                                                              \
  {                                                                                           \
    static int resident = 0;                                                                  \
    if (resident == 0) {                                                                      \
      int r = 0;                                                                              \
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(                                      \
              &r, router_topk_softmax_kernel<EE, KK>, threads, 0) != cudaSuccess ||          \
          r < 1)                                                                              \
        r = 4;                                                                                \
      resident = r;                                                                           \
    }                                                                                         \
    router_topk_softmax_kernel<EE, KK>                                                        \
        <<<grid_for(RouterGeom<EE>::kRpw, resident), threads, 0, stream>>>(                   \
            logits, w, idx, src, num_tokens, k, renorm);                                      \
    return 0;                                                                                 \
  }
#define CMOE_ROUTER_CASE(EE)                                                                    \
  case EE:                                                                                    \
    if (k == 2) CMOE_ROUTER_LAUNCH(EE, 2)                                                     \
    if (k == 8) CMOE_ROUTER_LAUNCH(EE, 8)                                                     \
    CMOE_ROUTER_LAUNCH(EE, 0)
  switch (num_experts) {
    CMOE_ROUTER_CASE(1)
    CMOE_ROUTER_CASE(2)
    CMOE_ROUTER_CASE(4)
    CMOE_ROUTER_CASE(8)
    CMOE_ROUTER_CASE(16)
    CMOE_ROUTER_CASE(32)
    CMOE_ROUTER_CASE(64)
    CMOE_ROUTER_CASE(128)
    CMOE_ROUTER_CASE(256)
    default:
      return 1;
  }
#undef CMOE_ROUTER_LAUNCH
#undef CMOE_ROUTER_CASE
}

}  // namespace cmoe
