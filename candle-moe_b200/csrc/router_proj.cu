// R0: the router's gate projection fused with the softmax + top-k (R1).
//
// The reference leaves the projection to its caller: a model computes the router logits with a
// Linear over the hidden states and hands them to apply_topk_softmax_inplace (README.md:67-73,
// src/lib.rs:124-155).  Here one kernel reads each token row once, computes its E logits
// x_t . W_r^T on the tensor cores (tcgen05.mma, f32 accumulation in TMEM) and turns them into
// the k picks in the epilogue, so the [T, E] logits never travel through HBM.
//
//   A = 128 token rows x 64 hidden  (TMA box of x [T, H], K-major, 128-byte swizzle)
//   B = E expert rows x 64 hidden   (TMA box of W_r [E, H], K-major; E < 16 is padded to 16
//                                    rows that the TMA fills with zeros and the epilogue skips)
//   D = [128 tokens, E experts] f32 in TMEM, double-buffered so one tile's epilogue overlaps the
//       next tile's MMAs.  Tiles of 128 tokens go round-robin to one CTA per SM.
//
// Epilogue: TMEM lane = token, so one thread holds its token's logits and needs no exchange.
// The softmax reproduces R1's arithmetic exactly (router.cu, compiled like this file with
// --use_fast_math): R1 gives each of its TPR lanes the columns g*ELTS + l*ELTS*TPR + i and sums
// a lane's exponentials in (l, i) order, then adds the lanes with an xor butterfly; this
// thread forms the same TPR partial sums and the same butterfly, so the probabilities -- and
// the picks (largest first, ties to the lower expert) and weights -- are bit-identical to R1
// run on the logits this kernel computes (moe_router_project_topk can write them out for that
// check).  Every wait is bounded (common.cuh).
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {

constexpr int kRpThreads = 256;
constexpr int kRpBM = 128;   // tokens per tile
constexpr int kRpBK = 64;    // hidden elements per stage
constexpr int kRpRingBytes = 220 * 1024;  // operand ring (+ staging, see kWarpPick)
constexpr int kRpMaxK = 16;

// R1's lane geometry for E experts (RouterGeom in router.cu).
template <int E>
struct RpGeom {
  static constexpr int kBytes = (4 * E < 16) ? 4 * E : 16;
  static constexpr int kElts = kBytes / 4;
  static constexpr int kVecs = (E / (kElts * 32)) > 1 ? (E / (kElts * 32)) : 1;
  static constexpr int kVpt = kVecs * kElts;
  static constexpr int kTpr = E / kVpt;
  static constexpr int kN = E < 16 ? 16 : E;           // MMA N (padded)
  static constexpr int kABytes = kRpBM * kRpBK * 2;    // 16 KB
  static constexpr int kBBytes = (kN * 128 + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // E = 64 / 128 pick per warp from probabilities staged in shared memory (4 warps x 16 rows
  // x (E + 1) floats), which takes room from the operand ring
  static constexpr bool kWarpPick = E == 64 || E == 128;
  static constexpr int kStageFloats = kWarpPick ? 4 * 16 * (E + 1) : 0;
  static constexpr int kRing = kRpRingBytes - (kWarpPick ? (kStageFloats * 4 + 1023) / 1024 * 1024 : 0);
  static constexpr int kStages = kRing / kStageBytes > 8 ? 8 : kRing / kStageBytes;
  static constexpr int kTmemCols = 2 * kN <= 32 ? 32 : 2 * kN <= 64 ? 64 : 2 * kN <= 128 ? 128
                                 : 2 * kN <= 256 ? 256 : 512;
};

// order-preserving 32-bit keys of non-NaN floats (as router.cu's order_key / from_order_key)
__device__ __forceinline__ uint32_t rp_order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float rp_from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <typename T> struct RpFmt;
template <> struct RpFmt<__half> { static constexpr uint32_t v = 0; };
template <> struct RpFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

// the logit of column c from TMEM (32 columns per load)
template <int E, int CH>
__device__ __forceinline__ void rp_load_chunk(uint32_t tb, int c0, float (&v)[CH]) {
  static_assert(CH == 16 || CH == 32, "chunk");
  if (CH == 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tb + c0, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < CH; ++i) v[i] = __uint_as_float(r[i]);
  } else {
    uint32_t r[16];
    tmem_ld_32x32b_x16(tb + c0, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < CH; ++i) v[i] = __uint_as_float(r[i]);
  }
}

template <typename T, int E, int KC>
__global__ void __launch_bounds__(kRpThreads, 1)
    router_project_kernel(const __grid_constant__ CUtensorMap tmX,
                          const __grid_constant__ CUtensorMap tmW, const RouterProjParams p) {
  using Gm = RpGeom<E>;
  constexpr int kN = Gm::kN, kStages = Gm::kStages;
  constexpr int kCh = E >= 32 ? 32 : 16;  // TMEM columns per load
  constexpr int kChunks = (E + kCh - 1) / kCh;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kStages];
  __shared__ __align__(8) uint64_t bar_empty[kStages];
  __shared__ __align__(8) uint64_t bar_accf[2];
  __shared__ __align__(8) uint64_t bar_acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const uint32_t smem_base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  // E = 64 and 128: the probabilities of 16 rows per epilogue warp, after the operand ring
  constexpr bool kWarpPick = RpGeom<E>::kWarpPick;
  float* s_stage = reinterpret_cast<float*>(smem_raw + (smem_base - smem_addr(smem_raw)) +
                                            static_cast<size_t>(RpGeom<E>::kStages) *
                                                RpGeom<E>::kStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k = KC > 0 ? KC : p.k;
  const int num_kb = p.H / kRpBK;
  const int tiles = (p.num_tokens + kRpBM - 1) / kRpBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&bar_full[s]), 1);
      mbar_init(smem_addr(&bar_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&bar_accf[b]), 1);
      mbar_init(smem_addr(&bar_acce[b]), 4);
    }
    s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 2) {
    tmem_alloc(smem_addr(&s_tmem), Gm::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                 kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_addr(&bar_full[stage]);
          mbar_arrive_expect_tx(full, Gm::kABytes + kN * kRpBK * 2);
          const uint32_t a_dst = smem_base + stage * Gm::kStageBytes;
          tma_load_2d(a_dst, &tmX, full, kb * kRpBK, tile * kRpBM);
          tma_load_2d(a_dst + Gm::kABytes, &tmW, full, kb * kRpBK, 0);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(RpFmt<T>::v, 0u, kRpBM, kN);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int lt = 0;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_bounded(smem_addr(&bar_acce[buf]), static_cast<uint32_t>((lt >> 1) & 1) ^ 1u,
                               &s_abort, p.err, kErrWaitAccEmpty))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_full[stage]), phase, &s_abort, p.err,
                                 kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_base + stage * Gm::kStageBytes;
          const uint32_t b_base = a_base + Gm::kABytes;
#pragma unroll
          for (int ks = 0; ks < kRpBK / 16; ++ks)
            umma_f16(d, umma_sdesc(a_base + ks * 32, 16, 1024),
                     umma_sdesc(b_base + ks * 32, 16, 1024), idesc, (kb | ks) != 0 ? 1u : 0u);
          umma_commit(smem_addr(&bar_empty[stage]));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_addr(&bar_accf[buf]));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue: softmax, top-k
    const int q = warp & 3;
    int lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int buf = lt & 1;
      bool got = mbar_wait_bounded(smem_addr(&bar_accf[buf]), static_cast<uint32_t>((lt >> 1) & 1),
                                   &s_abort, p.err, kErrWaitAccFull);
      got = __all_sync(0xffffffffu, got);
      if (!got) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * kN);
      const int64_t row = static_cast<int64_t>(tile) * kRpBM + q * 32 + lane;
      const bool live = row < p.num_tokens;

      // pass 1: max over the row (and the optional logits copy)
      float m = -INFINITY;
#pragma unroll 1
      for (int cb = 0; cb < kChunks; ++cb) {
        float v[kCh];
        rp_load_chunk<E, kCh>(tb, cb * kCh, v);
#pragma unroll
        for (int i = 0; i < kCh; ++i) {
          if (cb * kCh + i < E) {
            m = (cb * kCh + i == 0) ? v[i] : max(m, v[i]);
            if (p.logits && live) p.logits[row * E + cb * kCh + i] = v[i];
          }
        }
      }
      // pass 2: R1's TPR lane partial sums of the exponentials, then its xor butterfly
      float part[Gm::kTpr];
#pragma unroll
      for (int g = 0; g < Gm::kTpr; ++g) part[g] = 0.f;
#pragma unroll
      for (int cb = 0; cb < kChunks; ++cb) {
        float v[kCh];
        rp_load_chunk<E, kCh>(tb, cb * kCh, v);
#pragma unroll
        for (int i = 0; i < kCh; ++i) {
          const int c = cb * kCh + i;
          if (c < E) {
            // column c belongs to R1 lane (c / ELTS) % TPR; its (l, i) order is column order
            // (c is a compile-time index here, so part[] stays in registers)
            part[(c / Gm::kElts) % Gm::kTpr] += expf(v[i] - m);
          }
        }
      }
#pragma unroll
      for (int mask = Gm::kTpr / 2; mask > 0; mask /= 2) {
#pragma unroll
        for (int g = 0; g < Gm::kTpr; ++g)
          if ((g & mask) == 0) {
            const float t = part[g] + part[g | mask];
            part[g] = t;
            part[g | mask] = t;
          }
      }
      const float rs = 1.f / part[0];
      if (kWarpPick) {
        // pass 3 (E = 64, 128): the probabilities go through shared memory (16 of this warp's
        // rows at a time, row stride E + 1 floats: conflict-free both ways), then the warp picks
        // as R1 does when a warp owns a row -- each lane sorts its E/32 values (columns lane +
        // 32 l) by (value desc, expert asc), and every pick is a warp max over the lanes' heads
        // (as order-preserving keys) and a warp min over the experts at that max; eight rows
        // are picked side by side so that their reduction chains overlap.
        float* st = s_stage + static_cast<size_t>(q) * 16 * (E + 1);
        constexpr int kPer = E >= 32 ? E / 32 : 1;  // values per lane
        constexpr int kRows = 8;  // rows picked side by side: independent reduction chains
        const int64_t row0 = static_cast<int64_t>(tile) * kRpBM + q * 32;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          // lanes 16h..16h+15 stage their rows' probabilities (row stride E + 1 floats); the
          // TMEM loads are warp-wide (.sync.aligned), only the stores are per half
          const bool mine = (lane >> 4) == h;
#pragma unroll 1
          for (int cb = 0; cb < kChunks; ++cb) {
            float v[kCh];
            rp_load_chunk<E, kCh>(tb, cb * kCh, v);
            if (mine) {
#pragma unroll
              for (int i = 0; i < kCh; ++i)
                st[(lane & 15) * (E + 1) + cb * kCh + i] = expf(v[i] - m) * rs;
            }
          }
          if (h == 1) {
            // every probability is out of TMEM: release the accumulator
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&bar_acce[buf]));
          }
          __syncwarp();
#pragma unroll 1
          for (int r0 = 0; r0 < 16; r0 += kRows) {
            uint32_t key[kRows][kPer];
            int id[kRows][kPer];
#pragma unroll
            for (int rr = 0; rr < kRows; ++rr) {
#pragma unroll
              for (int l = 0; l < kPer; ++l) {
                key[rr][l] = rp_order_key(st[(r0 + rr) * (E + 1) + lane + 32 * l]);
                id[rr][l] = lane + 32 * l;
              }
              // odd-even transposition sort of this lane's values: (value desc, expert asc)
#pragma unroll
              for (int t = 0; t < kPer; ++t) {
#pragma unroll
                for (int a = t & 1; a + 1 < kPer; a += 2) {
                  const bool sw = key[rr][a + 1] > key[rr][a] ||
                                  (key[rr][a + 1] == key[rr][a] && id[rr][a + 1] < id[rr][a]);
                  const uint32_t ka = key[rr][a], kb2 = key[rr][a + 1];
                  const int ia = id[rr][a], ib = id[rr][a + 1];
                  key[rr][a] = sw ? kb2 : ka;
                  key[rr][a + 1] = sw ? ka : kb2;
                  id[rr][a] = sw ? ib : ia;
                  id[rr][a + 1] = sw ? ia : ib;
                }
              }
            }
            float mine_w[kRows], wsum[kRows];
            int mine_e[kRows];
#pragma unroll
            for (int rr = 0; rr < kRows; ++rr) {
              mine_w[rr] = 0.f;
              wsum[rr] = 0.f;
              mine_e[rr] = 0;
            }
#pragma unroll 1
            for (int j = 0; j < k; ++j) {
              uint32_t km[kRows];
#pragma unroll
              for (int rr = 0; rr < kRows; ++rr) km[rr] = __reduce_max_sync(0xffffffffu, key[rr][0]);
              int be[kRows];
#pragma unroll
              for (int rr = 0; rr < kRows; ++rr)
                be[rr] = static_cast<int>(__reduce_min_sync(
                    0xffffffffu,
                    key[rr][0] == km[rr] ? static_cast<uint32_t>(id[rr][0]) : 0xffffffffu));
#pragma unroll
              for (int rr = 0; rr < kRows; ++rr) {
                if (id[rr][0] == be[rr]) {  // this lane held the pick: pop it
#pragma unroll
                  for (int l = 0; l + 1 < kPer; ++l) {
                    key[rr][l] = key[rr][l + 1];
                    id[rr][l] = id[rr][l + 1];
                  }
                  key[rr][kPer - 1] = 0u;
                  id[rr][kPer - 1] = 0x7fffffff;
                }
                const float wv = rp_from_order_key(km[rr]);
                wsum[rr] += wv;
                if (lane == j) {
                  mine_w[rr] = wv;
                  mine_e[rr] = be[rr];
                }
              }
            }
#pragma unroll
            for (int rr = 0; rr < kRows; ++rr) {
              const int64_t rrow = row0 + 16 * h + r0 + rr;
              if (lane < k && rrow < p.num_tokens) {
                const int64_t o = rrow * k + lane;
                p.out_w[o] = p.renorm ? mine_w[rr] / wsum[rr] : mine_w[rr];
                p.out_idx[o] = mine_e[rr];
                p.out_src[o] =
                    static_cast<int32_t>(static_cast<int64_t>(lane) * p.num_tokens + rrow);
              }
            }
          }
          __syncwarp();
        }
        __syncwarp();
        continue;
      }
      // pass 3 (E <= 32 or 256): the k largest probabilities, ties to the lower expert, kept
      // sorted; a value enters only when strictly larger than the k-th (columns arrive in
      // ascending order, so an equal later value loses, as in R1)
      constexpr int KK = KC > 0 ? KC : kRpMaxK;
      float bw[KK];
      int be[KK];
#pragma unroll
      for (int j = 0; j < KK; ++j) {
        bw[j] = -INFINITY;
        be[j] = 0x7fffffff;
      }
      float thr = -INFINITY;  // the k-th largest so far
#pragma unroll 1
      for (int cb = 0; cb < kChunks; ++cb) {
        float v[kCh];
        rp_load_chunk<E, kCh>(tb, cb * kCh, v);
#pragma unroll
        for (int i = 0; i < kCh; ++i) {
          const int c = cb * kCh + i;
          if (c < E) {
            float pv = expf(v[i] - m) * rs;
            int pe = c;
            if (pv > thr) {
#pragma unroll
              for (int j = 0; j < KK; ++j) {
                if (j < k && pv > bw[j]) {
                  const float tw = bw[j];
                  const int te = be[j];
                  bw[j] = pv;
                  be[j] = pe;
                  pv = tw;
                  pe = te;
                }
              }
#pragma unroll
              for (int j = 0; j < KK; ++j)
                if (j == k - 1) thr = bw[j];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&bar_acce[buf]));
      if (live) {
        float wsum = 0.f;
#pragma unroll
        for (int j = 0; j < KK; ++j)
          if (j < k) wsum += bw[j];
#pragma unroll
        for (int j = 0; j < KK; ++j) {
          if (j < k) {
            const int64_t o = row * k + j;
            p.out_w[o] = p.renorm ? bw[j] / wsum : bw[j];
            p.out_idx[o] = be[j];
            p.out_src[o] = static_cast<int32_t>(static_cast<int64_t>(j) * p.num_tokens + row);
          }
        }
      }
    }
  }

  __syncthreads();
  if (s_abort) {
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Gm::kTmemCols);
  }
}

// ---- host side -------------------------------------------------------------------------------

int router_project_max_k() { return kRpMaxK; }

template <typename T, int E, int KC>
static size_t rp_smem() {
  return static_cast<size_t>(RpGeom<E>::kStages) * RpGeom<E>::kStageBytes + 1024 +
         static_cast<size_t>(RpGeom<E>::kStageFloats) * sizeof(float);
}

template <typename T, int E, int KC>
static int rp_launch(const CUtensorMap& x, const CUtensorMap& w, const RouterProjParams& p,
                     int grid, cudaStream_t s) {
  router_project_kernel<T, E, KC><<<grid, kRpThreads, rp_smem<T, E, KC>(), s>>>(x, w, p);
  return 0;
}

template <typename T, int E>
static bool rp_attr_e() {
  const auto a = cudaFuncAttributeMaxDynamicSharedMemorySize;
  bool ok = cudaFuncSetAttribute(router_project_kernel<T, E, 2>, a,
                                 static_cast<int>(rp_smem<T, E, 2>())) == cudaSuccess;
  ok &= cudaFuncSetAttribute(router_project_kernel<T, E, 8>, a,
                             static_cast<int>(rp_smem<T, E, 8>())) == cudaSuccess;
  ok &= cudaFuncSetAttribute(router_project_kernel<T, E, 0>, a,
                             static_cast<int>(rp_smem<T, E, 0>())) == cudaSuccess;
  return ok;
}

template <typename T>
static bool rp_attr_t() {
  return rp_attr_e<T, 1>() && rp_attr_e<T, 2>() && rp_attr_e<T, 4>() && rp_attr_e<T, 8>() &&
         rp_attr_e<T, 16>() && rp_attr_e<T, 32>() && rp_attr_e<T, 64>() &&
         rp_attr_e<T, 128>() && rp_attr_e<T, 256>();
}

// Once per device: the shared-memory sizes of every instantiation.
bool router_project_set_attributes() {
  return rp_attr_t<__nv_bfloat16>() && rp_attr_t<__half>();
}

template <typename T, int E>
static int rp_launch_e(const CUtensorMap& x, const CUtensorMap& w, const RouterProjParams& p,
                       int grid, cudaStream_t s) {
  if (p.k == 2) return rp_launch<T, E, 2>(x, w, p, grid, s);
  if (p.k == 8) return rp_launch<T, E, 8>(x, w, p, grid, s);
  return rp_launch<T, E, 0>(x, w, p, grid, s);
}

template <typename T>
static int rp_launch_t(int E, const CUtensorMap& x, const CUtensorMap& w,
                       const RouterProjParams& p, int grid, cudaStream_t s) {
  switch (E) {
    case 1: return rp_launch_e<T, 1>(x, w, p, grid, s);
    case 2: return rp_launch_e<T, 2>(x, w, p, grid, s);
    case 4: return rp_launch_e<T, 4>(x, w, p, grid, s);
    case 8: return rp_launch_e<T, 8>(x, w, p, grid, s);
    case 16: return rp_launch_e<T, 16>(x, w, p, grid, s);
    case 32: return rp_launch_e<T, 32>(x, w, p, grid, s);
    case 64: return rp_launch_e<T, 64>(x, w, p, grid, s);
    case 128: return rp_launch_e<T, 128>(x, w, p, grid, s);
    case 256: return rp_launch_e<T, 256>(x, w, p, grid, s);
    default: return 1;
  }
}

// 0 on success; 1 unsupported shape.
int launch_router_project(int dtype, int E, const CUtensorMap& x, const CUtensorMap& w,
                          const RouterProjParams& p, int grid, cudaStream_t s) {
  if (p.k < 1 || p.k > kRpMaxK || p.k > E || p.H % kRpBK != 0 || grid <= 0) return 1;
  if (dtype == kBF16) return rp_launch_t<__nv_bfloat16>(E, x, w, p, grid, s);
  if (dtype == kF16) return rp_launch_t<__half>(E, x, w, p, grid, s);
  return 1;
}

}  // namespace cmoe
