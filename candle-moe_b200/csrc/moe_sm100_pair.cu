// The Qwen3 expert GEMMs on CTA pairs: tcgen05.mma.cta_group::2 with M = 256, so each SM stages
// only half of the B tile.  GEMM-2 (y = h.D_e x routing weight, D_e [I,H] MN-major) is the
// default path for fused calls; GEMM-1 (gate|up with the activation epilogue, gathered rows) is
// opt-in (GEMM path 4): correct, and as fast as the one-CTA GEMM-1 at configs 4 and 5, not faster.
// The description below is GEMM-2's; GEMM-1's kernel says what differs.
//
// A cluster of two CTAs owns a pair tile: 256 sorted rows of one expert (each CTA 128 of them)
// by 256 output columns (each CTA stages 128 of the B columns).  Per CTA a stage is 16 KB of A +
// 16 KB of B, so six stages fit where the one-CTA kernel holds four of 48 KB: the same bytes in
// flight cover 1.5x the latency, and the L2 -> SM traffic per FLOP drops by a third.
//
// Roles (256 threads per CTA):
//   warp 0, one thread (both CTAs)  TMA loads of this CTA's A rows and B columns; the completion
//                                   bytes of both CTAs go to the even CTA's full barrier, whose
//                                   producer also posts the expected byte count of the pair;
//   warp 1, one thread (even CTA)   tcgen05.mma.cta_group::2 (M=256, N=256, K=16) reading both
//                                   CTAs' shared memory; tcgen05.commit to the stage-empty and
//                                   accumulator-full barriers of both CTAs (one commit each);
//   warp 2                          TMEM allocation of the pair (cta_group::2);
//   warps 4-7 (both CTAs)           epilogue of this CTA's 128 rows from its TMEM: x routing weight,
//                                   rounding, staged 128-byte row stores; arrival on the even
//                                   CTA's accumulator-empty barrier (remote from the odd CTA).
// Tiles are scheduled statically (pair p takes tiles p, p + pairs, ...), so both CTAs of a pair
// walk the same sequence with no exchange.  Every wait is bounded; the pair meets at a cluster
// barrier before the TMEM is released.  No load uses cluster multicast.
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {
namespace {

constexpr int kPBM = 128;          // rows per CTA (the pair covers 256)
constexpr int kPBN = 256;          // output columns of a pair tile
constexpr int kPBK = 64;
constexpr int kPStages = 6;
constexpr int kPAStage = kPBM * kPBK * 2;        // 16 KB
constexpr int kPBStage = (kPBN / 2) * kPBK * 2;  // 16 KB: this CTA's half of the B columns
constexpr int kPStageBytes = kPAStage + kPBStage;
constexpr int kPThreads = 256;
// GEMM-1: relay threads of the odd CTA (warp 1 and warps 8..), each taking every kP1Relays-th
// stage, so that one relay's wait for its stage does not delay the next stage's relay.
#ifndef CMOE_P1_RELAYS
#define CMOE_P1_RELAYS 4
#endif
constexpr int kP1Relays = CMOE_P1_RELAYS;
constexpr int kP1Threads = kPThreads + 32 * (kP1Relays - 1);
constexpr int kPStageOut = 4 * 4096;
constexpr size_t kPSmemBase = static_cast<size_t>(kPStages) * kPStageBytes + 1024 + kPStageOut;
constexpr size_t kPSmemMax = 232448 - 1024;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Arrival on a barrier of the other CTA of the pair, with the instruction's default semantics
// (release at CTA scope), as CUTLASS's 2-SM pipelines arrive on the leader CTA's barriers.  An
// explicit .release.cluster made each arrival wait 0.5-2.7 us for the SM's outstanding memory
// traffic (measured with %globaltimer stamps in GEMM-1's relay at config 5).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait with cluster-scope acquire (barriers that the peer CTA arrives on)
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity,
                                                          volatile int* abort_flag, uint32_t* err,
                                                          uint32_t code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((n & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        if (err) atomicOr(err, code);
        return false;
      }
    }
  }
}
// 2-D tiled load into this CTA's shared memory whose completion bytes go to `mbar` (a
// shared::cluster address, here the even CTA's barrier)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t mbar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (shared::cluster address) when the pair MMAs issued so far have completed
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

template <typename T> struct PairFmt;
template <> struct PairFmt<__half> { static constexpr uint32_t v = 0; };
template <> struct PairFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    sm100_gemm2_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB, const Sm100Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kPStages];
  __shared__ __align__(8) uint64_t bar_empty[kPStages];
  __shared__ __align__(8) uint64_t bar_accf[2];
  __shared__ __align__(8) uint64_t bar_acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const uint32_t rank = cluster_ctarank();
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t smem_base = (raw + 1023u) & ~1023u;
  const uint32_t stage_out_base = smem_base + static_cast<uint32_t>(kPStages * kPStageBytes);
  int32_t* s_tp = reinterpret_cast<int32_t*>(smem_raw + (smem_base - raw) +
                                             static_cast<size_t>(kPStages) * kPStageBytes +
                                             kPStageOut);
  int32_t* s_off = s_tp + (p.E + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const int num_kb = p.K / kPBK;

  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_off[i] = __ldg(p.offsets + i);
  __syncthreads();
  if (threadIdx.x == 0) {
    // pair-tile prefix: ceil(rows / 256) pair tiles per expert
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_tp[e] = acc;
      acc += (s_off[e + 1] - s_off[e] + 2 * kPBM - 1) / (2 * kPBM);
    }
    s_tp[E] = acc;
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(smem_addr(&bar_full[s]), 1);
      mbar_init(smem_addr(&bar_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&bar_accf[b]), 1);
      mbar_init(smem_addr(&bar_acce[b]), 8);  // 4 epilogue warps in each CTA of the pair
    }
    s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_addr(&s_tmem), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;
  const int total_tiles = s_tp[E] * p.n_tiles;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total_tiles; tile += pairs) {
        const int mt = tile / p.n_tiles;
        const int nt = tile - mt * p.n_tiles;
        const int e = expert_of_tile_smem(s_tp, E, mt);
        const int row0 = s_off[e] + (mt - s_tp[e]) * 2 * kPBM + static_cast<int>(rank) * kPBM;
        const int col0 = nt * kPBN + static_cast<int>(rank) * (kPBN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                 kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t full_local = smem_addr(&bar_full[stage]);
          const uint32_t full0 = mapa_shared(full_local, 0);
          if (rank == 0) mbar_arrive_expect_tx(full_local, 2u * kPStageBytes);
          const uint32_t a_dst = smem_base + stage * kPStageBytes;
          const uint32_t b_dst = a_dst + kPAStage;
          const int kc = kb * kPBK;
          tma_load_2d_pair(a_dst, &tmA, full0, kc, row0);
          const int krow = e * p.K + kc;
          tma_load_2d_pair(b_dst, &tmB, full0, col0, krow);
          tma_load_2d_pair(b_dst + 8192, &tmB, full0, col0 + 64, krow);
          if (++stage == kPStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = umma_idesc(PairFmt<T>::v, 1u, 2 * kPBM, kPBN);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int lt = 0;
      for (int tile = pair; ok && tile < total_tiles; tile += pairs, ++lt) {
        const int buf = lt & 1;
        const uint32_t par = static_cast<uint32_t>((lt >> 1) & 1) ^ 1u;
        if (!mbar_wait_cluster_bounded(smem_addr(&bar_acce[buf]), par, &s_abort, p.err,
                                       kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * 256);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_full[stage]), phase, &s_abort, p.err,
                                 kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_base + stage * kPStageBytes;
          const uint32_t b_base = a_base + kPAStage;
#pragma unroll
          for (int ks = 0; ks < kPBK / 16; ++ks) {
            const uint64_t adesc = umma_sdesc(a_base + ks * 32, 16, 1024);
            const uint64_t bdesc = umma_sdesc(b_base + ks * 2048, 8192, 1024);
            umma_f16_pair(d, adesc, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          const uint32_t empty_local = smem_addr(&bar_empty[stage]);
          umma_commit_pair(empty_local);
          umma_commit_pair(mapa_shared(empty_local, 1));
          if (++stage == kPStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t accf_local = smem_addr(&bar_accf[buf]);
        umma_commit_pair(accf_local);
        umma_commit_pair(mapa_shared(accf_local, 1));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp - 4;
    const int r = q * 32 + lane;
    T* out = static_cast<T*>(p.out);
    const uint32_t stg = stage_out_base + static_cast<uint32_t>(q * 4096);
    const int unit = lane & 7;
    int lt = 0;
    for (int tile = pair; tile < total_tiles; tile += pairs, ++lt) {
      const int mt = tile / p.n_tiles;
      const int nt = tile - mt * p.n_tiles;
      const int e = expert_of_tile_smem(s_tp, E, mt);
      const int m0 = (mt - s_tp[e]) * 2 * kPBM + static_cast<int>(rank) * kPBM;
      const int row_base = s_off[e] + m0;
      const int valid = min(kPBM, s_off[e + 1] - s_off[e] - m0);  // may be <= 0 for the odd CTA
      const int n0 = nt * kPBN;
      const int buf = lt & 1;
      const bool live = r < valid;
      int64_t orow = 0;
      float wgt = 1.f;
      if (live) {
        orow = __ldg(p.sorted_flat + row_base + r);
        if (p.out_row) orow = __ldg(p.out_row + orow);
        wgt = __ldg(p.sorted_w + row_base + r);
      }
      bool got = mbar_wait_bounded(smem_addr(&bar_accf[buf]), static_cast<uint32_t>((lt >> 1) & 1),
                                   &s_abort, p.err, kErrWaitAccFull);
      got = __all_sync(0xffffffffu, got);
      if (!got) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * 256);
      int64_t frow[8];
      bool flive[8];
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const int src = rr * 4 + (lane >> 3);
        frow[rr] = __shfl_sync(0xffffffffu, orow, src);
        flive[rr] = __shfl_sync(0xffffffffu, live ? 1 : 0, src) != 0;
      }
#pragma unroll 1
      for (int cc = 0; cc < kPBN; cc += 64) {
        uint32_t a[2][32];
        tmem_ld_32x32b_x32(tb + cc, a[0]);
        tmem_ld_32x32b_x32(tb + cc + 32, a[1]);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t w0 = pack2<T>(__uint_as_float(a[h][u * 8 + 0]) * wgt,
                                         __uint_as_float(a[h][u * 8 + 1]) * wgt);
            const uint32_t w1 = pack2<T>(__uint_as_float(a[h][u * 8 + 2]) * wgt,
                                         __uint_as_float(a[h][u * 8 + 3]) * wgt);
            const uint32_t w2 = pack2<T>(__uint_as_float(a[h][u * 8 + 4]) * wgt,
                                         __uint_as_float(a[h][u * 8 + 5]) * wgt);
            const uint32_t w3 = pack2<T>(__uint_as_float(a[h][u * 8 + 6]) * wgt,
                                         __uint_as_float(a[h][u * 8 + 7]) * wgt);
            const uint32_t addr = stg + lane * 128 + ((((4 * h + u) ^ (lane & 7))) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0),
                         "r"(w1), "r"(w2), "r"(w3)
                         : "memory");
          }
        }
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int srow = rr * 4 + (lane >> 3);
          uint4 val;
          const uint32_t addr = stg + srow * 128 + (((unit ^ (srow & 7))) << 4);
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                       : "r"(addr)
                       : "memory");
          if (flive[rr])
            *reinterpret_cast<uint4*>(out + frow[rr] * p.N + n0 + cc + unit * 8) = val;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t acce_local = smem_addr(&bar_acce[buf]);
        if (rank == 0) mbar_arrive(acce_local);
        else mbar_arrive_remote(mapa_shared(acce_local, 0));
      }
    }
  }

  __syncthreads();
  if (s_abort) {
    // a role gave up: leave time for copies and MMAs already in flight before releasing TMEM
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  cluster_sync_all();  // the peer's MMAs, loads and arrivals that touch this CTA are done
  tc_fence_after();
  if (warp == 2) tmem_dealloc_pair(tmem_base, 512);
}

// Relay `r` of the odd CTA (see sm100_gemm1_pair_kernel): for every kP1Relays-th stage, from
// the r-th on, wait for this CTA's gather threads, then fence and arrive on the even CTA's full
// barrier of that stage.
__device__ __forceinline__ void pair_gemm1_relay(uint64_t* bar_full, int r, int pair, int pairs,
                                                 int total_tiles, int num_kb, int* s_abort,
                                                 uint32_t* err) {
  uint32_t stage = 0, phase = 0;
  int n = 0;
  for (int tile = pair; tile < total_tiles; tile += pairs) {
    for (int kb = 0; kb < num_kb; ++kb, ++n) {
      if (n % kP1Relays == r) {
        const uint32_t full_local = smem_addr(&bar_full[stage]);
        if (!mbar_wait_bounded(full_local, phase, s_abort, err, kErrWaitFull)) return;
        fence_proxy_async_smem();  // the gathered rows before the even CTA's MMA reads them
        mbar_arrive_remote(mapa_shared(full_local, 0));
      }
      if (++stage == kPStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
}

// GEMM-1 of the Qwen3 FFN on CTA pairs: h = act(x.G_e) * (x.U_e) for 256 gathered rows of one
// expert and 128 intermediate columns.  Each CTA gathers its own 128 token rows with cp.async into
// the swizzled A layout (warps 2-3) and stages one half of the N = 256 B tile: the even CTA the
// gate columns, the odd CTA the up columns; both CTAs' TMEM then hold gate (columns 0-127) and
// up (128-255) of their own rows.  The even CTA's full barrier counts its producer (expected B
// bytes of both CTAs), its 64 gather threads and one relay arrival: a relay thread of the odd CTA
// waits for its own gather threads on its local full barrier, orders their generic-proxy writes
// before the tensor core's async-proxy reads (fence.proxy.async) and arrives remotely.  The
// stages are dealt round-robin to kP1Relays relay threads in separate warps (warp 1 and warps
// 8..), so that the fences and remote arrivals of consecutive stages overlap.
template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kP1Threads, 1)
    sm100_gemm1_pair_kernel(const __grid_constant__ CUtensorMap tmG,
                            const __grid_constant__ CUtensorMap tmU, const Sm100Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kPStages];
  __shared__ __align__(8) uint64_t bar_empty[kPStages];
  __shared__ __align__(8) uint64_t bar_accf[2];
  __shared__ __align__(8) uint64_t bar_acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const uint32_t rank = cluster_ctarank();
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t smem_base = (raw + 1023u) & ~1023u;
  const uint32_t stage_out_base = smem_base + static_cast<uint32_t>(kPStages * kPStageBytes);
  int32_t* s_tp = reinterpret_cast<int32_t*>(smem_raw + (smem_base - raw) +
                                             static_cast<size_t>(kPStages) * kPStageBytes +
                                             kPStageOut);
  int32_t* s_off = s_tp + (p.E + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const int num_kb = p.K / kPBK;
  constexpr int kGatherArrivals = 64;

  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_off[i] = __ldg(p.offsets + i);
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_tp[e] = acc;
      acc += (s_off[e + 1] - s_off[e] + 2 * kPBM - 1) / (2 * kPBM);
    }
    s_tp[E] = acc;
    for (int st = 0; st < kPStages; ++st) {
      // even CTA: producer + its gather threads + the odd CTA's relay; odd CTA: its gather
      mbar_init(smem_addr(&bar_full[st]), rank == 0 ? 1 + kGatherArrivals + 1 : kGatherArrivals);
      mbar_init(smem_addr(&bar_empty[st]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&bar_accf[b]), 1);
      mbar_init(smem_addr(&bar_acce[b]), 8);
    }
    s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmG);
    tma_prefetch_desc(&tmU);
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_addr(&s_tmem), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;
  const int total_tiles = s_tp[E] * p.n_tiles;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (B half)
    if (lane == 0) {
      const CUtensorMap* tmB = rank == 0 ? &tmG : &tmU;
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total_tiles; tile += pairs) {
        const int mt = tile / p.n_tiles;
        const int nt = tile - mt * p.n_tiles;
        const int e = expert_of_tile_smem(s_tp, E, mt);
        const int n0 = nt * (kPBN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                 kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t full_local = smem_addr(&bar_full[stage]);
          const uint32_t full0 = mapa_shared(full_local, 0);
          if (rank == 0) mbar_arrive_expect_tx(full_local, 2u * kPBStage);
          const uint32_t b_dst = smem_base + stage * kPStageBytes + kPAStage;
          const int krow = e * p.K + kb * kPBK;
          tma_load_2d_pair(b_dst, tmB, full0, n0, krow);
          tma_load_2d_pair(b_dst + 8192, tmB, full0, n0 + 64, krow);
          if (++stage == kPStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------------- MMA issuer (even CTA)
      constexpr uint32_t idesc = umma_idesc(PairFmt<T>::v, 1u, 2 * kPBM, kPBN);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int lt = 0;
      for (int tile = pair; ok && tile < total_tiles; tile += pairs, ++lt) {
        const int buf = lt & 1;
        const uint32_t par = static_cast<uint32_t>((lt >> 1) & 1) ^ 1u;
        if (!mbar_wait_cluster_bounded(smem_addr(&bar_acce[buf]), par, &s_abort, p.err,
                                       kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * 256);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster_bounded(smem_addr(&bar_full[stage]), phase, &s_abort, p.err,
                                         kErrWaitFull)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();  // this CTA's gathered rows (cp.async, generic proxy)
          tc_fence_after();
          const uint32_t a_base = smem_base + stage * kPStageBytes;
          const uint32_t b_base = a_base + kPAStage;
#pragma unroll
          for (int ks = 0; ks < kPBK / 16; ++ks) {
            const uint64_t adesc = umma_sdesc(a_base + ks * 32, 16, 1024);
            const uint64_t bdesc = umma_sdesc(b_base + ks * 2048, 8192, 1024);
            umma_f16_pair(d, adesc, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          const uint32_t empty_local = smem_addr(&bar_empty[stage]);
          umma_commit_pair(empty_local);
          umma_commit_pair(mapa_shared(empty_local, 1));
          if (++stage == kPStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t accf_local = smem_addr(&bar_accf[buf]);
        umma_commit_pair(accf_local);
        umma_commit_pair(mapa_shared(accf_local, 1));
      }
    } else if (lane == 0 && rank == 1) {
      pair_gemm1_relay(bar_full, 0, pair, pairs, total_tiles, num_kb, &s_abort, p.err);
    }
  } else if (warp >= 8) {
    if (lane == 0 && rank == 1)
      pair_gemm1_relay(bar_full, warp - 7, pair, pairs, total_tiles, num_kb, &s_abort, p.err);
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ A-row gather
    const int g = threadIdx.x - 64;
    const int c = g & 7;
    const int q = g >> 3;
    const T* x = static_cast<const T*>(p.a_rows);
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    // the row indices of this CTA's 128 rows of a tile, loaded while the previous tile streams
    int tok[16];
    auto load_rows = [&](int t) {
      const int mt = t / p.n_tiles;
      const int e = expert_of_tile_smem(s_tp, E, mt);
      const int pm0 = (mt - s_tp[e]) * 2 * kPBM;
      const int row_base = s_off[e] + pm0 + static_cast<int>(rank) * kPBM;
      const int valid = min(kPBM, s_off[e + 1] - s_off[e] - pm0 - static_cast<int>(rank) * kPBM);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // rows past the expert's last one repeat a valid row (their outputs are not written)
        const int sr = valid > 0 ? row_base + min(q + 8 * i, valid - 1) : s_off[e] + pm0;
        tok[i] = __ldg(p.sorted_token + sr);
      }
    };
    if (pair < total_tiles) load_rows(pair);
    for (int tile = pair; ok && tile < total_tiles; tile += pairs) {
      const T* src[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) src[i] = x + static_cast<size_t>(tok[i]) * p.K + c * 8;
      const uint32_t dst_off = static_cast<uint32_t>(q * 128 + ((c ^ q) << 4));
      for (int kb = 0; kb < num_kb; ++kb) {
        if (kb == (num_kb - 1) / 2 && tile + pairs < total_tiles) load_rows(tile + pairs);
        bool got = mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                     kErrWaitEmpty);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          break;
        }
        const uint32_t a_dst = smem_base + stage * kPStageBytes + dst_off;
#pragma unroll
        for (int i = 0; i < 16; ++i) cp_async16(a_dst + i * 8 * 128, src[i] + kb * kPBK);
        cp_async_mbar_arrive_noinc(smem_addr(&bar_full[stage]));
        if (++stage == kPStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp - 4;
    const int r = q * 32 + lane;
    T* out = static_cast<T*>(p.out);
    const uint32_t stg = stage_out_base + static_cast<uint32_t>(q * 4096);
    const int unit = lane & 7;
    int lt = 0;
    for (int tile = pair; tile < total_tiles; tile += pairs, ++lt) {
      const int mt = tile / p.n_tiles;
      const int nt = tile - mt * p.n_tiles;
      const int e = expert_of_tile_smem(s_tp, E, mt);
      const int m0 = (mt - s_tp[e]) * 2 * kPBM + static_cast<int>(rank) * kPBM;
      const int row_base = s_off[e] + m0;
      const int valid = min(kPBM, s_off[e + 1] - s_off[e] - m0);
      const int n0 = nt * (kPBN / 2);
      const int buf = lt & 1;
      bool got = mbar_wait_bounded(smem_addr(&bar_accf[buf]), static_cast<uint32_t>((lt >> 1) & 1),
                                   &s_abort, p.err, kErrWaitAccFull);
      got = __all_sync(0xffffffffu, got);
      if (!got) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * 256);
#pragma unroll 1
      for (int cc = 0; cc < kPBN / 2; cc += 64) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t gv[32], uv[32];
          tmem_ld_32x32b_x32(tb + cc + 32 * h, gv);
          tmem_ld_32x32b_x32(tb + kPBN / 2 + cc + 32 * h, uv);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              v[i] = act_apply(__uint_as_float(gv[u * 8 + i]), p.act) *
                     __uint_as_float(uv[u * 8 + i]);
            const uint32_t addr = stg + lane * 128 + ((((4 * h + u) ^ (lane & 7))) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                         "r"(pack2<T>(v[0], v[1])), "r"(pack2<T>(v[2], v[3])),
                         "r"(pack2<T>(v[4], v[5])), "r"(pack2<T>(v[6], v[7]))
                         : "memory");
          }
        }
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int srow = rr * 4 + (lane >> 3);
          uint4 val;
          const uint32_t addr = stg + srow * 128 + (((unit ^ (srow & 7))) << 4);
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                       : "r"(addr)
                       : "memory");
          if (q * 32 + srow < valid)
            *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row_base + q * 32 + srow) * p.N +
                                      n0 + cc + unit * 8) = val;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t acce_local = smem_addr(&bar_acce[buf]);
        if (rank == 0) mbar_arrive(acce_local);
        else mbar_arrive_remote(mapa_shared(acce_local, 0));
      }
      (void)r;
    }
  }

  __syncthreads();
  if (s_abort) {
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 2) tmem_dealloc_pair(tmem_base, 512);
}

}  // namespace

size_t sm100_pair_smem_bytes(int num_experts) {
  return kPSmemBase + static_cast<size_t>(2 * num_experts + 3) * sizeof(int32_t);
}

bool sm100_pair_set_attributes() {
  const int smax = static_cast<int>(kPSmemMax);
  const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
  bool ok = cudaFuncSetAttribute(sm100_gemm2_pair_kernel<__nv_bfloat16>, attr, smax) == cudaSuccess;
  ok &= cudaFuncSetAttribute(sm100_gemm2_pair_kernel<__half>, attr, smax) == cudaSuccess;
  ok &= cudaFuncSetAttribute(sm100_gemm1_pair_kernel<__nv_bfloat16>, attr, smax) == cudaSuccess;
  ok &= cudaFuncSetAttribute(sm100_gemm1_pair_kernel<__half>, attr, smax) == cudaSuccess;
  return ok;
}

// Clusters of two CTAs of the pair kernels that can be resident at once on the current device
// (both kernels use the same block size and shared-memory budget).  The static tile schedule
// hands pair p the tiles p, p + pairs, ...: a cluster that could not be resident would run its
// whole list after the others, so the launchers' callers cap `pairs` with this.  0 on error.
int sm100_pair_max_clusters() {
  cudaLaunchConfig_t cfg = {};
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmemMax;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, sm100_gemm2_pair_kernel<__nv_bfloat16>, &cfg) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

// GEMM-1, Qwen3 (gate|up with the activation epilogue), on CTA pairs.  g / u: maps over gate and
// up [E*H, I] with a 64 x 64 box; p.a_rows = x; p.out = the intermediate [rows, I]; p.n_tiles =
// I / 128; pairs <= num_sms / 2.  Returns non-zero if the request does not fit this kernel.
int launch_sm100_gemm1_pair(int dtype, const CUtensorMap& g, const CUtensorMap& u,
                            const Sm100Params& p, int pairs, cudaStream_t s) {
  if (pairs <= 0) return 3;  // no cluster fits: the caller takes the one-CTA kernel
  if (p.N % (kPBN / 2) != 0 || p.K % kPBK != 0) return 1;
  const size_t smem = sm100_pair_smem_bytes(p.E);
  if (smem > kPSmemMax) return 2;
  const dim3 grid(2 * pairs), block(kP1Threads);
  if (dtype == kBF16)
    sm100_gemm1_pair_kernel<__nv_bfloat16><<<grid, block, smem, s>>>(g, u, p);
  else if (dtype == kF16)
    sm100_gemm1_pair_kernel<__half><<<grid, block, smem, s>>>(g, u, p);
  else
    return 1;
  return 0;
}

// GEMM-2, Qwen3 (down projection, MN-major B), on CTA pairs.  a: A map (box 64 x 128 rows of the
// intermediate); b: B map over down [E*I, H] with a 64 x 64 box; p.n_tiles = H / 256;
// pairs <= num_sms / 2.  Returns non-zero if the request does not fit this kernel.
int launch_sm100_gemm2_pair(int dtype, const CUtensorMap& a, const CUtensorMap& b,
                            const Sm100Params& p, int pairs, cudaStream_t s) {
  if (pairs <= 0) return 3;  // no cluster fits: the caller takes the one-CTA kernel
  if (p.N % kPBN != 0 || p.K % kPBK != 0) return 1;
  const size_t smem = sm100_pair_smem_bytes(p.E);
  if (smem > kPSmemMax) return 2;
  const dim3 grid(2 * pairs), block(kPThreads);
  if (dtype == kBF16)
    sm100_gemm2_pair_kernel<__nv_bfloat16><<<grid, block, smem, s>>>(a, b, p);
  else if (dtype == kF16)
    sm100_gemm2_pair_kernel<__half><<<grid, block, smem, s>>>(a, b, p);
  else
    return 1;
  return 0;
}

}  // namespace cmoe
