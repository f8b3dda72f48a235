// G1/G2 for f32 operands on the 5th-generation tensor cores with three TF32 products.
//
// Replaces the reference's f32 grouped GEMMs (moe.cu:193-449, K9/K10), which run on FFMA, for
// hidden / intermediate sizes that are multiples of 128.  Each f32 operand value v is split into
// hi = v with its 13 low mantissa bits cleared (exactly a TF32 value) and lo = v - hi (exact in
// f32, |lo| < 2^-10 |v|); then a.b = hi_a.hi_b + hi_a.lo_b + lo_a.hi_b + lo_a.lo_b, and the first
// three products run as tcgen05.mma kind::tf32 into one f32 accumulator in TMEM.  The dropped
// term and the TF32 reading of lo are each below 2^-20 |a.b|, so a product carries a relative
// error of ~3e-6 against ~6e-8 for FFMA; the f32 tolerance of the reference comparison is 1e-4.
//
// One CTA per SM walks the tile list (m-tile of 128 sorted rows of one expert x n-tile) with a
// static schedule (tile = CTA, CTA + grid, ...).  Warp roles (384 threads):
//   warp 0      TMA producer (one thread): B tiles from the weights in their API layout (gate /
//               up [E,H,I] and down [E,I,H] MN-major in 32 x 32 boxes, Nomic's up [E,H,I] as
//               the K-major B of h.U^T), and GEMM-2's A (contiguous intermediate rows)
//   warps 2-3   GEMM-1's A: the 128 gathered token rows, 16-byte cp.async copies written into
//               the 128-byte-swizzled K-major layout; warp 2 also owns the TMEM allocation
//   warps 8-11  the split: once a stage has landed, each thread reads its 16-byte chunks and
//               writes lo = v - hi to the stage's lo half (same offsets, so the same swizzle),
//               then orders those writes before the tensor core's reads (fence.proxy.async) and
//               its warp arrives on the stage's split barrier.  hi stays the raw f32 value: the
//               TF32 MMA reads an f32 operand as its 13 low mantissa bits cleared (outputs
//               bit-identical to writing the cleared values, checked at config 2), so only lo is
//               written
//   warp 1      MMA issuer (one thread): per 8-deep K step hi.hi, hi.lo, lo.hi (M = 128, N = 64
//               or 128), commit to the stage-empty and accumulator-full barriers
//   warps 4-7   epilogue: TMEM -> registers (one lane per row), activation or routing weight in
//               f32, 32-column slabs staged through 4 KB of swizzled shared memory per warp and
//               written as full 128-byte row segments
// Shared-memory layouts: K-major operands use the 128-byte swizzle with 16-byte granules (as
// for f16/bf16); MN-major 32-bit operands must use the 128-byte swizzle with 32-byte granules
// (UMMA layout type 1; the TMA's SWIZZLE_128B_ATOM_32B writes it): 32-bit elements along N,
// 128-byte rows, the 32-byte chunk index XORed with the row index mod 4 (a 512-byte pattern).
// Stage (1024-aligned pieces): A hi 16 KB | A lo 16 KB | B hi | B lo, B = MMA_N x 128 bytes.
// Every wait is bounded (common.cuh); a timeout sets a bit in the device error word.
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {
namespace {

constexpr int kXBM = 128;                  // rows per tile
constexpr int kXBK = 32;                   // f32 per k-block: one 128-byte row
constexpr int kXThreads = 384;
constexpr int kXAHalf = kXBM * kXBK * 4;   // 16 KB
constexpr int kXStageOut = 4 * 4096;       // epilogue staging, 4 KB per warp
constexpr int kXRing = 192 * 1024;
constexpr size_t kXSmemMax = 232448 - 1024;

template <int MODE, int BN>
struct XCfg {
  static constexpr bool kGather = (MODE == kModeG1Dual || MODE == kModeG1Single);
  static constexpr bool kDual = MODE == kModeG1Dual;
  // Qwen3's gate and up columns of the tile side by side: one MMA of N = 2 * BN
  static constexpr int kMmaN = kDual ? 2 * BN : BN;
  static constexpr int kBHalf = kMmaN * kXBK * 4;
  static constexpr int kStageBytes = 2 * kXAHalf + 2 * kBHalf;
  static constexpr int kStages = kXRing / kStageBytes > 4 ? 4 : kXRing / kStageBytes;
  // bytes the TMA copies of one stage deliver (A too when it is not gathered)
  static constexpr uint32_t kTxBytes = kBHalf + (kGather ? 0 : kXAHalf);
  static constexpr uint32_t kFullCount = 1 + (kGather ? 64 : 0);
  static constexpr int kTmemCols = 2 * kMmaN <= 128 ? 128 : 256;
};

// D[tmem] (+)= A[smem] * B[smem], kind::tf32 (32-bit operands read as TF32, f32 accumulate).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Descriptor of an MN-major 32-bit operand in the 128-byte swizzle with 32-byte granules
// (layout type 1): 32-column boxes `lbo` bytes apart along N, 4-row groups 512 bytes apart
// along K.
__device__ __forceinline__ uint64_t umma_sdesc_mn32(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(1u) << 61;
  return d;
}

// hi (13 low mantissa bits cleared) and lo = v - hi of four values (hi is what the MMA reads
// from the raw value)
__device__ __forceinline__ void split4(const uint4& v, uint4& hi, uint4& lo) {
  hi.x = v.x & 0xFFFFE000u;
  hi.y = v.y & 0xFFFFE000u;
  hi.z = v.z & 0xFFFFE000u;
  hi.w = v.w & 0xFFFFE000u;
  lo.x = __float_as_uint(__uint_as_float(v.x) - __uint_as_float(hi.x));
  lo.y = __float_as_uint(__uint_as_float(v.y) - __uint_as_float(hi.y));
  lo.z = __float_as_uint(__uint_as_float(v.z) - __uint_as_float(hi.z));
  lo.w = __float_as_uint(__uint_as_float(v.w) - __uint_as_float(hi.w));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <int MODE, int BN>
__global__ void __launch_bounds__(kXThreads, 1)
    tf32x3_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                               const __grid_constant__ CUtensorMap tmB0,
                               const __grid_constant__ CUtensorMap tmB1, const Sm100Params p) {
  using C = XCfg<MODE, BN>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kStages];   // stage landed (TMA bytes + gather)
  __shared__ __align__(8) uint64_t bar_split[kStages];  // stage split into hi / lo
  __shared__ __align__(8) uint64_t bar_empty[kStages];  // stage consumed by the MMAs
  __shared__ __align__(8) uint64_t bar_accf[2];
  __shared__ __align__(8) uint64_t bar_acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t smem_base = (raw + 1023u) & ~1023u;
  const uint32_t stage_out_base = smem_base + static_cast<uint32_t>(kStages * C::kStageBytes);
  int32_t* s_tp = reinterpret_cast<int32_t*>(smem_raw + (smem_base - raw) +
                                             static_cast<size_t>(kStages) * C::kStageBytes +
                                             kXStageOut);
  int32_t* s_off = s_tp + (p.E + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const int num_kb = p.K / kXBK;

  // Launched as a programmatic dependent: the set-up below reads nothing the previous kernels
  // write and overlaps their end; the tables and operands are read after the wait.
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&bar_full[s]), C::kFullCount);
      mbar_init(smem_addr(&bar_split[s]), 4);
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
    if (!C::kGather) tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB0);
    if (C::kDual) tma_prefetch_desc(&tmB1);
  }
  if (warp == 2) {
    tmem_alloc(smem_addr(&s_tmem), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_tp[i] = __ldg(p.tile_prefix + i);
    s_off[i] = __ldg(p.offsets + i);
  }
  __syncthreads();
  const int total_tiles = s_tp[E] * p.n_tiles;
  const int G = static_cast<int>(gridDim.x);

  // tile -> (expert, first sorted row, rows present, first output column)
  auto decode = [&](int tile, int& e, int& row_base, int& valid, int& n0) {
    const int mt = tile / p.n_tiles;
    const int nt = tile - mt * p.n_tiles;
    e = expert_of_tile_smem(s_tp, E, mt);
    const int m0 = (mt - s_tp[e]) * kXBM;
    row_base = s_off[e] + m0;
    valid = min(kXBM, s_off[e + 1] - s_off[e] - m0);
    n0 = nt * BN;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += G) {
        int e, row_base, valid, n0;
        decode(tile, e, row_base, valid, n0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                 kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_addr(&bar_full[stage]);
          mbar_arrive_expect_tx(full, C::kTxBytes);
          const uint32_t a_dst = smem_base + stage * C::kStageBytes;
          const uint32_t b_dst = a_dst + 2 * kXAHalf;
          const int kc = kb * kXBK;
          if (!C::kGather) tma_load_2d(a_dst, &tmA, full, kc, row_base);
          if (MODE == kModeG2K) {
            tma_load_2d(b_dst, &tmB0, full, kc, e * p.N + n0);
          } else {
            const int krow = e * p.K + kc;
#pragma unroll
            for (int j = 0; j < BN / 32; ++j) {
              tma_load_2d(b_dst + j * 4096, &tmB0, full, n0 + j * 32, krow);
              if (C::kDual)
                tma_load_2d(b_dst + (BN / 32 + j) * 4096, &tmB1, full, n0 + j * 32, krow);
            }
          }
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
      constexpr uint32_t idesc = umma_idesc(2u, MODE == kModeG2K ? 0u : 1u, kXBM, C::kMmaN);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int lt = 0;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += G, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_bounded(smem_addr(&bar_acce[buf]),
                               static_cast<uint32_t>((lt >> 1) & 1) ^ 1u, &s_abort, p.err,
                               kErrWaitAccEmpty)) {
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * C::kMmaN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_split[stage]), phase, &s_abort, p.err,
                                 kErrWaitFull)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();
          tc_fence_after();
          const uint32_t a_hi = smem_base + stage * C::kStageBytes;
          const uint32_t a_lo = a_hi + kXAHalf;
          const uint32_t b_hi = a_hi + 2 * kXAHalf;
          const uint32_t b_lo = b_hi + C::kBHalf;
#pragma unroll
          for (int ks = 0; ks < kXBK / 8; ++ks) {
            // K-major A (and Nomic's B of h.U^T): +32 bytes per 8-deep step; MN-major B in
            // 32-column boxes 4 KB apart, +1024 bytes (8 K rows) per step
            const uint64_t ah = umma_sdesc(a_hi + ks * 32, 16, 1024);
            const uint64_t al = umma_sdesc(a_lo + ks * 32, 16, 1024);
            const uint64_t bh = MODE == kModeG2K ? umma_sdesc(b_hi + ks * 32, 16, 1024)
                                                 : umma_sdesc_mn32(b_hi + ks * 1024, 4096);
            const uint64_t bl = MODE == kModeG2K ? umma_sdesc(b_lo + ks * 32, 16, 1024)
                                                 : umma_sdesc_mn32(b_lo + ks * 1024, 4096);
            umma_tf32(d, ah, bh, idesc, (kb | ks) != 0 ? 1u : 0u);
            umma_tf32(d, ah, bl, idesc, 1u);
            umma_tf32(d, al, bh, idesc, 1u);
          }
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
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ A-row gather (GEMM-1)
    // Thread g copies 16-byte chunk c = g%8 (four f32) of rows q + 8i (q = g/8, i = 0..15),
    // into the swizzled K-major layout (chunk c of row r at chunk c ^ (r % 8) = c ^ q).
    if (C::kGather) {
      const int g = threadIdx.x - 64;
      const int c = g & 7;
      const int q = g >> 3;
      const float* x = static_cast<const float*>(p.a_rows);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += G) {
        int e, row_base, valid, n0;
        decode(tile, e, row_base, valid, n0);
        const float* src[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int tok = __ldg(p.sorted_token + row_base + min(q + 8 * i, valid - 1));
          src[i] = x + static_cast<size_t>(tok) * p.K + c * 4;
        }
        const uint32_t dst_off = static_cast<uint32_t>(q * 128 + ((c ^ q) << 4));
        for (int kb = 0; kb < num_kb; ++kb) {
          bool got = mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                       kErrWaitEmpty);
          got = __all_sync(0xffffffffu, got);
          if (!got) {
            ok = false;
            break;
          }
          const uint32_t a_dst = smem_base + stage * C::kStageBytes + dst_off;
#pragma unroll
          for (int i = 0; i < 16; ++i) cp_async16(a_dst + i * 8 * 128, src[i] + kb * kXBK);
          cp_async_mbar_arrive_noinc(smem_addr(&bar_full[stage]));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ hi / lo split
    const int t = threadIdx.x - 256;  // 0..127
    constexpr int kAChunks = kXAHalf / 16;
    constexpr int kBChunks = C::kBHalf / 16;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += G) {
      for (int kb = 0; kb < num_kb; ++kb) {
        bool got = mbar_wait_bounded(smem_addr(&bar_full[stage]), phase, &s_abort, p.err,
                                     kErrWaitFull);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          break;
        }
        const uint32_t a_hi = smem_base + stage * C::kStageBytes;
        const uint32_t b_hi = a_hi + 2 * kXAHalf;
#pragma unroll 4
        for (int i = t; i < kAChunks; i += 128) {
          uint4 hi, lo;
          split4(lds128(a_hi + i * 16), hi, lo);
          sts128(a_hi + kXAHalf + i * 16, lo);
        }
#pragma unroll 4
        for (int i = t; i < kBChunks; i += 128) {
          uint4 hi, lo;
          split4(lds128(b_hi + i * 16), hi, lo);
          sts128(b_hi + C::kBHalf + i * 16, lo);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&bar_split[stage]));
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 4-7)
    const int q = warp - 4;
    const int r = q * 32 + lane;
    float* out = static_cast<float*>(p.out);
    const uint32_t stg = stage_out_base + static_cast<uint32_t>(q * 4096);
    const int unit = lane & 7;
    int lt = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += G, ++lt) {
      int e, row_base, valid, n0;
      decode(tile, e, row_base, valid, n0);
      const int buf = lt & 1;
      const bool live = r < valid;
      int64_t orow = row_base + r;
      float wgt = 1.f;
      if (!C::kGather && live) {
        orow = __ldg(p.sorted_flat + row_base + r);
        if (p.out_row) orow = __ldg(p.out_row + orow);
        wgt = __ldg(p.sorted_w + row_base + r);
      }
      // rows this lane stores in flush round rr: row 4 rr + lane / 8 of the warp's 32
      int64_t frow[8];
      bool flive[8];
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const int src = rr * 4 + (lane >> 3);
        frow[rr] = __shfl_sync(0xffffffffu, orow, src);
        flive[rr] = __shfl_sync(0xffffffffu, live ? 1 : 0, src) != 0;
      }
      bool got = mbar_wait_bounded(smem_addr(&bar_accf[buf]), static_cast<uint32_t>((lt >> 1) & 1),
                                   &s_abort, p.err, kErrWaitAccFull);
      got = __all_sync(0xffffffffu, got);
      if (!got) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * C::kMmaN);
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 32) {
        float v[32];
        if (C::kDual) {
          uint32_t gv[32], uv[32];
          tmem_ld_32x32b_x32(tb + cc, gv);
          tmem_ld_32x32b_x32(tb + BN + cc, uv);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = act_apply(__uint_as_float(gv[i]), p.act) * __uint_as_float(uv[i]);
        } else {
          uint32_t a[32];
          tmem_ld_32x32b_x32(tb + cc, a);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = C::kGather ? act_apply(__uint_as_float(a[i]), p.act)
                              : __uint_as_float(a[i]) * wgt;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 w = make_uint4(__float_as_uint(v[4 * u]), __float_as_uint(v[4 * u + 1]),
                                     __float_as_uint(v[4 * u + 2]), __float_as_uint(v[4 * u + 3]));
          sts128(stg + lane * 128 + ((u ^ (lane & 7)) << 4), w);
        }
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int srow = rr * 4 + (lane >> 3);
          const uint4 val = lds128(stg + srow * 128 + ((unit ^ (srow & 7)) << 4));
          if (flive[rr])
            *reinterpret_cast<uint4*>(out + frow[rr] * p.N + n0 + cc + unit * 4) = val;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&bar_acce[buf]));
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
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int MODE, int BN>
size_t x_smem(int num_experts) {
  using C = XCfg<MODE, BN>;
  return static_cast<size_t>(C::kStages) * C::kStageBytes + 1024 + kXStageOut +
         static_cast<size_t>(2 * num_experts + 3) * sizeof(int32_t);
}

template <int MODE, int BN>
bool x_attr() {
  return cudaFuncSetAttribute(tf32x3_grouped_gemm_kernel<MODE, BN>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kXSmemMax)) == cudaSuccess;
}

template <int MODE, int BN>
int x_launch(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
             const Sm100Params& p, int grid, cudaStream_t s) {
  const size_t smem = x_smem<MODE, BN>(p.E);
  if (smem > kXSmemMax) return 2;
  // programmatic dependent of the previous kernel (the route preparation or GEMM-1)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kXThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tf32x3_grouped_gemm_kernel<MODE, BN>, a, b0, b1, p) ==
                 cudaSuccess
             ? 0
             : 4;
}

}  // namespace

bool tf32x3_set_attributes() {
  return x_attr<kModeG1Dual, 64>() && x_attr<kModeG1Single, 128>() && x_attr<kModeG2MN, 128>() &&
         x_attr<kModeG2MN, 64>() && x_attr<kModeG2K, 128>() && x_attr<kModeG2K, 64>();
}

int tf32x3_out_cols(int mode, int N) {
  if (mode == kModeG1Dual) return 64;
  if (mode == kModeG1Single) return 128;
  // GEMM-2: 64-column tiles when 128-column tiles would leave most SMs idle
  return N % 128 == 0 && N >= 2048 ? 128 : 64;
}

// f32 grouped GEMM of `mode` on the tensor cores (3xTF32).  a: GEMM-2's A map over the
// intermediate [rows, K] (box 32 x 128, 128-byte swizzle); b0 / b1: B maps (MN-major 32 x 32
// boxes over [E*K, N] in the 128-byte swizzle with 32-byte granules; Nomic's GEMM-2 K-major
// 32 x bn boxes over [E*N, K], 128-byte swizzle).  p.n_tiles = N / bn.
int launch_tf32x3_gemm(int mode, int bn, const CUtensorMap& a, const CUtensorMap& b0,
                       const CUtensorMap& b1, const Sm100Params& p, int grid, cudaStream_t s) {
  if (grid <= 0) return 3;
  if (p.K % kXBK != 0 || p.N % bn != 0) return 1;
  switch (mode) {
    case kModeG1Dual: return bn == 64 ? x_launch<kModeG1Dual, 64>(a, b0, b1, p, grid, s) : 1;
    case kModeG1Single:
      return bn == 128 ? x_launch<kModeG1Single, 128>(a, b0, b1, p, grid, s) : 1;
    case kModeG2MN:
      return bn == 128 ? x_launch<kModeG2MN, 128>(a, b0, b1, p, grid, s)
                       : x_launch<kModeG2MN, 64>(a, b0, b1, p, grid, s);
    case kModeG2K:
      return bn == 128 ? x_launch<kModeG2K, 128>(a, b0, b1, p, grid, s)
                       : x_launch<kModeG2K, 64>(a, b0, b1, p, grid, s);
    default: return 1;
  }
}

}  // namespace cmoe
