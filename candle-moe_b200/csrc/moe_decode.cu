// D1: the expert FFN of decode-sized calls on the 5th-generation tensor cores, as a weight stream.
//
// Replaces the reference's direct kernels (qwen3_moe.cu:85-263, nomic_moe.cu:6-174: one CTA per
// routed (token, slot), each streaming its expert's whole weight matrices, so an expert picked by
// several tokens is read several times).  With a few routed rows per expert the FFN is bound by
// reading each routed expert's weights once; the M = 128 row tiles of the grouped GEMMs would
// be almost empty and their tile count (experts x column tiles) leaves SMs idle.  Here the
// operands are swapped: the WEIGHTS are the MMA's A operand (M = 128 output columns of the
// weight matrix, streamed by TMA straight from the API layout) and the routed token rows are B
// (N = 16, 32 or 64 rows of one expert, gathered with cp.async), so one MMA produces 128 output
// columns for all of the expert's rows:
//   GEMM-1  [Qwen3]  g|u^T = G_e^T x^T, U_e^T x^T  (gate [E,H,I], up [E,H,I]: MN-major A)
//           [Nomic]  g^T   = G_e^T x^T
//           epilogue: act(g) * u (Qwen3) or act(g) (Nomic), rounded to the operand type, into
//           the intermediate rows (expert-sorted, as the route preparation orders them)
//   GEMM-2  [Qwen3]  y^T = D_e^T h^T  (down [E,I,H]: MN-major A)
//           [Nomic]  y^T = U_e h^T    (up [E,H,I] as h.U^T: K-major A)
//           epilogue: y * routing weight rounded to the operand type into the (token, slot)
//           row, then -- once every expert's contribution to a 128-column tile of the output
//           is in -- the slot-ordered sum of each token's k contributions (f32, one rounding)
//           into the output: the combine is fused, the same arithmetic as combine_slots_kernel.
//
// Work is split "stream-K": the units (expert row chunk x 128-column tile) each need K/64
// k-blocks; their concatenated k-block range is cut into gridDim.x equal contiguous pieces, one
// per CTA (one CTA per SM), so every SM streams the same number of weight bytes whatever the
// routing.  A unit cut between CTAs is finished by the last CTA to arrive: each piece's f32
// partial sum goes to scratch (`partials`, two slots per CTA: its first and its last unit), an
// atomic counter per (unit, 32-row quarter) elects the last arrival, which adds the pieces in
// CTA order -- a fixed order, so results are deterministic for a given grid.
//
// Warp roles (256 threads): warp 0 one thread = TMA producer of the weight tiles; warps 2-3 =
// cp.async gather of the B rows (warp 2 also owns TMEM); warp 1 one thread = tcgen05.mma
// issuer; warps 4-7 = epilogue (TMEM lane quarter warp % 4), each warp independent of the others
// (its own counters), so no CTA-wide barrier is needed after the set-up.  TMEM holds two
// accumulator buffers so the epilogue of one unit overlaps the MMAs of the next.  Every wait is
// bounded (common.cuh); a timeout sets a bit in the device error word and the kernel drains.
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {

constexpr int kDecThreads = 256;
constexpr int kDecM = 128;                 // weight output columns per unit (the MMA's M)
constexpr int kDecK = 64;                  // reduction elements per stage
// Operand ring per CTA: 96-110 KB, enough bytes in flight to stream at the HBM rate with one
// CTA per SM (a TMA stream of 64 x 64 boxes with 96 KB in flight per SM measured 6.9 TB/s on
// B200), and small enough that a GEMM-2 CTA fits beside a GEMM-1 CTA: GEMM-2 is launched as a
// programmatic dependent of GEMM-1, so its set-up and its first weight tiles overlap GEMM-1's
// last units.
constexpr int kDecRingBytes = 110 * 1024;
constexpr int kDecMaxExperts = 1024;
constexpr int kDecMaxGrid = 256;

template <int MODE, int N>
struct DecCfg {
  static constexpr bool kDual = MODE == kModeG1Dual;
  static constexpr bool kG1 = MODE == kModeG1Dual || MODE == kModeG1Single;
  static constexpr bool kAMN = MODE != kModeG2K;  // weights MN-major, except Nomic's h.U^T
  static constexpr int kAccs = kDual ? 2 : 1;
  static constexpr int kABytes = kAccs * kDecM * kDecK * 2;           // 16 or 32 KB
  static constexpr int kBBytes = (N * 128 + 1023) / 1024 * 1024;      // N rows x 64 x 2 B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages =
      kDecRingBytes / kStageBytes > 8 ? 8 : kDecRingBytes / kStageBytes;
  static_assert(kStages >= 2, "operand ring too small");
  static constexpr int kAccCols = kAccs * N;                          // TMEM columns / buffer
  static constexpr int kTmemCols = 2 * kAccCols <= 32 ? 32 : 2 * kAccCols <= 64 ? 64
                                 : 2 * kAccCols <= 128 ? 128 : 256;
  static constexpr uint32_t kFullCount = 1 + 64;  // TMA thread + the 64 gather threads
  static constexpr int kPartFloats = kAccs * N * kDecM;
};

template <typename T> struct DecFmt;
template <> struct DecFmt<__half> { static constexpr uint32_t v = 0; };
template <> struct DecFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

// kind::f16 instruction descriptor, f32 accumulate: A MN-major (weights) or K-major, B K-major.
__host__ __device__ constexpr uint32_t dec_idesc(uint32_t fmt, uint32_t a_mn, uint32_t n) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_mn << 15) | ((n >> 3) << 17) |
         ((static_cast<uint32_t>(kDecM) >> 4) << 24);
}

// First k-block of CTA c when W k-blocks are cut into G contiguous pieces.
__device__ __forceinline__ int64_t sk_start(int64_t c, int64_t W, int G) { return c * W / G; }

// The work of one CTA: first its stream-K share of the first U_sk units (W_sk = U_sk * KB
// k-blocks cut into G equal pieces; U_sk < G, so a share touches at most two units and is never
// a whole one), then the whole units U_sk + c, U_sk + c + G, ... below U.  With the split pieces
// first, the exchange that finishes a cut unit overlaps the streaming of the whole units, and a
// CTA's last piece (when it has whole units) needs no exchange.
struct DecWork {
  int64_t w, w1;      // stream-K k-block cursor and end
  int64_t u, u_end;   // next whole unit, end of the unit list
  int G;
};

__device__ __forceinline__ DecWork dec_work(int64_t U, int KB, int G, int c, int64_t* W_sk) {
  const int64_t rounds = U / G;
  const int64_t u_sk = U - rounds * G;
  *W_sk = u_sk * KB;
  DecWork d;
  d.w = sk_start(c, *W_sk, G);
  d.w1 = sk_start(c + 1, *W_sk, G);
  d.u = u_sk + c;
  d.u_end = U;
  d.G = G;
  return d;
}

// Next piece (unit u, k-blocks [kb_lo, kb_hi)) of a CTA's work; false when there is none.
__device__ __forceinline__ bool dec_next(DecWork& d, int KB, int64_t& u, int& kb_lo,
                                         int& kb_hi) {
  if (d.w < d.w1) {
    u = d.w / KB;
    kb_lo = static_cast<int>(d.w - u * KB);
    kb_hi = static_cast<int>(d.w1 - u * KB < KB ? d.w1 - u * KB : KB);
    d.w = u * KB + kb_hi;
    return true;
  }
  if (d.u < d.u_end) {
    u = d.u;
    kb_lo = 0;
    kb_hi = KB;
    d.u += d.G;
    return true;
  }
  return false;
}

// Programmatic dependent launch: let the next kernel in the stream (launched with the
// programmatic-serialization attribute) start its CTAs now / wait until the previous kernel's
// writes are visible.  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Arrival on a counter that publishes this thread's (and, through a preceding warp barrier, its
// warp's) earlier writes and, for the last arrival, acquires everyone else's.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}

// f32 value of the 16-bit storage of a T.
template <typename T> __device__ __forceinline__ float raw_to_f(unsigned short u);
template <> __device__ __forceinline__ float raw_to_f<__nv_bfloat16>(unsigned short u) {
  return __uint_as_float(static_cast<uint32_t>(u) << 16);
}
template <> __device__ __forceinline__ float raw_to_f<__half>(unsigned short u) {
  return __half2float(__ushort_as_half(u));
}

struct DecUnit {
  int e, mt, base, valid;
};

__device__ __forceinline__ DecUnit dec_unit(const int32_t* s_cp, const int32_t* s_off, int E,
                                            int MT, int64_t u) {
  DecUnit d;
  const int c = static_cast<int>(u / MT);
  d.mt = static_cast<int>(u - static_cast<int64_t>(c) * MT);
  d.e = expert_of_tile_smem(s_cp, E, c);
  return d;
}

template <typename T, int MODE, int N>
__global__ void __launch_bounds__(kDecThreads, 1)
    decode_ffn_kernel(const __grid_constant__ CUtensorMap tmA0,
                      const __grid_constant__ CUtensorMap tmA1, const DecodeParams p) {
  using C = DecCfg<MODE, N>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[C::kStages];
  __shared__ __align__(8) uint64_t bar_empty[C::kStages];
  __shared__ __align__(8) uint64_t bar_accf[2];
  __shared__ __align__(8) uint64_t bar_acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t smem_base = (raw + 1023u) & ~1023u;
  int32_t* s_cp = reinterpret_cast<int32_t*>(smem_raw + (smem_base - raw) +
                                             static_cast<size_t>(C::kStages) * C::kStageBytes);
  int32_t* s_off = s_cp + (p.E + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const int MT = p.M / kDecM;
  const int KB = p.K / kDecK;
  const int G = static_cast<int>(gridDim.x);

  // Set-up that reads nothing the previous kernels write (barriers, descriptors, TMEM) runs
  // before the wait, so that it overlaps the route preparation, which lets GEMM-1 launch early.
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_addr(&bar_full[s]), C::kFullCount);
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
    tma_prefetch_desc(&tmA0);
    if (C::kDual) tma_prefetch_desc(&tmA1);
  }
  if (warp == 2) {
    tmem_alloc(smem_addr(&s_tmem), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;

  // GEMM-1 waits for the route preparation's tables, then lets GEMM-2 launch: GEMM-2's CTAs
  // take the SMs' free shared memory, set up and stream their first weight tiles while GEMM-1
  // finishes (GEMM-2 reads the tables, complete by then, at once, and waits for GEMM-1's
  // intermediate rows before it reads them).
  if (C::kG1) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_launch_dependents();
  }
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_cp[i] = __ldg(p.chunk_prefix + i);
    s_off[i] = __ldg(p.offsets + i);
  }
  __syncthreads();
  const int chunks = s_cp[E];
  if (chunks == 0) {
    // no routed row at all: GEMM-2 still owes the caller an output of zeros
    if (!C::kG1) {
      T* out = static_cast<T*>(p.final_out);
      const int64_t n = static_cast<int64_t>(p.num_tokens) * p.M;
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
           i += static_cast<int64_t>(G) * blockDim.x)
        out[i] = Elem<T>::from_f(0.f);
    }
    if (warp == 2) {
      tc_fence_after();
      tmem_dealloc(tmem_base, C::kTmemCols);
    }
    return;
  }
  const int64_t U = static_cast<int64_t>(chunks) * MT;
  int64_t W = 0;  // k-blocks of the stream-K part
  const DecWork work0 = dec_work(U, KB, G, static_cast<int>(blockIdx.x), &W);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (weights)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      DecWork work = work0;
      int64_t u;
      int kb_lo, kb_hi;
      while (ok && dec_next(work, KB, u, kb_lo, kb_hi)) {
        const DecUnit d = dec_unit(s_cp, s_off, E, MT, u);
        const int m0 = d.mt * kDecM;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                 kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_addr(&bar_full[stage]);
          mbar_arrive_expect_tx(full, C::kABytes);
          const uint32_t a_dst = smem_base + stage * C::kStageBytes;
          if (C::kAMN) {
            // [E*K rows, M cols]: two 64 x 64 boxes side by side per weight matrix
            const int krow = d.e * p.K + kb * kDecK;
            tma_load_2d(a_dst, &tmA0, full, m0, krow);
            tma_load_2d(a_dst + 8192, &tmA0, full, m0 + 64, krow);
            if (C::kDual) {
              tma_load_2d(a_dst + 16384, &tmA1, full, m0, krow);
              tma_load_2d(a_dst + 16384 + 8192, &tmA1, full, m0 + 64, krow);
            }
          } else {
            // [E*M rows, K cols]: one 64 (K) x 128 (M) box
            tma_load_2d(a_dst, &tmA0, full, kb * kDecK, d.e * p.M + m0);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = dec_idesc(DecFmt<T>::v, C::kAMN ? 1u : 0u, N);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int piece = 0;
      DecWork work = work0;
      int64_t u;
      int kb_lo, kb_hi;
      for (; ok && dec_next(work, KB, u, kb_lo, kb_hi); ++piece) {
        const int buf = piece & 1;
        if (!mbar_wait_bounded(smem_addr(&bar_acce[buf]),
                               static_cast<uint32_t>((piece >> 1) & 1) ^ 1u, &s_abort, p.err,
                               kErrWaitAccEmpty)) {
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * C::kAccCols);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait_bounded(smem_addr(&bar_full[stage]), phase, &s_abort, p.err,
                                 kErrWaitFull)) {
            ok = false;
            break;
          }
          // the B rows were written by cp.async (generic proxy); the MMA reads them through
          // the async proxy
          fence_proxy_async_smem();
          tc_fence_after();
          const uint32_t a_base = smem_base + stage * C::kStageBytes;
          const uint32_t b_base = a_base + C::kABytes;
#pragma unroll
          for (int ks = 0; ks < kDecK / 16; ++ks) {
            const uint64_t bdesc = umma_sdesc(b_base + ks * 32, 16, 1024);
            const uint32_t acc = (kb != kb_lo || ks != 0) ? 1u : 0u;
            if (C::kAMN) {
              umma_f16(d, umma_sdesc(a_base + ks * 2048, 8192, 1024), bdesc, idesc, acc);
              if (C::kDual)
                umma_f16(d + N, umma_sdesc(a_base + 16384 + ks * 2048, 8192, 1024), bdesc,
                         idesc, acc);
            } else {
              umma_f16(d, umma_sdesc(a_base + ks * 32, 16, 1024), bdesc, idesc, acc);
            }
          }
          umma_commit(smem_addr(&bar_empty[stage]));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_addr(&bar_accf[buf]));
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ B-row gather
    // Thread g copies 16-byte chunk c = g % 8 of rows q + 8i (q = g / 8) of each stage into the
    // 128-byte-swizzled K-major layout (chunk c of row r at c ^ (r % 8)).  Rows past the unit's
    // valid ones repeat its last row; their accumulator columns are never stored.
    const int g = threadIdx.x - 64;
    const int c = g & 7;
    const int q = g >> 3;
    const T* src_base = static_cast<const T*>(p.b_src);
    // GEMM-2's B rows are GEMM-1's output: wait until GEMM-1 has completed
    if (!C::kG1) pdl_wait();
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    DecWork work = work0;
    int64_t u;
    int kb_lo, kb_hi;
    while (ok && dec_next(work, KB, u, kb_lo, kb_hi)) {
      const DecUnit d = dec_unit(s_cp, s_off, E, MT, u);
      const int chunk = static_cast<int>(u / MT);
      const int base = s_off[d.e] + (chunk - s_cp[d.e]) * N;
      const int last = min(N, s_off[d.e + 1] - base) - 1;
      const T* src[N / 8];
#pragma unroll
      for (int i = 0; i < N / 8; ++i) {
        const int r = base + min(q + 8 * i, last);
        const int row = C::kG1 ? __ldg(p.sorted_token + r) : r;
        src[i] = src_base + static_cast<size_t>(row) * p.K + c * 8;
      }
      const uint32_t dst_off = static_cast<uint32_t>(q * 128 + ((c ^ q) << 4));
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        bool got = mbar_wait_bounded(smem_addr(&bar_empty[stage]), phase ^ 1u, &s_abort, p.err,
                                     kErrWaitEmpty);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          break;
        }
        const uint32_t b_dst = smem_base + stage * C::kStageBytes + C::kABytes + dst_off;
#pragma unroll
        for (int i = 0; i < N / 8; ++i) cp_async16(b_dst + i * 8 * 128, src[i] + kb * kDecK);
        cp_async_mbar_arrive_noinc(smem_addr(&bar_full[stage]));
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 4-7)
    const int q = warp & 3;          // TMEM lane quarter
    const int m = q * 32 + lane;     // weight output column within the unit's 128
    int piece = 0;
    DecWork work = work0;
    int64_t u;
    int kb_lo, kb_hi;
    for (; dec_next(work, KB, u, kb_lo, kb_hi); ++piece) {
      const DecUnit d = dec_unit(s_cp, s_off, E, MT, u);
      const int chunk = static_cast<int>(u / MT);
      const int base = s_off[d.e] + (chunk - s_cp[d.e]) * N;
      const int valid = min(N, s_off[d.e + 1] - base);
      const int buf = piece & 1;
      bool got = mbar_wait_bounded(smem_addr(&bar_accf[buf]),
                                   static_cast<uint32_t>((piece >> 1) & 1), &s_abort, p.err,
                                   kErrWaitAccFull);
      got = __all_sync(0xffffffffu, got);
      if (!got) break;
      tc_fence_after();
      float v[C::kAccCols];
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * C::kAccCols);
#pragma unroll
      for (int c0 = 0; c0 < C::kAccCols; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tb + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) v[c0 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&bar_acce[buf]));

      if (kb_lo != 0 || kb_hi != KB) {
        // a piece of a unit cut between CTAs: publish it, and finish the unit if last
        const int64_t first_unit = work0.w / KB;
        float* sp = p.partials + (static_cast<size_t>(blockIdx.x) * 2 + (u == first_unit ? 0 : 1)) *
                                     C::kPartFloats;
#pragma unroll
        for (int i = 0; i < C::kAccCols; ++i) __stcg(sp + i * kDecM + m, v[i]);
        __syncwarp();
        // the CTAs holding pieces of u: c_lo.. while their range starts before the unit's end
        const int64_t lo = u * KB, hi = lo + KB;
        int64_t c_lo = lo * G / W;
        while (c_lo > 0 && sk_start(c_lo, W, G) > lo) --c_lo;
        while (sk_start(c_lo + 1, W, G) <= lo) ++c_lo;
        uint32_t pieces = 0;
        for (int64_t cc = c_lo; cc < G && sk_start(cc, W, G) < hi; ++cc)
          if (sk_start(cc + 1, W, G) > sk_start(cc, W, G)) ++pieces;
        uint32_t old = 0;
        if (lane == 0) old = atom_add_acq_rel_gpu(p.unit_counter + u * 4 + q, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old + 1 != pieces) continue;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < C::kAccCols; ++i) v[i] = 0.f;
        for (int64_t cc = c_lo; cc < G && sk_start(cc, W, G) < hi; ++cc) {
          const int64_t s0 = sk_start(cc, W, G);
          if (sk_start(cc + 1, W, G) <= s0) continue;
          const float* pp = p.partials +
                            (static_cast<size_t>(cc) * 2 + (u == s0 / KB ? 0 : 1)) * C::kPartFloats;
#pragma unroll
          for (int i = 0; i < C::kAccCols; ++i) v[i] += __ldcg(pp + i * kDecM + m);
        }
      }

      const int col = d.mt * kDecM + m;
      if (C::kG1) {
        T* inter = static_cast<T*>(p.out);
#pragma unroll
        for (int n = 0; n < N; ++n) {
          if (n < valid) {
            const float h = C::kDual ? act_apply(v[n], p.act) * v[N + n] : act_apply(v[n], p.act);
            inter[static_cast<size_t>(base + n) * p.M + col] = Elem<T>::from_f(h);
          }
        }
      } else {
        T* slot = static_cast<T*>(p.out);
        // the chunk's (flat index, routing weight) pairs: lane l holds rows l and l + 32, so
        // the stores below wait on no load
        constexpr int kR = N > 32 ? N / 32 : 1;
        int fl[kR];
        float wl[kR];
#pragma unroll
        for (int i = 0; i < kR; ++i) {
          const int r = i * 32 + lane;
          fl[i] = r < valid ? __ldg(p.sorted_flat + base + r) : 0;
          wl[i] = r < valid ? __ldg(p.sorted_w + base + r) : 0.f;
        }
#pragma unroll
        for (int n = 0; n < N; ++n) {
          const int flat = __shfl_sync(0xffffffffu, fl[n / 32], n % 32);
          const float wgt = __shfl_sync(0xffffffffu, wl[n / 32], n % 32);
          if (n < valid) slot[static_cast<size_t>(flat) * p.M + col] = Elem<T>::from_f(v[n] * wgt);
        }
        // the last unit of this 128-column tile (any expert) sums every token's slots
        __syncwarp();
        uint32_t old = 0;
        if (lane == 0) old = atom_add_acq_rel_gpu(p.tile_counter + d.mt * 4 + q, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old + 1 == static_cast<uint32_t>(chunks)) {
          __syncwarp();
          T* out = static_cast<T*>(p.final_out);
          const int k = p.k;
          const int T_ = p.num_tokens;
          const int tb = k < 32 ? 32 / k : 1;  // tokens per batch: their k slots in 32 lanes
          for (int t0 = 0; t0 < T_; t0 += tb) {
            const int nf = min(tb, T_ - t0) * k;
            const int f0 = t0 * k;
            const bool ok_j = lane < nf && __ldg(p.idx + f0 + lane) < static_cast<uint32_t>(E);
            const uint32_t okm = __ballot_sync(0xffffffffu, ok_j);
            // every load of the batch is issued before the sums: rows past the batch or of
            // skipped slots read row f0 (any readable address) and are masked out below
            unsigned short raw[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int f = (okm >> j) & 1u ? f0 + j : f0;
              raw[j] = __ldcg(reinterpret_cast<const unsigned short*>(slot) +
                              static_cast<size_t>(f) * p.M + col);
            }
            float acc = 0.f;
            int jj = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < nf) {
                // slot order, as combine_slots_kernel
                if ((okm >> j) & 1u) acc += raw_to_f<T>(raw[j]);
                if (++jj == k) {
                  out[static_cast<size_t>(t0 + j / k) * p.M + col] = Elem<T>::from_f(acc);
                  acc = 0.f;
                  jj = 0;
                }
              }
            }
          }
        }
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
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---- host side -------------------------------------------------------------------------------

int decode_max_experts() { return kDecMaxExperts; }
int decode_max_grid() { return kDecMaxGrid; }

int decode_chunk_rows(int64_t num_tokens) {
  if (num_tokens <= 16) return 16;
  if (num_tokens <= 32) return 32;
  return 64;
}

size_t decode_partial_bytes(int n, int grid) {
  // two slots per CTA of the widest accumulator (Qwen3 GEMM-1: gate and up)
  return static_cast<size_t>(grid) * 2 * 2 * n * kDecM * sizeof(float);
}

template <typename T, int MODE, int N>
static size_t dec_smem(int num_experts) {
  using C = DecCfg<MODE, N>;
  return static_cast<size_t>(C::kStages) * C::kStageBytes + 1024 +
         static_cast<size_t>(2 * num_experts + 2) * sizeof(int32_t);
}

template <typename T, int MODE, int N>
static bool dec_attr() {
  return cudaFuncSetAttribute(decode_ffn_kernel<T, MODE, N>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(dec_smem<T, MODE, N>(kDecMaxExperts))) ==
         cudaSuccess;
}

template <typename T, int N>
static bool dec_attr_n() {
  return dec_attr<T, kModeG1Dual, N>() && dec_attr<T, kModeG1Single, N>() &&
         dec_attr<T, kModeG2MN, N>() && dec_attr<T, kModeG2K, N>();
}

bool decode_set_attributes() {
  bool ok = dec_attr_n<__nv_bfloat16, 16>() && dec_attr_n<__nv_bfloat16, 32>() &&
            dec_attr_n<__nv_bfloat16, 64>();
  ok &= dec_attr_n<__half, 16>() && dec_attr_n<__half, 32>() && dec_attr_n<__half, 64>();
  return ok;
}

// Launch with the programmatic-serialization attribute: the kernel may start before the
// previous kernel in the stream completes (the kernels wait with griddepcontrol.wait before
// reading its outputs).
template <typename T, int MODE, int N>
static int dec_launch_one(const CUtensorMap& a0, const CUtensorMap& a1, const DecodeParams& p,
                          int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = dec_smem<T, MODE, N>(p.E);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_ffn_kernel<T, MODE, N>, a0, a1, p) == cudaSuccess ? 0
                                                                                          : 4;
}

template <typename T, int N>
static int dec_launch_n(int mode, const CUtensorMap& a0, const CUtensorMap& a1,
                        const DecodeParams& p, int grid, cudaStream_t s) {
#define CMOE_DEC(MODE) return dec_launch_one<T, MODE, N>(a0, a1, p, grid, s);
  switch (mode) {
    case kModeG1Dual: CMOE_DEC(kModeG1Dual)
    case kModeG1Single: CMOE_DEC(kModeG1Single)
    case kModeG2MN: CMOE_DEC(kModeG2MN)
    case kModeG2K: CMOE_DEC(kModeG2K)
    default: return 1;
  }
#undef CMOE_DEC
}

template <typename T>
static int dec_launch_t(int mode, int n, const CUtensorMap& a0, const CUtensorMap& a1,
                        const DecodeParams& p, int grid, cudaStream_t s) {
  if (n == 16) return dec_launch_n<T, 16>(mode, a0, a1, p, grid, s);
  if (n == 32) return dec_launch_n<T, 32>(mode, a0, a1, p, grid, s);
  if (n == 64) return dec_launch_n<T, 64>(mode, a0, a1, p, grid, s);
  return 1;
}

int launch_decode_ffn(int dtype, int mode, int n, const CUtensorMap& a0, const CUtensorMap& a1,
                      const DecodeParams& p, int grid, cudaStream_t s) {
  if (grid <= 0 || grid > kDecMaxGrid || p.E > kDecMaxExperts) return 3;
  if (p.M % kDecM != 0 || p.K % kDecK != 0) return 1;
  if (dtype == kBF16) return dec_launch_t<__nv_bfloat16>(mode, n, a0, a1, p, grid, s);
  if (dtype == kF16) return dec_launch_t<__half>(mode, n, a0, a1, p, grid, s);
  return 1;
}

}  // namespace cmoe
