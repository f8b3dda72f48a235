// SIMT grouped GEMMs and the slot combine.
//
// The f32 MoE (kernels/moe.cu:193-449 in the reference) and any f16/bf16 shape the tcgen05 path
// does not take (hidden / intermediate sizes that are not multiples of its tile sizes, or
// misaligned pointers) run here: 64x64 output tiles, 16-deep K slices staged through shared
// memory as f32, 4x4 outputs per thread, f32 accumulation.  The grid's y dimension enumerates
// the linear m-tiles of all experts (tile_prefix from route preparation, tile height 64), so no
// CTA is launched for rows an expert does not have.
//
// Modes (one template instance each):
//   0  Qwen3 GEMM-1: h = act(A.G_e) * (A.U_e), A = gathered x rows   (moe.cu:193-317, has_up)
//   1  Nomic GEMM-1: h = act(A.G_e)                                    (moe.cu:193-317)
//   2  Qwen3 GEMM-2: y = h.D_e (D_e [I,H], N contiguous) times the routing weight
//   3  Nomic GEMM-2: y = h.U_e^T (U_e [H,I], K contiguous) times the routing weight
//                                                                      (moe.cu:319-449)
// GEMM-1 writes the intermediate row of each sorted row in the operand type (the reference's
// f16/bf16 path rounds it there too, nomic_moe.cu:374, qwen3_moe.cu:493).  GEMM-2 writes each
// weighted contribution to its (token, slot) row of a slot buffer; combine_slots then sums the
// k slots of a token in slot order in f32 and rounds once.  With k = 1 GEMM-2 writes the output
// row directly.
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace cmoe {

constexpr int kSimtBM = 64, kSimtBN = 64, kSimtBK = 16, kSimtThreads = 256;


template <typename T, int MODE>
__global__ void __launch_bounds__(kSimtThreads) simt_grouped_gemm_kernel(SimtParams p) {
  __shared__ __align__(16) float As[kSimtBK][kSimtBM + 4];
  __shared__ __align__(16) float Bs[kSimtBK][kSimtBN + 4];
  __shared__ __align__(16) float Bs2[MODE == 0 ? kSimtBK : 1][kSimtBN + 4];
  __shared__ int64_t s_arow[kSimtBM];

  const int mt = blockIdx.y;
  const int E = p.E, N = p.N, K = p.K;
  if (mt >= __ldg(p.tile_prefix + E)) return;
  const int e = expert_of_tile(p.tile_prefix, E, mt);
  const int m0 = (mt - __ldg(p.tile_prefix + e)) * kSimtBM;
  const int row_base = __ldg(p.offsets + e) + m0;
  const int cnt = __ldg(p.offsets + e + 1) - __ldg(p.offsets + e);
  const int valid = min(kSimtBM, cnt - m0);
  const int n0 = blockIdx.x * kSimtBN;
  const int tid = threadIdx.x;
  if (tid < kSimtBM) {
    const int r = min(tid, valid - 1);
    s_arow[tid] = (MODE <= 1) ? static_cast<int64_t>(__ldg(p.sorted_token + row_base + r))
                              : static_cast<int64_t>(row_base + r);
  }
  __syncthreads();

  const T* A = static_cast<const T*>(p.a);
  const size_t wstride = static_cast<size_t>(K) * N;
  const T* B0 = static_cast<const T*>(p.b0) + static_cast<size_t>(e) * wstride;
  const T* B1 = (MODE == 0) ? static_cast<const T*>(p.b1) + static_cast<size_t>(e) * wstride : nullptr;
  const int tx = tid & 15, ty = tid >> 4;
  float acc[4][4], acc2[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = acc2[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += kSimtBK) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int li = tid + q * kSimtThreads;
      const int r = li >> 4, c = li & 15;
      const int kk = k0 + c;
      As[c][r] = kk < K ? Elem<T>::to_f(A[s_arow[r] * K + kk]) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int li = tid + q * kSimtThreads;
      if (MODE == 3) {
        // B[kk][n] = U[n][kk]: walk K fastest for coalescing
        const int n = li >> 4, c = li & 15;
        const int kk = k0 + c, nn = n0 + n;
        Bs[c][n] = (kk < K && nn < N) ? Elem<T>::to_f(B0[static_cast<size_t>(nn) * K + kk]) : 0.f;
      } else {
        const int c = li >> 6, n = li & 63;
        const int kk = k0 + c, nn = n0 + n;
        const bool ok = kk < K && nn < N;
        Bs[c][n] = ok ? Elem<T>::to_f(B0[static_cast<size_t>(kk) * N + nn]) : 0.f;
        if (MODE == 0) Bs2[c][n] = ok ? Elem<T>::to_f(B1[static_cast<size_t>(kk) * N + nn]) : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtBK; ++kk) {
      const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b4 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
      const float b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      if (MODE == 0) {
        const float4 u4 = *reinterpret_cast<const float4*>(&Bs2[kk][tx * 4]);
        const float u[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc2[i][j] = fmaf(a[i], u[j], acc2[i][j]);
      }
    }
    __syncthreads();
  }

  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty * 4 + i;
    if (r >= valid) continue;
    int64_t orow;
    float wgt = 1.f;
    if (MODE <= 1) {
      orow = row_base + r;
    } else {
      orow = __ldg(p.sorted_flat + row_base + r);
      if (p.out_row) orow = __ldg(p.out_row + orow);
      wgt = __ldg(p.sorted_w + row_base + r);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v;
      if (MODE == 0) v = act_apply(acc[i][j], p.act) * acc2[i][j];
      else if (MODE == 1) v = act_apply(acc[i][j], p.act);
      else v = acc[i][j] * wgt;
      out[orow * N + n] = Elem<T>::from_f(v);
    }
  }
}

// f32 operands whose rows start on 16-byte boundaries (K and N multiples of 4, aligned bases):
// float4 global loads, the next 16-deep K slice loaded into registers while the current one is
// multiplied out of shared memory (two buffers, one barrier per slice), 64 x BN tiles with 4 x 8
// (BN = 128) or 4 x 4 (BN = 64) outputs per thread; the column groups of a thread sit 64 apart.
// Same modes, tile list, rounding and epilogue as simt_grouped_gemm_kernel.
template <int MODE, int BN>
__global__ void __launch_bounds__(kSimtThreads) simt_f32v_kernel(SimtParams p) {
  constexpr int BM = 64, BK = 16, TN = BN / 16, NB = BN / 64;  // NB float4 of B per thread
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];
  __shared__ __align__(16) float Us[MODE == 0 ? 2 : 1][MODE == 0 ? BK : 1][BN + 4];
  __shared__ int64_t s_arow[BM];

  const int mt = blockIdx.y;
  const int E = p.E, N = p.N, K = p.K;
  if (mt >= __ldg(p.tile_prefix + E)) return;
  const int e = expert_of_tile(p.tile_prefix, E, mt);
  const int m0 = (mt - __ldg(p.tile_prefix + e)) * BM;
  const int row_base = __ldg(p.offsets + e) + m0;
  const int cnt = __ldg(p.offsets + e + 1) - __ldg(p.offsets + e);
  const int valid = min(BM, cnt - m0);
  const int n0 = blockIdx.x * BN;
  const int tid = threadIdx.x;
  if (tid < BM) {
    const int r = min(tid, valid - 1);
    s_arow[tid] = (MODE <= 1) ? static_cast<int64_t>(__ldg(p.sorted_token + row_base + r))
                              : static_cast<int64_t>(row_base + r);
  }
  __syncthreads();

  const float* A = static_cast<const float*>(p.a);
  const size_t wstride = static_cast<size_t>(K) * N;
  const float* B0 = static_cast<const float*>(p.b0) + static_cast<size_t>(e) * wstride;
  const float* B1 = MODE == 0 ? static_cast<const float*>(p.b1) + static_cast<size_t>(e) * wstride
                              : nullptr;
  // loader coordinates: A row tid/4, k quad (tid%4)*4; B float4 index tid + 256*i
  const int a_r = tid >> 2, a_c = (tid & 3) * 4;
  const float* a_src = A + s_arow[a_r] * K + a_c;
  float4 ra, rb[NB], ru[NB];
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  auto load_regs = [&](int k0) {
    ra = k0 + a_c < K ? __ldg(reinterpret_cast<const float4*>(a_src + k0)) : z4;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int idx = tid + kSimtThreads * i;
      if (MODE == 3) {  // B[k][n] = U[n][k]: 4 consecutive k of one n
        const int n = n0 + (idx >> 2), kk = k0 + (idx & 3) * 4;
        rb[i] = (n < N && kk < K)
                    ? __ldg(reinterpret_cast<const float4*>(B0 + static_cast<size_t>(n) * K + kk))
                    : z4;
      } else {  // 4 consecutive n of one k
        const int kk = k0 + idx / (BN / 4), n = n0 + (idx % (BN / 4)) * 4;
        const bool ok = kk < K && n < N;
        const size_t o = static_cast<size_t>(kk) * N + n;
        rb[i] = ok ? __ldg(reinterpret_cast<const float4*>(B0 + o)) : z4;
        if (MODE == 0) ru[i] = ok ? __ldg(reinterpret_cast<const float4*>(B1 + o)) : z4;
      }
    }
  };
  auto store_smem = [&](int buf) {
    As[buf][a_c + 0][a_r] = ra.x;
    As[buf][a_c + 1][a_r] = ra.y;
    As[buf][a_c + 2][a_r] = ra.z;
    As[buf][a_c + 3][a_r] = ra.w;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int idx = tid + kSimtThreads * i;
      if (MODE == 3) {
        const int n = idx >> 2, kq = (idx & 3) * 4;
        Bs[buf][kq + 0][n] = rb[i].x;
        Bs[buf][kq + 1][n] = rb[i].y;
        Bs[buf][kq + 2][n] = rb[i].z;
        Bs[buf][kq + 3][n] = rb[i].w;
      } else {
        const int kk = idx / (BN / 4), n = (idx % (BN / 4)) * 4;
        *reinterpret_cast<float4*>(&Bs[buf][kk][n]) = rb[i];
        if (MODE == 0) *reinterpret_cast<float4*>(&Us[buf][kk][n]) = ru[i];
      }
    }
  };

  const int tx = tid & 15, ty = tid >> 4;
  float acc[4][TN], acc2[MODE == 0 ? 4 : 1][MODE == 0 ? TN : 1];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      acc[i][j] = 0.f;
      if (MODE == 0) acc2[i][j] = 0.f;
    }

  load_regs(0);
  store_smem(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) load_regs(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
      float b[TN], u[MODE == 0 ? TN : 1];
#pragma unroll
      for (int g = 0; g < TN / 4; ++g) {
        const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][kk][g * 64 + tx * 4]);
        b[g * 4 + 0] = b4.x;
        b[g * 4 + 1] = b4.y;
        b[g * 4 + 2] = b4.z;
        b[g * 4 + 3] = b4.w;
        if (MODE == 0) {
          const float4 u4 = *reinterpret_cast<const float4*>(&Us[buf][kk][g * 64 + tx * 4]);
          u[g * 4 + 0] = u4.x;
          u[g * 4 + 1] = u4.y;
          u[g * 4 + 2] = u4.z;
          u[g * 4 + 3] = u4.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          if (MODE == 0) acc2[i][j] = fmaf(a[i], u[j], acc2[i][j]);
        }
    }
    if (more) store_smem(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

  float* out = static_cast<float*>(p.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty * 4 + i;
    if (r >= valid) continue;
    int64_t orow;
    float wgt = 1.f;
    if (MODE <= 1) {
      orow = row_base + r;
    } else {
      orow = __ldg(p.sorted_flat + row_base + r);
      if (p.out_row) orow = __ldg(p.out_row + orow);
      wgt = __ldg(p.sorted_w + row_base + r);
    }
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + (j / 4) * 64 + tx * 4 + (j % 4);
      if (n >= N) continue;
      float v;
      if (MODE == 0) v = act_apply(acc[i][j], p.act) * acc2[i][j];
      else if (MODE == 1) v = act_apply(acc[i][j], p.act);
      else v = acc[i][j] * wgt;
      out[orow * N + n] = v;
    }
  }
}

// out[t, :] = sum over slots j < k whose expert id is < E of slot[t*k + j, :], in slot order,
// accumulated in f32 and rounded once.  V elements (16 bytes) per thread when H allows it.  KC
// slots are handled per pass with all their loads in flight together (the expert ids first, then
// every present row), so a token's k rows are fetched concurrently instead of one DRAM round trip
// after another.
template <typename T, int V, int KC>
__global__ void __launch_bounds__(256) combine_slots_kernel(const T* __restrict__ slot,
                                                            const uint32_t* __restrict__ idx,
                                                            int64_t num_tokens, int k, int H,
                                                            int E, T* __restrict__ out) {
  const int vec_per_row = H / V;
  const int64_t total = num_tokens * vec_per_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = v / vec_per_row;
    const int c = static_cast<int>(v - t * vec_per_row) * V;
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int j0 = 0; j0 < k; j0 += KC) {
      bool ok[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j)
        ok[j] = j0 + j < k && __ldg(idx + t * k + j0 + j) < static_cast<uint32_t>(E);
      uint4 q[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const T* src = slot + (t * k + j0 + j) * H + c;
        if (V * sizeof(T) == 16) {
          q[j] = ok[j] ? __ldcs(reinterpret_cast<const uint4*>(src)) : make_uint4(0, 0, 0, 0);
        } else {
          T* qe = reinterpret_cast<T*>(&q[j]);
#pragma unroll
          for (int i = 0; i < V; ++i) qe[i] = ok[j] ? src[i] : Elem<T>::from_f(0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        if (!ok[j]) continue;  // slot order is kept: rows are added in j order
        const T* qe = reinterpret_cast<const T*>(&q[j]);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += Elem<T>::to_f(qe[i]);
      }
    }
    T* dst = out + t * H + c;
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

// ---- host launchers --------------------------------------------------------------------------

template <int BN>
static void simt_f32v_launch(int mode, const SimtParams& p, int64_t mtile_bound, cudaStream_t s) {
  dim3 grid((p.N + BN - 1) / BN, static_cast<unsigned>(mtile_bound));
  switch (mode) {
    case 0: simt_f32v_kernel<0, BN><<<grid, kSimtThreads, 0, s>>>(p); break;
    case 1: simt_f32v_kernel<1, BN><<<grid, kSimtThreads, 0, s>>>(p); break;
    case 2: simt_f32v_kernel<2, BN><<<grid, kSimtThreads, 0, s>>>(p); break;
    default: simt_f32v_kernel<3, BN><<<grid, kSimtThreads, 0, s>>>(p); break;
  }
}

template <typename T>
static void simt_launch_t(int mode, const SimtParams& p, int64_t mtile_bound, cudaStream_t s) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (sizeof(T) == 4 && p.K % 4 == 0 && p.N % 4 == 0 && a16(p.a) && a16(p.b0) &&
      (mode != 0 || a16(p.b1))) {
    if (p.N >= 1024) simt_f32v_launch<128>(mode, p, mtile_bound, s);
    else simt_f32v_launch<64>(mode, p, mtile_bound, s);
    return;
  }
  dim3 grid((p.N + kSimtBN - 1) / kSimtBN, static_cast<unsigned>(mtile_bound));
  switch (mode) {
    case 0: simt_grouped_gemm_kernel<T, 0><<<grid, kSimtThreads, 0, s>>>(p); break;
    case 1: simt_grouped_gemm_kernel<T, 1><<<grid, kSimtThreads, 0, s>>>(p); break;
    case 2: simt_grouped_gemm_kernel<T, 2><<<grid, kSimtThreads, 0, s>>>(p); break;
    default: simt_grouped_gemm_kernel<T, 3><<<grid, kSimtThreads, 0, s>>>(p); break;
  }
}

int simt_tile_m() { return kSimtBM; }

// mtile_bound: an upper bound of the number of linear m-tiles (grid y); CTAs past the real
// count exit at once.
int launch_simt_gemm(int dtype, int mode, const SimtParams& p, int64_t mtile_bound,
                     cudaStream_t s) {
  if (mtile_bound <= 0) return 0;
  if (mtile_bound > 65535) return 2;
  if (dtype == kF32) simt_launch_t<float>(mode, p, mtile_bound, s);
  else if (dtype == kBF16) simt_launch_t<__nv_bfloat16>(mode, p, mtile_bound, s);
  else simt_launch_t<__half>(mode, p, mtile_bound, s);
  return 0;
}

template <typename T>
static void combine_t(const void* slot, const uint32_t* idx, int64_t T_, int k, int H, int E,
                      void* out, int num_sms, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = (H % V) == 0 && (reinterpret_cast<uintptr_t>(slot) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) % 16) == 0;
  const int64_t work = T_ * (vec ? H / V : H);
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (vec) {
    if (k <= 2)
      combine_slots_kernel<T, V, 2><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
          static_cast<const T*>(slot), idx, T_, k, H, E, static_cast<T*>(out));
    else if (k <= 4)
      combine_slots_kernel<T, V, 4><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
          static_cast<const T*>(slot), idx, T_, k, H, E, static_cast<T*>(out));
    else
      combine_slots_kernel<T, V, 8><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
          static_cast<const T*>(slot), idx, T_, k, H, E, static_cast<T*>(out));
  } else {
    combine_slots_kernel<T, 1, 4><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const T*>(slot), idx, T_, k, H, E, static_cast<T*>(out));
  }
}

int launch_combine(int dtype, const void* slot, const uint32_t* idx, int64_t num_tokens, int k,
                   int H, int E, void* out, int num_sms, cudaStream_t s) {
  if (num_tokens <= 0) return 0;
  if (dtype == kF32) combine_t<float>(slot, idx, num_tokens, k, H, E, out, num_sms, s);
  else if (dtype == kBF16) combine_t<__nv_bfloat16>(slot, idx, num_tokens, k, H, E, out, num_sms, s);
  else combine_t<__half>(slot, idx, num_tokens, k, H, E, out, num_sms, s);
  return 0;
}

// ---- row movement for the expert-parallel exchange ------------------------------------------

// dst[r, :] = src[index[r], :], 16 bytes per thread where the row allows it.
template <typename V>
__global__ void __launch_bounds__(256) gather_rows_kernel(const V* __restrict__ src,
                                                          const int32_t* __restrict__ index,
                                                          int64_t rows, int vec_per_row,
                                                          V* __restrict__ dst) {
  const int64_t total = rows * vec_per_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = v / vec_per_row;
    const int c = static_cast<int>(v - r * vec_per_row);
    dst[v] = src[static_cast<int64_t>(__ldg(index + r)) * vec_per_row + c];
  }
}

// inv[flat[r]] = r for r < rows (inv pre-filled with -1 by the caller)
__global__ void __launch_bounds__(256) invert_rows_kernel(const int32_t* __restrict__ flat,
                                                          int64_t rows, int32_t* __restrict__ inv) {
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x)
    inv[__ldg(flat + r)] = static_cast<int32_t>(r);
}

// out[t, :] = sum over slots j (in slot order) with inv[t*k+j] >= 0 of rows_buf[inv[t*k+j], :],
// accumulated in f32 and rounded once -- the slot-ordered combine of combine_slots_kernel with
// one indirection, for contributions that come back from other ranks in exchange order.
template <typename T, int V, int KC>
__global__ void __launch_bounds__(256) combine_indirect_kernel(const T* __restrict__ rows_buf,
                                                               const int32_t* __restrict__ inv,
                                                               int64_t num_tokens, int k, int H,
                                                               T* __restrict__ out) {
  const int vec_per_row = H / V;
  const int64_t total = num_tokens * vec_per_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = v / vec_per_row;
    const int c = static_cast<int>(v - t * vec_per_row) * V;
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int j0 = 0; j0 < k; j0 += KC) {
      int32_t r[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j) r[j] = j0 + j < k ? __ldg(inv + t * k + j0 + j) : -1;
      uint4 q[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const T* src = rows_buf + static_cast<int64_t>(r[j] < 0 ? 0 : r[j]) * H + c;
        if (V * sizeof(T) == 16) {
          q[j] = r[j] >= 0 ? __ldcs(reinterpret_cast<const uint4*>(src)) : make_uint4(0, 0, 0, 0);
        } else {
          T* qe = reinterpret_cast<T*>(&q[j]);
#pragma unroll
          for (int i = 0; i < V; ++i) qe[i] = r[j] >= 0 ? src[i] : Elem<T>::from_f(0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        if (r[j] < 0) continue;
        const T* qe = reinterpret_cast<const T*>(&q[j]);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += Elem<T>::to_f(qe[i]);
      }
    }
    T* dst = out + t * H + c;
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

static unsigned grid_for(int64_t work, int num_sms) {
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

int launch_gather_rows(int dtype, const void* src, const int32_t* index, int64_t rows, int H,
                       void* dst, int num_sms, cudaStream_t s) {
  if (rows <= 0) return 0;
  const size_t row_bytes = static_cast<size_t>(H) * (dtype == kF32 ? 4 : 2);
  if (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src) % 16) == 0 &&
      (reinterpret_cast<uintptr_t>(dst) % 16) == 0) {
    const int vpr = static_cast<int>(row_bytes / 16);
    gather_rows_kernel<uint4><<<grid_for(rows * vpr, num_sms), 256, 0, s>>>(
        static_cast<const uint4*>(src), index, rows, vpr, static_cast<uint4*>(dst));
  } else if (row_bytes % 4 == 0) {
    const int vpr = static_cast<int>(row_bytes / 4);
    gather_rows_kernel<uint32_t><<<grid_for(rows * vpr, num_sms), 256, 0, s>>>(
        static_cast<const uint32_t*>(src), index, rows, vpr, static_cast<uint32_t*>(dst));
  } else {
    const int vpr = static_cast<int>(row_bytes / 2);
    gather_rows_kernel<uint16_t><<<grid_for(rows * vpr, num_sms), 256, 0, s>>>(
        static_cast<const uint16_t*>(src), index, rows, vpr, static_cast<uint16_t*>(dst));
  }
  return 0;
}

template <typename T>
static void combine_indirect_t(const void* rows_buf, const int32_t* inv, int64_t T_, int k, int H,
                               void* out, int num_sms, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = (H % V) == 0 && (reinterpret_cast<uintptr_t>(rows_buf) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) % 16) == 0;
  if (vec) {
    if (k <= 2)
      combine_indirect_kernel<T, V, 2><<<grid_for(T_ * (H / V), num_sms), 256, 0, s>>>(
          static_cast<const T*>(rows_buf), inv, T_, k, H, static_cast<T*>(out));
    else if (k <= 4)
      combine_indirect_kernel<T, V, 4><<<grid_for(T_ * (H / V), num_sms), 256, 0, s>>>(
          static_cast<const T*>(rows_buf), inv, T_, k, H, static_cast<T*>(out));
    else
      combine_indirect_kernel<T, V, 8><<<grid_for(T_ * (H / V), num_sms), 256, 0, s>>>(
          static_cast<const T*>(rows_buf), inv, T_, k, H, static_cast<T*>(out));
  } else {
    combine_indirect_kernel<T, 1, 4><<<grid_for(T_ * H, num_sms), 256, 0, s>>>(
        static_cast<const T*>(rows_buf), inv, T_, k, H, static_cast<T*>(out));
  }
}

// inv: caller scratch of num_tokens*k int32.
int launch_combine_indirect(int dtype, const void* rows_buf, const int32_t* flat, int64_t rows,
                            int64_t num_tokens, int k, int H, int32_t* inv, void* out,
                            int num_sms, cudaStream_t s) {
  if (num_tokens <= 0) return 0;
  if (cudaMemsetAsync(inv, 0xff, sizeof(int32_t) * static_cast<size_t>(num_tokens) * k, s) !=
      cudaSuccess)
    return 3;
  if (rows > 0)
    invert_rows_kernel<<<grid_for(rows, num_sms), 256, 0, s>>>(flat, rows, inv);
  if (dtype == kF32) combine_indirect_t<float>(rows_buf, inv, num_tokens, k, H, out, num_sms, s);
  else if (dtype == kBF16) combine_indirect_t<__nv_bfloat16>(rows_buf, inv, num_tokens, k, H, out, num_sms, s);
  else combine_indirect_t<__half>(rows_buf, inv, num_tokens, k, H, out, num_sms, s);
  return 0;
}

}  // namespace cmoe
