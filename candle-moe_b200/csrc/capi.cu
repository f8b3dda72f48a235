// C ABI of candle-moe-b200 (declared in include/candle_moe.h): argument checks, per-device
// state, the stream-ordered workspace pool, TMA tensor maps and the dispatch of the router,
// route-preparation, grouped-GEMM and combine kernels.
//
// Reference counterparts: topk_softmax -> kernels/topk_softmax.cu:331-353; fused_moe ->
// kernels/moe.cu:451-773 (direct/GEMM path selection, per-call workspace, preprocessing,
// per-dtype dispatch); moe_route_prep -> kernels/preprocessing.cuh:253-313.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/candle_moe.h"
#include "common.cuh"
#include "kernels.h"

#define CMOE_API extern "C" __attribute__((visibility("default")))

namespace cmoe {
namespace {

thread_local int t_last_status = MOE_OK;
thread_local int t_last_path = 0;
std::atomic<int> g_gemm_path{0};
std::atomic<int> g_sm_reserve{0};  // SMs the persistent GEMMs leave free (moe_set_sm_reserve)

constexpr int kMaxDevices = 64;

struct DeviceState {
  std::atomic<bool> ready{false};
  int num_sms = 0;
  int max_pairs = 0;  // 2-CTA clusters of the pair GEMMs resident at once
  int cc_major = 0, cc_minor = 0;
  cudaMemPool_t pool = nullptr;
  uint32_t* err_word = nullptr;
};

DeviceState g_dev[kMaxDevices];

// ---- benchmark instrumentation: kernel launch counter and per-phase CUDA events ------------
std::atomic<int64_t> g_launches{0};
constexpr int kPhases = 4;  // route preparation, GEMM-1, GEMM-2, combine
struct PhaseTimer {
  std::mutex mu;
  bool on = false;
  std::vector<cudaEvent_t> events;  // kPhases + 1 per recorded call
  int64_t calls = 0;
};
PhaseTimer g_timer;

// Events for the next timed call (nullptr when timing is off).
cudaEvent_t* timer_slots() {
  std::lock_guard<std::mutex> lk(g_timer.mu);
  if (!g_timer.on) return nullptr;
  const size_t need = static_cast<size_t>(g_timer.calls + 1) * (kPhases + 1);
  while (g_timer.events.size() < need) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g_timer.events.push_back(e);
  }
  cudaEvent_t* slot = g_timer.events.data() + g_timer.calls * (kPhases + 1);
  ++g_timer.calls;
  return slot;
}
std::mutex g_dev_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int init_device(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return MOE_ERR_UNSUPPORTED;
  DeviceState& d = g_dev[dev];
  if (d.ready.load(std::memory_order_acquire)) {
    *out = &d;
    return MOE_OK;
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!d.ready.load(std::memory_order_relaxed)) {
    if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return MOE_ERR_CUDA;
    cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaMemPoolProps props;
    std::memset(&props, 0, sizeof(props));
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    if (cudaMemPoolCreate(&d.pool, &props) != cudaSuccess) return MOE_ERR_CUDA;
    uint64_t keep = UINT64_MAX;  // keep freed blocks cached for the next call
    cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep);
    if (cudaMalloc(&d.err_word, sizeof(uint32_t)) != cudaSuccess) return MOE_ERR_CUDA;
    if (cudaMemset(d.err_word, 0, sizeof(uint32_t)) != cudaSuccess) return MOE_ERR_CUDA;
    const bool attrs_ok = route_prep_set_attributes() && sm100_set_attributes() &&
                          sm100_pair_set_attributes() && decode_set_attributes() &&
                          router_project_set_attributes() && tf32x3_set_attributes();
    cudaGetLastError();  // attribute failures are reported here, not by a later call
    if (!attrs_ok) return MOE_ERR_CUDA;
    d.max_pairs = sm100_pair_max_clusters();
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
              cudaSuccess &&
          q == cudaDriverEntryPointSuccess)
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    d.ready.store(true, std::memory_order_release);
  }
  *out = &d;
  return MOE_OK;
}

int current_device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  return init_device(dev, out);
}

inline size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// 2-D tensor map over a row-major [outer, inner] matrix of 16-bit elements, 128-byte swizzle.
// swizzle: the 128-byte swizzle with 16-byte granules, or (MN-major f32 operands of the TF32
// MMA) with 32-byte granules.
bool make_map_2d(CUtensorMap* map, int dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (!g_encode) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * (dtype == kF32 ? 4 : 2)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == kF32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Largest token count the decode kernels take by default (the reference's direct path takes
// T <= 32 as well, moe.cu:481); above it the grouped GEMMs' 128-row tiles fill up.
constexpr int64_t kDecodeMaxTokens = 32;

// Rows per expert chunk of the decode kernels (moe_decode.cu) for this call, or 0 when the
// grouped GEMMs serve it: f16/bf16 with 128-aligned H and I, at most kDecodeMaxTokens tokens
// (any count with GEMM path 6), not with GEMM paths 1, 4 and 5.  Pointer alignment and the
// device are checked by the caller (sm100_shape_ok).
int decode_rows(int64_t T, int H, int I, int E, int dtype, int gpath) {
  if (dtype == kF32 || H % 128 != 0 || I % 128 != 0 || E > decode_max_experts()) return 0;
  if (gpath == 1 || gpath == 4 || gpath == 5) return 0;
  if (T > kDecodeMaxTokens && gpath != 6) return 0;
  return decode_chunk_rows(T);
}

// Workspace of one fused call (byte offsets into one buffer).
struct FusedLayout {
  size_t offsets, tile_prefix, counters, sorted_token, sorted_flat, sorted_w, prep_scratch, inter,
      slot, dec_part, dec_cnt, total;
  int64_t dec_units1, dec_units2;  // unit-counter capacity of the decode GEMMs
};

// dec_n: rows per chunk of the decode kernels (0: the grouped GEMMs run).
FusedLayout fused_layout(int64_t T, int H, int I, int E, int k, int dtype, int dec_n = 0) {
  const int64_t rows = T * k;
  const size_t elt = dtype == kF32 ? 4 : 2;
  FusedLayout L;
  size_t o = 0;
  L.offsets = o;        o += align256(sizeof(int32_t) * (E + 2));
  L.tile_prefix = o;    o += align256(sizeof(int32_t) * (E + 1));
  L.counters = o;       o += align256(sizeof(uint32_t) * 2);  // tile counters of the 2 GEMMs
  L.sorted_token = o;   o += align256(sizeof(int32_t) * rows);
  L.sorted_flat = o;    o += align256(sizeof(int32_t) * rows);
  L.sorted_w = o;       o += align256(sizeof(float) * rows);
  L.prep_scratch = o;   o += align256(route_prep_scratch_bytes(rows, E));
  L.inter = o;          o += align256(elt * static_cast<size_t>(rows) * I);
  // the decode kernels always combine through the (token, slot) rows, also for k = 1
  L.slot = o;           o += (k > 1 || dec_n) ? align256(elt * static_cast<size_t>(rows) * H) : 0;
  L.dec_part = o;
  L.dec_units1 = L.dec_units2 = 0;
  if (dec_n) {
    // one region per GEMM: GEMM-2 starts while GEMM-1's last units are being finished
    o += 2 * align256(decode_partial_bytes(dec_n, decode_max_grid()));
    const int64_t chunks = rows / dec_n + (E < rows ? E : rows);
    L.dec_units1 = chunks * (I / 128);
    L.dec_units2 = chunks * (H / 128);
  }
  L.dec_cnt = o;
  if (dec_n) o += align256(sizeof(uint32_t) * 4 * (L.dec_units1 + L.dec_units2 + H / 128));
  L.total = o;
  return L;
}

int finish(int status) {
  if (status == MOE_OK) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) status = MOE_ERR_CUDA;
  }
  return status;
}

// SMs the persistent tensor-core GEMMs may use: all but the reserve, and at least one (the
// reserve is a performance hint; a GEMM is never skipped because of it).
int gemm_sms(const DeviceState* ds) {
  const int sms = ds->num_sms - g_sm_reserve.load();
  return sms < 1 ? 1 : sms;
}

// 2-CTA clusters for the pair GEMMs: one per two usable SMs, no more than can be resident at
// once (0: the pair kernels cannot run; the one-CTA kernel takes the GEMM).
int pair_grid(const DeviceState* ds, int sms) {
  const int pairs = sms / 2;
  return pairs < ds->max_pairs ? pairs : ds->max_pairs;
}

bool sm100_shape_ok(int dtype, const void* x, const void* g, const void* u, const void* d,
                    const void* out, int H, int I, int E, int moe_type) {
  if (dtype == kF32) return false;
  if (E > sm100_max_experts()) return false;
  if (H % 128 != 0 || I % 128 != 0) return false;
  if (!aligned16(x) || !aligned16(g) || !aligned16(u) || !aligned16(out)) return false;
  if (moe_type == 0 && !aligned16(d)) return false;
  return true;
}

// f32 operands on the tensor cores (moe_tf32.cu): the same tile constraints as f16/bf16.
bool tf32_shape_ok(int dtype, const void* x, const void* g, const void* u, const void* d,
                   const void* out, int H, int I, int E, int moe_type) {
  if (dtype != kF32) return false;
  if (E > sm100_max_experts()) return false;
  if (H % 128 != 0 || I % 128 != 0) return false;
  if (!aligned16(x) || !aligned16(g) || !aligned16(u) || !aligned16(out)) return false;
  if (moe_type == 0 && !aligned16(d)) return false;
  return true;
}

// out_row == nullptr: the drop-in semantics (output [T,H], the k slots of a token combined).
// out_row != nullptr: no combine; the weighted contribution of every routed (t, j) is written to
// row out_row[t*k + j] of `output` (rows must be distinct).
int fused_impl(const void* input, const void* gate, const void* up, const void* down,
               const float* rw, const uint32_t* idx, void* output, int64_t T, int H, int I, int E,
               int k, int act, uint32_t moe_type, uint32_t dtype, void* workspace,
               size_t workspace_bytes, cudaStream_t stream, const int32_t* out_row = nullptr) {
  t_last_path = 0;
  if (dtype > 2 || moe_type > 1) return MOE_ERR_INVALID_ARG;
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0) return MOE_ERR_INVALID_ARG;
  if (T == 0) return MOE_OK;
  if (!input || !gate || !up || !rw || !idx || !output) return MOE_ERR_INVALID_ARG;
  if (moe_type == 0 && !down) return MOE_ERR_INVALID_ARG;
  if (E > route_prep_max_experts()) return MOE_ERR_UNSUPPORTED;
  if (T * k > INT32_MAX) return MOE_ERR_UNSUPPORTED;

  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;

  const int gpath = g_gemm_path.load();
  bool use_sm100 = sm100_shape_ok(static_cast<int>(dtype), input, gate, up, down, output, H, I,
                                  E, static_cast<int>(moe_type)) &&
                   ds->cc_major == 10 && g_encode != nullptr;
  bool use_tf32 = tf32_shape_ok(static_cast<int>(dtype), input, gate, up, down, output, H, I, E,
                                static_cast<int>(moe_type)) &&
                  ds->cc_major == 10 && g_encode != nullptr;
  if (gpath == 1) use_sm100 = use_tf32 = false;
  if (gpath == 2 && !use_sm100 && !use_tf32) return MOE_ERR_UNSUPPORTED;

  const bool scatter = out_row != nullptr;
  // decode-sized calls: weight-streaming tensor-core kernels with the combine fused
  const int dec_n = (use_sm100 && !scatter)
                        ? decode_rows(T, H, I, E, static_cast<int>(dtype), gpath)
                        : 0;
  const int bm = dec_n ? dec_n : (use_sm100 || use_tf32) ? sm100_tile_m() : simt_tile_m();
  // scatter writes each contribution to its own output row: no slot buffer, no combine
  FusedLayout L = fused_layout(T, H, I, E, k, static_cast<int>(dtype), dec_n);
  if (scatter) L.total = L.slot;
  char* ws = static_cast<char*>(workspace);
  bool owned = false;
  if (ws == nullptr) {
    void* p = nullptr;
    if (cudaMallocFromPoolAsync(&p, L.total, ds->pool, stream) != cudaSuccess) {
      cudaGetLastError();
      return MOE_ERR_NO_MEMORY;
    }
    ws = static_cast<char*>(p);
    owned = true;
  } else if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) {
    return MOE_ERR_WORKSPACE;
  }

  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* tile_prefix = reinterpret_cast<int32_t*>(ws + L.tile_prefix);
  int32_t* s_token = reinterpret_cast<int32_t*>(ws + L.sorted_token);
  int32_t* s_flat = reinterpret_cast<int32_t*>(ws + L.sorted_flat);
  float* s_w = reinterpret_cast<float*>(ws + L.sorted_w);
  void* prep_scratch = ws + L.prep_scratch;
  void* inter = ws + L.inter;
  void* slot = (k > 1 && !scatter) ? static_cast<void*>(ws + L.slot) : output;

  const int64_t rows = T * k;
  const int64_t mtile_bound = rows / bm + (E < rows ? E : rows);
  const size_t elt = dtype == kF32 ? 4 : 2;
  cudaEvent_t* ev = timer_slots();
  if (ev) cudaEventRecord(ev[0], stream);
  int64_t launches = route_prep_scratch_bytes(rows, E) ? 3 : 1;

  // the decode kernels' counters are cleared by the route preparation itself, so that GEMM-1
  // follows it directly (it is launched as the route preparation's programmatic dependent)
  const int64_t dec_ncnt = dec_n ? 4 * (L.dec_units1 + L.dec_units2 + H / 128) : 0;
  if (st == MOE_OK)
    st = launch_route_prep(idx, rw, T, k, E, bm, offsets, tile_prefix, s_token, s_w, s_flat,
                           prep_scratch, stream,
                           reinterpret_cast<uint32_t*>(ws + L.dec_cnt), dec_ncnt) == 0
             ? MOE_OK
             : MOE_ERR_UNSUPPORTED;
  if (st == MOE_OK && k == 1 && !scatter && !dec_n)
    if (cudaMemsetAsync(output, 0, elt * static_cast<size_t>(T) * H, stream) != cudaSuccess)
      st = MOE_ERR_CUDA;
  if (ev) cudaEventRecord(ev[1], stream);

  uint32_t* counters = reinterpret_cast<uint32_t*>(ws + L.counters);
  if (st == MOE_OK && dec_n) {
    // ---------------------------------------------------------------- decode kernels (D1)
    uint32_t* dcnt = reinterpret_cast<uint32_t*>(ws + L.dec_cnt);
    const int grid = std::min(gemm_sms(ds), decode_max_grid());
    DecodeParams p;
    p.offsets = offsets;
    p.chunk_prefix = tile_prefix;
    p.sorted_token = s_token;
    p.sorted_flat = s_flat;
    p.sorted_w = s_w;
    p.idx = idx;
    p.partials = reinterpret_cast<float*>(ws + L.dec_part);
    p.err = ds->err_word;
    p.E = E;
    p.act = act;
    p.k = k;
    p.num_tokens = static_cast<int>(T);
    CUtensorMap mA0, mA1, mW2;
    const int mode1 = moe_type == 0 ? kModeG1Dual : kModeG1Single;
    const int mode2 = moe_type == 0 ? kModeG2MN : kModeG2K;
    bool ok = st == MOE_OK &&
              make_map_2d(&mA0, dtype, gate, I, static_cast<uint64_t>(E) * H, 64, 64) &&
              make_map_2d(&mA1, dtype, up, I, static_cast<uint64_t>(E) * H, 64, 64) &&
              (mode2 == kModeG2MN
                   ? make_map_2d(&mW2, dtype, down, H, static_cast<uint64_t>(E) * I, 64, 64)
                   : make_map_2d(&mW2, dtype, up, I, static_cast<uint64_t>(E) * H, 64, 128));
    if (ok) {
      p.b_src = input;
      p.out = inter;
      p.final_out = nullptr;
      p.unit_counter = dcnt;
      p.tile_counter = nullptr;
      p.M = I;
      p.K = H;
      ok = launch_decode_ffn(static_cast<int>(dtype), mode1, dec_n, mA0, mA1, p, grid, stream) == 0;
    }
    if (ev) cudaEventRecord(ev[2], stream);
    if (ok) {
      p.b_src = inter;
      p.out = ws + L.slot;
      p.final_out = output;
      p.partials = reinterpret_cast<float*>(
          ws + L.dec_part + align256(decode_partial_bytes(dec_n, decode_max_grid())));
      p.unit_counter = dcnt + 4 * L.dec_units1;
      p.tile_counter = dcnt + 4 * (L.dec_units1 + L.dec_units2);
      p.M = H;
      p.K = I;
      ok = launch_decode_ffn(static_cast<int>(dtype), mode2, dec_n, mW2, mW2, p, grid, stream) == 0;
    }
    if (!ok && st == MOE_OK) st = MOE_ERR_CUDA;
    if (ev) cudaEventRecord(ev[3], stream);
    t_last_path = 3;
  } else if (st == MOE_OK && use_sm100) {
    if (cudaMemsetAsync(counters, 0, 2 * sizeof(uint32_t), stream) != cudaSuccess) st = MOE_ERR_CUDA;
  }
  if (st == MOE_OK && use_sm100 && !dec_n) {
    // GEMM-1
    CUtensorMap mA, mB0, mB1;
    const int mode1 = moe_type == 0 ? kModeG1Dual : kModeG1Single;
    // Output tiles as wide as the shape allows, also for decode-sized calls: a tile's weight
    // stream runs at (bytes in flight per SM) / latency, which grows with the tile width, so
    // narrower tiles on more SMs move the weights no faster and add waves (measured on B200:
    // 64-wide gate|up tiles took GEMM-1 of a top-2 decode step at 8 tokens to 92 us).
    auto pick_bn = [](int n, int widest, int narrowest) {
      int bn = widest;
      while (bn > narrowest && n % bn != 0) bn /= 2;
      return bn;
    };
    const int bn1 = mode1 == kModeG1Dual ? pick_bn(I, 128, 64) : pick_bn(I, 256, 128);
    const int cols1 = sm100_out_cols(mode1, bn1);
    // GEMM-1 gathers its A rows with cp.async; mA is an unused placeholder there
    bool ok = make_map_2d(&mA, dtype, input, H, T, 64, 64) &&
              make_map_2d(&mB0, dtype, gate, I, static_cast<uint64_t>(E) * H, 64, 64) &&
              make_map_2d(&mB1, dtype, up, I, static_cast<uint64_t>(E) * H, 64, 64);
    Sm100Params p;
    p.out_row = nullptr;
    p.a_rows = input;
    p.offsets = offsets;
    p.tile_prefix = tile_prefix;
    p.sorted_token = s_token;
    p.sorted_flat = s_flat;
    p.sorted_w = s_w;
    p.E = E;
    p.act = act;
    p.err = ds->err_word;
    if (ok) {
      p.out = inter;
      p.tile_counter = counters;
      p.N = I;
      p.K = H;
      p.n_tiles = I / cols1;
      const int64_t tiles = mtile_bound * p.n_tiles;
      const int sms = gemm_sms(ds);
      bool done = false;
      if (g_gemm_path.load() == 4 && !scatter && mode1 == kModeG1Dual && bn1 == 128) {
        // CTA pairs (cta_group::2) as for GEMM-2 below; opt-in only: correct, and measured as
        // fast as the one-CTA GEMM-1 at configs 4 and 5, not faster
        const int64_t pair_tiles = (rows / 256 + (E < rows ? E : rows)) * p.n_tiles;
        const int pairs = static_cast<int>(std::min<int64_t>(pair_tiles, pair_grid(ds, sms)));
        done = launch_sm100_gemm1_pair(static_cast<int>(dtype), mB0, mB1, p, pairs, stream) == 0;
      }
      const int grid = static_cast<int>(tiles < sms ? tiles : sms);
      if (!done &&
          launch_sm100_gemm(static_cast<int>(dtype), mode1, bn1, mA, mB0, mB1, p, grid, stream))
        ok = false;
    }
    if (ev) cudaEventRecord(ev[2], stream);
    // GEMM-2
    const int mode2 = moe_type == 0 ? kModeG2MN : kModeG2K;
    const int bn2 = pick_bn(H, 256, 128);
    if (ok) {
      ok = make_map_2d(&mA, dtype, inter, I, static_cast<uint64_t>(rows), 64, 128);
      if (mode2 == kModeG2MN)
        ok = ok && make_map_2d(&mB0, dtype, down, H, static_cast<uint64_t>(E) * I, 64, 64);
      else
        ok = ok && make_map_2d(&mB0, dtype, up, I, static_cast<uint64_t>(E) * H, 64, bn2);
    }
    if (ok) {
      p.out = slot;
      p.out_row = out_row;
      p.tile_counter = counters + 1;
      p.N = H;
      p.K = I;
      p.n_tiles = H / sm100_out_cols(mode2, bn2);
      const int64_t tiles = mtile_bound * p.n_tiles;
      const int sms = gemm_sms(ds);
      bool done = false;
      if (g_gemm_path.load() != 3 && (!scatter || g_sm_reserve.load() == 0) &&
          mode2 == kModeG2MN && bn2 == 256) {
        // CTA pairs (cta_group::2): tiles of 256 rows, static schedule; shapes it does not take
        // fall through to the one-CTA kernel, which also serves the scatter calls that leave
        // SMs to other kernels (the collective exchange: a static schedule would wait for CTAs
        // held back by them, where the one-CTA kernel's dynamic one does not)
        const int64_t pair_tiles = (rows / 256 + (E < rows ? E : rows)) * p.n_tiles;
        const int pairs = static_cast<int>(std::min<int64_t>(pair_tiles, pair_grid(ds, sms)));
        done = launch_sm100_gemm2_pair(static_cast<int>(dtype), mA, mB0, p, pairs, stream) == 0;
      }
      if (!done) {
        const int grid = static_cast<int>(tiles < sms ? tiles : sms);
        if (launch_sm100_gemm(static_cast<int>(dtype), mode2, bn2, mA, mB0, mB0, p, grid,
                              stream))
          ok = false;
      }
    }
    if (!ok) st = MOE_ERR_CUDA;
    t_last_path = 2;
  } else if (st == MOE_OK && use_tf32) {
    // ---------------------------------------------------------------- f32: 3xTF32 GEMMs
    const int mode1 = moe_type == 0 ? kModeG1Dual : kModeG1Single;
    const int mode2 = moe_type == 0 ? kModeG2MN : kModeG2K;
    const int bn1 = tf32x3_out_cols(mode1, I), bn2 = tf32x3_out_cols(mode2, H);
    const int sms = gemm_sms(ds);
    const CUtensorMapSwizzle mn32 = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    CUtensorMap mA, mB0, mB1;
    Sm100Params p;
    p.a_rows = input;
    p.offsets = offsets;
    p.tile_prefix = tile_prefix;
    p.sorted_token = s_token;
    p.sorted_flat = s_flat;
    p.sorted_w = s_w;
    p.out_row = nullptr;
    p.E = E;
    p.act = act;
    p.err = ds->err_word;
    p.tile_counter = nullptr;
    // GEMM-1 gathers its A rows with cp.async; mA (the intermediate) serves GEMM-2
    bool ok = make_map_2d(&mA, dtype, inter, I, static_cast<uint64_t>(rows), 32, 128) &&
              make_map_2d(&mB0, dtype, gate, I, static_cast<uint64_t>(E) * H, 32, 32, mn32) &&
              make_map_2d(&mB1, dtype, up, I, static_cast<uint64_t>(E) * H, 32, 32, mn32);
    if (ok) {
      p.out = inter;
      p.N = I;
      p.K = H;
      p.n_tiles = I / bn1;
      const int64_t tiles = mtile_bound * p.n_tiles;
      ok = launch_tf32x3_gemm(mode1, bn1, mA, mB0, mB1, p,
                              static_cast<int>(tiles < sms ? tiles : sms), stream) == 0;
    }
    if (ev) cudaEventRecord(ev[2], stream);
    if (ok) {
      ok = mode2 == kModeG2MN
               ? make_map_2d(&mB0, dtype, down, H, static_cast<uint64_t>(E) * I, 32, 32, mn32)
               : make_map_2d(&mB0, dtype, up, I, static_cast<uint64_t>(E) * H, 32, bn2);
    }
    if (ok) {
      p.out = slot;
      p.out_row = out_row;
      p.N = H;
      p.K = I;
      p.n_tiles = H / bn2;
      const int64_t tiles = mtile_bound * p.n_tiles;
      ok = launch_tf32x3_gemm(mode2, bn2, mA, mB0, mB0, p,
                              static_cast<int>(tiles < sms ? tiles : sms), stream) == 0;
    }
    if (!ok) st = MOE_ERR_CUDA;
    t_last_path = 2;
  } else if (st == MOE_OK && !dec_n) {
    SimtParams p;
    p.out_row = nullptr;
    p.offsets = offsets;
    p.tile_prefix = tile_prefix;
    p.sorted_token = s_token;
    p.sorted_flat = s_flat;
    p.sorted_w = s_w;
    p.E = E;
    p.act = act;
    p.a = input;
    p.b0 = gate;
    p.b1 = up;
    p.out = inter;
    p.N = I;
    p.K = H;
    st = launch_simt_gemm(static_cast<int>(dtype), moe_type == 0 ? 0 : 1, p, mtile_bound, stream) == 0
             ? MOE_OK
             : MOE_ERR_UNSUPPORTED;
    if (ev) cudaEventRecord(ev[2], stream);
    if (st == MOE_OK) {
      p.a = inter;
      p.b0 = moe_type == 0 ? down : up;
      p.b1 = nullptr;
      p.out = slot;
      p.out_row = out_row;
      p.N = H;
      p.K = I;
      st = launch_simt_gemm(static_cast<int>(dtype), moe_type == 0 ? 2 : 3, p, mtile_bound, stream) == 0
               ? MOE_OK
               : MOE_ERR_UNSUPPORTED;
    }
    t_last_path = 1;
  }
  if (ev && !dec_n) cudaEventRecord(ev[3], stream);
  launches += 2;
  if (st == MOE_OK && k > 1 && !scatter && !dec_n) {
    launch_combine(static_cast<int>(dtype), slot, idx, T, k, H, E, output, ds->num_sms, stream);
    ++launches;
  }
  if (ev) cudaEventRecord(ev[4], stream);
  if (st == MOE_OK) g_launches += launches;
  if (owned) cudaFreeAsync(ws, stream);
  return finish(st);
}

}  // namespace

// Kernel launches made by entry points defined in other translation units.
void add_launches(int64_t n) { g_launches += n; }

}  // namespace cmoe

using namespace cmoe;

CMOE_API int moe_last_status(void) { return t_last_status; }

CMOE_API const char* moe_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_UNSUPPORTED: return "unsupported";
    case MOE_ERR_CUDA: return "cuda error";
    case MOE_ERR_WORKSPACE: return "workspace too small or misaligned";
    case MOE_ERR_NO_MEMORY: return "out of device memory";
    default: return "unknown status";
  }
}

CMOE_API int moe_topk_softmax_v2(const float* gating_output, float* topk_weights,
                                 int32_t* topk_indices, int32_t* token_expert_indices,
                                 int32_t num_experts, int64_t num_tokens, int32_t topk,
                                 int32_t renormalize, void* stream) {
  if (num_tokens < 0 || topk <= 0 || num_experts <= 0) return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0) return MOE_OK;
  if (num_tokens > INT32_MAX) return MOE_ERR_UNSUPPORTED;
  if (!gating_output || !topk_weights || !topk_indices || !token_expert_indices)
    return MOE_ERR_INVALID_ARG;
  if ((num_experts & (num_experts - 1)) != 0 || num_experts > 256) return MOE_ERR_UNSUPPORTED;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (launch_router(gating_output, topk_weights, topk_indices, token_expert_indices, num_experts,
                    static_cast<int>(num_tokens), topk, renormalize, ds->num_sms,
                    static_cast<cudaStream_t>(stream)) != 0)
    return MOE_ERR_UNSUPPORTED;
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_router_project_topk(const void* input, const void* gate_proj,
                                     int64_t num_tokens, int32_t hidden_dim, int32_t num_experts,
                                     int32_t topk, int32_t renormalize, uint32_t dtype,
                                     float* topk_weights, int32_t* topk_indices,
                                     int32_t* token_expert_indices, float* logits, void* stream) {
  if (num_tokens < 0 || hidden_dim <= 0 || num_experts <= 0 || topk <= 0 || dtype > 2)
    return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0) return MOE_OK;
  if (!input || !gate_proj || !topk_weights || !topk_indices || !token_expert_indices)
    return MOE_ERR_INVALID_ARG;
  if (dtype == kF32 || (num_experts & (num_experts - 1)) != 0 || num_experts > 256 ||
      topk > num_experts || topk > router_project_max_k() || hidden_dim % 64 != 0 ||
      num_tokens > INT32_MAX / num_experts || !aligned16(input) || !aligned16(gate_proj))
    return MOE_ERR_UNSUPPORTED;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (ds->cc_major != 10 || !g_encode) return MOE_ERR_UNSUPPORTED;
  // x [T, H] in 64 x 128-row boxes; W_r [E, H] in 64 x max(E, 16)-row boxes (rows past E are
  // outside the tensor: the TMA fills them with zeros)
  CUtensorMap mx, mw;
  const int n_box = num_experts < 16 ? 16 : num_experts;
  if (!make_map_2d(&mx, static_cast<int>(dtype), input, hidden_dim,
                   static_cast<uint64_t>(num_tokens), 64, 128) ||
      !make_map_2d(&mw, static_cast<int>(dtype), gate_proj, hidden_dim, num_experts, 64, n_box))
    return MOE_ERR_CUDA;
  RouterProjParams p;
  p.out_w = topk_weights;
  p.out_idx = topk_indices;
  p.out_src = token_expert_indices;
  p.logits = logits;
  p.err = ds->err_word;
  p.num_tokens = static_cast<int>(num_tokens);
  p.H = hidden_dim;
  p.k = topk;
  p.renorm = renormalize;
  const int64_t tiles = (num_tokens + 127) / 128;
  const int sms = ds->num_sms;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  if (launch_router_project(static_cast<int>(dtype), num_experts, mx, mw, p, grid,
                            static_cast<cudaStream_t>(stream)) != 0)
    return MOE_ERR_UNSUPPORTED;
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API void topk_softmax(void* gating_output, void* topk_weights, void* topk_indices,
                           void* token_expert_indices, int32_t num_experts, int32_t num_tokens,
                           int32_t topk, void* stream) {
  t_last_status = moe_topk_softmax_v2(
      static_cast<const float*>(gating_output), static_cast<float*>(topk_weights),
      static_cast<int32_t*>(topk_indices), static_cast<int32_t*>(token_expert_indices),
      num_experts, num_tokens, topk, 0, stream);
}

CMOE_API int moe_route_prep(const uint32_t* expert_indices, const float* routing_weights,
                            int64_t num_tokens, int32_t topk, int32_t num_experts,
                            int32_t* expert_offsets, int32_t* sorted_token_ids,
                            float* sorted_weights, void* stream) {
  if (num_tokens < 0 || topk <= 0 || num_experts <= 0) return MOE_ERR_INVALID_ARG;
  // an empty request reads nothing: only the offsets (all zero) are written
  if ((num_tokens > 0 && (!expert_indices || !routing_weights)) || !expert_offsets)
    return MOE_ERR_INVALID_ARG;
  if (num_experts > route_prep_max_experts() || num_tokens * topk > INT32_MAX)
    return MOE_ERR_UNSUPPORTED;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t scratch_bytes = route_prep_scratch_bytes(num_tokens * topk, num_experts);
  void* scratch = nullptr;
  if (scratch_bytes) {
    if (cudaMallocFromPoolAsync(&scratch, scratch_bytes, ds->pool, s) != cudaSuccess) {
      cudaGetLastError();
      return MOE_ERR_NO_MEMORY;
    }
  }
  st = launch_route_prep(expert_indices, routing_weights, num_tokens, topk, num_experts, 1,
                         expert_offsets, nullptr, sorted_token_ids, sorted_weights, nullptr,
                         scratch, s) == 0
           ? MOE_OK
           : MOE_ERR_UNSUPPORTED;
  if (st == MOE_OK) g_launches += scratch_bytes ? 3 : 1;
  if (scratch) cudaFreeAsync(scratch, s);
  return finish(st);
}

CMOE_API int moe_route_prep_ex(const uint32_t* expert_indices, const float* routing_weights,
                               int64_t num_tokens, int32_t topk, int32_t num_experts,
                               int32_t* expert_offsets, int32_t* sorted_token_ids,
                               float* sorted_weights, int32_t* sorted_flat, void* stream) {
  if (num_tokens < 0 || topk <= 0 || num_experts <= 0) return MOE_ERR_INVALID_ARG;
  // an empty request reads nothing: only the offsets (all zero) are written
  if ((num_tokens > 0 && (!expert_indices || !routing_weights)) || !expert_offsets)
    return MOE_ERR_INVALID_ARG;
  if (num_experts > route_prep_max_experts() || num_tokens * topk > INT32_MAX)
    return MOE_ERR_UNSUPPORTED;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t scratch_bytes = route_prep_scratch_bytes(num_tokens * topk, num_experts);
  void* scratch = nullptr;
  if (scratch_bytes) {
    if (cudaMallocFromPoolAsync(&scratch, scratch_bytes, ds->pool, s) != cudaSuccess) {
      cudaGetLastError();
      return MOE_ERR_NO_MEMORY;
    }
  }
  st = launch_route_prep(expert_indices, routing_weights, num_tokens, topk, num_experts, 1,
                         expert_offsets, nullptr, sorted_token_ids, sorted_weights, sorted_flat,
                         scratch, s) == 0
           ? MOE_OK
           : MOE_ERR_UNSUPPORTED;
  if (st == MOE_OK) g_launches += scratch_bytes ? 3 : 1;
  if (scratch) cudaFreeAsync(scratch, s);
  return finish(st);
}

CMOE_API int moe_gather_rows(const void* src, const int32_t* index, int64_t rows,
                             int32_t hidden_dim, uint32_t dtype, void* dst, void* stream) {
  if (rows < 0 || hidden_dim <= 0 || dtype > 2) return MOE_ERR_INVALID_ARG;
  if (rows == 0) return MOE_OK;
  if (!src || !index || !dst) return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  launch_gather_rows(static_cast<int>(dtype), src, index, rows, hidden_dim, dst, ds->num_sms,
                     static_cast<cudaStream_t>(stream));
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_combine_rows(const void* rows_buf, const int32_t* sorted_flat, int64_t rows,
                              int64_t num_tokens, int32_t topk, int32_t hidden_dim,
                              uint32_t dtype, void* output, void* stream) {
  if (rows < 0 || num_tokens < 0 || topk <= 0 || hidden_dim <= 0 || dtype > 2)
    return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0) return MOE_OK;
  if (!output || (rows > 0 && (!rows_buf || !sorted_flat))) return MOE_ERR_INVALID_ARG;
  if (rows > num_tokens * topk) return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* inv = nullptr;
  if (cudaMallocFromPoolAsync(&inv, sizeof(int32_t) * static_cast<size_t>(num_tokens) * topk,
                              ds->pool, s) != cudaSuccess) {
    cudaGetLastError();
    return MOE_ERR_NO_MEMORY;
  }
  st = launch_combine_indirect(static_cast<int>(dtype), rows_buf, sorted_flat, rows, num_tokens,
                               topk, hidden_dim, static_cast<int32_t*>(inv), output, ds->num_sms,
                               s) == 0
           ? MOE_OK
           : MOE_ERR_CUDA;
  if (st == MOE_OK) g_launches += rows > 0 ? 2 : 1;
  cudaFreeAsync(inv, s);
  return finish(st);
}

CMOE_API int moe_ep_dest_groups(const uint32_t* expert_indices, int64_t num_tokens, int32_t topk,
                                int32_t num_experts, int32_t num_ranks,
                                int64_t tokens_per_chunk, int32_t* groups, int32_t num_chunks,
                                int64_t* assignment_counts, void* stream) {
  if (num_tokens < 0 || topk <= 0 || num_experts <= 0 || num_ranks <= 0 || tokens_per_chunk <= 0)
    return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0 && !assignment_counts) return MOE_OK;
  if ((num_tokens > 0 && (!expert_indices || !groups)) || (assignment_counts && num_chunks <= 0))
    return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (launch_ep_dest_groups(expert_indices, num_tokens, topk, num_experts, num_ranks,
                            tokens_per_chunk, groups, assignment_counts, num_chunks, ds->num_sms,
                            static_cast<cudaStream_t>(stream)))
    return MOE_ERR_UNSUPPORTED;
  if (num_tokens > 0) ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_ep_pack(const void* input, const int32_t* pair_token, const int32_t* pair_flat,
                         int64_t num_pairs, const int32_t* num_pairs_device,
                         const uint32_t* expert_indices, const float* routing_weights,
                         int32_t topk, int32_t num_experts, int32_t num_ranks,
                         int32_t hidden_dim, uint32_t dtype, void* rows, int32_t* meta,
                         int32_t* slot_count, void* stream) {
  if (num_pairs < 0 || topk <= 0 || num_experts <= 0 || num_ranks <= 0 || hidden_dim <= 0 ||
      dtype > 2)
    return MOE_ERR_INVALID_ARG;
  if (num_pairs == 0) return MOE_OK;
  if (!input || !pair_token || !pair_flat || !expert_indices || !routing_weights || !rows ||
      !meta || !slot_count)
    return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (launch_ep_pack(static_cast<int>(dtype), input, pair_token, pair_flat, num_pairs,
                     num_pairs_device, expert_indices, routing_weights, topk, num_experts,
                     num_ranks, hidden_dim,
                     rows, meta, slot_count, ds->num_sms, static_cast<cudaStream_t>(stream)))
    return MOE_ERR_UNSUPPORTED;
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_ep_entry_flat(const int32_t* pair_token, const int32_t* pair_flat,
                               const int64_t* pair_start, int64_t num_pairs,
                               const uint32_t* expert_indices, int32_t topk, int32_t num_experts,
                               int32_t num_ranks, int32_t* flat, void* stream) {
  if (num_pairs < 0 || topk <= 0 || num_experts <= 0 || num_ranks <= 0)
    return MOE_ERR_INVALID_ARG;
  if (num_pairs == 0) return MOE_OK;
  if (!pair_token || !pair_flat || !pair_start || !expert_indices || !flat)
    return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (launch_ep_entry_flat(pair_token, pair_flat, pair_start, num_pairs, expert_indices, topk,
                           num_experts, num_ranks, flat, ds->num_sms,
                           static_cast<cudaStream_t>(stream)))
    return MOE_ERR_UNSUPPORTED;
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_segment_sum_rows(const void* rows_in, const int64_t* segment_start,
                                 int64_t num_segments, int32_t hidden_dim, uint32_t dtype,
                                 void* output, void* stream) {
  if (num_segments < 0 || hidden_dim <= 0 || dtype > 2) return MOE_ERR_INVALID_ARG;
  if (num_segments == 0) return MOE_OK;
  if (!rows_in || !segment_start || !output) return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  launch_segment_sum_rows(static_cast<int>(dtype), rows_in, segment_start, num_segments,
                          hidden_dim, output, ds->num_sms, static_cast<cudaStream_t>(stream));
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API size_t moe_fused_workspace_size(int64_t num_tokens, int32_t hidden_dim,
                                         int32_t intermediate_dim, int32_t num_experts,
                                         int32_t topk, uint32_t moe_type, uint32_t dtype) {
  (void)moe_type;
  if (num_tokens <= 0 || hidden_dim <= 0 || intermediate_dim <= 0 || num_experts <= 0 ||
      topk <= 0 || dtype > 2)
    return 0;
  // the decode layout when the shape allows it (pointer alignment is only known at the call;
  // a call that takes the grouped GEMMs needs less)
  const int dec_n = decode_rows(num_tokens, hidden_dim, intermediate_dim, num_experts,
                                static_cast<int>(dtype), g_gemm_path.load());
  return fused_layout(num_tokens, hidden_dim, intermediate_dim, num_experts, topk,
                      static_cast<int>(dtype), dec_n)
      .total;
}

CMOE_API int moe_fused_v2(const void* input, const void* gate_weights, const void* up_weights,
                          const void* down_weights, const float* routing_weights,
                          const uint32_t* expert_indices, void* output, int64_t num_tokens,
                          int32_t hidden_dim, int32_t intermediate_dim, int32_t num_experts,
                          int32_t topk, int32_t activation_type, uint32_t moe_type,
                          uint32_t dtype, void* workspace, size_t workspace_bytes,
                          void* stream) {
  return fused_impl(input, gate_weights, up_weights, down_weights, routing_weights,
                    expert_indices, output, num_tokens, hidden_dim, intermediate_dim,
                    num_experts, topk, activation_type, moe_type, dtype, workspace,
                    workspace_bytes, static_cast<cudaStream_t>(stream));
}

CMOE_API int moe_fused_scatter(const void* input, const void* gate_weights,
                               const void* up_weights, const void* down_weights,
                               const float* routing_weights, const uint32_t* expert_indices,
                               const int32_t* out_row, void* output, int64_t num_tokens,
                               int32_t hidden_dim, int32_t intermediate_dim, int32_t num_experts,
                               int32_t topk, int32_t activation_type, uint32_t moe_type,
                               uint32_t dtype, void* stream) {
  if (!out_row) return MOE_ERR_INVALID_ARG;
  return fused_impl(input, gate_weights, up_weights, down_weights, routing_weights,
                    expert_indices, output, num_tokens, hidden_dim, intermediate_dim,
                    num_experts, topk, activation_type, moe_type, dtype, nullptr, 0,
                    static_cast<cudaStream_t>(stream), out_row);
}

CMOE_API void fused_moe(void* input, void* gate_weights, void* up_weights, void* down_weights,
                        void* routing_weights, void* expert_indices, void* output,
                        int num_tokens, int hidden_dim, int intermediate_dim, int num_experts,
                        int num_selected_experts, int activation_type, uint32_t moe_type,
                        uint32_t dtype, void* stream) {
  t_last_status = fused_impl(input, gate_weights, up_weights, down_weights,
                             static_cast<const float*>(routing_weights),
                             static_cast<const uint32_t*>(expert_indices), output, num_tokens,
                             hidden_dim, intermediate_dim, num_experts, num_selected_experts,
                             activation_type, moe_type, dtype, nullptr, 0,
                             static_cast<cudaStream_t>(stream));
}

CMOE_API uint32_t moe_device_error_bits(int32_t device, int32_t clear) {
  DeviceState* ds = nullptr;
  if (init_device(device, &ds) != MOE_OK) return 0xffffffffu;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  uint32_t v = 0;
  cudaDeviceSynchronize();
  cudaMemcpy(&v, ds->err_word, sizeof(v), cudaMemcpyDeviceToHost);
  if (clear) cudaMemset(ds->err_word, 0, sizeof(uint32_t));
  cudaSetDevice(prev);
  return v;
}

CMOE_API int32_t moe_set_gemm_path(int32_t path) {
  if (path < 0 || path > 6) return -1;
  return g_gemm_path.exchange(path);
}

CMOE_API int32_t moe_last_gemm_path(void) { return t_last_path; }

CMOE_API int32_t moe_set_sm_reserve(int32_t sms) {
  if (sms < 0 || sms > 128) return -1;
  return g_sm_reserve.exchange(sms);
}

CMOE_API int64_t moe_kernel_launches(void) { return g_launches.load(); }

CMOE_API int moe_phase_timing(int32_t enable) {
  std::lock_guard<std::mutex> lk(g_timer.mu);
  if (enable) g_timer.calls = 0;
  g_timer.on = enable != 0;
  return MOE_OK;
}

CMOE_API int moe_phase_times(double* ms, int64_t* calls) {
  std::lock_guard<std::mutex> lk(g_timer.mu);
  for (int i = 0; i < kPhases; ++i) ms[i] = 0.0;
  for (int64_t c = 0; c < g_timer.calls; ++c) {
    cudaEvent_t* e = g_timer.events.data() + c * (kPhases + 1);
    if (cudaEventSynchronize(e[kPhases]) != cudaSuccess) return MOE_ERR_CUDA;
    for (int i = 0; i < kPhases; ++i) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, e[i], e[i + 1]) != cudaSuccess) return MOE_ERR_CUDA;
      ms[i] += t;
    }
  }
  if (calls) *calls = g_timer.calls;
  return MOE_OK;
}

// ---- peer-mapped buffers and arrival flags (expert-parallel exchange) ------------------------

static_assert(sizeof(cudaIpcMemHandle_t) == MOE_PEER_HANDLE_BYTES, "IPC handle size");

CMOE_API int moe_peer_alloc(size_t bytes, void** ptr, uint8_t* handle) {
  if (!ptr || !handle || bytes == 0) return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return MOE_ERR_NO_MEMORY;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return MOE_ERR_CUDA;
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return MOE_OK;
}

CMOE_API int moe_peer_free(void* ptr) {
  if (!ptr) return MOE_ERR_INVALID_ARG;
  return finish(cudaFree(ptr) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA);
}

CMOE_API int moe_peer_open(const uint8_t* handle, void** ptr) {
  if (!handle || !ptr) return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return MOE_ERR_CUDA;
  }
  *ptr = p;
  return MOE_OK;
}

CMOE_API int moe_peer_close(void* ptr) {
  if (!ptr) return MOE_ERR_INVALID_ARG;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
    cudaGetLastError();
    return MOE_ERR_CUDA;
  }
  return MOE_OK;
}

CMOE_API int moe_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MOE_OK;
  if (!dst || !src) return MOE_ERR_INVALID_ARG;
  if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    cudaGetLastError();
    return MOE_ERR_CUDA;
  }
  return MOE_OK;
}

CMOE_API int moe_peer_signal(uint32_t* const* flag_addrs, int32_t count, uint32_t value,
                             void* stream) {
  if (count < 0 || count > kMaxPeerFlags || (count > 0 && !flag_addrs))
    return MOE_ERR_INVALID_ARG;
  if (count == 0) return MOE_OK;
  PeerFlagPtrs t{};
  for (int i = 0; i < count; ++i) {
    if (!flag_addrs[i] || (reinterpret_cast<uintptr_t>(flag_addrs[i]) & 3u))
      return MOE_ERR_INVALID_ARG;
    t.p[i] = flag_addrs[i];
  }
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  launch_peer_signal(t, count, value, static_cast<cudaStream_t>(stream));
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_peer_wait(const uint32_t* flags, int32_t count, uint32_t value,
                           int64_t timeout_ns, void* stream) {
  if (count < 0 || count > kMaxPeerFlags || timeout_ns <= 0 || (count > 0 && !flags) ||
      (reinterpret_cast<uintptr_t>(flags) & 3u))
    return MOE_ERR_INVALID_ARG;
  if (count == 0) return MOE_OK;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  launch_peer_wait(flags, count, value, static_cast<unsigned long long>(timeout_ns), ds->err_word,
                   static_cast<cudaStream_t>(stream));
  ++g_launches;
  return finish(MOE_OK);
}


CMOE_API int moe_ep_push_pairs(const void* input, const int32_t* pair_token,
                               const int32_t* pair_flat, const int32_t* pair_offsets,
                               int32_t chunk, const uint32_t* expert_indices,
                               const float* routing_weights, int32_t topk, int32_t num_experts,
                               int32_t num_ranks, int32_t hidden_dim, uint32_t dtype,
                               void* const* dst_rows, void* const* dst_meta, int32_t* slot_count,
                               int32_t blocks, void* stream) {
  if (topk <= 0 || num_experts <= 0 || num_ranks <= 0 || num_ranks > kMaxEpRanks ||
      hidden_dim <= 0 || dtype > 2 || chunk < 0 || blocks < 0)
    return MOE_ERR_INVALID_ARG;
  if (!input || !pair_token || !pair_flat || !pair_offsets || !expert_indices ||
      !routing_weights || !dst_rows || !dst_meta)
    return MOE_ERR_INVALID_ARG;
  EpPeerRows tab{};
  for (int d = 0; d < num_ranks; ++d) {
    if (!dst_rows[d] || !dst_meta[d]) return MOE_ERR_INVALID_ARG;
    tab.rows[d] = static_cast<char*>(dst_rows[d]);
    tab.meta[d] = static_cast<char*>(dst_meta[d]);
  }
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (launch_ep_push_pairs(static_cast<int>(dtype), input, pair_token, pair_flat, pair_offsets,
                           chunk, expert_indices, routing_weights, topk, num_experts, num_ranks,
                           hidden_dim, tab, slot_count, blocks ? blocks : ds->num_sms,
                           static_cast<cudaStream_t>(stream)))
    return MOE_ERR_UNSUPPORTED;
  ++g_launches;
  return finish(MOE_OK);
}

CMOE_API int moe_segment_sum_push(const void* rows_in, const int64_t* segment_start,
                                  int64_t num_segments, int32_t hidden_dim, uint32_t dtype,
                                  int32_t num_ranks, void* const* dst, const int64_t* first_row,
                                  int32_t blocks, void* stream) {
  if (num_segments < 0 || hidden_dim <= 0 || dtype > 2 || num_ranks <= 0 ||
      num_ranks > kMaxEpRanks || blocks < 0)
    return MOE_ERR_INVALID_ARG;
  if (num_segments == 0) return MOE_OK;
  if (!rows_in || !segment_start || !dst || !first_row) return MOE_ERR_INVALID_ARG;
  EpPeerReturn tab{};
  for (int s = 0; s <= num_ranks; ++s) {
    if (s < num_ranks) {
      if (!dst[s]) return MOE_ERR_INVALID_ARG;
      tab.dst[s] = static_cast<char*>(dst[s]);
    }
    if (first_row[s] < 0 || (s > 0 && first_row[s] < first_row[s - 1]))
      return MOE_ERR_INVALID_ARG;
    tab.first[s] = first_row[s];
  }
  if (tab.first[0] != 0 || tab.first[num_ranks] != num_segments) return MOE_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int st = current_device_state(&ds);
  if (st != MOE_OK) return st;
  if (launch_segment_sum_push(static_cast<int>(dtype), rows_in, segment_start, num_segments,
                              hidden_dim, num_ranks, tab, blocks ? blocks : ds->num_sms,
                              static_cast<cudaStream_t>(stream)))
    return MOE_ERR_UNSUPPORTED;
  ++g_launches;
  return finish(MOE_OK);
}
