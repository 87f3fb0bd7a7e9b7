// moe_api.cu — the C ABI (include/moe_fp8_ds.h): argument checks, cached
// device workspace, TMA tensor maps and the launch sequence
//   route+plan+permute -> GEMM1(+SwiGLU+requant) -> GEMM2(+weight) -> finalize
// on the caller's stream, with no host synchronisation.
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "moe_fp8_ds.h"
#include "moe_kernels.h"

using namespace moe;

namespace {

std::mutex g_mu;
// Cached workspaces, one per (device, layout): the full expert pipeline per
// number of local experts, plus a small routing-only layout (key suffix 0).
std::unordered_map<int64_t, Workspace> g_ws;
inline int64_t ws_key(int dev, int e_local, bool routing_only) { return (int64_t)dev * 1024 + (routing_only ? 0 : e_local); }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2D byte matrix [rows][cols] (row stride = cols bytes), 128x128 box,
// 128-byte swizzle (matches the UMMA K-major SWIZZLE_128B operand layout).
// Encoded maps are cached by (base, cols, rows): a map holds no state beyond
// those, and callers typically reuse their weight and workspace buffers.
struct MapKey {
  const void* base;
  uint64_t cols, rows;
  uint32_t box_rows;
};
constexpr int kMapCache = 32;
MapKey g_map_key[kMapCache];
CUtensorMap g_map_val[kMapCache];
int g_map_next = 0;

bool encode_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows);

bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows = 128) {
  for (int i = 0; i < kMapCache; ++i) {
    if (g_map_key[i].base == base && g_map_key[i].cols == cols && g_map_key[i].rows == rows &&
        g_map_key[i].box_rows == box_rows && base) {
      *m = g_map_val[i];
      return true;
    }
  }
  if (!encode_map(m, base, cols, rows, box_rows)) return false;
  g_map_key[g_map_next] = MapKey{base, cols, rows, box_rows};
  g_map_val[g_map_next] = *m;
  g_map_next = (g_map_next + 1) % kMapCache;
  return true;
}

bool encode_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Rows of the expert-major padded layout: every routed assignment, padding
// of up to 127 rows per expert, and with a shared expert its T rows (+ padding).
int64_t rows_cap_for(int64_t T, int e_local, bool shared = false) {
  const int64_t per_tok = e_local < kTopK ? e_local : kTopK;
  return ((T * per_tok + kTileM - 1) / kTileM) * kTileM + (int64_t)e_local * kTileM +
         (shared ? ((T + kTileM - 1) / kTileM) * kTileM : 0);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Computes the layout; when `base` is non-null also assigns the pointers.
// `zero_bytes` receives the length of the prefix that must start zeroed
// (self-resetting counters, the combine accumulator, split-K scratch).
size_t layout(Workspace& w, int64_t T, int e_local, uint8_t* base, size_t* zero_bytes, bool routing_only = false,
              bool shared = false) {
  const int64_t rows = routing_only ? 0 : rows_cap_for(T, e_local, shared);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += align256(bytes);
    return base ? base + o : nullptr;
  };
  const size_t Tz = static_cast<size_t>(T > 0 ? T : 1);
  w.expert_fill = reinterpret_cast<int32_t*>(take((size_t)kExperts * 4));
  w.done_ctas = reinterpret_cast<uint32_t*>(take(4));
  w.bar_cnt = reinterpret_cast<uint32_t*>(take(4));
  w.leave_cnt = reinterpret_cast<uint32_t*>(take(4));
  w.status = reinterpret_cast<unsigned*>(take(4));
  if (routing_only) {
    if (zero_bytes) *zero_bytes = off;
    w.plan = reinterpret_cast<Plan*>(take(sizeof(Plan)));
    w.topk_ids = reinterpret_cast<int32_t*>(take(Tz * kTopK * 4));
    w.topk_w = reinterpret_cast<float*>(take(Tz * kTopK * 4));
    w.topk_rank = reinterpret_cast<int32_t*>(take(Tz * kTopK * 4));
    w.rows_cap = 0;
    w.t_cap = T;
    w.e_local = e_local;
    return off;
  }
  w.tile_sem = reinterpret_cast<int32_t*>(take((size_t)kMaxSplitMTiles * kNT1 * 4 * 4));
  w.tile_sem2 = reinterpret_cast<int32_t*>(take((size_t)kMaxSplitMTiles * kNT2 * kEpiWarps * 4));
  w.g_part = reinterpret_cast<float*>(take((size_t)kMaxSplitMTiles * kTileM * kGemm1N * 4));
  w.g2_part = reinterpret_cast<float*>(take((size_t)kMaxSplitMTiles * kTileM * kHidden * 4));
  // fused decode kernel scratch (independent of T)
  const int grid = device_sm_count();
  w.dec.grid = grid;
  w.dec.slots_cap = e_local;
  w.dec.g1_cnt = reinterpret_cast<int*>(take((size_t)grid * 4));
  w.dec.ready = reinterpret_cast<int*>(take((size_t)e_local * 4));
  w.dec.h_cnt = reinterpret_cast<int*>(take((size_t)kNT2 * 4));
  w.dec.done = reinterpret_cast<int*>(take(4));
  w.dec.zero = reinterpret_cast<const float*>(take(4));
  if (zero_bytes) *zero_bytes = off;
  w.dec.g1_part = reinterpret_cast<float*>(take((size_t)grid * 2 * kDecMaxT * 2 * kBlk * 4));
  w.dec.g2_part = reinterpret_cast<float*>(take((size_t)grid * 2 * kDecMaxT * 2 * kBlk * 4));
  w.dec.inter = take((size_t)e_local * kDecMaxT * kInterCols);
  w.dec.inter_scale = reinterpret_cast<float*>(take((size_t)e_local * kInterBlocks * kDecMaxT * 4));
  w.dec.status = w.status;
  w.token_rows = reinterpret_cast<int32_t*>(take(Tz * kTopK * 4));
  w.out_rows = reinterpret_cast<__nv_bfloat16*>(take((size_t)rows * kHidden * 2));
  w.plan = reinterpret_cast<Plan*>(take(sizeof(Plan)));
  w.topk_ids = reinterpret_cast<int32_t*>(take(Tz * kTopK * 4));
  w.topk_w = reinterpret_cast<float*>(take(Tz * kTopK * 4));
  w.topk_rank = reinterpret_cast<int32_t*>(take(Tz * kTopK * 4));
  w.a1 = take((size_t)rows * kHidden);
  w.a1_scale = reinterpret_cast<float*>(take((size_t)rows * kHiddenBlocks * 4));
  w.row_token = reinterpret_cast<int32_t*>(take((size_t)rows * 4));
  w.row_weight = reinterpret_cast<float*>(take((size_t)rows * 4));
  w.inter = take((size_t)rows * kInterCols);
  w.inter_scale = reinterpret_cast<float*>(take((size_t)rows * kInterBlocks * 4));
  w.rows_cap = rows;
  w.t_cap = T;
  w.e_local = e_local;
  w.shared_cap = shared;
  return off;
}

void forget_maps(const void* base, size_t bytes) {
  const uint8_t* b = static_cast<const uint8_t*>(base);
  for (int i = 0; i < kMapCache; ++i) {
    const uint8_t* k = static_cast<const uint8_t*>(g_map_key[i].base);
    if (k >= b && k < b + bytes) g_map_key[i] = MapKey{nullptr, 0, 0, 0};
  }
}

int get_workspace(int64_t T, int e_local, bool routing_only, Workspace** out, bool shared = false) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  Workspace& w = g_ws[ws_key(dev, e_local, routing_only)];
  if (w.base && w.t_cap >= T && (w.shared_cap || !shared)) {
    *out = &w;
    return MOE_OK;
  }
  // grow: keep the larger token capacity and any shared-expert capacity
  const int64_t t_new = (w.base && w.t_cap > T) ? w.t_cap : T;
  shared = shared || (w.base && w.shared_cap);
  if (w.base) {
    cudaDeviceSynchronize();
    forget_maps(w.base, w.bytes);
    cudaFree(w.base);
    w = Workspace{};
  }
  Workspace nw;
  size_t zero_bytes = 0;
  const size_t bytes = layout(nw, t_new, e_local, nullptr, &zero_bytes, routing_only, shared);
  void* base = nullptr;
  if (cudaMalloc(&base, bytes) != cudaSuccess) {
    cudaGetLastError();
    return MOE_ERR_WORKSPACE;
  }
  if (cudaMemset(base, 0, zero_bytes) != cudaSuccess) {
    cudaFree(base);
    return MOE_ERR_CUDA;
  }
  layout(nw, t_new, e_local, static_cast<uint8_t*>(base), nullptr, routing_only, shared);
  nw.base = base;
  nw.bytes = bytes;
  nw.zero_bytes = zero_bytes;
  w = nw;
  *out = &w;
  return MOE_OK;
}

int check_device() {
  static int major_cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOE_ERR_NO_DEVICE;
  if (!major_cache[dev]) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return MOE_ERR_NO_DEVICE;
    major_cache[dev] = major;
  }
  return major_cache[dev] == 10 ? MOE_OK : MOE_ERR_NO_DEVICE;
}

// Optional per-kernel CUDA events (moe_fp8_ds_profile_enable): routing with
// the permutation, GEMM1, GEMM2, finalize.
constexpr int kProfKernels = 4;
bool g_prof_on = false;
bool g_prof_valid = false;
int g_prof_n = kProfKernels;  // intervals recorded by the last call (1 for the fused decode kernel)
cudaEvent_t g_prof_ev[kProfKernels + 1] = {};

inline void prof_mark(int i, cudaStream_t s) {
  if (g_prof_on) cudaEventRecord(g_prof_ev[i], s);
}

// Calls with 1..kDecMaxT tokens can be served by the fused decode kernel.
// It is off by default (the four-kernel pipeline measured faster on the
// decode sweep); MOE_FP8_DS_FUSED_DECODE=1 in the environment or
// moe_fp8_ds_set_fused_decode(1) turns it on.
int g_fused_decode = -1;
bool fused_decode_enabled() {
  if (g_fused_decode < 0) {
    const char* v = getenv("MOE_FP8_DS_FUSED_DECODE");
    g_fused_decode = (v && v[0] == '1') ? 1 : 0;
  }
  return g_fused_decode == 1;
}

// Failure-path test hook (moe_fp8_ds_test_route_barrier), off by default.
uint64_t g_test_wait_limit_ns = 0;
int g_test_skip_arrival = -1;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_e_local(int64_t e) { return e == 32 || e == 64 || e == 128 || e == 256; }

// The common expert pipeline: plan (from logits or from given ids), permute,
// both GEMMs and the finalize cast. sw1/ss1/sw2/ss2: an optional shared
// expert (all four or none), scheduled as local expert E_l with every token.
int run_pipeline(const float* logits, const void* bias, const int32_t* given_ids, const float* given_w,
                 const void* hidden, const float* hidden_scale, const void* w1, const float* s1, const void* w2,
                 const float* s2, int64_t offset, double scale, void* out, int out_fp32, int64_t T, int64_t E_l,
                 int32_t* user_ids, float* user_w, int32_t* user_counts, void* stream, bool route_only,
                 const void* sw1 = nullptr, const float* ss1 = nullptr, const void* sw2 = nullptr,
                 const float* ss2 = nullptr) {
  if (T < 0 || T > (int64_t(1) << 24) || !valid_e_local(E_l)) return MOE_ERR_INVALID_ARG;
  const bool shared = sw1 != nullptr;
  if (shared) {
    if (!ss1 || !sw2 || !ss2 || E_l > 128) return MOE_ERR_INVALID_ARG;
    if (!aligned16(sw1) || !aligned16(sw2)) return MOE_ERR_ALIGNMENT;
  } else if (ss1 || sw2 || ss2) {
    return MOE_ERR_INVALID_ARG;
  }
  if (offset < -(int64_t(1) << 30) || offset > (int64_t(1) << 30)) return MOE_ERR_INVALID_ARG;
  if (T == 0) return check_device();  // empty tensors may carry null data pointers
  if (logits) {
    if (!bias) return MOE_ERR_INVALID_ARG;
    if (!aligned16(logits) || !aligned16(bias)) return MOE_ERR_ALIGNMENT;
  } else if (!given_ids || !given_w) {
    return MOE_ERR_INVALID_ARG;
  }
  if (!route_only) {
    if (!hidden || !hidden_scale || !w1 || !s1 || !w2 || !s2 || !out) return MOE_ERR_INVALID_ARG;
    if (!aligned16(hidden) || !aligned16(w1) || !aligned16(w2) || !aligned16(out)) return MOE_ERR_ALIGNMENT;
  }
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  std::lock_guard<std::mutex> lk(g_mu);
  Workspace* ws = nullptr;
  rc = get_workspace(T, static_cast<int>(E_l), route_only, &ws, shared);
  if (rc) return rc;

  if (logits && !route_only && !out_fp32 && !shared && T <= kDecMaxT && fused_decode_enabled()) {
    // one persistent kernel for routing, both GEMMs and the combine
    CUtensorMap mw1, mw2, mx1, mx2;
    if (!make_map(&mw1, w1, kHidden, static_cast<uint64_t>(E_l) * kGemm1N) ||
        !make_map(&mw2, w2, kInter, static_cast<uint64_t>(E_l) * kHidden) ||
        !make_map(&mx1, hidden, kHidden, static_cast<uint64_t>(T), kDecMaxT) ||
        !make_map(&mx2, ws->dec.inter, kInterCols, static_cast<uint64_t>(ws->dec.slots_cap) * kDecMaxT, kDecMaxT))
      return MOE_ERR_CUDA;
    DecodeCall dc{};
    dc.logits = logits;
    dc.bias = static_cast<const uint16_t*>(bias);
    dc.hidden_scale = hidden_scale;
    dc.w13_scale = s1;
    dc.w2_scale = s2;
    dc.T = static_cast<int>(T);
    dc.offset = static_cast<int>(offset);
    dc.e_local = static_cast<int>(E_l);
    dc.scale = static_cast<float>(scale);
    dc.out = out;
    dc.user_ids = user_ids;
    dc.user_w = user_w;
    dc.user_counts = user_counts;
    prof_mark(0, s);
    if (launch_decode(ws->dec, mw1, mw2, mx1, mx2, dc, s) != cudaSuccess) return MOE_ERR_CUDA;
    prof_mark(1, s);
    g_prof_n = 1;
    g_prof_valid = g_prof_on;
    return MOE_OK;
  }

  RouteArgs ra{};
  ra.logits = logits;
  ra.bias = static_cast<const uint16_t*>(bias);
  ra.given_ids = given_ids;
  ra.given_w = given_w;
  ra.T = static_cast<int>(T);
  ra.offset = static_cast<int>(offset);
  ra.e_local = static_cast<int>(E_l);
  ra.scale = static_cast<float>(scale);
  ra.user_ids = user_ids;
  ra.user_w = user_w;
  ra.user_counts = user_counts;
  if (route_only) {
    ra.tokens_per_cta = tokens_per_cta_for(static_cast<int>(T));
    return launch_route(*ws, ra, s) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
  }
  if (route_permute_grid(static_cast<int>(T), &ra.tokens_per_cta) < 1) return MOE_ERR_CUDA;
  ra.wait_limit_ns = g_test_wait_limit_ns;
  ra.skip_arrival_cta = g_test_skip_arrival;

  // calls with at most 64 rows use the skinny GEMM configuration (64-row
  // token tiles, one more stage of weights in flight)
  const bool skinny = T <= kSkinnyMaxRows;
  const uint32_t a_box = skinny ? kSkinnyMaxRows : kTileM;
  // small calls: GEMM1 gathers its few rows straight from hidden_states
  // (one-row boxes), so the routing kernel copies no rows
  CUtensorMap ma1, mw1, ma2, mw2;
  if (!(skinny ? make_map(&ma1, hidden, kHidden, static_cast<uint64_t>(T), 1)
               : make_map(&ma1, ws->a1, kHidden, ws->rows_cap, a_box)) ||
      !make_map(&mw1, w1, kHidden, static_cast<uint64_t>(E_l) * kGemm1N) ||
      !make_map(&ma2, ws->inter, kInterCols, ws->rows_cap, a_box) ||
      !make_map(&mw2, w2, kInter, static_cast<uint64_t>(E_l) * kHidden))
    return MOE_ERR_CUDA;
  // the shared expert's weights (one expert each); unused copies otherwise
  CUtensorMap mws1 = mw1, mws2 = mw2;
  if (shared && (!make_map(&mws1, sw1, kHidden, kGemm1N) || !make_map(&mws2, sw2, kInter, kHidden)))
    return MOE_ERR_CUDA;
  const int shared_e = shared ? static_cast<int>(E_l) : -1;

  PermuteArgs pa{};
  pa.hidden = static_cast<const uint8_t*>(hidden);
  pa.hidden_scale = hidden_scale;
  pa.T = static_cast<int>(T);
  pa.offset = static_cast<int>(offset);
  pa.tokens_per_cta = ra.tokens_per_cta;
  pa.copy_rows = skinny ? 0 : 1;
  pa.shared = shared ? 1 : 0;
  prof_mark(0, s);
  if (launch_route_permute(*ws, ra, pa, s) != cudaSuccess) return MOE_ERR_CUDA;
  prof_mark(1, s);
  if (launch_gemm1(*ws, ma1, mw1, s1, s, skinny, hidden_scale, T, mws1, ss1, shared_e) != cudaSuccess)
    return MOE_ERR_CUDA;
  prof_mark(2, s);
  if (launch_gemm2(*ws, ma2, mw2, s2, s, skinny, mws2, ss2, shared_e, static_cast<int>(T)) != cudaSuccess) return MOE_ERR_CUDA;
  prof_mark(3, s);
  if (launch_finalize(*ws, static_cast<int>(T), out, out_fp32, s, shared_e) != cudaSuccess) return MOE_ERR_CUDA;
  prof_mark(4, s);
  g_prof_n = kProfKernels;
  g_prof_valid = g_prof_on;
  return MOE_OK;
}

}  // namespace

extern "C" {

int moe_fp8_ds_kernel_ex(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                         const float* hidden_states_scale, const void* gemm1_weights,
                         const float* gemm1_weights_scale, const void* gemm2_weights,
                         const float* gemm2_weights_scale, int64_t local_expert_offset,
                         double routed_scaling_factor, void* output, int64_t seq_len, int64_t num_local_experts,
                         int32_t* topk_ids_out, float* topk_weights_out, int32_t* expert_counts_out,
                         void* stream) {
  if (!routing_logits && seq_len != 0) return MOE_ERR_INVALID_ARG;
  return run_pipeline(routing_logits, routing_bias, nullptr, nullptr, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                      routed_scaling_factor, output, 0, seq_len, num_local_experts, topk_ids_out, topk_weights_out,
                      expert_counts_out, stream, false);
}

int moe_fp8_ds_kernel(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                      const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                      const void* gemm2_weights, const float* gemm2_weights_scale, int64_t local_expert_offset,
                      double routed_scaling_factor, void* output, int64_t seq_len, int64_t num_local_experts,
                      void* stream) {
  return moe_fp8_ds_kernel_ex(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                              routed_scaling_factor, output, seq_len, num_local_experts, nullptr, nullptr, nullptr,
                              stream);
}

int moe_fp8_ds_kernel_shared(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                             const float* hidden_states_scale, const void* gemm1_weights,
                             const float* gemm1_weights_scale, const void* gemm2_weights,
                             const float* gemm2_weights_scale, int64_t local_expert_offset,
                             double routed_scaling_factor, const void* shared_gemm1_weights,
                             const float* shared_gemm1_weights_scale, const void* shared_gemm2_weights,
                             const float* shared_gemm2_weights_scale, void* output, int64_t seq_len,
                             int64_t num_local_experts, void* stream) {
  if (seq_len != 0 && (!routing_logits || !shared_gemm1_weights)) return MOE_ERR_INVALID_ARG;
  return run_pipeline(routing_logits, routing_bias, nullptr, nullptr, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                      routed_scaling_factor, output, 0, seq_len, num_local_experts, nullptr, nullptr, nullptr, stream,
                      false, shared_gemm1_weights, shared_gemm1_weights_scale, shared_gemm2_weights,
                      shared_gemm2_weights_scale);
}

int moe_fp8_ds_route(const float* routing_logits, const void* routing_bias, int64_t seq_len,
                     int64_t local_expert_offset, int64_t num_local_experts, double routed_scaling_factor,
                     int32_t* topk_ids_out, float* topk_weights_out, int32_t* expert_counts_out, void* stream) {
  if (seq_len != 0 && (!routing_logits || !topk_ids_out || !topk_weights_out)) return MOE_ERR_INVALID_ARG;
  return run_pipeline(routing_logits, routing_bias, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                      nullptr, local_expert_offset, routed_scaling_factor, nullptr, 0, seq_len, num_local_experts,
                      topk_ids_out, topk_weights_out, expert_counts_out, stream, true);
}

int moe_fp8_ds_experts(const void* hidden_states, const float* hidden_states_scale, const int32_t* topk_ids,
                       const float* topk_weights, const void* gemm1_weights, const float* gemm1_weights_scale,
                       const void* gemm2_weights, const float* gemm2_weights_scale, int64_t local_expert_offset,
                       int64_t num_rows, int64_t num_local_experts, void* output, int output_fp32, void* stream) {
  if (num_rows != 0 && (!topk_ids || !topk_weights)) return MOE_ERR_INVALID_ARG;
  return run_pipeline(nullptr, nullptr, topk_ids, topk_weights, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset, 1.0, output,
                      output_fp32 ? 1 : 0, num_rows, num_local_experts, nullptr, nullptr, nullptr, stream, false);
}

int moe_fp8_ds_quantize_act(const void* hidden_bf16, int64_t seq_len, void* hidden_fp8_out, float* hidden_scale_out,
                            void* stream) {
  if (seq_len < 0 || seq_len > (int64_t(1) << 24)) return MOE_ERR_INVALID_ARG;
  if (seq_len == 0) return check_device();  // empty tensors may carry null data pointers
  if (!hidden_bf16 || !hidden_fp8_out || !hidden_scale_out) return MOE_ERR_INVALID_ARG;
  if (!aligned16(hidden_bf16) || !aligned16(hidden_fp8_out) ||
      (reinterpret_cast<uintptr_t>(hidden_scale_out) & 3u))
    return MOE_ERR_ALIGNMENT;
  int rc = check_device();
  if (rc) return rc;
  if (launch_quant_rows(hidden_bf16, static_cast<int>(seq_len), hidden_fp8_out, hidden_scale_out,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int moe_fp8_ds_add_norm_quant(const void* x_bf16, void* residual_bf16, const void* norm_weight_bf16, float eps,
                              int64_t seq_len, void* out_fp8, float* out_scale, void* stream) {
  if (seq_len < 0 || seq_len > (int64_t(1) << 24) || !(eps >= 0.f)) return MOE_ERR_INVALID_ARG;
  if (seq_len == 0) return check_device();
  if (!x_bf16 || !out_fp8 || !out_scale) return MOE_ERR_INVALID_ARG;
  if (!aligned16(x_bf16) || !aligned16(out_fp8) || (residual_bf16 && !aligned16(residual_bf16)) ||
      (norm_weight_bf16 && !aligned16(norm_weight_bf16)) || (reinterpret_cast<uintptr_t>(out_scale) & 3u))
    return MOE_ERR_ALIGNMENT;
  int rc = check_device();
  if (rc) return rc;
  if (launch_add_norm_quant(x_bf16, residual_bf16, norm_weight_bf16, eps, static_cast<int>(seq_len), out_fp8,
                            out_scale, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int moe_fp8_ds_ep_pack(const void* hidden_states, const float* hidden_states_scale, const int32_t* topk_ids,
                       const float* topk_weights, int64_t seq_len, const int64_t* send_idx, int64_t num_send,
                       void* send_buf, void* stream) {
  if (seq_len < 0 || num_send < 0 || seq_len > (int64_t(1) << 24) || num_send > (int64_t(1) << 27))
    return MOE_ERR_INVALID_ARG;
  if (num_send == 0) return check_device();
  if (!hidden_states || !hidden_states_scale || !topk_ids || !topk_weights || !send_idx || !send_buf)
    return MOE_ERR_INVALID_ARG;
  if (!aligned16(hidden_states) || !aligned16(send_buf)) return MOE_ERR_ALIGNMENT;
  int rc = check_device();
  if (rc) return rc;
  if (launch_ep_pack(hidden_states, hidden_states_scale, topk_ids, topk_weights, static_cast<int>(seq_len), send_idx,
                     static_cast<int>(num_send), send_buf, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int moe_fp8_ds_ep_unpack(const void* recv_buf, int64_t num_rows, void* hidden_states, float* hidden_states_scale,
                         int32_t* topk_ids, float* topk_weights, void* stream) {
  if (num_rows < 0 || num_rows > (int64_t(1) << 27)) return MOE_ERR_INVALID_ARG;
  if (num_rows == 0) return check_device();
  if (!recv_buf || !hidden_states || !hidden_states_scale || !topk_ids || !topk_weights) return MOE_ERR_INVALID_ARG;
  if (!aligned16(recv_buf) || !aligned16(hidden_states)) return MOE_ERR_ALIGNMENT;
  int rc = check_device();
  if (rc) return rc;
  if (launch_ep_unpack(recv_buf, static_cast<int>(num_rows), hidden_states, hidden_states_scale, topk_ids,
                       topk_weights, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int moe_fp8_ds_ep_plan(const int32_t* topk_ids, int64_t seq_len, int64_t world, int64_t* send_idx,
                       int64_t* send_counts, int32_t* row_of, void* stream) {
  if (seq_len < 0 || seq_len > (int64_t(1) << 24) || world < 1 || world > 64 || (kExperts % world) != 0)
    return MOE_ERR_INVALID_ARG;
  if (!send_counts) return MOE_ERR_INVALID_ARG;
  if (seq_len > 0 && (!topk_ids || !send_idx || !row_of)) return MOE_ERR_INVALID_ARG;
  int rc = check_device();
  if (rc) return rc;
  // seq_len 0 still writes the (zero) counts
  if (launch_ep_plan(topk_ids, static_cast<int>(seq_len), static_cast<int>(world), send_idx, send_counts, row_of,
                     static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int moe_fp8_ds_ep_combine(const void* partials, const int32_t* row_of, int64_t seq_len, int64_t world, void* output,
                          void* stream) {
  if (seq_len < 0 || seq_len > (int64_t(1) << 24) || world < 1 || world > 64) return MOE_ERR_INVALID_ARG;
  if (seq_len == 0) return check_device();
  if (!row_of || !output) return MOE_ERR_INVALID_ARG;
  if ((partials && !aligned16(partials)) || !aligned16(output)) return MOE_ERR_ALIGNMENT;
  int rc = check_device();
  if (rc) return rc;
  if (launch_ep_combine(partials, row_of, static_cast<int>(seq_len), static_cast<int>(world), output,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

const char* moe_fp8_ds_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument (size, null pointer or unsupported value)";
    case MOE_ERR_ALIGNMENT: return "tensor base address is not 16-byte aligned";
    case MOE_ERR_CUDA: return "CUDA runtime/driver call failed";
    case MOE_ERR_NO_DEVICE: return "no sm_100 (B200) device is current";
    case MOE_ERR_WORKSPACE: return "device workspace allocation failed";
    case MOE_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    default: return "unknown status";
  }
}

int moe_fp8_ds_device_status(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return MOE_ERR_CUDA;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  int rc = MOE_OK;
  for (auto& kv : g_ws) {
    if (kv.first / 1024 != dev || !kv.second.base) continue;
    unsigned v = 0;
    if (cudaMemcpy(&v, kv.second.status, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return MOE_ERR_CUDA;
    if (v) {
      // a kernel gave up part-way: counters and partial sums that are normally
      // left at zero may not be; clear them (this also clears the status word)
      cudaMemset(kv.second.base, 0, kv.second.zero_bytes);
      rc = MOE_ERR_DEVICE_TIMEOUT;
    }
  }
  return rc;
}

int moe_fp8_ds_last_rows(int64_t seq_len, int64_t num_local_experts, int32_t* rows_out, void* stream) {
  if (seq_len < 0 || !valid_e_local(num_local_experts)) return MOE_ERR_INVALID_ARG;
  if (seq_len > 0 && !rows_out) return MOE_ERR_INVALID_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (seq_len == 0) return MOE_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_ws.find(ws_key(dev, static_cast<int>(num_local_experts), false));
  if (it == g_ws.end() || !it->second.base || it->second.t_cap < seq_len) return MOE_ERR_INVALID_ARG;
  if (cudaMemcpyAsync(rows_out, it->second.token_rows, static_cast<size_t>(seq_len) * kTopK * 4,
                      cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

size_t moe_fp8_ds_workspace_bytes(int64_t seq_len, int64_t num_local_experts) {
  if (seq_len < 0 || !valid_e_local(num_local_experts)) return 0;
  Workspace w;
  return layout(w, seq_len, static_cast<int>(num_local_experts), nullptr, nullptr);
}

int moe_fp8_ds_release_workspace(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  cudaDeviceSynchronize();
  for (auto it = g_ws.begin(); it != g_ws.end();) {
    if (it->first / 1024 == dev) {
      if (it->second.base) {
        forget_maps(it->second.base, it->second.bytes);
        cudaFree(it->second.base);
      }
      it = g_ws.erase(it);
    } else {
      ++it;
    }
  }
  return MOE_OK;
}

int moe_fp8_ds_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (on && !g_prof_ev[0]) {
    for (int i = 0; i <= kProfKernels; ++i)
      if (cudaEventCreate(&g_prof_ev[i]) != cudaSuccess) return MOE_ERR_CUDA;
  }
  g_prof_on = on != 0;
  g_prof_valid = false;
  return MOE_OK;
}

int moe_fp8_ds_profile_last(float* ms_out, int n) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!ms_out || n <= 0) return -MOE_ERR_INVALID_ARG;
  if (!g_prof_valid) return 0;
  if (cudaEventSynchronize(g_prof_ev[g_prof_n]) != cudaSuccess) return -MOE_ERR_CUDA;
  int k = n < g_prof_n ? n : g_prof_n;
  for (int i = 0; i < k; ++i) {
    if (cudaEventElapsedTime(&ms_out[i], g_prof_ev[i], g_prof_ev[i + 1]) != cudaSuccess) return -MOE_ERR_CUDA;
  }
  return k;
}

int moe_fp8_ds_test_route_barrier(uint64_t wait_limit_ns, int skip_arrival_cta) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_test_wait_limit_ns = wait_limit_ns;
  g_test_skip_arrival = skip_arrival_cta;
  return MOE_OK;
}

int moe_fp8_ds_set_fused_decode(int on) {
  std::lock_guard<std::mutex> lk(g_mu);
  const int prev = fused_decode_enabled() ? 1 : 0;
  if (on >= 0) g_fused_decode = on ? 1 : 0;
  return prev;
}

const char* moe_fp8_ds_version(void) { return "moe_fp8_ds 0.1 sm_100a"; }

}  // extern "C"
