// moe_kernels.h — host-side launch interface of the MoE kernels (internal).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "moe_common.cuh"

namespace moe {

// ---- fused decode kernel (1 <= T <= kDecMaxT) ----
// Scratch of the fused decode kernel (device memory; the counters, partial
// sums and the combine accumulator start at zero and are left at zero).
struct DecodeBuffers {
  int grid = 0;                // CTAs of the launch (the device's SM count)
  int slots_cap = 0;           // touched local experts it can hold
  uint8_t* inter = nullptr;    // [slots_cap][64][4096] two-term e4m3 intermediate
  float* inter_scale = nullptr;  // [slots_cap][16][64]
  float* g1_part = nullptr;    // [grid][2][64][256] pieces of split GEMM1 units
  float* g2_part = nullptr;    // [grid][2][64][256] pieces of GEMM2 units
  int* g1_cnt = nullptr;       // [grid]
  int* ready = nullptr;        // [slots_cap]
  int* h_cnt = nullptr;        // [28]
  int* done = nullptr;         // [1]
  const float* zero = nullptr;  // one 0.0f
  unsigned* status = nullptr;
};

struct DecodeCall {
  const float* logits;
  const uint16_t* bias;
  const float* hidden_scale;
  const float* w13_scale;
  const float* w2_scale;
  int T;
  int offset;
  int e_local;
  float scale;
  void* out;                   // bf16 [T][7168]
  int32_t* user_ids;
  float* user_w;
  int32_t* user_counts;
};

// Device workspace of one call (all pointers device memory).
struct Workspace {
  int64_t t_cap = 0;       // tokens (rows of the caller's tensors) it was sized for
  int e_local = 0;         // local experts it was sized for
  int64_t rows_cap = 0;    // rows of the expert-major padded layout

  int32_t* topk_ids = nullptr;     // [t_cap][8] global expert ids
  float* topk_w = nullptr;         // [t_cap][8]
  int32_t* topk_rank = nullptr;    // [t_cap][8] rank inside (routing CTA, expert), -1 = not local
  int32_t* expert_fill = nullptr;  // [e_local] running counters (self-resetting)
  uint32_t* done_ctas = nullptr;   // routing CTAs finished (self-resetting)
  uint32_t* bar_cnt = nullptr;     // fused routing kernel: CTAs at the grid barrier (self-resetting)
  uint32_t* leave_cnt = nullptr;   // fused routing kernel: CTAs past the barrier (self-resetting)
  Plan* plan = nullptr;
  uint8_t* a1 = nullptr;           // [rows_cap][7168] permuted e4m3 token rows
  float* a1_scale = nullptr;       // [56][rows_cap]
  int32_t* row_token = nullptr;    // [rows_cap] source token of each permuted row
  float* row_weight = nullptr;     // [rows_cap] routing weight of each permuted row
  uint8_t* inter = nullptr;        // [rows_cap][4096] two-term e4m3 intermediate (hi | lo)
  float* inter_scale = nullptr;    // [16][rows_cap] hi scales (lo = hi / 16)
  float* g_part = nullptr;         // [kMaxSplitMTiles*128][4096] GEMM1 split-K partial sums (kept zero)
  int32_t* tile_sem = nullptr;     // [kMaxSplitMTiles][16][4] GEMM1 split-K arrival counters (kept zero)
  float* g2_part = nullptr;        // [kMaxSplitMTiles*128][7168] GEMM2 split-K partial sums by row, or by token in a direct-combine call (kept zero)
  int32_t* tile_sem2 = nullptr;    // [kMaxSplitMTiles][28][16] GEMM2 split-K arrival counters (kept zero)
  __nv_bfloat16* out_rows = nullptr;  // [rows_cap][7168] routing-weighted expert output of every permuted row (bf16)
  int32_t* token_rows = nullptr;   // [t_cap][8] permuted rows of each token, ascending expert id, -1 padded
  unsigned* status = nullptr;      // device status word (kErrTimeout ...)
  DecodeBuffers dec;               // scratch of the fused decode kernel
  void* base = nullptr;            // single allocation backing everything above
  size_t bytes = 0;
  size_t zero_bytes = 0;           // length of the prefix that must be zero between calls
  bool shared_cap = false;         // rows_cap includes a shared expert's T rows
};

struct RouteArgs {
  const float* logits;        // [T][256] (route mode) or nullptr
  const uint16_t* bias;       // bf16 [256]
  const int32_t* given_ids;   // [T][8] (pre-routed mode) or nullptr
  const float* given_w;       // [T][8]
  int T;
  int offset;
  int e_local;
  float scale;
  int tokens_per_cta;
  int32_t* user_ids;          // optional outputs
  float* user_w;
  int32_t* user_counts;
  // Fused routing kernel: the grid-barrier wait limit (0 = the default) and
  // a CTA that skips its barrier arrival (-1 = none). Set only by the
  // failure-path test hook moe_fp8_ds_test_route_barrier.
  uint64_t wait_limit_ns;
  int skip_arrival_cta;
};

struct PermuteArgs {
  const uint8_t* hidden;      // [T][7168]
  const float* hidden_scale;  // [56][T]
  int T;
  int offset;
  int tokens_per_cta;
  int copy_rows;              // 0: record the row maps only (GEMM1 gathers the rows itself)
  int shared;                 // 1: a shared expert is local expert e_local, every token's row t
};

// Launch `kernel` on `s`; with `pdl` the launch may overlap the tail of the
// previous kernel on the stream (the kernel must call griddep_wait() before
// touching that kernel's outputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Routing grid: tokens per routing CTA and the CTA count for T tokens, with up
// to ctas_per_sm CTAs per SM for large T.
constexpr int kRouteCtasPerSm = 4;
int route_ctas_for(int T, int ctas_per_sm = kRouteCtasPerSm);
int device_sm_count();  // cached per device
int tokens_per_cta_for(int T, int ctas_per_sm = kRouteCtasPerSm);

// Routing alone (no permutation): route_ctas_for() CTAs, no CTA waits for another.
cudaError_t launch_route(const Workspace& ws, const RouteArgs& a, cudaStream_t s);
// Routing fused with the permutation: one cooperative launch. The grid and
// a.tokens_per_cta must come from route_permute_grid (-1: no device).
int route_permute_grid(int T, int* tokens_per_cta);
cudaError_t launch_route_permute(const Workspace& ws, const RouteArgs& a, const PermuteArgs& pa, cudaStream_t s);
// skinny: every m-tile has at most kSkinnyMaxRows valid rows. GEMM1 then
// gathers its rows from hidden_states (map_a: hidden_states [T][7168] with
// one-row boxes, x_scale its [56][T] scales); otherwise map_a is the permuted
// rows with 128-row boxes. GEMM2's map_a has kSkinnyMaxRows-row boxes when skinny.
// shared_e >= 0: local expert shared_e is a shared expert whose weights come
// through map_ws / ws_scale (one expert); otherwise map_ws is unused.
cudaError_t launch_gemm1(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                         const float* w_scale, cudaStream_t s, bool skinny, const float* x_scale, int64_t T,
                         const CUtensorMap& map_ws, const float* ws_scale, int shared_e);
cudaError_t launch_gemm2(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                         const float* w_scale, cudaStream_t s, bool skinny, const CUtensorMap& map_ws,
                         const float* ws_scale, int shared_e, int T);
// shared_e >= 0: every token also adds its row of the shared expert (last);
// a direct-combine call (direct_combine) casts the per-token sums instead
cudaError_t launch_finalize(const Workspace& ws, int T, void* out, int out_fp32, cudaStream_t s, int shared_e);

// Expert-parallel token exchange (packed 7456-byte rows, see moe_ep.cu)
cudaError_t launch_ep_pack(const void* hidden, const float* hidden_scale, const int32_t* ids, const float* w, int T,
                           const int64_t* idx, int S, void* out, cudaStream_t s);
cudaError_t launch_ep_unpack(const void* in, int R, void* hidden, float* hidden_scale, int32_t* ids, float* w,
                             cudaStream_t s);
cudaError_t launch_ep_combine(const void* back, const int32_t* row_of, int T, int world, void* out, cudaStream_t s);
cudaError_t launch_ep_plan(const int32_t* ids, int T, int world, int64_t* send_idx, int64_t* send_counts,
                           int32_t* row_of, cudaStream_t s);

// BF16 [T][7168] -> e4m3 [T][7168] + f32 scales [56][T] (1x128 blocks, amax / 448)
cudaError_t launch_quant_rows(const void* x, int T, void* q, float* scale, cudaStream_t s);
cudaError_t launch_add_norm_quant(const void* x, void* residual, const void* w, float eps, int T, void* q,
                                  float* scale, cudaStream_t s);

size_t decode_smem_bytes();
// map_w13: W13 [E_l*4096][7168] 128-row boxes; map_w2: W2 [E_l*7168][2048]
// 128-row boxes; map_x1: hidden_states [T][7168] 64-row boxes (rows >= T read
// as zero); map_x2: DecodeBuffers::inter [slots_cap*64][4096] 64-row boxes.
cudaError_t launch_decode(const DecodeBuffers& d, const CUtensorMap& map_w13, const CUtensorMap& map_w2,
                          const CUtensorMap& map_x1, const CUtensorMap& map_x2, const DecodeCall& c,
                          cudaStream_t s);


}  // namespace moe
