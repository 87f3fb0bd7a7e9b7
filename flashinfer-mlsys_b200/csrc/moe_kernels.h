// moe_kernels.h — host-side launch interface of the MoE kernels (internal).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "moe_common.cuh"

namespace moe {

// Device workspace of one call (all pointers device memory).
struct Workspace {
  int64_t t_cap = 0;       // tokens (rows of the caller's tensors) it was sized for
  int e_local = 0;         // local experts it was sized for
  int64_t rows_cap = 0;    // rows of the expert-major padded layout
  int route_ctas_cap = 0;  // routing CTAs it was sized for

  int32_t* topk_ids = nullptr;     // [t_cap][8] global expert ids
  float* topk_w = nullptr;         // [t_cap][8]
  int32_t* topk_rank = nullptr;    // [t_cap][8] rank inside (routing CTA, expert), -1 = not local
  int32_t* cta_off = nullptr;      // [route_ctas_cap][e_local] first slot of each CTA in an expert
  int32_t* expert_fill = nullptr;  // [e_local] running counters (self-resetting)
  uint32_t* done_ctas = nullptr;   // routing CTAs finished (self-resetting)
  Plan* plan = nullptr;
  uint8_t* a1 = nullptr;           // [rows_cap][7168] permuted e4m3 token rows
  float* a1_scale = nullptr;       // [56][rows_cap]
  int32_t* row_token = nullptr;    // [rows_cap] source token of each permuted row
  float* row_weight = nullptr;     // [rows_cap] routing weight of each permuted row
  uint8_t* inter = nullptr;        // [rows_cap][4096] two-term e4m3 intermediate (hi | lo)
  float* inter_scale = nullptr;    // [16][rows_cap] hi scales (lo = hi / 16)
  float* g_part = nullptr;         // [kMaxSplitMTiles*128][4096] GEMM1 split-K partial sums (kept zero)
  int32_t* tile_sem = nullptr;     // [kMaxSplitMTiles][16] GEMM1 split-K arrival counters (kept zero)
  float* g2_part = nullptr;        // [kMaxSplitMTiles*128][7168] GEMM2 split-K partial sums (kept zero)
  int32_t* tile_sem2 = nullptr;    // [kMaxSplitMTiles][28] GEMM2 split-K arrival counters (kept zero)
  float* out_rows = nullptr;       // [rows_cap][7168] routing-weighted expert output of every permuted row
  int32_t* token_rows = nullptr;   // [t_cap][8] permuted rows of each token, ascending expert id, -1 padded
  unsigned* status = nullptr;      // device status word (kErrTimeout ...)
  void* base = nullptr;            // single allocation backing everything above
  size_t bytes = 0;
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
};

struct PermuteArgs {
  const uint8_t* hidden;      // [T][7168]
  const float* hidden_scale;  // [56][T]
  int T;
  int offset;
  int tokens_per_cta;
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

int route_ctas_for(int T);
int device_sm_count();  // cached per device
int tokens_per_cta_for(int T);

cudaError_t launch_route(const Workspace& ws, const RouteArgs& a, cudaStream_t s);
cudaError_t launch_permute(const Workspace& ws, const PermuteArgs& a, cudaStream_t s);
// skinny: every m-tile has at most kSkinnyMaxRows valid rows (map_a then has
// kSkinnyMaxRows-row boxes)
cudaError_t launch_gemm1(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                         const float* w_scale, cudaStream_t s, bool skinny);
cudaError_t launch_gemm2(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                         const float* w_scale, cudaStream_t s, bool skinny);
cudaError_t launch_finalize(const Workspace& ws, int T, void* out, int out_fp32, cudaStream_t s);


}  // namespace moe
