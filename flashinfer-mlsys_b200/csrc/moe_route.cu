// moe_route.cu — K1: DeepSeek-V3 no-aux routing + local histogram + the
// expert-major token lists and the device-side tile plan that both GEMMs
// read (no host synchronisation).
//
// Routing semantics follow reference moe/ref_moe.py:95-126:
//   s = 1 / (1 + exp(-logit)); sb = s + bias
//   group score = sum of the two largest sb in each of 8 groups of 32
//   keep the 4 best groups; take the 8 largest sb inside them
//   weight_k = s[id_k] / (sum_k s[id_k] + 1e-20) * routed_scaling_factor
// and the local dispatch of ref_moe.py:131-148 / kernel.cu:201-232
// (expert id - local_expert_offset in [0, E_local)).
#include "moe_kernels.h"
#include "moe_routing.cuh"

namespace moe {

namespace {

constexpr int kRouteThreads = 256;  // 8 warps, one token per warp at a time
constexpr int kMinTokensPerCta = 8;
// Cost of one extra work unit (its output stage and pipeline refill) in K
// blocks, used when choosing the K split.
#ifndef MOE_SPLIT_UNIT_OVERHEAD
#define MOE_SPLIT_UNIT_OVERHEAD 16
#endif
constexpr int kSplitUnitOverhead = MOE_SPLIT_UNIT_OVERHEAD;

// One warp, one token, after its routing CTA knows its base slot inside every
// expert (`s_off`): record the token in the expert-major lists GEMM1 gathers
// from (etok/ew, slot = base + rank inside the CTA), its local (expert, slot)
// pairs in ascending expert id (the order in which ref_moe.py:134-166
// accumulates the experts, -1 padded) and their number; a token with no local
// expert gets its output row zeroed here (kernel.cu:206-209: every element of
// the DPS output is written).
__device__ __forceinline__ void scatter_token(int t, int lane, const RouteArgs& a, const int* s_off,
                                              const Workspace& ws) {
  int le = -1, slot = -1;
  if (lane < kTopK) {
    const size_t o = (size_t)t * kTopK + lane;
    const int r = ws.topk_rank[o];
    if (r >= 0) {
      le = ws.topk_ids[o] - a.offset;
      slot = s_off[le] + r;
      ws.etok[(size_t)le * ws.t_cap + slot] = t;
      ws.ew[(size_t)le * ws.t_cap + slot] = ws.topk_w[o];
    }
  }
  // a token's experts are distinct, so the rank among its local ones is unique
  const int key = le >= 0 ? le : 0x7fffffff;
  int rank = 0;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) rank += (__shfl_sync(0xffffffffu, key, k) < key) ? 1 : 0;
  const int n_loc = __popc(__ballot_sync(0xffffffffu, le >= 0));
  if (lane < kTopK) {
    if (le >= 0) {
      ws.tok_e[(size_t)t * kTopK + rank] = le;
      ws.tok_slot[(size_t)t * kTopK + rank] = slot;
    }
    if (lane >= n_loc) {
      ws.tok_e[(size_t)t * kTopK + lane] = -1;
      ws.tok_slot[(size_t)t * kTopK + lane] = -1;
    }
  }
  if (lane == 0) ws.tok_n[t] = n_loc;
  if (n_loc == 0) {
    const int n16 = a.out_fp32 ? kHidden * 4 / 16 : kHidden * 2 / 16;
    uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + (size_t)t * (n16 * 16));
    for (int i = lane; i < n16; i += 32) o[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

__global__ void __launch_bounds__(kRouteThreads) route_plan_kernel(RouteArgs a, Workspace ws) {
  __shared__ int hist[kExperts];
  __shared__ int s_off[kExperts];  // this CTA's first slot inside every expert
  __shared__ int is_last;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int E_l = a.e_local;
  // first kernel of a call: launched with normal stream ordering; let GEMM1
  // get scheduled early (it runs its prologue, then waits for this grid).
  griddep_launch_dependents();
  for (int e = tid; e < E_l; e += blockDim.x) hist[e] = 0;
  __syncthreads();

  const int t_begin = blockIdx.x * a.tokens_per_cta;
  const int t_end = min(a.T, t_begin + a.tokens_per_cta);
  const int nwarps = blockDim.x >> 5;
  for (int t = t_begin + warp; t < t_end; t += nwarps) {
    int my_id = -1;     // lane k < 8 holds the k-th selected expert
    float my_w = 0.f;
    if (a.logits != nullptr) {
      route_token_warp(a.logits + (size_t)t * kExperts, a.bias, a.scale, lane, my_id, my_w);
    } else if (lane < kTopK) {
      my_id = __ldg(a.given_ids + (size_t)t * kTopK + lane);
      my_w = __ldg(a.given_w + (size_t)t * kTopK + lane);
    }
    if (lane < kTopK) {
      const size_t o = (size_t)t * kTopK + lane;
      ws.topk_ids[o] = my_id;
      ws.topk_w[o] = my_w;
      if (a.user_ids) a.user_ids[o] = my_id;
      if (a.user_w) a.user_w[o] = my_w;
      const int le = my_id - a.offset;
      int r = -1;
      if (my_id >= 0 && le >= 0 && le < E_l) r = atomicAdd(&hist[le], 1);
      ws.topk_rank[o] = r;
    }
  }
  __syncthreads();

  // ---- this CTA's base slot inside every expert ----
  const bool single = gridDim.x == 1;
  for (int e = tid; e < E_l; e += blockDim.x) {
    const int h = hist[e];
    s_off[e] = (single || !h) ? 0 : atomicAdd(&ws.expert_fill[e], h);
  }
  __syncthreads();
  // ---- expert-major token lists and per-token slots (full pipeline only) ----
  if (ws.etok != nullptr) {
    for (int t = t_begin + warp; t < t_end; t += nwarps) scatter_token(t, lane, a, s_off, ws);
  }
  int c = 0;
  if (single) {
    // single CTA: the shared histogram is the whole story
    if (tid < E_l) c = hist[tid];
  } else {
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(ws.done_ctas, 1u) == gridDim.x - 1) ? 1 : 0;
    __syncthreads();
    if (!is_last) return;
    // ---- last CTA: per-expert counts ----
    __threadfence();
    if (tid < E_l) c = atomicExch(&ws.expert_fill[tid], 0);  // read and reset for the next call
  }
  // ---- m-tile prefix and K-split plan ----
  __shared__ int warp_tot[2][kRouteThreads / 32];
  if (tid < E_l) {
    ws.plan->count[tid] = c;
    if (a.user_counts) a.user_counts[tid] = c;
  }
  int m = (c + kTileM - 1) / kTileM;
  // block-wide exclusive scan of m-tiles and total of rows over the experts
  int incl = m, csum = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
    csum += __shfl_xor_sync(0xffffffffu, csum, off);
  }
  if (lane == 31) warp_tot[0][warp] = incl;
  if (lane == 0) warp_tot[1][warp] = csum;
  __syncthreads();
  int base = 0, total = 0, nas = 0;
  for (int w = 0; w < nwarps; ++w) {
    if (w < warp) base += warp_tot[0][w];
    total += warp_tot[0][w];
    nas += warp_tot[1][w];
  }
  if (tid < E_l) ws.plan->mtile_prefix[tid] = base + incl - m;
  if (warp == 0) {
    // K split: minimise waves * (K blocks per unit + per-unit overhead); lane = split - 1
    auto cost = [&](int tiles, int nkb, int smax, int sp) -> long long {
      if (sp > smax || tiles <= 0) return 0x7fffffffffffLL;
      const long long units = (long long)tiles * sp;
      return ((units + kSMs - 1) / kSMs) * ((nkb + sp - 1) / sp + kSplitUnitOverhead);
    };
    const int sp = lane + 1;
    const long long c1 = (total <= kMaxSplitMTiles) ? cost(total * kNT1, kKB1, 14, sp) : (sp == 1 ? 0 : 0x7fffffffffffLL);
    const long long c2 = (total <= kMaxSplitMTiles) ? cost(total * kNT2, kKB2, 4, sp) : (sp == 1 ? 0 : 0x7fffffffffffLL);
    // pack (cost, split) so that the minimum prefers the smaller split on ties
    unsigned long long k1 = (static_cast<unsigned long long>(c1) << 8) | sp;
    unsigned long long k2 = (static_cast<unsigned long long>(c2) << 8) | sp;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const unsigned long long o1 = __shfl_xor_sync(0xffffffffu, k1, off);
      const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, k2, off);
      k1 = o1 < k1 ? o1 : k1;
      k2 = o2 < k2 ? o2 : k2;
    }
    if (lane == 0) {
      ws.plan->mtile_prefix[E_l] = total;
      ws.plan->total_mtiles = total;
      ws.plan->n_assign = nas;
      ws.plan->split1 = total > 0 ? static_cast<int>(k1 & 0xFF) : 1;
      ws.plan->split2 = total > 0 ? static_cast<int>(k2 & 0xFF) : 1;
      *ws.done_ctas = 0u;
    }
  }
}

}  // namespace

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kSMs;
  if (!cache[dev]) {
    int n = kSMs;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n;
  }
  return cache[dev];
}

int tokens_per_cta_for(int T, int ctas_per_sm) {
  // one token per warp for small T (a call with T <= 8 is a single CTA and
  // needs no cross-CTA handshake); at most ~ctas_per_sm * kSMs routing CTAs
  // for large T (routing a token is a few hundred dependent warp
  // instructions, so large calls want several resident CTAs per SM)
  const int ctas = kSMs * (ctas_per_sm > 0 ? ctas_per_sm : 1);
  int per = (T + ctas - 1) / ctas;
  per = ((per + 7) / 8) * 8;
  return per < kMinTokensPerCta ? kMinTokensPerCta : per;
}

int route_ctas_for(int T, int ctas_per_sm) {
  if (T <= 0) return 1;
  const int per = tokens_per_cta_for(T, ctas_per_sm);
  return (T + per - 1) / per;
}

cudaError_t launch_route(const Workspace& ws, const RouteArgs& a, cudaStream_t s) {
  const int grid = (a.T + a.tokens_per_cta - 1) / a.tokens_per_cta;
  return launch_k(route_plan_kernel, dim3(grid), dim3(kRouteThreads), 0, s, false, a, ws);
}

}  // namespace moe
