// moe_route.cu — K1 (DeepSeek-V3 no-aux routing + local histogram + plan,
// fused with the token permutation into the expert-major padded layout in one
// cooperative launch; a routing-only variant for the routing entry points)
// and K4 (the per-token combine of GEMM2's rows, or the cast of the per-token
// fp32 sums of a direct-combine call, to bf16/fp32 output).
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
// The same for GEMM2 of a call of at most 64 tokens: its partials add into
// per-token sums (no arrival counting, no read-back), so a unit costs little
// beyond its K blocks.
#ifndef MOE_DIRECT_UNIT_OVERHEAD
#define MOE_DIRECT_UNIT_OVERHEAD 2
#endif
constexpr int kDirectUnitOverhead = MOE_DIRECT_UNIT_OVERHEAD;
constexpr uint64_t kRouteWaitLimitNs = 2000000000ull;  // 2 s: only reached if something is broken

// One warp, one token: copy the e4m3 row (7168 B) and its 56 block scales to
// every local expert slot the token was routed to, and record the token's
// rows. `prefix` is the m-tile prefix of the local experts, `base` the first
// slot of the token's routing CTA inside every expert.
// shared_row >= 0: the token's row of the shared expert (weight 1), which is
// not listed in token_rows (the finalize adds it after the routed rows).
__device__ __forceinline__ void permute_token(int t, int lane, const uint8_t* __restrict__ hidden,
                                              const float* __restrict__ hidden_scale, int T, int offset,
                                              const int* prefix, const int* base, const Workspace& ws,
                                              bool copy_rows, int shared_row) {
  int row = -1;
  float w = 0.f;
  if (lane < kTopK) {
    const size_t o = (size_t)t * kTopK + lane;
    const int r = ws.topk_rank[o];
    if (r >= 0) {
      const int le = ws.topk_ids[o] - offset;
      row = prefix[le] * kTileM + base[le] + r;
      w = ws.topk_w[o];
    }
  }
  // token_rows[t]: this token's rows in ascending expert id (the order in which
  // ref_moe.py:134-166 accumulates the experts), -1 padded
  {
    const int my_e = (row >= 0) ? ws.topk_ids[(size_t)t * kTopK + lane] : 0x7fffffff;
    int rank = 0, n_loc = 0;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int ek = __shfl_sync(0xffffffffu, my_e, k);
      const int rk = __shfl_sync(0xffffffffu, row, k);
      rank += (rk >= 0 && (ek < my_e || (ek == my_e && k < lane))) ? 1 : 0;
      n_loc += (rk >= 0) ? 1 : 0;
    }
    if (lane < kTopK) {
      if (row >= 0) ws.token_rows[(size_t)t * kTopK + rank] = row;
      if (lane >= n_loc) ws.token_rows[(size_t)t * kTopK + lane] = -1;
    }
  }
  const unsigned has = __ballot_sync(0xffffffffu, row >= 0) | (shared_row >= 0 ? (1u << 31) : 0u);
  if (!has) return;
  const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * kHidden);
  const float sc0 = copy_rows ? __ldg(hidden_scale + (size_t)lane * T + t) : 0.f;
  const float sc1 = (copy_rows && lane + 32 < kHiddenBlocks) ? __ldg(hidden_scale + (size_t)(lane + 32) * T + t) : 0.f;
  // the row in two halves of 7 chunks of 16 B per lane: each half is loaded
  // once (its loads in flight together) and stored to every destination
  constexpr int kChunks = kHidden / 16 / 32;  // 14
  constexpr int kHalf = kChunks / 2;
  for (int h = 0; h < 2; ++h) {
    uint4 v[kHalf];
    if (copy_rows) {
#pragma unroll
      for (int i = 0; i < kHalf; ++i) v[i] = __ldg(src + lane + 32 * (h * kHalf + i));
    }
    unsigned m = has;
    while (m) {
      const int k = __ffs(m) - 1;
      m &= m - 1;
      const int r = k == 31 ? shared_row : __shfl_sync(0xffffffffu, row, k);
      if (copy_rows) {
        uint4* dst = reinterpret_cast<uint4*>(ws.a1 + (size_t)r * kHidden);
#pragma unroll
        for (int i = 0; i < kHalf; ++i) dst[lane + 32 * (h * kHalf + i)] = v[i];
        if (h == 0) {
          ws.a1_scale[(size_t)lane * ws.rows_cap + r] = sc0;
          if (lane + 32 < kHiddenBlocks) ws.a1_scale[(size_t)(lane + 32) * ws.rows_cap + r] = sc1;
        }
      }
    }
  }
  unsigned m = has;
  while (m) {
    const int k = __ffs(m) - 1;
    m &= m - 1;
    const int r = k == 31 ? shared_row : __shfl_sync(0xffffffffu, row, k);
    const float wk = k == 31 ? 1.0f : __shfl_sync(0xffffffffu, w, k);
    if (lane == 0) {
      ws.row_token[r] = t;
      ws.row_weight[r] = wk;
    }
  }
}

// The device-side plan from the per-expert counts (thread e < E_l holds the
// count `c` of local expert e): m-tile prefix (also left in `s_prefix`,
// E_l + 1 entries), the number of (token, local expert) pairs and the K split
// of both GEMMs for a call of T tokens. With `write`, the plan and the
// optional user counts are stored. Called by every thread of the CTA.
__device__ __forceinline__ void build_plan(int c, int E_l, int* s_prefix, bool write, int32_t* user_counts,
                                           int n_user, const Workspace& ws, int T) {
  __shared__ int warp_tot[2][kRouteThreads / 32];
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  if (write && tid < E_l) {
    ws.plan->count[tid] = c;
    if (user_counts && tid < n_user) user_counts[tid] = c;
  }
  const int m = (c + kTileM - 1) / kTileM;
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
  if (tid < E_l) {
    s_prefix[tid] = base + incl - m;
    if (write) ws.plan->mtile_prefix[tid] = base + incl - m;
  }
  if (tid == 0) s_prefix[E_l] = total;
  if (write && warp == 0) {
    // K split: minimise waves * (K blocks per unit + per-unit overhead); lane = split - 1
    auto cost = [&](int tiles, int nkb, int smax, int sp, int overhead) -> long long {
      if (sp > smax || tiles <= 0) return 0x7fffffffffffLL;
      const long long units = (long long)tiles * sp;
      return ((units + kSMs - 1) / kSMs) * ((nkb + sp - 1) / sp + overhead);
    };
    const int sp = lane + 1;
    const int oh2 = T <= kSkinnyMaxRows ? kDirectUnitOverhead : kSplitUnitOverhead;
    const long long c1 =
        (total <= kMaxSplitMTiles) ? cost(total * kNT1, kKB1, 14, sp, kSplitUnitOverhead) : (sp == 1 ? 0 : 0x7fffffffffffLL);
    const long long c2 =
        (total <= kMaxSplitMTiles) ? cost(total * kNT2, kKB2, 4, sp, oh2) : (sp == 1 ? 0 : 0x7fffffffffffLL);
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
    }
  }
  __syncthreads();
}

// Routes the CTA's tokens (one warp per token) and counts its local
// assignments per expert in `hist`; writes ids, weights and per-(CTA, expert)
// ranks to the workspace and the optional user outputs.
__device__ __forceinline__ void route_tokens(const RouteArgs& a, const Workspace& ws, int* hist, int t_begin,
                                             int t_end) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
      if (my_id >= 0 && le >= 0 && le < a.e_local) r = atomicAdd(&hist[le], 1);
      ws.topk_rank[o] = r;
    }
  }
}

// Routing alone (moe_fp8_ds_route and the allocation-free router): the last
// CTA to finish builds the plan, so no CTA ever waits for another.
__global__ void __launch_bounds__(kRouteThreads) route_plan_kernel(RouteArgs a, Workspace ws) {
  __shared__ int hist[kExperts];
  __shared__ int s_prefix[kExperts + 1];
  __shared__ int is_last;
  const int tid = threadIdx.x;
  const int E_l = a.e_local;
  for (int e = tid; e < E_l; e += blockDim.x) hist[e] = 0;
  __syncthreads();

  const int t_begin = blockIdx.x * a.tokens_per_cta;
  const int t_end = min(a.T, t_begin + a.tokens_per_cta);
  route_tokens(a, ws, hist, t_begin, t_end);
  __syncthreads();

  int c = 0;
  if (gridDim.x == 1) {
    // single CTA: the shared histogram is the whole story
    if (tid < E_l) c = hist[tid];
  } else {
    // ---- publish this CTA's histogram ----
    for (int e = tid; e < E_l; e += blockDim.x) {
      const int h = hist[e];
      if (h) atomicAdd(&ws.expert_fill[e], h);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(ws.done_ctas, 1u) == gridDim.x - 1) ? 1 : 0;
    __syncthreads();
    if (!is_last) return;
    // ---- last CTA: per-expert counts ----
    __threadfence();
    if (tid < E_l) c = atomicExch(&ws.expert_fill[tid], 0);  // read and reset for the next call
  }
  build_plan(c, E_l, s_prefix, true, a.user_counts, E_l, ws, a.T);
  if (tid == 0) *ws.done_ctas = 0u;
}

// Routing fused with the histogram, the prefix sum and the token
// permutation (kernel.cu:157-232, ref_moe.py:95-148) in one cooperative launch
// (every CTA is resident). Each CTA routes its tokens, takes its base slot
// inside every expert from the running per-expert counters, and meets the
// others at a grid barrier; then every CTA reads the final counts, computes
// the m-tile prefix itself and copies its own tokens' e4m3 rows and scales to
// their slots of the expert-major padded layout. CTA 0 writes the plan the
// GEMMs read. The barrier wait is bounded (status bit and no permutation on
// timeout); the last CTA to leave resets the counters for the next call.
__global__ void __launch_bounds__(kRouteThreads) route_permute_kernel(RouteArgs a, PermuteArgs pa, Workspace ws) {
  __shared__ int hist[kExperts];
  __shared__ int s_base[kExperts];
  __shared__ int s_prefix[kExperts + 2];
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int E_l = a.e_local;
  const int E_tot = E_l + (pa.shared ? 1 : 0);  // the shared expert, if any, is local expert E_l
  const int G = gridDim.x;
  // first kernel of a call: let GEMM1 get scheduled early (it runs its
  // prologue, then waits for this grid)
  griddep_launch_dependents();
  for (int e = tid; e < E_l; e += blockDim.x) hist[e] = 0;
  if (tid == 0) s_ok = 1;
  __syncthreads();
  const int t_begin = blockIdx.x * a.tokens_per_cta;
  const int t_end = min(a.T, t_begin + a.tokens_per_cta);
  route_tokens(a, ws, hist, t_begin, t_end);
  __syncthreads();
  int c = 0;
  if (G == 1) {
    for (int e = tid; e < E_l; e += blockDim.x) s_base[e] = 0;
    if (tid < E_l) c = hist[tid];
    if (tid == E_l && pa.shared) c = a.T;
  } else {
    for (int e = tid; e < E_l; e += blockDim.x) {
      const int h = hist[e];
      s_base[e] = h ? atomicAdd(&ws.expert_fill[e], h) : 0;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0 && static_cast<int>(blockIdx.x) != a.skip_arrival_cta) {
      atomicAdd(ws.bar_cnt, 1u);
      const uint64_t limit = a.wait_limit_ns ? a.wait_limit_ns : kRouteWaitLimitNs;
      bool ok = true;
      uint64_t t0 = 0;
      for (uint32_t spin = 0;; ++spin) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ws.bar_cnt) : "memory");
        if (v >= static_cast<uint32_t>(G)) break;
        if (spin == 0) t0 = global_timer_ns();
        else if (global_timer_ns() - t0 > limit) { ok = false; break; }
        __nanosleep(64);
      }
      if (!ok) {
        atomicOr(ws.status, kErrTimeout);
        s_ok = 0;
      }
    } else if (tid == 0) {
      s_ok = 0;  // test hook: this CTA stays away from the barrier
    }
    __syncthreads();
    if (tid < E_l) c = __ldcg(&ws.expert_fill[tid]);
    if (tid == E_l && pa.shared) c = a.T;
  }
  // a CTA whose barrier wait gave up plans nothing (CTA 0's plan is the
  // GEMMs': an empty plan launches no work on rows that were never written)
  build_plan(s_ok ? c : 0, E_tot, s_prefix, blockIdx.x == 0, a.user_counts, E_l, ws, a.T);
  if (s_ok) {
    for (int t = t_begin + warp; t < t_end; t += kRouteThreads / 32)
      permute_token(t, lane, pa.hidden, pa.hidden_scale, pa.T, pa.offset, s_prefix, s_base, ws, pa.copy_rows != 0,
                    pa.shared ? s_prefix[E_l] * kTileM + t : -1);
  } else {
    // the barrier gave up: no rows for these tokens (the finalize writes
    // zeros; the GEMMs only read rows inside the padded layout)
    for (int t = t_begin + warp; t < t_end; t += kRouteThreads / 32)
      if (lane < kTopK) ws.token_rows[(size_t)t * kTopK + lane] = -1;
  }
  if (G > 1) {
    __syncthreads();
    if (tid == 0 && atomicAdd(ws.leave_cnt, 1u) == static_cast<uint32_t>(G) - 1) {
      // every CTA has read the counts: reset them for the next call
      for (int e = 0; e < E_l; ++e) ws.expert_fill[e] = 0;
      *ws.bar_cnt = 0u;
      *ws.leave_cnt = 0u;
    }
  }
}

// out[t, :] = sum over the token's local rows (ascending expert id) of the
// routing-weighted expert outputs (bf16 rows written by GEMM2), in fp32, then
// cast once (ref_moe.py:166-167). Eight columns per thread. A direct-combine
// call (direct_combine) has its fp32 sums in `tok_sum` already: they are cast
// and cleared for the next call.
__global__ void __launch_bounds__(256) finalize_kernel(const __nv_bfloat16* __restrict__ rows_buf,
                                                       const int32_t* __restrict__ token_rows,
                                                       void* __restrict__ out, int T, int out_fp32,
                                                       const Plan* __restrict__ plan, int shared_e,
                                                       float* __restrict__ tok_sum) {
  griddep_wait();
  const bool direct = direct_combine(plan->split2, T);
  // the shared expert's rows (one per token, in token order), added last
  const int64_t shared_base = (shared_e >= 0 && !direct) ? (int64_t)plan->mtile_prefix[shared_e] * kTileM : -1;
  constexpr int kC8 = kHidden / 8;  // 896 eight-column chunks per token
  const int64_t n = (int64_t)T * kC8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(i / kC8);
    const int c8 = static_cast<int>(i - (int64_t)t * kC8);
    float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
    if (direct) {
      // tok_sum is [T][7168], i.e. eight-column chunk i at float4 2i, 2i+1
      float4* g = reinterpret_cast<float4*>(tok_sum) + 2 * i;
      s0 = __ldcg(g);
      s1 = __ldcg(g + 1);
      __stcg(g, make_float4(0.f, 0.f, 0.f, 0.f));
      __stcg(g + 1, make_float4(0.f, 0.f, 0.f, 0.f));
    } else {
      const int4* tr = reinterpret_cast<const int4*>(token_rows + (size_t)t * kTopK);
      const int4 r0 = __ldg(tr), r1 = __ldg(tr + 1);
      const int r[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        if (r[k] < 0) break;
        // 8 bf16 columns of the row; bf16 -> f32 is exact (upper half of the word)
        const uint4 q = __ldcs(reinterpret_cast<const uint4*>(rows_buf + (size_t)r[k] * kHidden) + c8);
        s0.x += __uint_as_float(q.x << 16); s0.y += __uint_as_float(q.x & 0xFFFF0000u);
        s0.z += __uint_as_float(q.y << 16); s0.w += __uint_as_float(q.y & 0xFFFF0000u);
        s1.x += __uint_as_float(q.z << 16); s1.y += __uint_as_float(q.z & 0xFFFF0000u);
        s1.z += __uint_as_float(q.w << 16); s1.w += __uint_as_float(q.w & 0xFFFF0000u);
      }
      if (shared_base >= 0) {
        const uint4 q = __ldcs(reinterpret_cast<const uint4*>(rows_buf + (size_t)(shared_base + t) * kHidden) + c8);
        s0.x += __uint_as_float(q.x << 16); s0.y += __uint_as_float(q.x & 0xFFFF0000u);
        s0.z += __uint_as_float(q.y << 16); s0.w += __uint_as_float(q.y & 0xFFFF0000u);
        s1.x += __uint_as_float(q.z << 16); s1.y += __uint_as_float(q.z & 0xFFFF0000u);
        s1.z += __uint_as_float(q.w << 16); s1.w += __uint_as_float(q.w & 0xFFFF0000u);
      }
    }
    if (out_fp32) {
      float4* o = reinterpret_cast<float4*>(out) + 2 * i;
      o[0] = s0;
      o[1] = s1;
    } else {
      __nv_bfloat162 b0 = __floats2bfloat162_rn(s0.x, s0.y);
      __nv_bfloat162 b1 = __floats2bfloat162_rn(s0.z, s0.w);
      __nv_bfloat162 b2 = __floats2bfloat162_rn(s1.x, s1.y);
      __nv_bfloat162 b3 = __floats2bfloat162_rn(s1.z, s1.w);
      uint4 u;
      u.x = *reinterpret_cast<uint32_t*>(&b0);
      u.y = *reinterpret_cast<uint32_t*>(&b1);
      u.z = *reinterpret_cast<uint32_t*>(&b2);
      u.w = *reinterpret_cast<uint32_t*>(&b3);
      reinterpret_cast<uint4*>(out)[i] = u;
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

int route_permute_grid(int T, int* tokens_per_cta) {
  // all CTAs must be resident at once (cooperative launch): at most as many
  // as the device holds, up to kRouteCtasPerSm per SM
  static int occ_cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  if (!occ_cache[dev]) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, route_permute_kernel, kRouteThreads, 0) != cudaSuccess ||
        occ < 1)
      return -1;
    occ_cache[dev] = occ < kRouteCtasPerSm ? occ : kRouteCtasPerSm;
  }
  const int ctas = device_sm_count() * occ_cache[dev];
  int per = (T + ctas - 1) / ctas;
  per = ((per + 7) / 8) * 8;
  if (per < kMinTokensPerCta) per = kMinTokensPerCta;
  *tokens_per_cta = per;
  return (T + per - 1) / per;
}

cudaError_t launch_route_permute(const Workspace& ws, const RouteArgs& a, const PermuteArgs& pa, cudaStream_t s) {
  const int grid = (a.T + a.tokens_per_cta - 1) / a.tokens_per_cta;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = grid > 1 ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, route_permute_kernel, a, pa, ws);
}

cudaError_t launch_finalize(const Workspace& ws, int T, void* out, int out_fp32, cudaStream_t s, int shared_e) {
  const int64_t n8 = (int64_t)T * kHidden / 8;
  if (n8 == 0) return cudaSuccess;
  int64_t blocks = (n8 + 255) / 256;
  if (blocks > 16 * kSMs) blocks = 16 * kSMs;
  return launch_k(finalize_kernel, dim3((unsigned)blocks), dim3(256), 0, s, true,
                  static_cast<const __nv_bfloat16*>(ws.out_rows), static_cast<const int32_t*>(ws.token_rows), out, T,
                  out_fp32, static_cast<const Plan*>(ws.plan), shared_e, ws.g2_part);
}

}  // namespace moe
