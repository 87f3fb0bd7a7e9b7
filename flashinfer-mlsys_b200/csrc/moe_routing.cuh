// moe_routing.cuh — DeepSeek-V3 no-aux routing of one token by one warp,
// shared by the routing kernel and the fused decode kernel.
//
// Semantics follow reference moe/ref_moe.py:95-126:
//   s = 1 / (1 + exp(-logit)); sb = s + bias
//   group score = sum of the two largest sb in each of 8 groups of 32
//   keep the 4 best groups; take the 8 largest sb inside them
//   weight_k = s[id_k] / (sum_k s[id_k] + 1e-20) * routed_scaling_factor
#pragma once
#include "moe_common.cuh"

namespace moe {

// Sort 8 composite keys descending (19-comparator network, all-0/1-input verified).
__device__ __forceinline__ void cmpswap(uint64_t& a, uint64_t& b) {
  const uint64_t hi = a > b ? a : b, lo = a > b ? b : a;
  a = hi;
  b = lo;
}
__device__ __forceinline__ void sort8_desc(uint64_t (&c)[8]) {
  cmpswap(c[0], c[2]); cmpswap(c[1], c[3]); cmpswap(c[4], c[6]); cmpswap(c[5], c[7]);
  cmpswap(c[0], c[4]); cmpswap(c[1], c[5]); cmpswap(c[2], c[6]); cmpswap(c[3], c[7]);
  cmpswap(c[0], c[1]); cmpswap(c[2], c[3]); cmpswap(c[4], c[5]); cmpswap(c[6], c[7]);
  cmpswap(c[2], c[4]); cmpswap(c[3], c[5]);
  cmpswap(c[1], c[4]); cmpswap(c[3], c[6]);
  cmpswap(c[1], c[2]); cmpswap(c[3], c[4]); cmpswap(c[5], c[6]);
}

// Loads lane l's 8 logits (experts 8l..8l+7) of one token.
__device__ __forceinline__ void route_load_warp(const float* __restrict__ logits_row, int lane, float (&x)[8]) {
  const float4* lp = reinterpret_cast<const float4*>(logits_row + lane * 8);
  const float4 x0 = __ldg(lp), x1 = __ldg(lp + 1);
  x[0] = x0.x; x[1] = x0.y; x[2] = x0.z; x[3] = x0.w;
  x[4] = x1.x; x[5] = x1.y; x[6] = x1.z; x[7] = x1.w;
}

// Loads lane l's 8 routing biases (bf16 bits of experts 8l..8l+7).
__device__ __forceinline__ uint4 route_load_bias(const uint16_t* __restrict__ bias, int lane) {
  return __ldg(reinterpret_cast<const uint4*>(bias + lane * 8));
}

// Routes one token whose logits the warp holds (x from route_load_warp, braw
// from route_load_bias). Lanes 0..7 receive the k-th selected global expert id
// (`my_id`) and its routing weight (`my_w`), ordered by (sb desc, id asc).
__device__ __forceinline__ void route_compute_warp(const float (&x)[8], uint4 braw, float scale, int lane,
                                                   int& my_id, float& my_w) {
  // ---- lane l owns experts [8l, 8l+8): group g = l / 4 ----
  const uint32_t bw[4] = {braw.x, braw.y, braw.z, braw.w};
  float s[8], sb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t bits = (i & 1) ? (bw[i >> 1] & 0xFFFF0000u) : (bw[i >> 1] << 16);
    float b = __uint_as_float(bits);
    s[i] = 1.0f / (1.0f + expf(-x[i]));
    sb[i] = s[i] + b;
  }
  // ---- top-2 of the group (4 lanes) ----
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v = sb[i];
    if (v > m1) { m2 = m1; m1 = v; } else if (v > m2) { m2 = v; }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    float o1 = __shfl_xor_sync(0xffffffffu, m1, off);
    float o2 = __shfl_xor_sync(0xffffffffu, m2, off);
    float n1 = fmaxf(m1, o1);
    float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
    m1 = n1; m2 = n2;
  }
  const float gscore = m1 + m2;
  const int g = lane >> 2;
  int rank = 0;
#pragma unroll
  for (int gg = 0; gg < kGroups; ++gg) {
    float o = __shfl_sync(0xffffffffu, gscore, gg * 4);
    rank += (o > gscore || (o == gscore && gg < g)) ? 1 : 0;
  }
  const bool kept = rank < kTopKGroups;
  // ---- top-8 of the kept candidates, ordered by (sb desc, expert id asc) ----
  // composite key: order-preserving bits of sb in the high word, 0xFFFF - id
  // in the low word; 0 marks a candidate of a dropped group.
  uint64_t c[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t u = __float_as_uint(sb[i]);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    c[i] = kept ? ((static_cast<uint64_t>(ord) << 32) | static_cast<uint32_t>(0xFFFF - (lane * 8 + i))) : 0ull;
  }
  sort8_desc(c);
  // 8 rounds: warp max of the lane heads (key word, then id word), the
  // winning lane pops its head.
  int sel = 0;
#pragma unroll 1
  for (int k = 0; k < kTopK; ++k) {
    const uint32_t hk = static_cast<uint32_t>(c[0] >> 32);
    const uint32_t mk = __reduce_max_sync(0xffffffffu, hk);
    const uint32_t lo = (hk == mk) ? static_cast<uint32_t>(c[0]) : 0u;
    const uint32_t ml = __reduce_max_sync(0xffffffffu, lo);
    const bool win = (hk == mk) && (lo == ml);
    if (lane == k) sel = 0xFFFF - static_cast<int>(ml);
    if (win) {
#pragma unroll
      for (int i = 0; i < 7; ++i) c[i] = c[i + 1];
      c[7] = 0ull;
    }
  }
  // weight numerators: the un-biased sigmoid of the chosen expert, fetched
  // from the lane that owns it (lane sel / 8, element sel % 8)
  float sel_s = 0.f;
  {
    const int src = (sel >> 3) & 31, idx = sel & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = __shfl_sync(0xffffffffu, s[i], src);
      if (i == idx) sel_s = v;
    }
  }
  if (lane < kTopK) {
    my_id = sel;
  } else {
    sel_s = 0.f;
  }
  float ssum = sel_s;
#pragma unroll
  for (int off = 4; off >= 1; off >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, off);
  my_w = (sel_s / (ssum + 1e-20f)) * scale;
}

// Loads and routes one token (route_load_warp + route_compute_warp).
__device__ __forceinline__ void route_token_warp(const float* __restrict__ logits_row,
                                                 const uint16_t* __restrict__ bias, float scale, int lane,
                                                 int& my_id, float& my_w) {
  float x[8];
  route_load_warp(logits_row, lane, x);
  route_compute_warp(x, route_load_bias(bias, lane), scale, lane, my_id, my_w);
}

}  // namespace moe
