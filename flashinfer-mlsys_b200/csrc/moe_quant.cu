// moe_quant.cu — the step upstream of the layer: BF16 hidden states to the
// layer's FP8 input format, e4m3 rows with one fp32 scale per 1x128 block,
// scales stored transposed [56][T] (the hidden_states / hidden_states_scale
// pair of reference moe/ref_moe.json).
//
// Per block of 128 columns of a token: s = max(amax(|x|) / 448, 1e-12),
// q = e4m3(x / s) rounded to nearest even (x / s <= 448 up to one rounding of
// the division, which rounds back to 448). This is the recipe of the layer's
// input definition (amax / 448 per 1x128 block) and of the intermediate
// requantisation in reference solution/triton/dsl-temp1.py:479-481. The
// quotient must be the correctly rounded float32 x / s (e4m3 rounding of a
// 1-ulp-off quotient can differ), so the bytes match a float32 host
// computation exactly. It is formed with Markstein's correction (P. Markstein,
// IA-64 division, 1990): with r = RN(1/s), q0 = RN(x r), e = x - q0 s
// (exact, one fma) and q = RN(q0 + e r) is the correctly rounded quotient
// when x and s are normal numbers (s >= 1e-12 here; a quotient small enough
// for e to underflow rounds to e4m3 zero either way). Two fmas per element
// instead of an IEEE division.
//
// One warp handles one token at a time, two 128-column blocks per step: lanes
// 0-15 hold block 2c, lanes 16-31 block 2c+1, 8 bf16 (16 bytes) per lane.
// HBM-bound: 14,336 B read and 7,392 B written per token.
#include "moe_kernels.h"

namespace moe {

namespace {

constexpr int kQuantWarps = 8;
constexpr int kQuantSteps = kHidden / 256;  // 28 steps of two blocks

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__global__ void __launch_bounds__(kQuantWarps * 32)
    quant_rows_kernel(const uint4* __restrict__ x, int T, uint2* __restrict__ q, float* __restrict__ scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kQuantWarps + warp;
  if (t >= T) return;
  const uint4* src = x + (size_t)t * (kHidden / 8);
  uint2* dst = q + (size_t)t * (kHidden / 8);
  constexpr int kUnroll = 4;
#pragma unroll 1
  for (int c0 = 0; c0 < kQuantSteps; c0 += kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) v[j] = __ldcs(src + (c0 + j) * 32 + lane);
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const int c = c0 + j;
      float f[8] = {bf16_lo(v[j].x), bf16_hi(v[j].x), bf16_lo(v[j].y), bf16_hi(v[j].y),
                    bf16_lo(v[j].z), bf16_hi(v[j].z), bf16_lo(v[j].w), bf16_hi(v[j].w)};
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
      // max over the 16 lanes of this block (|x| bits order like the values)
      unsigned mb = __float_as_uint(m);
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      const float s = fmaxf(__fdiv_rn(__uint_as_float(mb), 448.0f), 1e-12f);
      const float r = __frcp_rn(s);
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float q0 = f[i] * r;
        const float e = fmaf(-q0, s, f[i]);
        y[i] = copysignf(fmaf(e, r, q0), q0);  // keeps -0 for x = -0
      }
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        w0 |= static_cast<uint32_t>(f2_to_e4m3x2(y[i], y[i + 1])) << (8 * i);
        w1 |= static_cast<uint32_t>(f2_to_e4m3x2(y[4 + i], y[5 + i])) << (8 * i);
      }
      __stcs(dst + c * 32 + lane, make_uint2(w0, w1));
      if ((lane & 15) == 0) scale[(size_t)(2 * c + (lane >> 4)) * T + t] = s;
    }
  }
}

}  // namespace

cudaError_t launch_quant_rows(const void* x, int T, void* q, float* scale, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int grid = (T + kQuantWarps - 1) / kQuantWarps;
  return launch_k(quant_rows_kernel, dim3(grid), dim3(kQuantWarps * 32), 0, s, false,
                  static_cast<const uint4*>(x), T, static_cast<uint2*>(q), scale);
}

}  // namespace moe
