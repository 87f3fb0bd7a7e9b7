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
//
// The step downstream of the layer, add_norm_quant_kernel: the decoder's
// residual add, the next layer's input RMSNorm and the same 1x128
// quantisation, in one pass over the layer's bf16 output (DeepSeek-V3 decoder
// layer: h = residual + moe_out in bf16, then RMSNorm(h) with weight w and
// eps, as HF transformers' DeepseekV3RMSNorm computes it):
//   h  = bf16(residual + x)                        written back to residual
//   ss = sum of h^2 in float32, in the order below
//   r  = 1 / sqrt(ss / 7168 + eps)                 each step correctly rounded
//   y  = bf16(w * bf16(h * r))                     (y = h without a weight)
//   q, s = the 1x128 quantisation of y
// One 128-thread CTA per token; thread i holds chunks c = 128 j + i (j = 0..6)
// of 8 columns. ss order: each thread sums its 56 squares in column order
// (h^2 of a bf16 value is exact in float32, so an fma equals a multiply and
// add), then an xor-butterfly over the warp (offsets 16, 8, 4, 2, 1), then
// ((w0 + w1) + w2) + w3 over the 4 warps. The CPU restatement follows the same
// order, so the bytes match. HBM-bound: 28,672 B read and 21,728 B written
// per token (plus the 14,336-byte weight, read once from L2).
#include "moe_kernels.h"

namespace moe {

namespace {

constexpr int kQuantWarps = 8;
constexpr int kQuantSteps = kHidden / 256;  // 28 steps of two blocks

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// 1x128 quantisation of 8 consecutive columns held by this lane; the 16 lanes
// of a half warp hold one 128-column block. Returns the 8 e4m3 bytes, and the
// block scale in s.
__device__ __forceinline__ uint2 quant8_1x128(const float (&f)[8], float& s) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
  // max over the 16 lanes of this block (|x| bits order like the values)
  unsigned mb = __float_as_uint(m);
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, off));
  s = fmaxf(__fdiv_rn(__uint_as_float(mb), 448.0f), 1e-12f);
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
  return make_uint2(w0, w1);
}

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
      const float f[8] = {bf16_lo(v[j].x), bf16_hi(v[j].x), bf16_lo(v[j].y), bf16_hi(v[j].y),
                          bf16_lo(v[j].z), bf16_hi(v[j].z), bf16_lo(v[j].w), bf16_hi(v[j].w)};
      float s;
      __stcs(dst + c * 32 + lane, quant8_1x128(f, s));
      if ((lane & 15) == 0) scale[(size_t)(2 * c + (lane >> 4)) * T + t] = s;
    }
  }
}

constexpr int kAnqThreads = 128;
constexpr int kAnqChunks = kHidden / 8 / kAnqThreads;  // 7 chunks of 8 columns per thread
static_assert(kAnqChunks * 8 * kAnqThreads == kHidden, "a token is 7 chunks of 8 columns per thread");

// residual == nullptr: h = x, nothing written back; w == nullptr: y = h.
__global__ void __launch_bounds__(kAnqThreads)
    add_norm_quant_kernel(const uint4* __restrict__ x, uint4* __restrict__ residual, const uint4* __restrict__ w,
                          float eps, int T, uint2* __restrict__ q, float* __restrict__ scale) {
  __shared__ float warp_ss[kAnqThreads / 32];
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint4* xr = x + (size_t)t * (kHidden / 8);
  uint4* rr = residual ? residual + (size_t)t * (kHidden / 8) : nullptr;
  uint4 h[kAnqChunks];
#pragma unroll
  for (int j = 0; j < kAnqChunks; ++j) h[j] = __ldcs(xr + j * kAnqThreads + tid);
  if (rr) {
    uint4 r[kAnqChunks];
#pragma unroll
    for (int j = 0; j < kAnqChunks; ++j) r[j] = __ldcs(rr + j * kAnqThreads + tid);
#pragma unroll
    for (int j = 0; j < kAnqChunks; ++j) {
      const uint32_t a[4] = {h[j].x, h[j].y, h[j].z, h[j].w}, b[4] = {r[j].x, r[j].y, r[j].z, r[j].w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = bf16x2_rn(bf16_lo(b[k]) + bf16_lo(a[k]), bf16_hi(b[k]) + bf16_hi(a[k]));
      h[j] = make_uint4(o[0], o[1], o[2], o[3]);
      __stcs(rr + j * kAnqThreads + tid, h[j]);
    }
  }
  float inv = 1.f;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kAnqChunks; ++j) {
      const uint32_t a[4] = {h[j].x, h[j].y, h[j].z, h[j].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float lo = bf16_lo(a[k]), hi = bf16_hi(a[k]);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) warp_ss[warp] = ss;
    __syncthreads();
    const float tot = ((warp_ss[0] + warp_ss[1]) + warp_ss[2]) + warp_ss[3];
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(kHidden)), eps)));
  }
#pragma unroll
  for (int j = 0; j < kAnqChunks; ++j) {
    const int c = j * kAnqThreads + tid;
    const uint32_t a[4] = {h[j].x, h[j].y, h[j].z, h[j].w};
    float f[8];
    if (w) {
      const uint4 wv = __ldg(w + c);
      const uint32_t b[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t n = bf16x2_rn(bf16_lo(a[k]) * inv, bf16_hi(a[k]) * inv);
        const uint32_t y = bf16x2_rn(bf16_lo(b[k]) * bf16_lo(n), bf16_hi(b[k]) * bf16_hi(n));
        f[2 * k] = bf16_lo(y);
        f[2 * k + 1] = bf16_hi(y);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        f[2 * k] = bf16_lo(a[k]);
        f[2 * k + 1] = bf16_hi(a[k]);
      }
    }
    float sc;
    __stcs(q + (size_t)t * (kHidden / 8) + c, quant8_1x128(f, sc));
    // chunk c holds columns 8c..8c+7, i.e. 128-column block c / 16
    if ((lane & 15) == 0) scale[(size_t)(c >> 4) * T + t] = sc;
  }
}

}  // namespace

cudaError_t launch_quant_rows(const void* x, int T, void* q, float* scale, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int grid = (T + kQuantWarps - 1) / kQuantWarps;
  return launch_k(quant_rows_kernel, dim3(grid), dim3(kQuantWarps * 32), 0, s, false,
                  static_cast<const uint4*>(x), T, static_cast<uint2*>(q), scale);
}

cudaError_t launch_add_norm_quant(const void* x, void* residual, const void* w, float eps, int T, void* q,
                                  float* scale, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(add_norm_quant_kernel, dim3(T), dim3(kAnqThreads), 0, s, false, static_cast<const uint4*>(x),
                  static_cast<uint4*>(residual), static_cast<const uint4*>(w), eps, T, static_cast<uint2*>(q),
                  scale);
}

}  // namespace moe
