// moe_ep.cu — the token exchange around the expert computation when experts
// are sharded over GPUs (expert parallelism): packing the rows a rank sends,
// unpacking what it receives, and the per-token combine of the partial
// outputs that come back. The collectives themselves are NCCL all-to-alls
// issued by the host (flashinfer-mlsys_b200/ep.py).
//
// Packed row (7456 bytes, 16-byte aligned rows):
//   [0, 7168)     e4m3 hidden row
//   [7168, 7392)  56 f32 block scales of the row
//   [7392, 7424)  8 int32 global expert ids
//   [7424, 7456)  8 f32 routing weights
// All three kernels are memory copies / sums: HBM-bound.
#include "moe_kernels.h"

namespace moe {

namespace {

constexpr int kRowBytes = kHidden + kHiddenBlocks * 4 + kTopK * 4 + kTopK * 4;  // 7456
static_assert(kRowBytes % 16 == 0, "packed rows are copied in 16-byte chunks");
constexpr int kEpWarps = 8;

// One warp per sent row: row i of the send buffer is token idx[i].
__global__ void __launch_bounds__(kEpWarps * 32)
    ep_pack_kernel(const uint8_t* __restrict__ hidden, const float* __restrict__ hidden_scale,
                   const int32_t* __restrict__ ids, const float* __restrict__ w, int T,
                   const int64_t* __restrict__ idx, int S, uint8_t* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kEpWarps + warp;
  if (i >= S) return;
  const int64_t t = idx[i];
  const uint4* src = reinterpret_cast<const uint4*>(hidden + t * kHidden);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)i * kRowBytes);
#pragma unroll 7
  for (int j = lane; j < kHidden / 16; j += 32) dst[j] = __ldg(src + j);
  float* ds = reinterpret_cast<float*>(out + (size_t)i * kRowBytes + kHidden);
  for (int b = lane; b < kHiddenBlocks; b += 32) ds[b] = __ldg(hidden_scale + (size_t)b * T + t);
  if (lane < kTopK) {
    int32_t* di = reinterpret_cast<int32_t*>(out + (size_t)i * kRowBytes + kHidden + kHiddenBlocks * 4);
    di[lane] = __ldg(ids + t * kTopK + lane);
    di[kTopK + lane] = __float_as_int(__ldg(w + t * kTopK + lane));
  }
}

// One warp per received row: split it into the expert entry's input arrays.
__global__ void __launch_bounds__(kEpWarps * 32)
    ep_unpack_kernel(const uint8_t* __restrict__ in, int R, uint8_t* __restrict__ hidden,
                     float* __restrict__ hidden_scale, int32_t* __restrict__ ids, float* __restrict__ w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kEpWarps + warp;
  if (r >= R) return;
  const uint4* src = reinterpret_cast<const uint4*>(in + (size_t)r * kRowBytes);
  uint4* dst = reinterpret_cast<uint4*>(hidden + (size_t)r * kHidden);
#pragma unroll 7
  for (int j = lane; j < kHidden / 16; j += 32) dst[j] = __ldcs(src + j);
  const float* ss = reinterpret_cast<const float*>(in + (size_t)r * kRowBytes + kHidden);
  for (int b = lane; b < kHiddenBlocks; b += 32) hidden_scale[(size_t)b * R + r] = ss[b];
  if (lane < kTopK) {
    const int32_t* si = reinterpret_cast<const int32_t*>(in + (size_t)r * kRowBytes + kHidden + kHiddenBlocks * 4);
    ids[(size_t)r * kTopK + lane] = si[lane];
    w[(size_t)r * kTopK + lane] = __int_as_float(si[kTopK + lane]);
  }
}

// out[t, :] = sum over ranks q = 0..world-1 (ascending, i.e. ascending expert
// id blocks) of back[row_of[t][q], :] in fp32, cast once to bf16; -1 = the
// token sent nothing to rank q. Eight columns per thread.
__global__ void __launch_bounds__(256)
    ep_combine_kernel(const __nv_bfloat16* __restrict__ back, const int32_t* __restrict__ row_of, int T, int world,
                      __nv_bfloat16* __restrict__ out) {
  constexpr int kC8 = kHidden / 8;
  const int64_t n = (int64_t)T * kC8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(i / kC8);
    const int c8 = static_cast<int>(i - (int64_t)t * kC8);
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < world; ++q) {
      const int r = __ldg(row_of + (size_t)t * world + q);
      if (r < 0) continue;
      const uint4 v = __ldcs(reinterpret_cast<const uint4*>(back + (size_t)r * kHidden) + c8);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s[2 * k] += __uint_as_float(u[k] << 16);
        s[2 * k + 1] += __uint_as_float(u[k] & 0xFFFF0000u);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 b = __floats2bfloat162_rn(s[2 * k], s[2 * k + 1]);
      o[k] = *reinterpret_cast<uint32_t*>(&b);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The dispatch plan of one layer call, in one CTA. Rank q owns experts
// [q*e_local, (q+1)*e_local). For every q, the tokens with at least one
// expert there, in ascending token order, concatenated rank after rank
// (send_idx), the count per rank (send_counts) and row_of[t][q] = the row of
// token t in that concatenation (-1: nothing sent to q). Pass 1 counts with
// shared-memory atomics; pass 2 places 1024 tokens at a time with a ballot
// scan per rank, so positions ascend with the token index.
constexpr int kPlanThreads = 1024;
__global__ void __launch_bounds__(kPlanThreads)
    ep_plan_kernel(const int32_t* __restrict__ ids, int T, int world, int64_t* __restrict__ send_idx,
                   int64_t* __restrict__ send_counts, int32_t* __restrict__ row_of) {
  __shared__ int cnt[64], off[64], running[64];
  __shared__ int warp_tot[kPlanThreads / 32], warp_pre[kPlanThreads / 32], chunk_tot;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int e_local = kExperts / world;
  if (tid < world) cnt[tid] = running[tid] = 0;
  __syncthreads();
  auto dest_mask = [&](int t) -> uint64_t {
    uint64_t m = 0;
    if (t < T) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        int q = __ldg(ids + (size_t)t * kTopK + k) / e_local;
        q = q < 0 ? 0 : (q >= world ? world - 1 : q);
        m |= 1ull << q;
      }
    }
    return m;
  };
  for (int t = tid; t < T; t += kPlanThreads) {
    uint64_t m = dest_mask(t);
    while (m) {
      const int q = __ffsll(static_cast<long long>(m)) - 1;
      m &= m - 1;
      atomicAdd(&cnt[q], 1);
    }
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0;
    for (int q = 0; q < world; ++q) {
      off[q] = o;
      o += cnt[q];
      send_counts[q] = cnt[q];
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int base = 0; base < T; base += kPlanThreads) {
    const int t = base + tid;
    const uint64_t m = dest_mask(t);
    for (int q = 0; q < world; ++q) {
      const bool f = (m >> q) & 1ull;
      const unsigned bal = __ballot_sync(0xffffffffu, f);
      if (lane == 0) warp_tot[warp] = __popc(bal);
      __syncthreads();
      if (warp == 0) {
        const int v = warp_tot[lane];
        int incl = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, d);
          if (lane >= d) incl += y;
        }
        warp_pre[lane] = incl - v;
        if (lane == 31) chunk_tot = incl;
      }
      __syncthreads();
      if (t < T) {
        int r = -1;
        if (f) {
          r = off[q] + running[q] + warp_pre[warp] + __popc(bal & lt);
          send_idx[r] = t;
        }
        row_of[(size_t)t * world + q] = r;
      }
      __syncthreads();
      if (tid == 0) running[q] += chunk_tot;
    }
  }
}

}  // namespace

cudaError_t launch_ep_plan(const int32_t* ids, int T, int world, int64_t* send_idx, int64_t* send_counts,
                           int32_t* row_of, cudaStream_t s) {
  return launch_k(ep_plan_kernel, dim3(1), dim3(kPlanThreads), 0, s, false, ids, T, world, send_idx, send_counts,
                  row_of);
}

cudaError_t launch_ep_pack(const void* hidden, const float* hidden_scale, const int32_t* ids, const float* w, int T,
                           const int64_t* idx, int S, void* out, cudaStream_t s) {
  if (S <= 0) return cudaSuccess;
  return launch_k(ep_pack_kernel, dim3((S + kEpWarps - 1) / kEpWarps), dim3(kEpWarps * 32), 0, s, false,
                  static_cast<const uint8_t*>(hidden), hidden_scale, ids, w, T, idx, S, static_cast<uint8_t*>(out));
}

cudaError_t launch_ep_unpack(const void* in, int R, void* hidden, float* hidden_scale, int32_t* ids, float* w,
                             cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  return launch_k(ep_unpack_kernel, dim3((R + kEpWarps - 1) / kEpWarps), dim3(kEpWarps * 32), 0, s, false,
                  static_cast<const uint8_t*>(in), R, static_cast<uint8_t*>(hidden), hidden_scale, ids, w);
}

cudaError_t launch_ep_combine(const void* back, const int32_t* row_of, int T, int world, void* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int64_t n = (int64_t)T * (kHidden / 8);
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  return launch_k(ep_combine_kernel, dim3((unsigned)blocks), dim3(256), 0, s, false,
                  static_cast<const __nv_bfloat16*>(back), row_of, T, world, static_cast<__nv_bfloat16*>(out));
}

}  // namespace moe
