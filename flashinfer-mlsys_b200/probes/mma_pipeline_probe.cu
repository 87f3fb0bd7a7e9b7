// Measurement program (not part of the library): raw throughput of the TMA + tcgen05 MMA
// pipeline without epilogue, one-SM tiles (M128 N256) vs CTA-pair tiles
// (cta_group::2, M256 N256, each CTA stages its 128 A rows and half of B).
// Accumulators are never read: the MMA alternates two TMEM buffers freely.
// It bounds what the GEMM kernels' TMA + MMA pipeline can reach on this part
// (random e4m3 operands, 16384 x 4096 x 7168, 148 CTAs / 74 CTA pairs).
//
// Build and run (one B200):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -I include \
//        -o mma_pipeline_probe flashinfer-mlsys_b200/probes/mma_pipeline_probe.cu
//   ./mma_pipeline_probe
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdint>
#include <vector>
#include "../csrc/moe_common.cuh"
using namespace moe;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn enc() {
  void* p = nullptr; cudaDriverEntryPointQueryResult q;
  cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
  return (EncodeTiledFn)p;
}
static bool make_map(CUtensorMap* m, void* base, uint64_t cols, uint64_t rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  return enc()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---- pair helpers ----
__device__ __forceinline__ uint32_t ctarank() { uint32_t r; asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r)); return r; }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cl_addr(const void* p, uint32_t rank) {
  uint32_t r; asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank)); return r;
}
__device__ __forceinline__ void tma_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cl) {
  asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cl) : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst, uint32_t n) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(n) : "memory");
}
__device__ __forceinline__ void tmem_relinq2() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_dealloc2(uint32_t t, uint32_t n) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(t), "r"(n) : "memory");
}
__device__ __forceinline__ void mma2(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
               ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
// arrive once on the barrier at shared::cluster address `bar_cl` when this thread's prior pair MMAs complete
__device__ __forceinline__ void commit2(uint32_t bar_cl) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cl) : "memory");
}

struct Args {
  int m_tiles, n_tiles, nkb;  // m tiles of 128 rows, n tiles of 256 rows, K blocks of 128
  int stages;
  unsigned* err;
};
constexpr uint64_t kLim = 2000000000ull;

template <int kPair>
__global__ void __launch_bounds__(64, 1) probe_kernel(const __grid_constant__ CUtensorMap ma,
                                                      const __grid_constant__ CUtensorMap mb, Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full[8], empty[8], done;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = kPair ? ctarank() : 0;
  constexpr int kA = 128 * 128;                       // A tile bytes
  constexpr int kB = kPair ? 128 * 128 : 256 * 128;   // B bytes this CTA stages
  constexpr int kStage = kA + kB;
  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    if (kPair) { tmem_alloc2(&tbase, 512); tmem_relinq2(); }
    else { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  }
  tc_fence_before();
  __syncthreads();
  if (kPair) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = tbase;
  const int units = kPair ? (a.m_tiles / 2) * a.n_tiles : a.m_tiles * a.n_tiles;
  const int u0 = kPair ? blockIdx.x / 2 : blockIdx.x;
  const int ustep = kPair ? gridDim.x / 2 : gridDim.x;
  if (warp == 0 && lane == 0) {
    uint32_t it = 0;
    bool ok = true;
    for (int u = u0; u < units && ok; u += ustep) {
      const int n = u % a.n_tiles, mt = u / a.n_tiles;
      const int arow = kPair ? (2 * mt + rank) * 128 : mt * 128;
      for (int kb = 0; kb < a.nkb; ++kb, ++it) {
        const int s = it % a.stages;
        if (!mbar_wait_bounded(&empty[s], ((it / a.stages) & 1u) ^ 1u, kLim)) { atomicOr(a.err, 1u); ok = false; break; }
        uint8_t* sa = smem + s * kStage;
        if (kPair) {
          const uint32_t fb = cl_addr(&full[s], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kStage);
          tma_pair(sa, &ma, kb * 128, arow, fb);
          tma_pair(sa + kA, &mb, kb * 128, n * 256 + rank * 128, fb);
        } else {
          mbar_arrive_expect_tx(&full[s], kStage);
          tma_load_2d(sa, &ma, kb * 128, arow, &full[s]);
          tma_load_2d(sa + kA, &mb, kb * 128, n * 256, &full[s]);
          tma_load_2d(sa + kA + 128 * 128, &mb, kb * 128, n * 256 + 128, &full[s]);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    constexpr uint32_t idesc = idesc_e4m3_f32(kPair ? 256 : 128, 256);
    uint32_t it = 0;
    bool any = false, ok = true;
    for (int u = u0; u < units && ok; u += ustep) {
      for (int kb = 0; kb < a.nkb; ++kb, ++it) {
        const int s = it % a.stages;
        if (!mbar_wait_bounded(&full[s], (it / a.stages) & 1u, kLim)) { atomicOr(a.err, 2u); ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kStage);
        const uint64_t da = smem_desc_sw128(sa), db = smem_desc_sw128(sa + kA);
        const uint32_t d = tmem + (it & 1u) * 256;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (kPair) mma2(d, da + 2 * k, db + 2 * k, idesc, k > 0);
          else mma_f8f6f4(d, da + 2 * k, db + 2 * k, idesc, k > 0);
        }
        any = true;
        if (kPair) { commit2(cl_addr(&empty[s], 0)); commit2(cl_addr(&empty[s], 1)); }
        else mma_commit(&empty[s]);
      }
    }
    if (any) {
      if (kPair) commit2(cl_addr(&done, 0)); else mma_commit(&done);
      if (!mbar_wait_bounded(&done, 0, kLim)) atomicOr(a.err, 4u);
    }
  }
  tc_fence_before();
  __syncthreads();
  // the leader's MMAs read the peer's shared memory: neither leaves early
  if (kPair) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if (kPair) tmem_dealloc2(tmem, 512); else tmem_dealloc(tmem, 512);
  }
}

__global__ void fill_random(uint8_t* p, size_t n, uint32_t seed) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    uint32_t h = (uint32_t)i * 2654435761u ^ seed;
    h ^= h >> 13; h *= 0x5bd1e995u; h ^= h >> 15;
    p[i] = (uint8_t)(h & 0xF7u);  // bit 3 clear: never the NaN codes 0x7f / 0xff
  }
}

int main() {
  const int M = 16384, N = 4096, K = 7168;
  uint8_t *A, *B;
  unsigned* err;
  cudaMalloc(&A, (size_t)M * K);
  cudaMalloc(&B, (size_t)N * K);
  cudaMalloc(&err, 4);
  fill_random<<<1184, 256>>>(A, (size_t)M * K, 1u);
  fill_random<<<1184, 256>>>(B, (size_t)N * K, 2u);
  cudaMemset(err, 0, 4);
  CUtensorMap ma, mb;
  if (!make_map(&ma, A, K, M) || !make_map(&mb, B, K, N)) { printf("map failed\n"); return 1; }
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  const size_t smem = 192 * 1024 + 1024;
  cudaFuncSetAttribute(probe_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaFuncSetAttribute(probe_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0); cudaEventCreate(&e1);
  const double flops = 2.0 * M * N * K;
  for (int pair = 0; pair < 2; ++pair) {
    Args a{M / 128, N / 256, K / 128, pair ? 6 : 4, err};
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(sms - (sms % 2));
    cfg.blockDim = dim3(64);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = pair ? 2 : 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    float best = 1e9, last = 0.f;
    for (int rep = 0; rep < 40; ++rep) {
      cudaEventRecord(e0);
      cudaError_t le = pair ? cudaLaunchKernelEx(&cfg, probe_kernel<1>, ma, mb, a)
                            : cudaLaunchKernelEx(&cfg, probe_kernel<0>, ma, mb, a);
      cudaEventRecord(e1);
      cudaError_t se = cudaEventSynchronize(e1);
      if (le != cudaSuccess || se != cudaSuccess) {
        printf("pair=%d launch %s sync %s\n", pair, cudaGetErrorString(le), cudaGetErrorString(se));
        return 1;
      }
      float ms; cudaEventElapsedTime(&ms, e0, e1);
      if (rep >= 2 && ms < best) best = ms;
      if (rep >= 30) last += ms / 10.f;
    }
    unsigned h = 0;
    cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
    printf("%s: best %.1f us %.0f TFLOP/s | last-10 mean %.1f us %.0f TFLOP/s  err=%u\n",
           pair ? "pair M256xN256 (cta_group::2)" : "one-SM M128xN256", best * 1e3, flops / (best * 1e-3) / 1e12,
           last * 1e3, flops / (last * 1e-3) / 1e12, h);
  }
  return 0;
}
