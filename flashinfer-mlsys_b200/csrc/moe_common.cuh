// moe_common.cuh — geometry, workspace layout and sm_100a PTX helpers shared by
// the fused FP8 DeepSeek-V3 MoE kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// The kernels use tcgen05, TMEM and TMA: device code exists for sm_100a only.
#if defined(__CUDA_ARCH__) && !defined(__CUDA_ARCH_FEAT_SM100_ALL)
#error "build for sm_100a only: nvcc -gencode arch=compute_100a,code=sm_100a"
#endif

namespace moe {

// ---------------------------------------------------------------------------
// Fixed DeepSeek-V3 geometry (reference moe/ref_moe.py:33-63, kernel.cu:25-33).
// ---------------------------------------------------------------------------
constexpr int kHidden = 7168;                 // H
constexpr int kInter = 2048;                  // I
constexpr int kGemm1N = 2 * kInter;           // 4096 rows of W13 (gate | up)
constexpr int kExperts = 256;                 // global experts
constexpr int kTopK = 8;
constexpr int kGroups = 8;
constexpr int kTopKGroups = 4;
constexpr int kGroupSize = kExperts / kGroups;  // 32
constexpr int kBlk = 128;                     // quantisation block
constexpr int kHiddenBlocks = kHidden / kBlk; // 56
constexpr int kInterBlocks = kInter / kBlk;   // 16
constexpr int kGemm1NBlocks = kGemm1N / kBlk; // 32

// ---------------------------------------------------------------------------
// Tiling of the grouped GEMMs.
//   A operand = token rows (M = 128 per tile, expert-major padded layout)
//   B operand = expert weight rows (N = 256 per tile, two 128-row slabs)
//   K step    = one 128-wide quantisation block per pipeline stage
// GEMM1: N tile = 128 gate rows + the matching 128 up rows -> 16 N tiles,
//        56 K blocks, stage = A (128 token rows) + B (2 x 128 weight rows).
// GEMM2: N tile = 256 rows of W2 -> 28 N tiles, 16 K blocks; the two-term
//        e4m3 intermediate (hi and lo halves of every row, same block scale)
//        is contracted as two A tiles against the same B tile into ONE TMEM
//        partial, so a stage = A_hi + A_lo + B.
// ---------------------------------------------------------------------------
constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kNT1 = kInter / kBlk;           // 16
constexpr int kNT2 = kHidden / kTileN;        // 28
constexpr int kKB1 = kHiddenBlocks;           // 56
constexpr int kKB2 = kInterBlocks;            // 16
constexpr int kInterCols = 2 * kInter;        // 4096 bytes per intermediate row (hi | lo)

constexpr int kStageA = kTileM * kBlk;        // 16 KB of e4m3 (one 128-row A tile)
constexpr int kStageB = kTileN * kBlk;        // 32 KB of e4m3
// kSkinny = 1: calls with at most 64 tokens load 64-row token tiles (8 KB),
// which leaves room for one more stage of weights in flight. kSkinny = 2
// (GEMM1 of calls with at most kTinyMaxRows tokens): 16-row token tiles
// (2 KB) and six stages of weights in flight. The MMA still reads 128 rows;
// the rows past the tile then see unrelated shared memory (inside the ring)
// and only produce accumulator rows that are never stored.
constexpr int kTinyMaxRows = 16;
template <int kMode, int kSkinny = 0>
struct GemmCfg {
  static constexpr int kATiles = (kMode == 1) ? 1 : 2;          // GEMM2: hi and lo
  static constexpr int kARows = kSkinny == 2 ? kTinyMaxRows : (kSkinny ? 64 : kTileM);
  static constexpr int kABytes = kARows * kBlk;                 // bytes loaded (and slot size) per A tile
  static constexpr int kStageBytes = kATiles * kABytes + kStageB;
  static constexpr int kStages = kSkinny == 2 ? 6 : (kSkinny ? ((kMode == 1) ? 5 : 4) : ((kMode == 1) ? 4 : 3));
  static constexpr int kRing = kStages * kStageBytes;
  static constexpr int kNKB = (kMode == 1) ? kKB1 : kKB2;
  static constexpr int kNT = (kMode == 1) ? kNT1 : kNT2;
};
constexpr int kMaxStages = 6;
constexpr int kRingBytes = 204 * 1024;          // >= kRing of every configuration
constexpr int kSkinnyMaxRows = 64;
constexpr int kDecMaxT = 64;                   // largest call served by the fused decode kernel

constexpr int kGemmThreads = 608;             // 19 warps
constexpr int kScaleWarp = 2;                 // warp 2 streams block scales into shared memory
constexpr int kEpiWarp0 = 3;                  // warps 3..18 run the epilogue
constexpr int kEpiWarps = 16;                 // four per TMEM lane quarter, 64 columns each
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kScaleSlots = 8;                // depth of the scale ring (K blocks ahead)

// Split-K of GEMM1 reduces fp32 partial tiles in a bounded scratch area.
constexpr int kMaxSplitMTiles = 32;
// Calls of at most kSkinnyMaxRows tokens, and calls of at most kDirectMaxT
// tokens whose GEMM2 is split along K, combine directly: every GEMM2 partial
// adds its routing-weighted product into a per-token fp32 sum (GEMM2's split-K
// scratch, [kDirectMaxT][7168]), which the finalize kernel casts to the output
// and clears.
constexpr int kDirectMaxT = kMaxSplitMTiles * 128;
__host__ __device__ __forceinline__ bool direct_combine(int split2, int T) {
  return T <= kSkinnyMaxRows || (split2 > 1 && T <= kDirectMaxT);
}

constexpr int kSMs = 148;

// ---------------------------------------------------------------------------
// Per-call plan written by the routing kernel's last CTA, read by the GEMMs.
// ---------------------------------------------------------------------------
struct Plan {
  int total_mtiles;   // sum over local experts of ceil(count / 128)
  int split1;         // K split of GEMM1 (1 = no split)
  int split2;         // K split of GEMM2
  int n_assign;       // number of (token, local expert) pairs
  int mtile_prefix[kExperts + 2];  // first m-tile of each local expert (+ the shared expert, + the end)
  int count[kExperts + 1];         // rows (tokens) of each local expert (+ the shared expert)
};

// Status word bits written by kernels (never trap).
constexpr unsigned kErrTimeout = 1u;

// ---------------------------------------------------------------------------
// PTX helpers (sm_100a).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One try_wait with a suspend-time hint: the thread sleeps in hardware until
// the phase completes or the hint (ns) expires, instead of spinning on issue
// slots the working warps need.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity, uint32_t hint_ns = 1000000u) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and the caller must abort) if the phase has
// not completed within ~limit_ns of wall time.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// 2D TMA tile load global -> shared, completion counted on `bar` (bytes).
// Plain load: every CTA fetches its own tiles.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Four rows y0..y3 of a 2D tensor map whose box is one row high (x: 128
// bytes at column x) into four consecutive 128-byte rows of shared memory;
// the 128-byte swizzle follows the destination address, so row i lands as
// row (dst/128 + i) of its 1024-byte swizzle atom. Plain load (no multicast).
__device__ __forceinline__ void tma_gather4(void* smem_dst, const CUtensorMap* map, int x, int y0, int y1, int y2,
                                            int y3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5, %6}], [%7];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 (5th-generation tensor core, accumulators in TMEM) -----------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> f32, issued by one thread.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp receives row
// (lane base + i), columns [col, col+16). Waits for completion.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms).
// Field layout (sm_100 UMMA descriptor): start address >> 4 in bits [0,14),
// leading byte offset >> 4 in [16,30) (unused for swizzled K-major, set to 1),
// stride byte offset >> 4 in [32,46) (1024 B between 8-row groups),
// descriptor version 1 in [46,48), layout type 2 (SWIZZLE_128B) in [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::f8f6f4: D f32, A e4m3, B e4m3, both
// K-major, shape M x N. Bits: c_format [4,6)=1 (f32), a_format [7,10)=0,
// b_format [10,13)=0, a_major bit 15 = 0, b_major bit 16 = 0,
// N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---- cp.async (per-thread asynchronous global -> shared copies) ------------
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
// Arrive on `bar` once this thread's earlier cp.async copies have landed
// (the barrier's expected count includes this arrival).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---- programmatic dependent launch ---------------------------------------
// Kernels after the first of a call are launched with programmatic stream
// serialisation: they may start while the previous kernel drains, run their
// prologue, and block in griddep_wait() until it has completed and its memory
// is visible. Each kernel releases its dependent only after its own wait, so
// the kernel two steps back has always completed when a kernel starts.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- misc -----------------------------------------------------------------
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// e4m3 conversion of two floats (round to nearest even, saturating).
__device__ __forceinline__ uint16_t f2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %2, %1;\n\tmov.b16 %0, t;\n\t}"
      : "=h"(r)
      : "f"(lo), "f"(hi));
  return r;
}

}  // namespace moe
