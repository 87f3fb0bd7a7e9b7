// moe_decode.cu — the whole MoE layer in one persistent kernel for decode-size
// calls (1 <= T <= 64 tokens).
//
// At decode sizes the layer streams the FP8 weights of the touched experts
// from HBM and does almost no arithmetic per byte. The multi-kernel pipeline
// pays a routing kernel, a permutation kernel, two GEMM kernels with their
// tails and a combine kernel for that; here one cooperative launch of one CTA
// per SM does all of it:
//
//  1. Routing (reference moe/ref_moe.py:95-126): every CTA routes all T tokens
//     itself (a few microseconds, identical results in every CTA), so no CTA
//     waits for another before it starts streaming weights. The touched local
//     experts get "slots" in ascending expert id.
//  2. GEMM1 (ref_moe.py:153-159) with swapped operands: the weight rows are the
//     MMA's M = 128 side and all T tokens (padded to 64 with TMA zero fill) are
//     its N side, read straight from the caller's hidden_states; no permuted
//     copy of the activations exists. A work unit is (slot, 128 intermediate
//     columns): the gate rows and the up rows of W13 against the tokens, 56 K
//     blocks. The K blocks of all units are dealt to the CTAs as equal
//     contiguous ranges ("stream-K"), so every SM streams the same number of
//     weight bytes whatever the number of touched experts. A unit split between
//     CTAs meets in fp32 scratch; the CTA that completes it runs SwiGLU and the
//     two-term e4m3 quantisation (hi + lo, one scale per token and 128
//     columns) and publishes the slot's progress counter.
//  3. GEMM2 and the combine (ref_moe.py:162-167), also swapped: a work unit
//     is one 256-column slice of the output (two 128-row W2 tiles) over all
//     touched experts, 16 K blocks (hi and lo intermediate tiles) per expert.
//     The routing weight of (token, expert) is folded into each K block's
//     promotion factor, so the sum over experts builds up in the same
//     registers. Its K blocks are dealt the same way; a CTA may stream its W2
//     tiles into shared memory while GEMM1 still runs elsewhere and only loads
//     an expert's intermediate once that expert's 16 GEMM1 units are
//     published. The CTA that completes a slice adds its pieces in CTA order
//     (deterministic), casts once to bf16 and writes the output.
//
// Warp roles (608 threads): warp 0 streams weight tiles (TMA), warp 1 owns
// TMEM and issues tcgen05.mma (M128 N64 K32, e4m3 x e4m3 -> f32), warp 2
// loads the token-side tiles (TMA) and the block scales, warps 3-18 promote
// the per-K-block partials with a_scale[token] * w_scale and run the unit
// epilogues. Every wait is bounded; a CTA that gives up sets the status word.
#include "moe_kernels.h"
#include "moe_routing.cuh"

namespace moe {

namespace {

constexpr int kDecStages = 4;
constexpr int kDecW = 2 * kStageA;                 // two 128x128 weight tiles per stage
constexpr int kDecX = 2 * kDecMaxT * kBlk;         // GEMM1: one 64x128 token tile; GEMM2: hi + lo tiles
constexpr int kDecStage = kDecW + kDecX;           // 48 KB
constexpr int kDecRing = kDecStages * kDecStage;   // 192 KB
constexpr int kDecBufs = 4;                        // TMEM partial buffers of 128 columns
constexpr int kDecBufCols = 2 * kDecMaxT;
constexpr int kDecScaleSlots = 8;
constexpr int kDecU1 = kNT1;                       // GEMM1 units per slot (128 intermediate columns)
constexpr int kDecU2 = kNT2;                       // GEMM2 units (256 output columns, all slots)
constexpr int kDecKB1 = kKB1;                      // 56
constexpr int kDecKB2 = kKB2;                      // 16
constexpr uint64_t kDecWaitNs = 2000000000ull;

static_assert(kDecBufs * kDecBufCols <= 512, "TMEM buffers");
static_assert(kDecStages <= kDecBufs, "stage index doubles as nothing else");

struct __align__(16) DecScaleSlot {
  float a[kDecMaxT];   // per token column: hidden_scale (GEMM1) or intermediate scale (GEMM2)
  float wr[kDecMaxT];  // GEMM2: routing weight of (token, this K block's expert), 0 if not routed
  float w[4];          // weight-block scales: GEMM1 {gate, up}; GEMM2 {tile 0, tile 1}
};

struct __align__(16) DecCtl {
  DecScaleSlot scales[kDecScaleSlots];
  uint64_t sfull[kDecScaleSlots];
  uint64_t sempty[kDecScaleSlots];
  uint64_t full[kDecStages];
  uint64_t empty[kDecStages];
  uint64_t tfull[kDecBufs];
  uint64_t tempty[kDecBufs];
  uint64_t mma_done;
  uint64_t epi_bar;
  uint32_t tmem_base;
  int abort_flag;
  int flag;
  int n_slots;
  int slot_exp[kExperts];          // local expert of each slot
  int slot_of[kExperts];           // slot of each local expert, -1 if untouched
  int hist[kExperts];              // tokens per local expert
  int warp_cnt[8];
  int tok_slot[kDecMaxT][kTopK];   // slot of each (token, k), -1 if not local
  float tok_w[kDecMaxT][kTopK];
  float amax[4][kDecMaxT];
};

__device__ __forceinline__ void dec_abort(DecCtl* c, unsigned* status) {
  atomicOr(status, kErrTimeout);
  *reinterpret_cast<volatile int*>(&c->abort_flag) = 1;
}
__device__ __forceinline__ bool dec_aborted(DecCtl* c) {
  return *reinterpret_cast<volatile int*>(&c->abort_flag) != 0;
}

// bounded barrier among the 16 epilogue warps (an mbarrier, so it can give up)
struct DecEpiSync {
  uint32_t phase = 0;
  __device__ __forceinline__ bool sync(DecCtl* c, unsigned* status) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&c->epi_bar);
    bool ok = mbar_wait_bounded(&c->epi_bar, phase, kDecWaitNs);
    phase ^= 1u;
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) dec_abort(c, status);
    return ok;
  }
};

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// order this thread's generic-proxy global accesses with async-proxy (TMA) ones
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// First K block of CTA c in a range of `total` K blocks dealt over `g` CTAs.
__device__ __forceinline__ int range_begin(int c, int total, int g) {
  return static_cast<int>((static_cast<long long>(c) * total) / g);
}
// CTA whose range holds K block k.
__device__ __forceinline__ int range_owner(int k, int total, int g) {
  return static_cast<int>(((static_cast<long long>(k) + 1) * g - 1) / total);
}

// Walks the CTA's K blocks in order: its GEMM1 range, then its GEMM2 range,
// split into segments (runs of K blocks inside one unit).
struct Walk {
  int r1b, r1e, r2b, r2e;  // [begin, end) of the two ranges
  int ph, k;               // phase (0: GEMM1, 1: GEMM2, 2: done) and next K block
  int nkb2;                // K blocks of a GEMM2 unit (16 per slot)
  __device__ __forceinline__ void init(int c, int g, int n_slots) {
    nkb2 = n_slots * kDecKB2;
    const int t1 = n_slots * kDecU1 * kDecKB1, t2 = kDecU2 * nkb2;
    r1b = range_begin(c, t1, g);
    r1e = range_begin(c + 1, t1, g);
    r2b = range_begin(c, t2, g);
    r2e = range_begin(c + 1, t2, g);
    ph = 0;
    k = r1b;
    if (k >= r1e) {
      ph = 1;
      k = r2b;
      if (k >= r2e) ph = 2;
    }
  }
  // next segment: unit u, K blocks [kb0, kb1) of it
  __device__ __forceinline__ bool next(int& p, int& u, int& kb0, int& kb1) {
    if (ph == 2) return false;
    const int nkb = ph == 0 ? kDecKB1 : nkb2;
    const int end = ph == 0 ? r1e : r2e;
    p = ph;
    u = k / nkb;
    kb0 = k - u * nkb;
    kb1 = min(nkb, kb0 + (end - k));
    k += kb1 - kb0;
    if (k >= end) {
      if (ph == 0) {
        ph = 1;
        k = r2b;
        if (k >= r2e) ph = 2;
      } else {
        ph = 2;
      }
    }
    return true;
  }
};

struct DecArgs {
  const float* logits;        // [T][256]
  const uint16_t* bias;       // bf16 [256]
  const float* hidden_scale;  // [56][T]
  const float* w13_scale;     // [E_l][32][56]
  const float* w2_scale;      // [E_l][56][16]
  int T;
  int offset;
  int e_local;
  float scale;
  uint8_t* inter;             // [slots][64][4096] hi | lo
  float* inter_scale;         // [slots][16][64]
  float* g1_part;             // [grid][2][64][256] partial sums of the pieces of split GEMM1 units
  int* g1_cnt;                // [grid] K blocks accumulated per split unit (kept zero)
  int* ready;                 // [slots] GEMM1 units published per slot (reset at kernel end)
  float* g2_part;             // [grid][2][64][256] partial sums of the pieces of GEMM2 units
  int* h_cnt;                 // [28] K blocks accumulated per GEMM2 unit (kept zero)
  int* done;                  // CTAs finished (kept zero)
  const float* zero;          // one 0.0f in device memory
  __nv_bfloat16* out;         // [T][7168]
  int32_t* user_ids;          // optional [T][8]
  float* user_w;              // optional [T][8]
  int32_t* user_counts;       // optional [E_l]
  unsigned* status;
};

// acc[i] += (a[i] * w) * v[i] as packed f32x2 operations (each component
// rounds like the scalar fmul + fmaf)
__device__ __forceinline__ void dec_promote16(float (&acc)[16], const float (&a)[16], float w, const float (&v)[16]) {
  const float2 ww = make_float2(w, w);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const float2 f = __fmul2_rn(make_float2(a[i], a[i + 1]), ww);
    const float2 r = __ffma2_rn(f, make_float2(v[i], v[i + 1]), make_float2(acc[i], acc[i + 1]));
    acc[i] = r.x;
    acc[i + 1] = r.y;
  }
}

// x * sigmoid(x) with the fast exponential and reciprocal intrinsics (relative
// error ~1e-7, far below the e4m3 quantisation that follows)
__device__ __forceinline__ float dec_silu(float x) { return x * __frcp_rn(1.0f + __expf(-x)); }

__device__ __forceinline__ float dec_e4m3_to_f32(uint32_t b) {
  uint32_t h2;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(h2) : "r"(b));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_decode_kernel(const __grid_constant__ CUtensorMap map_w13, const __grid_constant__ CUtensorMap map_w2,
                      const __grid_constant__ CUtensorMap map_x1, const __grid_constant__ CUtensorMap map_x2,
                      DecArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  DecCtl* ctl = reinterpret_cast<DecCtl*>(smem + kDecRing);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int T = p.T, E_l = p.e_local;
  const int G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < kDecBufs; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], kEpiWarps);
    }
    for (int j = 0; j < kDecScaleSlots; ++j) {
      mbar_init(&ctl->sfull[j], 33);  // 32 cp.async arrivals + the routing weights' writer
      mbar_init(&ctl->sempty[j], kEpiWarps);
    }
    mbar_init(&ctl->mma_done, 1);
    mbar_init(&ctl->epi_bar, kEpiWarps);
    ctl->abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&map_w13);
    prefetch_tensormap(&map_w2);
    prefetch_tensormap(&map_x1);
    prefetch_tensormap(&map_x2);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  for (int e = tid; e < kExperts; e += blockDim.x) {
    ctl->hist[e] = 0;
    ctl->slot_of[e] = -1;
  }
  __syncthreads();

  // ---------------- 1. routing of all T tokens (every CTA) ----------------
  // Each warp first loads the logits of all its tokens (at most
  // kRouteTokPerWarp), so their memory latencies overlap, then routes them.
  const int nwarps = blockDim.x >> 5;
  constexpr int kRouteTokPerWarp = (kDecMaxT + kGemmThreads / 32 - 1) / (kGemmThreads / 32);
  float xs[kRouteTokPerWarp][8];
  const uint4 braw = route_load_bias(p.bias, lane);
#pragma unroll
  for (int j = 0; j < kRouteTokPerWarp; ++j) {
    const int t = warp + j * nwarps;
    if (t < T) route_load_warp(p.logits + (size_t)t * kExperts, lane, xs[j]);
  }
#pragma unroll
  for (int j = 0; j < kRouteTokPerWarp; ++j) {
    const int t = warp + j * nwarps;
    if (t >= T) break;
    int id = -1;
    float w = 0.f;
    route_compute_warp(xs[j], braw, p.scale, lane, id, w);
    if (lane < kTopK) {
      const int le = id - p.offset;
      const bool local = le >= 0 && le < E_l;
      ctl->tok_slot[t][lane] = local ? le : -1;  // local expert for now, slot below
      ctl->tok_w[t][lane] = w;
      if (local) atomicAdd(&ctl->hist[le], 1);
      if (blockIdx.x == 0) {
        if (p.user_ids) p.user_ids[(size_t)t * kTopK + lane] = id;
        if (p.user_w) p.user_w[(size_t)t * kTopK + lane] = w;
      }
    }
  }
  __syncthreads();
  // slots: touched local experts in ascending id (warps 0..7 cover 256 experts)
  if (warp < 8) {
    const int e = warp * 32 + lane;
    const bool used = e < E_l && ctl->hist[e] > 0;
    const unsigned m = __ballot_sync(0xffffffffu, used);
    if (lane == 0) ctl->warp_cnt[warp] = __popc(m);
    if (blockIdx.x == 0 && p.user_counts && e < E_l) p.user_counts[e] = ctl->hist[e];
  }
  __syncthreads();
  if (warp < 8) {
    const int e = warp * 32 + lane;
    const bool used = e < E_l && ctl->hist[e] > 0;
    const unsigned m = __ballot_sync(0xffffffffu, used);
    int base = 0;
    for (int w = 0; w < warp; ++w) base += ctl->warp_cnt[w];
    if (used) {
      const int s = base + __popc(m & ((1u << lane) - 1u));
      ctl->slot_of[e] = s;
      ctl->slot_exp[s] = e;
    }
    if (warp == 7 && lane == 0) ctl->n_slots = base + __popc(m);
  }
  __syncthreads();
  for (int i = tid; i < T * kTopK; i += blockDim.x) {
    const int t = i / kTopK, k = i % kTopK;
    const int le = ctl->tok_slot[t][k];
    ctl->tok_slot[t][k] = le >= 0 ? ctl->slot_of[le] : -1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const int n_slots = ctl->n_slots;
  const uint32_t tmem = ctl->tmem_base;

  if (n_slots == 0) {
    // no token uses a local expert: the output is zero
    const int64_t n8 = (int64_t)T * kHidden / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < n8; i += (int64_t)G * blockDim.x)
      reinterpret_cast<uint4*>(p.out)[i] = make_uint4(0u, 0u, 0u, 0u);
  } else if (warp == 0) {
    // ======================= weight producer =======================
    if (lane == 0) {
      Walk wk;
      wk.init(blockIdx.x, G, n_slots);
      int ph, u, kb0, kb1;
      uint32_t it = 0;
      bool ok = true;
      while (ok && wk.next(ph, u, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kDecStages;
          if (!mbar_wait_bounded(&ctl->empty[s], ((it / kDecStages) & 1u) ^ 1u, kDecWaitNs) || dec_aborted(ctl)) {
            if (!dec_aborted(ctl)) dec_abort(ctl, p.status);
            ok = false;
            break;
          }
          uint8_t* sw = ring + s * kDecStage;
          if (ph == 0) {
            const int e = ctl->slot_exp[u / kDecU1], n = u % kDecU1;
            mbar_arrive_expect_tx(&ctl->full[s], kDecW + kDecMaxT * kBlk);
            tma_load_2d(sw, &map_w13, kb * kBlk, e * kGemm1N + n * kBlk, &ctl->full[s]);
            tma_load_2d(sw + kStageA, &map_w13, kb * kBlk, e * kGemm1N + kInter + n * kBlk, &ctl->full[s]);
          } else {
            const int e = ctl->slot_exp[kb / kDecKB2], kb2 = kb % kDecKB2, h2 = u;
            mbar_arrive_expect_tx(&ctl->full[s], kDecW + 2 * kDecMaxT * kBlk);
            tma_load_2d(sw, &map_w2, kb2 * kBlk, e * kHidden + h2 * kTileN, &ctl->full[s]);
            tma_load_2d(sw + kStageA, &map_w2, kb2 * kBlk, e * kHidden + h2 * kTileN + kBlk, &ctl->full[s]);
          }
        }
      }
      if (!ok) {
        for (uint32_t j = (it > (uint32_t)kDecStages ? it - kDecStages : 0); j < it; ++j)
          mbar_wait_bounded(&ctl->full[j % kDecStages], (j / kDecStages) & 1u, kDecWaitNs);
      }
    }
  } else if (warp == 2) {
    // ============ token-side tiles (TMA), block scales and routing weights ============
    Walk wk;
    wk.init(blockIdx.x, G, n_slots);
    int ph, u, kb0, kb1;
    uint32_t it = 0;
    int ready_slot = -1, wr_slot = -1;
    float wr0 = 0.f, wr1 = 0.f;  // routing weights of tokens lane and lane + 32 for wr_slot
    bool ok = true;
    while (ok && wk.next(ph, u, kb0, kb1)) {
      for (int kbu = kb0; kbu < kb1; ++kbu, ++it) {
        // GEMM1: unit (slot, n), K block kbu; GEMM2: unit h2, K block kbu of slot kbu / 16
        const int slot = ph == 0 ? u / kDecU1 : kbu / kDecKB2;
        const int kb = ph == 0 ? kbu : kbu % kDecKB2;
        const int e = ctl->slot_exp[slot];
        if (ph == 1 && slot != ready_slot) {
          // the slot's intermediate is complete once its 16 GEMM1 units are published
          bool got = false;
          const uint64_t t0 = global_timer_ns();
          while (true) {
            if (ld_acquire(p.ready + slot) >= kDecU1) { got = true; break; }
            if (dec_aborted(ctl) || global_timer_ns() - t0 > kDecWaitNs) break;
            __nanosleep(64);
          }
          got = __all_sync(0xffffffffu, got);
          if (!got) {
            if (lane == 0 && !dec_aborted(ctl)) dec_abort(ctl, p.status);
            ok = false;
            break;
          }
          fence_proxy_async_global();
          ready_slot = slot;
        }
        if (ph == 1 && slot != wr_slot) {
          wr0 = wr1 = 0.f;
#pragma unroll
          for (int k = 0; k < kTopK; ++k) {
            if (lane < T && ctl->tok_slot[lane][k] == slot) wr0 = ctl->tok_w[lane][k];
            if (lane + 32 < T && ctl->tok_slot[lane + 32][k] == slot) wr1 = ctl->tok_w[lane + 32][k];
          }
          wr_slot = slot;
        }
        // token-side tile(s) of this K block
        const int s = it % kDecStages;
        if (lane == 0) {
          if (!mbar_wait_bounded(&ctl->empty[s], ((it / kDecStages) & 1u) ^ 1u, kDecWaitNs)) {
            dec_abort(ctl, p.status);
          } else {
            uint8_t* sx = ring + s * kDecStage + kDecW;
            if (ph == 0) {
              tma_load_2d(sx, &map_x1, kb * kBlk, 0, &ctl->full[s]);
            } else {
              tma_load_2d(sx, &map_x2, kb * kBlk, slot * kDecMaxT, &ctl->full[s]);
              tma_load_2d(sx + kDecMaxT * kBlk, &map_x2, kInter + kb * kBlk, slot * kDecMaxT, &ctl->full[s]);
            }
          }
        }
        // scales of this K block
        const int j = it % kDecScaleSlots;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&ctl->sempty[j], ((it / kDecScaleSlots) & 1u) ^ 1u,
                                                       kDecWaitNs)) || dec_aborted(ctl)) {
          if (lane == 0 && !dec_aborted(ctl)) dec_abort(ctl, p.status);
          ok = false;
          break;
        }
        DecScaleSlot* sl = &ctl->scales[j];
        if (ph == 0) {
          const int n = u % kDecU1;
          for (int t = lane; t < kDecMaxT; t += 32)
            cp_async_4(&sl->a[t], t < T ? p.hidden_scale + (size_t)kb * T + t : p.zero);
          if (lane < 2)
            cp_async_4(&sl->w[lane], p.w13_scale + ((size_t)e * kGemm1NBlocks + lane * kNT1 + n) * kHiddenBlocks + kb);
        } else {
          const int h2 = u;
          if (lane < kDecMaxT / 4)
            cp_async_16(&sl->a[4 * lane], p.inter_scale + ((size_t)slot * kInterBlocks + kb) * kDecMaxT + 4 * lane);
          if (lane < 2)
            cp_async_4(&sl->w[lane], p.w2_scale + ((size_t)e * kHiddenBlocks + 2 * h2 + lane) * kInterBlocks + kb);
          sl->wr[lane] = wr0;
          sl->wr[lane + 32] = wr1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sfull[j]);
        cp_async_arrive_noinc(&ctl->sfull[j]);
        if (__shfl_sync(0xffffffffu, dec_aborted(ctl) ? 1 : 0, 0)) {
          ok = false;
          break;
        }
      }
    }
    cp_async_wait_all();
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(kTileM, kDecMaxT);
      Walk wk;
      wk.init(blockIdx.x, G, n_slots);
      int ph, u, kb0, kb1;
      uint32_t it = 0;
      bool issued = false, ok = true;
      while (ok && wk.next(ph, u, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t b = it % kDecBufs;
          const int s = it % kDecStages;
          if (!mbar_wait_bounded(&ctl->tempty[b], ((it / kDecBufs) & 1u) ^ 1u, kDecWaitNs) ||
              !mbar_wait_bounded(&ctl->full[s], (it / kDecStages) & 1u, kDecWaitNs) || dec_aborted(ctl)) {
            if (!dec_aborted(ctl)) dec_abort(ctl, p.status);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sw = smem_u32(ring + s * kDecStage);
          const uint32_t sx = sw + kDecW;
          const uint32_t d0 = tmem + b * kDecBufCols, d1 = d0 + kDecMaxT;
          const uint64_t a0 = smem_desc_sw128(sw), a1 = smem_desc_sw128(sw + kStageA);
          const uint64_t xh = smem_desc_sw128(sx);
#pragma unroll
          for (int k = 0; k < kBlk / 32; ++k) mma_f8f6f4(d0, a0 + 2 * k, xh + 2 * k, idesc, k > 0 ? 1u : 0u);
          if (ph == 1) {
            const uint64_t xl = smem_desc_sw128(sx + kDecMaxT * kBlk);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) mma_f8f6f4(d0, a0 + 2 * k, xl + 2 * k, idesc, 1u);
          }
#pragma unroll
          for (int k = 0; k < kBlk / 32; ++k) mma_f8f6f4(d1, a1 + 2 * k, xh + 2 * k, idesc, k > 0 ? 1u : 0u);
          if (ph == 1) {
            const uint64_t xl = smem_desc_sw128(sx + kDecMaxT * kBlk);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) mma_f8f6f4(d1, a1 + 2 * k, xl + 2 * k, idesc, 1u);
          }
          issued = true;
          mma_commit(&ctl->empty[s]);
          mma_commit(&ctl->tfull[b]);
        }
      }
      if (!ok && issued) {
        mma_commit(&ctl->mma_done);
        mbar_wait_bounded(&ctl->mma_done, 0, kDecWaitNs);
      }
    }
  } else {
    // ======================= epilogue (16 warps) =======================
    const int q = warp & 3;                      // TMEM lane quarter of this warp
    const int cg = (warp - kEpiWarp0) >> 2;      // token columns [16cg, 16cg + 16)
    const int r = q * 32 + lane;                 // weight row inside the 128-row tile
    const int t0 = cg * 16;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const bool lead = (warp == kEpiWarp0 && lane == 0);
    DecEpiSync es;
    Walk wk;
    wk.init(blockIdx.x, G, n_slots);
    const int tot1 = n_slots * kDecU1 * kDecKB1;
    const int tot2 = kDecU2 * n_slots * kDecKB2;
    int ph, u, kb0, kb1;
    uint32_t it = 0;
    bool ok = true;
    while (ok && wk.next(ph, u, kb0, kb1)) {
      float acc0[16], acc1[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc0[i] = acc1[i] = 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int j = it % kDecScaleSlots;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&ctl->sfull[j], (it / kDecScaleSlots) & 1u, kDecWaitNs))) {
          dec_abort(ctl, p.status);
          ok = false;
          break;
        }
        float a[16], w0, w1;
        {
          const DecScaleSlot* sl = &ctl->scales[j];
          w0 = sl->w[0];
          w1 = sl->w[1];
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 a4 = *reinterpret_cast<const float4*>(&sl->a[t0 + i]);
            a[i] = a4.x; a[i + 1] = a4.y; a[i + 2] = a4.z; a[i + 3] = a4.w;
          }
          if (ph == 1) {
            // GEMM2: the routing weight of (token, this K block's expert) joins the factor
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 r4 = *reinterpret_cast<const float4*>(&sl->wr[t0 + i]);
              a[i] *= r4.x; a[i + 1] *= r4.y; a[i + 2] *= r4.z; a[i + 3] *= r4.w;
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sempty[j]);
        const uint32_t b = it % kDecBufs;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&ctl->tfull[b], (it / kDecBufs) & 1u, kDecWaitNs))) {
          dec_abort(ctl, p.status);
          ok = false;
          break;
        }
        tc_fence_after();
        {
          float v[16];
          tmem_ld_32x32b_x16(t_lane + b * kDecBufCols + t0, v);
          dec_promote16(acc0, a, w0, v);
          tmem_ld_32x32b_x16(t_lane + b * kDecBufCols + kDecMaxT + t0, v);
          dec_promote16(acc1, a, w1, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->tempty[b]);
      }
      if (!ok) break;

      if (ph == 0) {
        // ---- GEMM1 unit (slot, n): complete it, then SwiGLU + two-term quantisation ----
        const int slot = u / kDecU1, n = u % kDecU1;
        bool finish = (kb0 == 0 && kb1 == kDecKB1);
        if (!finish) {
          // split unit: every piece stores its partial sums to its CTA's
          // scratch (side 0: a unit's first piece, side 1: a later piece);
          // the CTA that completes the unit adds the pieces in CTA order
          const int side = kb0 > 0 ? 1 : 0;
          float* mine = p.g1_part + ((size_t)blockIdx.x * 2 + side) * kDecMaxT * 2 * kBlk;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (t0 + i < T) {
              __stcg(mine + (size_t)(t0 + i) * 2 * kBlk + r, acc0[i]);
              __stcg(mine + (size_t)(t0 + i) * 2 * kBlk + kBlk + r, acc1[i]);
            }
          }
          if (!es.sync(ctl, p.status)) break;
          const int first = u * kDecKB1;
          const int ps = range_owner(first, tot1, G);
          if (lead) {
            const int add = kb1 - kb0;
            __threadfence();
            const int old = atomicAdd(p.g1_cnt + ps, add);
            const int last = (old + add == kDecKB1) ? 1 : 0;
            if (last) {
              __threadfence();
              p.g1_cnt[ps] = 0;
            }
            ctl->flag = last;
          }
          if (!es.sync(ctl, p.status)) break;
          finish = ctl->flag != 0;
          if (finish) {
            const int pl = range_owner(first + kDecKB1 - 1, tot1, G);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc0[i] = acc1[i] = 0.f;
            for (int c = ps; c <= pl; ++c) {
              const float* src = p.g1_part + ((size_t)c * 2 + (c == ps ? 0 : 1)) * kDecMaxT * 2 * kBlk;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (t0 + i < T) {
                  acc0[i] += __ldcg(src + (size_t)(t0 + i) * 2 * kBlk + r);
                  acc1[i] += __ldcg(src + (size_t)(t0 + i) * 2 * kBlk + kBlk + r);
                }
              }
            }
          }
        }
        if (finish) {
          // C[t][col] = G[t][col] * silu(G[t][2048 + col]) (ref_moe.py:153-159), one
          // scale per (token, 128 columns): s = amax / 448, hi = e4m3(C / s),
          // lo = e4m3(C / s - hi)
          float c[16];
          float* am = ctl->amax[q];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            c[i] = (t0 + i < T) ? acc0[i] * dec_silu(acc1[i]) : 0.f;
            // |c| as bits orders like the value (non-negative floats)
            const unsigned m = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(c[i])));
            if (lane == i) am[t0 + i] = __uint_as_float(m);
          }
          if (!es.sync(ctl, p.status)) break;
          uint8_t* ib = p.inter + (size_t)slot * kDecMaxT * kInterCols + n * kBlk + r;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = t0 + i;
            if (t < T) {
              const float amax = fmaxf(fmaxf(ctl->amax[0][t], ctl->amax[1][t]), fmaxf(ctl->amax[2][t], ctl->amax[3][t]));
              const float inv = amax > 0.f ? 448.0f / amax : 0.f;
              const float uq = c[i] * inv;
              const uint16_t hb = f2_to_e4m3x2(uq, 0.f);
              const float qh = dec_e4m3_to_f32(hb & 0xFFu);
              const uint16_t lb = f2_to_e4m3x2(uq - qh, 0.f);
              ib[(size_t)t * kInterCols] = static_cast<uint8_t>(hb & 0xFFu);
              ib[(size_t)t * kInterCols + kInter] = static_cast<uint8_t>(lb & 0xFFu);
              if (q == 0 && lane == i) p.inter_scale[((size_t)slot * kInterBlocks + n) * kDecMaxT + t] = amax / 448.0f;
            }
          }
          fence_proxy_async_global();
          if (!es.sync(ctl, p.status)) break;
          if (lead) {
            __threadfence();
            atomicAdd(p.ready + slot, 1);
          }
        }
      } else {
        // ---- GEMM2 unit h2: columns [256 h2, 256 h2 + 256) summed over all slots ----
        const int h2 = u;
        const int nkb2 = n_slots * kDecKB2;
        bool finish = (kb0 == 0 && kb1 == nkb2);
        if (!finish) {
          // pieces meet as in GEMM1: side 0 = the unit's first piece, side 1 = later ones
          const int side = kb0 > 0 ? 1 : 0;
          float* mine = p.g2_part + ((size_t)blockIdx.x * 2 + side) * kDecMaxT * 2 * kBlk;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (t0 + i < T) {
              __stcg(mine + (size_t)(t0 + i) * 2 * kBlk + r, acc0[i]);
              __stcg(mine + (size_t)(t0 + i) * 2 * kBlk + kBlk + r, acc1[i]);
            }
          }
          if (!es.sync(ctl, p.status)) break;
          const int first = h2 * nkb2;
          const int ps = range_owner(first, tot2, G);
          if (lead) {
            const int add = kb1 - kb0;
            __threadfence();
            const int old = atomicAdd(p.h_cnt + h2, add);
            const int last = (old + add == nkb2) ? 1 : 0;
            if (last) {
              __threadfence();
              p.h_cnt[h2] = 0;
            }
            ctl->flag = last;
          }
          if (!es.sync(ctl, p.status)) break;
          finish = ctl->flag != 0;
          if (finish) {
            const int pl = range_owner(first + nkb2 - 1, tot2, G);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc0[i] = acc1[i] = 0.f;
            for (int c = ps; c <= pl; ++c) {
              const float* src = p.g2_part + ((size_t)c * 2 + (c == ps ? 0 : 1)) * kDecMaxT * 2 * kBlk;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (t0 + i < T) {
                  acc0[i] += __ldcg(src + (size_t)(t0 + i) * 2 * kBlk + r);
                  acc1[i] += __ldcg(src + (size_t)(t0 + i) * 2 * kBlk + kBlk + r);
                }
              }
            }
          }
        }
        if (finish) {
          // the expert sum is complete: cast once to bf16 (ref_moe.py:167)
          __nv_bfloat16* o = p.out + h2 * kTileN + r;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (t0 + i < T) {
              o[(size_t)(t0 + i) * kHidden] = __float2bfloat16_rn(acc0[i]);
              o[(size_t)(t0 + i) * kHidden + kBlk] = __float2bfloat16_rn(acc1[i]);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (tid == 0) {
    // the last CTA to finish clears the per-slot progress counters for the next call
    __threadfence();
    if (atomicAdd(p.done, 1) == G - 1) {
      __threadfence();
      for (int s = 0; s < n_slots; ++s) p.ready[s] = 0;
      *p.done = 0;
    }
  }
}

}  // namespace

size_t decode_smem_bytes() { return kDecRing + sizeof(DecCtl) + 1024; }

cudaError_t launch_decode(const DecodeBuffers& d, const CUtensorMap& map_w13, const CUtensorMap& map_w2,
                          const CUtensorMap& map_x1, const CUtensorMap& map_x2, const DecodeCall& c,
                          cudaStream_t s) {
  static int configured_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const size_t smem = decode_smem_bytes();
  if (configured_dev != dev) {
    e = cudaFuncSetAttribute(moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  DecArgs a{};
  a.logits = c.logits;
  a.bias = c.bias;
  a.hidden_scale = c.hidden_scale;
  a.w13_scale = c.w13_scale;
  a.w2_scale = c.w2_scale;
  a.T = c.T;
  a.offset = c.offset;
  a.e_local = c.e_local;
  a.scale = c.scale;
  a.inter = d.inter;
  a.inter_scale = d.inter_scale;
  a.g1_part = d.g1_part;
  a.g1_cnt = d.g1_cnt;
  a.ready = d.ready;
  a.g2_part = d.g2_part;
  a.h_cnt = d.h_cnt;
  a.done = d.done;
  a.zero = d.zero;
  a.out = static_cast<__nv_bfloat16*>(c.out);
  a.user_ids = c.user_ids;
  a.user_w = c.user_w;
  a.user_counts = c.user_counts;
  a.status = d.status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(d.grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  // all CTAs must be resident at once: GEMM2 work waits for GEMM1 work of other CTAs
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_decode_kernel, map_w13, map_w2, map_x1, map_x2, a);
}

}  // namespace moe
