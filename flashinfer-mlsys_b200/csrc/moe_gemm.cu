// moe_gemm.cu — K2/K3: persistent grouped block-scaled FP8 GEMMs on tcgen05.
//
//   GEMM1 (kMode = 1): G[r, :] = A1[r, :] (e4m3, 1x128 scales) x W13[e]^T
//     (e4m3, 128x128 scales), K = 7168, then SwiGLU (ref_moe.py:153-159:
//     C = G[:, :2048] * silu(G[:, 2048:]), silu(x) = x / (1 + exp(-x))) and
//     re-quantisation of C into a two-term e4m3 intermediate per 1x128 block:
//     hi = e4m3(C / s), lo = e4m3(C / s - hi), s = amax / 448, so
//     C ~= s * (hi + lo).
//   GEMM2 (kMode = 2): O[r, :] = (hi + lo)[r, :] x W2[e]^T over 16 K blocks:
//     per block the hi and lo tiles are both multiplied against the same W2
//     tile into one TMEM partial (they share the scale s), then
//     out_rows[r, :] = bf16(routing_weight(r) * O[r, :])  (ref_moe.py:162-166;
//     the combine sums these rows in fp32). Direct-combine calls (small or
//     split-K ones, see direct_combine) instead add routing_weight(r) *
//     O[r, :] into their token's fp32 sum, cast once by the finalize kernel;
//     with 64-row tiles their hi and lo tiles form one 128-row operand: one
//     MMA per K slice puts hi x W in TMEM lanes 0-63 and lo x W in 64-127.
//
// Warp roles (608 threads, one CTA per SM):
//   warp 0      TMA producer (one elected lane): A tile 128x128 + two B slabs
//               128x128 per K block into a shared-memory ring of 3-6 stages
//               (GemmCfg); GEMM1 of calls with at most 64 tokens gathers its
//               A rows from hidden_states with all 32 lanes (tile::gather4).
//   warp 1      TMEM owner + MMA issuer (one lane): 4 x tcgen05.mma
//               (M128 N256 K32, e4m3 x e4m3 -> f32) per K block into one of
//               two 256-column TMEM partial accumulators.
//   warp 2      scale loader: cp.async copies of the 128 row scales and the
//               weight-block scales of every K block into an 8-deep shared
//               ring, running ahead of the epilogue.
//   warps 3-18  epilogue: per K block, read the fresh partial from TMEM and
//               promote it in fp32 registers with a_scale[row,kb] *
//               w_scale[nblk,kb] (the block scales are arbitrary fp32, so no
//               hardware block-scale mode applies); after the last K block
//               run the fused output stage.
// Work units (expert, m-tile, n-tile, k-split) come from the device-side plan
// written by the routing kernel; CTAs walk them with a static stride.
#include "moe_kernels.h"

namespace moe {

namespace {

struct GemmArgs {
  const Plan* plan;
  const float* a_scale;     // GEMM1: [56][rows_cap]; GEMM2: [16][rows_cap]
  // GEMM1 of calls with at most 64 tokens gathers its rows from
  // hidden_states instead: the token of every padded row and the [56][T]
  // activation scales
  const int32_t* row_token;
  const float* x_scale;
  int64_t x_ld;
  const float* w_scale;     // GEMM1: [E_l][32][56];  GEMM2: [E_l][56][16]
  const float* ws_scale;    // the shared expert's scales ([32][56] / [56][16]) when shared_e >= 0
  int shared_e;             // local expert index of the shared expert, or -1
  int rows_cap;
  int e_local;
  uint8_t* inter;           // GEMM1 out: [rows_cap][4096]
  float* inter_scale;       // GEMM1 out: [16][rows_cap]
  float* g_part;            // GEMM1 split-K scratch: [kMaxSplitMTiles*128][4096]
  int32_t* tile_sem;        // GEMM1 split-K counters: [kMaxSplitMTiles][16][4 lane quarters]
  const float* row_weight;  // GEMM2: routing weight of each permuted row
  __nv_bfloat16* out_rows;  // GEMM2 out: [rows_cap][7168] weighted expert outputs (bf16)
  float* g2_part;           // GEMM2 split-K scratch: [kMaxSplitMTiles*128][7168]
  int32_t* tile_sem2;       // GEMM2 split-K counters: [kMaxSplitMTiles][28][16 epilogue warps]
  int T;                    // tokens of the call (GEMM2: direct combine, see direct_combine)
  unsigned* status;
  int plan_early;           // 1: the plan was complete before the previous kernel released this one
};

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: only reached if something is broken

struct Unit {
  int e, m, n, gm, kb0, kb1, rows;
};

template <int kMode>
__device__ __forceinline__ Unit decode_unit(int u, int split, const int* prefix, const int* count, int e_local) {
  constexpr int NT = GemmCfg<kMode>::kNT;
  constexpr int NKB = GemmCfg<kMode>::kNKB;
  Unit x;
  const int ks = u % split;
  const int tile = u / split;
  x.n = tile % NT;
  x.gm = tile / NT;
  // last expert whose first m-tile is <= gm (empty experts share prefixes)
  int lo = 0, hi = e_local - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= x.gm) lo = mid; else hi = mid - 1;
  }
  x.e = lo;
  x.m = x.gm - prefix[lo];
  x.rows = min(kTileM, count[lo] - x.m * kTileM);
  x.kb0 = (ks * NKB) / split;
  x.kb1 = ((ks + 1) * NKB) / split;
  return x;
}

struct __align__(16) ScaleSlot {
  float a[kTileM];  // a_scale of the 128 rows of the m-tile for this K block
  float w[4];       // weight-block scales: GEMM1 {gate, up}; GEMM2 {slab 0, slab 1}
};

struct __align__(16) SmemCtl {
  ScaleSlot scales[kScaleSlots];
  uint64_t sfull[kScaleSlots];
  uint64_t sempty[kScaleSlots];
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  uint64_t epi_bar;   // barrier among the 16 epilogue warps (bounded waits)
  uint32_t tmem_base;
  int abort_flag;
  int plan_total;      // total m-tiles of the call
  int plan_split;      // K split of this GEMM
  int prefix[kExperts + 2];
  int count[kExperts + 1];
  float amax[4][kTileM];
};

__device__ __forceinline__ void signal_abort(SmemCtl* c, unsigned* status) {
  atomicOr(status, kErrTimeout);
  *reinterpret_cast<volatile int*>(&c->abort_flag) = 1;
}
__device__ __forceinline__ bool aborted(SmemCtl* c) { return *reinterpret_cast<volatile int*>(&c->abort_flag) != 0; }

// Barrier among the epilogue warps built on an mbarrier so that every wait is
// bounded (a plain bar.sync could never give up). Returns false on timeout.
struct EpiSync {
  uint32_t phase = 0;
  __device__ __forceinline__ bool sync(SmemCtl* c, unsigned* status) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&c->epi_bar);
    bool ok = mbar_wait_bounded(&c->epi_bar, phase, kWaitLimitNs);
    phase ^= 1u;
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) signal_abort(c, status);
    return ok;
  }
};

// acc[i] += f * v[i] for 16 values, as eight packed f32x2 FMAs (each
// component rounds exactly like fmaf).
__device__ __forceinline__ void promote16(float* acc, const float (&v)[16], float f) {
  const float2 ff = make_float2(f, f);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const float2 r = __ffma2_rn(ff, make_float2(v[i], v[i + 1]), make_float2(acc[i], acc[i + 1]));
    acc[i] = r.x;
    acc[i + 1] = r.y;
  }
}

// x * sigmoid(x) (ref_moe.py:157) with the fast exponential and reciprocal
// intrinsics: relative error ~1e-7, far below the e4m3 requantisation that
// follows, and a short code path (no division slow path).
// 16 consecutive bf16 values w * v[0..15] (round to nearest even) as two uint4
__device__ __forceinline__ void store_bf16x16(__nv_bfloat16* dst, float w, const float* v) {
  uint32_t u[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_bfloat162 b = __floats2bfloat162_rn(w * v[2 * i], w * v[2 * i + 1]);
    u[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(u[0], u[1], u[2], u[3]);
  d[1] = make_uint4(u[4], u[5], u[6], u[7]);
}

__device__ __forceinline__ float silu_ref(float x) { return x * __frcp_rn(1.0f + __expf(-x)); }

__device__ __forceinline__ float e4m3_byte_to_f32(uint32_t b) {
  uint32_t h2;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(h2) : "r"(b));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}

// SwiGLU of N (gate, up) pairs of one row, in place (gate[i] becomes the
// intermediate value), and their absolute maximum. Padding rows (past the
// expert's token count) hold garbage partials; they are kept out of the
// exponential and reciprocal, whose special-value paths would stall the warp.
template <int N>
__device__ __forceinline__ float swiglu_n(float* gate, const float* up, bool valid) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float g = valid ? gate[i] : 0.f;
    const float u = valid ? up[i] : 0.f;
    gate[i] = g * silu_ref(u);
    amax = fmaxf(amax, fabsf(gate[i]));
  }
  return amax;
}

// Two-term e4m3 quantisation of N intermediate values of padded row `row`,
// columns n * 128 + col .. + N, with the amax of their 128-wide block:
// hi = e4m3(c / s), lo = e4m3(c / s - hi), s = amax / 448; the piece at
// column 0 also stores the block's scale.
template <int N>
__device__ __forceinline__ void quant_store_n(const float* c, float amax, size_t row, int n, int col,
                                              const GemmArgs& p) {
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  const float scale = amax / 448.0f;
  uint32_t hi_w[N / 4], lo_w[N / 4];
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    uint32_t hw = 0, lw = 0;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const float u0 = c[i + j] * inv, u1 = c[i + j + 1] * inv;
      const uint16_t h = f2_to_e4m3x2(u0, u1);
      const float q0 = e4m3_byte_to_f32(h & 0xFFu), q1 = e4m3_byte_to_f32(h >> 8);
      const uint16_t l = f2_to_e4m3x2(u0 - q0, u1 - q1);
      hw |= static_cast<uint32_t>(h) << (8 * j);
      lw |= static_cast<uint32_t>(l) << (8 * j);
    }
    hi_w[i / 4] = hw;
    lo_w[i / 4] = lw;
  }
  uint8_t* base = p.inter + row * kInterCols + n * kBlk + col;
  uint4* dh = reinterpret_cast<uint4*>(base);
  uint4* dl = reinterpret_cast<uint4*>(base + kInter);
#pragma unroll
  for (int i = 0; i < N / 16; ++i) {
    dh[i] = make_uint4(hi_w[4 * i], hi_w[4 * i + 1], hi_w[4 * i + 2], hi_w[4 * i + 3]);
    dl[i] = make_uint4(lo_w[4 * i], lo_w[4 * i + 1], lo_w[4 * i + 2], lo_w[4 * i + 3]);
  }
  if (col == 0) p.inter_scale[(size_t)n * p.rows_cap + row] = scale;
}

// SwiGLU of 32 (gate, up) pairs of one row + two-term e4m3 quantisation of the
// 128-wide intermediate block shared by the 4 column-group warps of the row
// (their amax meets in shared memory).
__device__ __forceinline__ void swiglu_quant_store(float* gate, const float* up, int cg, int row_in_tile,
                                                   bool valid, size_t row, int n, SmemCtl* ctl,
                                                   const GemmArgs& p, EpiSync& es) {
  float amax = swiglu_n<32>(gate, up, valid);
  ctl->amax[cg][row_in_tile] = amax;
  if (!es.sync(ctl, p.status)) return;
  amax = fmaxf(fmaxf(ctl->amax[0][row_in_tile], ctl->amax[1][row_in_tile]),
               fmaxf(ctl->amax[2][row_in_tile], ctl->amax[3][row_in_tile]));
  if (!es.sync(ctl, p.status)) return;
  if (valid) quant_store_n<32>(gate, amax, row, n, cg * 32, p);
}

// Split GEMM1, after the last partial of one TMEM lane quarter (rows
// q*32 .. q*32+31 of m-tile gm, n-tile n) has arrived: the finished sums are
// read back from the fp32 scratch (which is cleared for the next call) and
// turned into the two-term intermediate. Eight lanes per row (lane & 7 picks
// 16 of the 128 columns), four rows per pass; the block amax meets by
// shuffles, so no other warp takes part. `buf` holds 32 floats of scratch.
__device__ __forceinline__ void fixup_quarter_g1(const GemmArgs& p, int gm, int n, int rows, int q, int lane,
                                                 float* buf) {
  const int r_end = min(rows, q * 32 + 32);
  const int col = (lane & 7) * 16;
  for (int rb = q * 32; rb < r_end; rb += 4) {
    const int r = rb + (lane >> 3);
    const bool valid = r < r_end;
    const size_t row = (size_t)gm * kTileM + r;
    if (valid) {
      float4* pg = reinterpret_cast<float4*>(p.g_part + row * kGemm1N + n * kBlk + col);
      float4* pu = reinterpret_cast<float4*>(p.g_part + row * kGemm1N + kInter + n * kBlk + col);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a4 = __ldcg(pg + i), b4 = __ldcg(pu + i);
        buf[4 * i] = a4.x; buf[4 * i + 1] = a4.y; buf[4 * i + 2] = a4.z; buf[4 * i + 3] = a4.w;
        buf[16 + 4 * i] = b4.x; buf[17 + 4 * i] = b4.y; buf[18 + 4 * i] = b4.z; buf[19 + 4 * i] = b4.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __stcg(pg + i, make_float4(0.f, 0.f, 0.f, 0.f));
        __stcg(pu + i, make_float4(0.f, 0.f, 0.f, 0.f));
      }
    }
    float amax = swiglu_n<16>(buf, buf + 16, valid);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    if (valid) quant_store_n<16>(buf, amax, row, n, col, p);
  }
}

// The weight slabs of K block kb of unit x: GEMM1 128 gate rows + the matching
// 128 up rows of W13[e]; GEMM2 256 rows of W2[e]. The shared expert (local
// expert shared_e) is read through its own tensor map as expert 0.
template <int kMode>
__device__ __forceinline__ void load_weights(uint8_t* sb, const CUtensorMap* map_w, const CUtensorMap* map_ws,
                                             const Unit& x, int kb, uint64_t* bar, int shared_e) {
  const bool sh = x.e == shared_e;
  const CUtensorMap* m = sh ? map_ws : map_w;
  const int e = sh ? 0 : x.e;
  if (kMode == 1) {
    const int y0 = e * kGemm1N + x.n * kBlk;
    tma_load_2d(sb, m, kb * kBlk, y0, bar);
    tma_load_2d(sb + kStageA, m, kb * kBlk, y0 + kInter, bar);
  } else {
    const int y0 = e * kHidden + x.n * kTileN;
    tma_load_2d(sb, m, kb * kBlk, y0, bar);
    tma_load_2d(sb + kStageA, m, kb * kBlk, y0 + kBlk, bar);
  }
}

// Bytes one pipeline stage receives: the two weight slabs plus the token
// tile(s); GEMM1 of small calls gathers its rows in groups of four (the last
// group repeats the unit's last row) instead of loading a 64-row box.
template <int kMode, int kSkinny>
__device__ __forceinline__ uint32_t stage_tx_bytes(int rows) {
  if (kMode == 1 && kSkinny) return static_cast<uint32_t>(kStageB + ((rows + 3) >> 2) * 4 * kBlk);
  return static_cast<uint32_t>(GemmCfg<kMode, kSkinny>::kStageBytes);
}

template <int kMode, int kSkinny>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                    const __grid_constant__ CUtensorMap map_ws, GemmArgs p) {
  using Cfg = GemmCfg<kMode, kSkinny>;
  static_assert(Cfg::kRing <= kRingBytes && Cfg::kStages <= kMaxStages, "stage ring does not fit");
  static_assert((Cfg::kATiles * Cfg::kABytes) % 1024 == 0 && Cfg::kStageBytes % 1024 == 0,
                "128-byte-swizzled tiles need 1024-byte alignment");
  constexpr int NT = Cfg::kNT;
  constexpr int kStages = Cfg::kStages;
  constexpr int kStageBytes = Cfg::kStageBytes;
  constexpr int kABytes = Cfg::kABytes;
  constexpr int kBOff = Cfg::kATiles * kABytes;  // B tile offset inside a stage
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment (in the shared window) for the 128-byte-swizzled tiles
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* tiles = smem;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + kRingBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // local experts including a shared expert (the last one) when there is one
  const int E_l = p.e_local + (p.shared_e >= 0 ? 1 : 0);

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], kEpiWarps);
    }
    for (int j = 0; j < kScaleSlots; ++j) {
      mbar_init(&ctl->sfull[j], 32);
      mbar_init(&ctl->sempty[j], kEpiWarps);
    }
    mbar_init(&ctl->mma_done, 1);
    mbar_init(&ctl->epi_bar, kEpiWarps);
    ctl->abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_w);
    if (p.shared_e >= 0) prefetch_tensormap(&map_ws);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  // The device plan (per-expert rows, m-tile prefix, K split) goes to shared
  // memory in one pass. When it was complete before this kernel was released
  // (it is written by the routing kernel, at least two kernels back), that
  // happens before waiting for the previous kernel, and so does the issue of
  // the first stages' weight tiles, which depend on nothing produced there.
  auto load_plan = [&]() {
    for (int e = tid; e <= E_l; e += blockDim.x) ctl->prefix[e] = p.plan->mtile_prefix[e];
    for (int e = tid; e < E_l; e += blockDim.x) ctl->count[e] = p.plan->count[e];
    if (tid == 0) {
      ctl->plan_total = p.plan->total_mtiles;
      ctl->plan_split = (kMode == 1) ? p.plan->split1 : p.plan->split2;
    }
  };
  if (p.plan_early) load_plan();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  int n_pre = 0;
  if (p.plan_early && tid == 0) {
    const int split0 = ctl->plan_split;
    const int units0 = ctl->plan_total * NT * split0;
    for (int u = blockIdx.x; u < units0 && n_pre < kStages; u += gridDim.x) {
      const Unit x = decode_unit<kMode>(u, split0, ctl->prefix, ctl->count, E_l);
      for (int kb = x.kb0; kb < x.kb1 && n_pre < kStages; ++kb, ++n_pre) {
        uint8_t* sb = tiles + n_pre * kStageBytes + kBOff;
        mbar_arrive_expect_tx(&ctl->full[n_pre], stage_tx_bytes<kMode, kSkinny>(x.rows));
        load_weights<kMode>(sb, &map_w, &map_ws, x, kb, &ctl->full[n_pre], p.shared_e);
      }
    }
  }
  // from here on we read what the previous kernel produced
  griddep_wait();
  griddep_launch_dependents();
  if (!p.plan_early) {
    load_plan();
    __syncthreads();
  }

  const int total_mtiles = ctl->plan_total;
  const int split = ctl->plan_split;
  // GEMM2 of a direct-combine call (direct_combine) adds its partials into
  // per-token sums; with 64-row tiles its hi and lo rows share one M=128 MMA
  // (their products land in different TMEM lanes and meet in those sums).
  const bool direct = (kMode == 2) && direct_combine(split, p.T);
  const bool stacked = (kMode == 2 && kSkinny == 1 && direct);
  const int units = total_mtiles * NT * split;
  const uint32_t tmem = ctl->tmem_base;

  constexpr bool kGather = (kMode == 1 && kSkinny >= 1);
  if (warp == 0 && kGather) {
    // ============ TMA producer, rows gathered from hidden_states ============
    // lane 0 waits for a free stage and loads the weights; lane l gathers
    // rows 4l..4l+3 of the unit (tile::gather4, one-row boxes)
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      if (__shfl_sync(0xffffffffu, aborted(ctl) ? 1 : 0, 0)) break;
      const Unit x = decode_unit<kMode>(u, split, ctl->prefix, ctl->count, E_l);
      const int ngroups = (x.rows + 3) >> 2;
      int y[4] = {0, 0, 0, 0};
      if (lane < ngroups) {
        const int32_t* rt = p.row_token + (size_t)x.gm * kTileM;
#pragma unroll
        for (int i = 0; i < 4; ++i) y[i] = __ldg(rt + min(4 * lane + i, x.rows - 1));
      }
      for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1u;
        uint8_t* sa = tiles + s * kStageBytes;
        if (lane == 0 && static_cast<int>(it) >= n_pre) {
          ok = mbar_wait_bounded(&ctl->empty[s], ph ^ 1u, kWaitLimitNs);
          if (ok) {
            mbar_arrive_expect_tx(&ctl->full[s], stage_tx_bytes<kMode, kSkinny>(x.rows));
            load_weights<kMode>(sa + kBOff, &map_w, &map_ws, x, kb, &ctl->full[s], p.shared_e);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        if (lane < ngroups) tma_gather4(sa + lane * 4 * kBlk, &map_a, kb * kBlk, y[0], y[1], y[2], y[3], &ctl->full[s]);
      }
      if (!ok) break;
    }
    if (lane == 0) {
      if (!ok) signal_abort(ctl, p.status);
      if (aborted(ctl)) {
        // drain: wait (bounded) for the loads this warp may still have in flight
        const uint32_t n_issued = it > static_cast<uint32_t>(n_pre) ? it : static_cast<uint32_t>(n_pre);
        for (uint32_t j = (n_issued > (uint32_t)kStages ? n_issued - kStages : 0); j < n_issued; ++j)
          mbar_wait_bounded(&ctl->full[j % kStages], (j / kStages) & 1u, kWaitLimitNs);
      }
    }
  } else if (warp == 0) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      uint32_t it = 0;
      for (int u = blockIdx.x; u < units && !aborted(ctl); u += gridDim.x) {
        const Unit x = decode_unit<kMode>(u, split, ctl->prefix, ctl->count, E_l);
        for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1u;
          uint8_t* sa = tiles + s * kStageBytes;
          uint8_t* sb = sa + kBOff;
          if (static_cast<int>(it) >= n_pre) {
            if (!mbar_wait_bounded(&ctl->empty[s], ph ^ 1u, kWaitLimitNs)) { signal_abort(ctl, p.status); break; }
            mbar_arrive_expect_tx(&ctl->full[s], kStageBytes);
            load_weights<kMode>(sb, &map_w, &map_ws, x, kb, &ctl->full[s], p.shared_e);
          }
          // token tile(s); the weights of a prefetched stage are already in flight
          tma_load_2d(sa, &map_a, kb * kBlk, x.gm * kTileM, &ctl->full[s]);
          if (kMode == 2) tma_load_2d(sa + kABytes, &map_a, kInter + kb * kBlk, x.gm * kTileM, &ctl->full[s]);
        }
        if (aborted(ctl)) break;
      }
      if (aborted(ctl)) {
        // drain: wait (bounded) for the loads this thread may still have in flight
        const uint32_t n_issued = it;
        for (uint32_t j = (n_issued > (uint32_t)kStages ? n_issued - kStages : 0); j < n_issued; ++j)
          mbar_wait_bounded(&ctl->full[j % kStages], (j / kStages) & 1u, kWaitLimitNs);
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(kTileM, kTileN);
      // stacked GEMM2: the 64-row hi and lo tiles are adjacent in the stage,
      // i.e. one 128-row operand; a single MMA per K slice gives hi x W in
      // TMEM lanes 0-63 and lo x W in lanes 64-127
      const int n_atiles = stacked ? 1 : Cfg::kATiles;
      uint32_t it = 0, gkb = 0;
      bool issued_any = false;
      for (int u = blockIdx.x; u < units && !aborted(ctl); u += gridDim.x) {
        const Unit x = decode_unit<kMode>(u, split, ctl->prefix, ctl->count, E_l);
        for (int kb = x.kb0; kb < x.kb1; ++kb, ++it, ++gkb) {
          const uint32_t buf = gkb & 1u;
          if (!mbar_wait_bounded(&ctl->tempty[buf], ((gkb >> 1) & 1u) ^ 1u, kWaitLimitNs)) {
            signal_abort(ctl, p.status);
            break;
          }
          const int s = it % kStages;
          if (!mbar_wait_bounded(&ctl->full[s], (it / kStages) & 1u, kWaitLimitNs)) {
            signal_abort(ctl, p.status);
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(tiles + s * kStageBytes);
          const uint32_t sb = sa + kBOff;
          const uint64_t db = smem_desc_sw128(sb);
#pragma unroll
          for (int a = 0; a < Cfg::kATiles; ++a) {
            if (a >= n_atiles) break;
            const uint64_t da = smem_desc_sw128(sa + a * kABytes);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) {
              // advance 32 bytes (one K=32 slice) inside the swizzle atom
              mma_f8f6f4(tmem + buf * kTileN, da + 2 * k, db + 2 * k, idesc, (a > 0 || k > 0) ? 1u : 0u);
            }
          }
          issued_any = true;
          mma_commit(&ctl->empty[s]);
          mma_commit(&ctl->tfull[buf]);
        }
        if (aborted(ctl)) break;
      }
      if (aborted(ctl) && issued_any) {
        mma_commit(&ctl->mma_done);
        mbar_wait_bounded(&ctl->mma_done, 0, kWaitLimitNs);
      }
    }
  } else if (warp == kScaleWarp) {
    // ======================= scale loader =======================
    uint32_t it = 0;
    for (int u = blockIdx.x; u < units && !aborted(ctl); u += gridDim.x) {
      const Unit x = decode_unit<kMode>(u, split, ctl->prefix, ctl->count, E_l);
      // gathered GEMM1 rows: the tokens of rows 4l..4l+3 (-1 past the last row)
      int y[4] = {-1, -1, -1, -1};
      if (kGather) {
        const int32_t* rt = p.row_token + (size_t)x.gm * kTileM;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (4 * lane + i < x.rows) y[i] = __ldg(rt + 4 * lane + i);
      }
      bool ok = true;
      for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
        const int j = it % kScaleSlots;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&ctl->sempty[j], ((it / kScaleSlots) & 1u) ^ 1u,
                                                       kWaitLimitNs));
        if (!ok) {
          signal_abort(ctl, p.status);
          break;
        }
        ScaleSlot* sl = &ctl->scales[j];
        const int ka = kb;
        if (kGather) {
          // hidden_states_scale [56][T]: block kb of each gathered token
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (static_cast<uint64_t>(y[i]) < static_cast<uint64_t>(p.x_ld))
              cp_async_4(&sl->a[4 * lane + i], p.x_scale + (size_t)kb * p.x_ld + y[i]);
        } else {
          cp_async_16(&sl->a[4 * lane], p.a_scale + (size_t)ka * p.rows_cap + (size_t)x.gm * kTileM + 4 * lane);
        }
        if (lane < 2) {
          const bool sh = x.e == p.shared_e;
          const float* wsc = sh ? p.ws_scale : p.w_scale;
          const size_t e = sh ? 0 : x.e;
          const float* src;
          if (kMode == 1)
            src = wsc + (e * kGemm1NBlocks + lane * kNT1 + x.n) * kHiddenBlocks + kb;
          else
            src = wsc + (e * kHiddenBlocks + 2 * x.n + lane) * kInterBlocks + ka;
          cp_async_4(&sl->w[lane], src);
        }
        cp_async_arrive_noinc(&ctl->sfull[j]);
      }
      if (!ok) break;
    }
    cp_async_wait_all();
  } else {
    // ======================= epilogue (16 warps) =======================
    const int q = warp & 3;              // TMEM lane quarter accessible to this warp
    const int cg = (warp - kEpiWarp0) >> 2;  // column group 0..3
    // padded row of this thread's TMEM lane (stacked GEMM2: lanes 64-127 hold
    // the lo products of rows 0-63)
    const int row_in_tile = stacked ? ((q & 1) * 32 + lane) : q * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t gkb = 0;
    EpiSync es;
    float acc[64];
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      if (aborted(ctl)) break;
      const Unit x = decode_unit<kMode>(u, split, ctl->prefix, ctl->count, E_l);
      const size_t row = (size_t)x.gm * kTileM + row_in_tile;
      const bool valid = row_in_tile < x.rows;
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0.f;
      bool ok = true;
      for (int kb = x.kb0; kb < x.kb1; ++kb, ++gkb) {
        const uint32_t buf = gkb & 1u;
        const int j = gkb % kScaleSlots;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&ctl->sfull[j], (gkb / kScaleSlots) & 1u, kWaitLimitNs))) {
          signal_abort(ctl, p.status);
          ok = false;
          break;
        }
        float f0, f1;
        {
          const ScaleSlot* sl = &ctl->scales[j];
          const float as = sl->a[row_in_tile];
          if (kMode == 1) {
            f0 = as * sl->w[0];
            f1 = as * sl->w[1];
          } else {
            f0 = f1 = as * sl->w[cg >> 1];
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sempty[j]);
        const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(&ctl->tfull[buf], (gkb >> 1) & 1u, kWaitLimitNs));
        if (!got) {
          signal_abort(ctl, p.status);
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        const uint32_t tb = t_lane + buf * kTileN;
        // columns of this warp: GEMM1 gate [32cg, 32cg+32) and up [128+32cg, ...);
        // GEMM2 [64cg, 64cg+64)
        const uint32_t c0 = (kMode == 1) ? cg * 32 : cg * 64;
        const uint32_t c1 = (kMode == 1) ? kBlk + cg * 32 : cg * 64 + 32;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float v[16];
          const uint32_t col = (h < 2) ? c0 + 16 * h : c1 + 16 * (h - 2);
          const float f = (h < 2) ? f0 : f1;
          tmem_ld_32x32b_x16(tb + col, v);
          promote16(acc + 16 * h, v, f);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->tempty[buf]);
      }
      if (!ok) break;

      if (kMode == 1) {
        // one call site of the SwiGLU stage (its code is fetched once)
        bool do_swiglu = (split == 1);
        if (split > 1) {
          // split-K: promoted partials meet in fp32 scratch. Arrivals are
          // counted per (m-tile, n-tile, lane quarter) over the 4 column-group
          // warps of every split; the last warp to arrive finishes that
          // quarter's rows (no barrier among the epilogue warps).
          float* g = p.g_part + row * kGemm1N;
          if (valid) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              red_add_v4(g + x.n * kBlk + cg * 32 + i, acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
              red_add_v4(g + kInter + x.n * kBlk + cg * 32 + i, acc[32 + i], acc[33 + i], acc[34 + i],
                         acc[35 + i]);
            }
          }
          __threadfence();
          __syncwarp();
          int32_t* sem = p.tile_sem + ((size_t)x.gm * kNT1 + x.n) * 4 + q;
          int last = 0;
          if (lane == 0) last = (atomicAdd(sem, 1) == 4 * split - 1) ? 1 : 0;
          last = __shfl_sync(0xffffffffu, last, 0);
          if (last) {
            __threadfence();
            if (lane == 0) *sem = 0;
            fixup_quarter_g1(p, x.gm, x.n, x.rows, q, lane, acc);
          }
        }
        if (do_swiglu) swiglu_quant_store(acc, acc + 32, cg, row_in_tile, valid, row, x.n, ctl, p, es);
      } else {
        const float w = valid ? __ldg(p.row_weight + row) : 0.f;
        __nv_bfloat16* dst = p.out_rows + row * kHidden + x.n * kTileN + cg * 64;
        if (direct) {
          // direct combine: the weighted partial goes straight into its
          // token's fp32 sum; no arrival counting (the finalize kernel, which
          // runs after this grid completes, casts the sums)
          // (a row's token is checked: after a routing timeout its slot may be stale)
          const int tok = valid ? __ldg(p.row_token + row) : -1;
          if (static_cast<unsigned>(tok) < static_cast<unsigned>(p.T)) {
            float* g = p.g2_part + (size_t)tok * kHidden + x.n * kTileN + cg * 64;
#pragma unroll
            for (int i = 0; i < 64; i += 4)
              red_add_v4(g + i, w * acc[i], w * acc[i + 1], w * acc[i + 2], w * acc[i + 3]);
          }
        } else if (split == 1) {
          if (valid) {
#pragma unroll
            for (int i = 0; i < 64; i += 16) store_bf16x16(dst + i, w, acc + i);
          }
        } else {
          // split-K: partial sums meet in fp32 scratch. Arrivals are counted
          // per (m-tile, n-tile, epilogue warp); the last split to arrive
          // writes that warp's 32 rows x 64 columns.
          float* g = p.g2_part + row * kHidden + x.n * kTileN + cg * 64;
          if (valid) {
#pragma unroll
            for (int i = 0; i < 64; i += 4)
              red_add_v4(g + i, w * acc[i], w * acc[i + 1], w * acc[i + 2], w * acc[i + 3]);
          }
          __threadfence();
          __syncwarp();
          int32_t* sem = p.tile_sem2 + ((size_t)x.gm * kNT2 + x.n) * kEpiWarps + (warp - kEpiWarp0);
          int last = 0;
          if (lane == 0) last = (atomicAdd(sem, 1) == split - 1) ? 1 : 0;
          last = __shfl_sync(0xffffffffu, last, 0);
          if (last) {
            __threadfence();
            if (lane == 0) *sem = 0;
            if (valid) {
              // all loads first (independent), then the stores
              float4* pg = reinterpret_cast<float4*>(g);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float4 a4 = __ldcg(pg + i);
                acc[4 * i] = a4.x; acc[4 * i + 1] = a4.y; acc[4 * i + 2] = a4.z; acc[4 * i + 3] = a4.w;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) __stcg(pg + i, make_float4(0.f, 0.f, 0.f, 0.f));
#pragma unroll
              for (int i = 0; i < 64; i += 16) store_bf16x16(dst + i, 1.0f, acc + i);
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
}

size_t gemm_smem_bytes() { return kRingBytes + sizeof(SmemCtl) + 1024; }

template <int kMode, int kSkinny>
cudaError_t launch_gemm(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                        const float* w_scale, cudaStream_t s, int plan_early, const CUtensorMap& map_ws,
                        const float* ws_scale, int shared_e, const float* x_scale = nullptr, int64_t x_ld = 0,
                        int T = 0) {
  // The shared-memory opt-in is a per-device function attribute: one bit per
  // device that has it (launches run under the library's host mutex).
  static uint64_t configured = 0;
  const size_t smem = gemm_smem_bytes();
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
  if (!(configured & bit) || !bit) {
    e = cudaFuncSetAttribute(moe_gemm_kernel<kMode, kSkinny>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured |= bit;
  }
  const int sms = device_sm_count();
  GemmArgs p{};
  p.plan = ws.plan;
  p.a_scale = (kMode == 1) ? ws.a1_scale : ws.inter_scale;
  p.w_scale = w_scale;
  p.ws_scale = ws_scale;
  p.shared_e = shared_e;
  p.rows_cap = static_cast<int>(ws.rows_cap);
  p.e_local = ws.e_local;
  p.inter = ws.inter;
  p.inter_scale = ws.inter_scale;
  p.g_part = ws.g_part;
  p.tile_sem = ws.tile_sem;
  p.row_weight = ws.row_weight;
  p.row_token = ws.row_token;
  p.x_scale = x_scale;
  p.x_ld = x_ld;
  p.out_rows = ws.out_rows;
  p.g2_part = ws.g2_part;
  p.tile_sem2 = ws.tile_sem2;
  p.status = ws.status;
  p.plan_early = plan_early;
  p.T = T;
  return launch_k(moe_gemm_kernel<kMode, kSkinny>, dim3(sms), dim3(kGemmThreads), smem, s, true, map_a, map_w,
                  map_ws, p);
}

}  // namespace

// GEMM1 of calls with at most this many tokens uses 16-row token tiles and
// six weight stages (a shared expert adds no rows beyond T).
#ifndef MOE_TINY_MAX_T
#define MOE_TINY_MAX_T 16
#endif
constexpr int kTinyMaxT = MOE_TINY_MAX_T;
static_assert(kTinyMaxT <= kTinyMaxRows, "tiny GEMM1 tiles hold kTinyMaxRows rows");

// GEMM1 directly follows the routing kernel that writes the plan, so it reads
// the plan after its programmatic-launch wait. GEMM2 was released by GEMM1
// after that wait: the plan is complete when GEMM2 starts, and GEMM2 loads it
// and issues its first weight tiles before waiting for GEMM1.
cudaError_t launch_gemm1(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                         const float* w_scale, cudaStream_t s, bool skinny, const float* x_scale, int64_t T,
                         const CUtensorMap& map_ws, const float* ws_scale, int shared_e) {
  if (skinny && T <= kTinyMaxT)
    return launch_gemm<1, 2>(ws, map_a, map_w, w_scale, s, 0, map_ws, ws_scale, shared_e, x_scale, T);
  return skinny ? launch_gemm<1, 1>(ws, map_a, map_w, w_scale, s, 0, map_ws, ws_scale, shared_e, x_scale, T)
                : launch_gemm<1, 0>(ws, map_a, map_w, w_scale, s, 0, map_ws, ws_scale, shared_e);
}

cudaError_t launch_gemm2(const Workspace& ws, const CUtensorMap& map_a, const CUtensorMap& map_w,
                         const float* w_scale, cudaStream_t s, bool skinny, const CUtensorMap& map_ws,
                         const float* ws_scale, int shared_e, int T) {
  return skinny ? launch_gemm<2, 1>(ws, map_a, map_w, w_scale, s, 1, map_ws, ws_scale, shared_e, nullptr, 0, T)
                : launch_gemm<2, 0>(ws, map_a, map_w, w_scale, s, 1, map_ws, ws_scale, shared_e, nullptr, 0, T);
}

}  // namespace moe
