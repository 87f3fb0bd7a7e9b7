/*
 * moe_fp8_ds.h — C ABI of the B200 (sm_100a) fused FP8 DeepSeek-V3 MoE layer.
 *
 * Operator: moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048
 * (reference definition: "reference moe/ref_moe.json", semantics:
 * "reference moe/ref_moe.py:5-167").
 *
 * All pointers are DEVICE pointers unless stated otherwise; all tensors are
 * contiguous row-major. Byte types: e4m3 tensors are passed as `const void*`
 * (one byte per element, float8_e4m3fn bit pattern), bf16 tensors as
 * `const void*` / `void*` (two bytes per element). Every call is enqueued on
 * `stream` (a cudaStream_t, NULL = legacy default stream) and returns without
 * synchronising the host; errors detected before launch are returned as a
 * status code and nothing is launched. The library caches its device
 * workspace per device (grown on demand with cudaMalloc on the first call of
 * a larger size), so calls on one device must be stream-ordered with respect
 * to each other.
 *
 * Fixed geometry: hidden 7168, intermediate 2048, 256 global experts, top-8,
 * 8 groups, top-4 groups, 128x128 / 1x128 quantisation blocks.
 */
#ifndef MOE_FP8_DS_H_
#define MOE_FP8_DS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARG 1   /* bad size, null pointer or unsupported value */
#define MOE_ERR_ALIGNMENT 2     /* a tensor base is not 16-byte aligned          */
#define MOE_ERR_CUDA 3          /* a CUDA runtime/driver call failed             */
#define MOE_ERR_NO_DEVICE 4     /* no sm_100 device current                      */
#define MOE_ERR_WORKSPACE 5     /* workspace allocation failed                   */
#define MOE_ERR_DEVICE_TIMEOUT 6 /* a bounded device-side wait gave up (read by moe_fp8_ds_device_status) */

/*
 * The drop-in entry point. Replaces the destination-passing `kernel(...)` of
 * solution/cuda/kernel.cu:134-146 (bound to Python at kernel.cu:296-298 and
 * wrapped by solution/cuda/binding.py:149-161). Same 11 arguments in the same
 * order and meaning, plus the sizes a C ABI cannot infer from tensors and the
 * stream:
 *   routing_logits      f32  [seq_len, 256]
 *   routing_bias        bf16 [256]
 *   hidden_states       e4m3 [seq_len, 7168]
 *   hidden_states_scale f32  [56, seq_len]        (transposed block scales)
 *   gemm1_weights       e4m3 [num_local_experts, 4096, 7168]
 *   gemm1_weights_scale f32  [num_local_experts, 32, 56]
 *   gemm2_weights       e4m3 [num_local_experts, 7168, 2048]
 *   gemm2_weights_scale f32  [num_local_experts, 56, 16]
 *   local_expert_offset first global expert id held by this rank
 *   routed_scaling_factor
 *   output              bf16 [seq_len, 7168]     (every element is written)
 * num_local_experts is 32 for the reference definition; 64, 128 and 256 are
 * accepted for expert-parallel layouts with fewer ranks. seq_len may be 0.
 */
int moe_fp8_ds_kernel(const float* routing_logits, const void* routing_bias,
                      const void* hidden_states, const float* hidden_states_scale,
                      const void* gemm1_weights, const float* gemm1_weights_scale,
                      const void* gemm2_weights, const float* gemm2_weights_scale,
                      int64_t local_expert_offset, double routed_scaling_factor,
                      void* output, int64_t seq_len, int64_t num_local_experts,
                      void* stream);

/*
 * Same as moe_fp8_ds_kernel, and additionally exposes the routing decision of
 * this very call (any of the three may be NULL):
 *   topk_ids_out       int32 [seq_len, 8]   global expert ids, best first
 *   topk_weights_out   f32   [seq_len, 8]   normalised un-biased sigmoid x scale
 *   expert_counts_out  int32 [num_local_experts] tokens routed to each local expert
 * Reference counterpart: the routing/dispatch tensors topk_idx, weights and
 * the per-expert counts of kernel.cu:175-232 / ref_moe.py:95-148.
 */
int moe_fp8_ds_kernel_ex(const float* routing_logits, const void* routing_bias,
                         const void* hidden_states, const float* hidden_states_scale,
                         const void* gemm1_weights, const float* gemm1_weights_scale,
                         const void* gemm2_weights, const float* gemm2_weights_scale,
                         int64_t local_expert_offset, double routed_scaling_factor,
                         void* output, int64_t seq_len, int64_t num_local_experts,
                         int32_t* topk_ids_out, float* topk_weights_out,
                         int32_t* expert_counts_out, void* stream);

/*
 * The layer with DeepSeek-V3's always-on shared expert fused in (no
 * counterpart in the reference, whose operator has routed experts only; the
 * shared expert follows DeepSeek-V3's MoE block: output = routed sum + shared
 * expert of every token, weight 1). The shared expert has the routed experts'
 * shapes and format: shared_gemm1_weights e4m3 [4096, 7168] with f32 scales
 * [32, 56], shared_gemm2_weights e4m3 [7168, 2048] with f32 scales [56, 16].
 * It is scheduled as one more local expert that every token uses, inside the
 * same persistent GEMMs (no extra launch), and its row is added after the
 * routed rows in the fp32 sum before the single bf16 cast. Other arguments as
 * moe_fp8_ds_kernel; num_local_experts in {32, 64, 128}.
 */
int moe_fp8_ds_kernel_shared(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                             const float* hidden_states_scale, const void* gemm1_weights,
                             const float* gemm1_weights_scale, const void* gemm2_weights,
                             const float* gemm2_weights_scale, int64_t local_expert_offset,
                             double routed_scaling_factor, const void* shared_gemm1_weights,
                             const float* shared_gemm1_weights_scale, const void* shared_gemm2_weights,
                             const float* shared_gemm2_weights_scale, void* output, int64_t seq_len,
                             int64_t num_local_experts, void* stream);

/*
 * Routing only: DeepSeek-V3 no-aux grouped top-k (ref_moe.py:95-126,
 * kernel.cu:157-198) plus the local per-expert histogram (kernel.cu:201-232).
 * Outputs as in moe_fp8_ds_kernel_ex; topk_ids_out and topk_weights_out are
 * required, expert_counts_out may be NULL.
 */
int moe_fp8_ds_route(const float* routing_logits, const void* routing_bias,
                     int64_t seq_len, int64_t local_expert_offset,
                     int64_t num_local_experts, double routed_scaling_factor,
                     int32_t* topk_ids_out, float* topk_weights_out,
                     int32_t* expert_counts_out, void* stream);

/*
 * Allocation-free routing. No counterpart in the reference: it exists for
 * callers that cannot call cudaMalloc when they route (a process whose device
 * memory is owned by a fixed-size pool or arena, an engine that reserves all
 * memory at start-up, or code that must not take the CUDA allocator's locks on
 * its hot path). Same arguments, outputs and status codes as
 * moe_fp8_ds_route(), but all scratch lives in one fixed array of 790,272
 * bytes in the library's own device memory, present on every GPU that loads
 * the library until the process exits; the call makes no allocation of any
 * kind. Limits: seq_len <= 8192 (larger requests return MOE_ERR_INVALID_ARG
 * and launch nothing); num_local_experts in {32, 64, 128, 256}.
 * The first call on a device looks up the array's device address (once per
 * device); make that first call before capturing a stream into a CUDA graph.
 * The address is kept for the life of the process: after the device's primary
 * context is destroyed (cudaDeviceReset) the array moves, so do not call this
 * function again in that process.
 * Every call reuses the same array: calls that may run at the same time on the
 * GPU (different streams without ordering, or different host threads) race on
 * it and must be serialised by the caller.
 */
int moe_fp8_ds_route_noalloc(const float* routing_logits, const void* routing_bias,
                             int64_t seq_len, int64_t local_expert_offset,
                             int64_t num_local_experts, double routed_scaling_factor,
                             int32_t* topk_ids_out, float* topk_weights_out,
                             int32_t* expert_counts_out, void* stream);

/*
 * Expert computation for pre-routed tokens (the expert loop of
 * kernel.cu:235-291 / ref_moe.py:131-167, without the routing step). Used by
 * the expert-parallel layer on the rank that owns the experts:
 *   hidden_states       e4m3 [num_rows, 7168], hidden_states_scale f32 [56, num_rows]
 *   topk_ids            int32 [num_rows, 8] global expert ids (ids outside
 *                       [local_expert_offset, +num_local_experts) are skipped)
 *   topk_weights        f32 [num_rows, 8]
 *   output              f32 [num_rows, 7168] if output_fp32 != 0, else bf16;
 *                       row r = sum over its local experts of weight * expert(row r).
 */
int moe_fp8_ds_experts(const void* hidden_states, const float* hidden_states_scale,
                       const int32_t* topk_ids, const float* topk_weights,
                       const void* gemm1_weights, const float* gemm1_weights_scale,
                       const void* gemm2_weights, const float* gemm2_weights_scale,
                       int64_t local_expert_offset, int64_t num_rows,
                       int64_t num_local_experts, void* output, int output_fp32,
                       void* stream);

/*
 * Per-kernel timing of this library's launches (instrumentation; the
 * reference times its kernels with CUDA events in scripts/ncu_profile.py:191-240).
 * While enabled, every pipeline call records CUDA events on its own stream
 * around each of its kernels. moe_fp8_ds_profile_last() synchronises on the
 * last call's final event and writes the milliseconds of its kernels
 * (route with the permutation, gemm1, gemm2, finalize) to ms_out[0..3]; returns the number
 * written, or a negative status. A call served by the fused decode kernel
 * records one interval (that kernel) and returns 1. Disabled by default;
 * enabling costs one event record per kernel.
 */
int moe_fp8_ds_profile_enable(int on);
int moe_fp8_ds_profile_last(float* ms_out, int n);

/*
 * Selects how moe_fp8_ds_kernel / moe_fp8_ds_kernel_ex serve calls with
 * 1 <= seq_len <= 64 (no reference counterpart: path selection of this
 * library). on = 1: one persistent kernel does routing, both GEMMs and the
 * combine. on = 0 (the default, unless the environment sets
 * MOE_FP8_DS_FUSED_DECODE=1): the kernel pipeline that larger calls use.
 * on < 0 only queries. Returns the previous setting. Both give results within
 * the same tolerance of the reference.
 */
int moe_fp8_ds_set_fused_decode(int on);

/*
 * Failure-path test hook (no counterpart in the reference; off by default).
 * Calls with more than 8 tokens route in one cooperative kernel whose CTAs
 * meet at a grid barrier with a bounded wait (2 s). wait_limit_ns > 0 lowers
 * that limit; skip_arrival_cta >= 0 makes that CTA stay away from the
 * barrier, so the others give up after the limit, set the device status bit
 * and return without permuting (the call's output is then undefined and
 * moe_fp8_ds_device_status reports MOE_ERR_DEVICE_TIMEOUT and clears the
 * counters). (0, -1) restores normal operation.
 */
int moe_fp8_ds_test_route_barrier(uint64_t wait_limit_ns, int skip_arrival_cta);

/*
 * The step upstream of the layer (no counterpart in the reference's solution;
 * its harness supplies pre-quantised inputs, reference moe/ref_moe.json:57-80):
 * BF16 hidden states [seq_len][7168] -> hidden_fp8_out e4m3 [seq_len][7168]
 * and hidden_scale_out f32 [56][seq_len] (transposed, the layer's input
 * format). Per 1x128 block: s = max(amax|x| / 448, 1e-12), q = e4m3(x / s)
 * with an IEEE division and round-to-nearest-even, the recipe of the layer's
 * input definition. Asynchronous on `stream`; 16-byte aligned rows.
 */
int moe_fp8_ds_quantize_act(const void* hidden_bf16, int64_t seq_len, void* hidden_fp8_out, float* hidden_scale_out,
                            void* stream);

/*
 * The step downstream of the layer (no counterpart in the reference, whose
 * operator ends at the bf16 output, solution/cuda/kernel.cu:288-291): the
 * decoder's residual add, the next layer's input RMSNorm and its FP8 1x128
 * quantisation in one pass over the layer's output `x_bf16` [seq_len][7168].
 *   h = bf16(residual + x)                  written back to residual_bf16
 *   y = bf16(w * bf16(h / sqrt(mean(h^2) + eps)))   (DeepSeek-V3 RMSNorm)
 *   out_fp8, out_scale = the quantisation of moe_fp8_ds_quantize_act of y
 * residual_bf16 == NULL: h = x (nothing is written back). norm_weight_bf16
 * [7168] == NULL: y = h (no normalisation). The float32 sum of squares and
 * every rounding follow a fixed order, so the result is deterministic.
 * Asynchronous on `stream`; 16-byte aligned rows; eps >= 0.
 */
int moe_fp8_ds_add_norm_quant(const void* x_bf16, void* residual_bf16, const void* norm_weight_bf16, float eps,
                              int64_t seq_len, void* out_fp8, float* out_scale, void* stream);

/*
 * Expert parallelism: the token exchange around moe_fp8_ds_experts when the
 * 256 experts are sharded over GPUs (no counterpart in the reference, which
 * runs one rank; the collectives are the caller's NCCL all-to-alls). A packed
 * row is 7456 bytes: the e4m3 hidden row (7168), its 56 f32 block scales, its
 * 8 int32 global expert ids and 8 f32 routing weights.
 *
 * moe_fp8_ds_ep_pack: send_buf[i] = packed row of token send_idx[i]
 *   (int64 [num_send]); hidden/scale/ids/weights as for the layer, seq_len rows.
 * moe_fp8_ds_ep_unpack: splits num_rows packed rows into hidden e4m3
 *   [num_rows][7168], hidden_scale f32 [56][num_rows], ids int32 [num_rows][8],
 *   weights f32 [num_rows][8].
 * moe_fp8_ds_ep_combine: output bf16 [seq_len][7168], output[t] = sum over
 *   q = 0..world-1 of partials[row_of[t][q]] (bf16 rows, -1 = none) in fp32 in
 *   rank order, cast once.
 * moe_fp8_ds_ep_plan: the dispatch plan from topk_ids int32 [seq_len][8]
 *   (global expert ids) for `world` ranks (1..64, dividing 256; rank q owns
 *   experts [q*256/world, (q+1)*256/world)). send_counts int64 [world]:
 *   tokens with at least one expert on rank q. send_idx int64 [world*seq_len]
 *   (first sum(send_counts) written): those tokens, ascending, rank after rank.
 *   row_of int32 [seq_len][world]: the row of token t in send_idx for rank q,
 *   -1 if none (the combine's input).
 */
int moe_fp8_ds_ep_pack(const void* hidden_states, const float* hidden_states_scale, const int32_t* topk_ids,
                       const float* topk_weights, int64_t seq_len, const int64_t* send_idx, int64_t num_send,
                       void* send_buf, void* stream);
int moe_fp8_ds_ep_unpack(const void* recv_buf, int64_t num_rows, void* hidden_states, float* hidden_states_scale,
                         int32_t* topk_ids, float* topk_weights, void* stream);
int moe_fp8_ds_ep_plan(const int32_t* topk_ids, int64_t seq_len, int64_t world, int64_t* send_idx,
                       int64_t* send_counts, int32_t* row_of, void* stream);
int moe_fp8_ds_ep_combine(const void* partials, const int32_t* row_of, int64_t seq_len, int64_t world, void* output,
                          void* stream);

/* Human-readable text for a status code (static storage, never NULL). */
const char* moe_fp8_ds_status_string(int status);

/*
 * Synchronises `stream` and returns MOE_ERR_DEVICE_TIMEOUT if any kernel of
 * this library gave up a bounded device-side wait since the last call of this
 * function (and clears the flag), MOE_ERR_CUDA on a CUDA error, else MOE_OK.
 */
int moe_fp8_ds_device_status(void* stream);

/*
 * Diagnostic (no counterpart in the reference): where the last layer call on
 * this device with `num_local_experts` (moe_fp8_ds_kernel, _kernel_ex or
 * _experts) placed each token's expert rows. rows_out int32 [seq_len][8]:
 * row rows_out[t][j] of the expert-major padded layout holds token t for its
 * j-th local expert in ascending id (-1 padded); the row belongs to m-tile
 * row / 128 of the grouped GEMMs, and every m-tile to exactly one expert.
 * seq_len must not exceed the last call's. An asynchronous device-to-device
 * copy on `stream`; tests use it to choose rows that cover every m-tile.
 */
int moe_fp8_ds_last_rows(int64_t seq_len, int64_t num_local_experts, int32_t* rows_out, void* stream);

/* Bytes of device workspace the library holds for (seq_len, num_local_experts). */
size_t moe_fp8_ds_workspace_bytes(int64_t seq_len, int64_t num_local_experts);

/* Frees the cached workspace of the current device (next call re-allocates). */
int moe_fp8_ds_release_workspace(void);

/* Library version string, e.g. "moe_fp8_ds 0.1 sm_100a". */
const char* moe_fp8_ds_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MOE_FP8_DS_H_ */
