// moe_noalloc.cu — allocation-free variant of the routing entry point.
//
// Some callers cannot call cudaMalloc at the point where they route tokens:
// code running inside a memory pool that forbids foreign allocations, an
// inference engine that reserves all device memory up front and hands out
// fixed buffers, or a host thread that must not take the allocator's locks.
// moe_fp8_ds_route() itself allocates its workspace on first use; this
// variant instead keeps its scratch in a fixed-size array that lives in the
// library's own device memory image (loaded with the module, held by every GPU
// that loads the library until the process exits), so a call never allocates.
#include <mutex>

#include "moe_fp8_ds.h"
#include "moe_kernels.h"

using namespace moe;

namespace {

// Limits of the allocation-free router.
constexpr int kNoAllocMaxTokens = 8192;
constexpr int kNoAllocMaxCtas = 256;  // route_ctas_for(T, 1) <= 148 for any T <= 8192

// Scratch layout inside the static array (byte offsets, 256-byte aligned).
constexpr size_t a256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr size_t kOffFill = 0;                                                  // int32 [256]
constexpr size_t kOffDone = kOffFill + a256(kExperts * 4);                      // uint32
constexpr size_t kOffStatus = kOffDone + 256;                                   // uint32
constexpr size_t kZeroBytes = kOffStatus + 256;                                 // cleared every call
constexpr size_t kOffPlan = kZeroBytes;                                         // Plan
constexpr size_t kOffIds = kOffPlan + a256(sizeof(Plan));                       // int32 [T][8]
constexpr size_t kOffW = kOffIds + a256((size_t)kNoAllocMaxTokens * kTopK * 4); // f32 [T][8]
constexpr size_t kOffRank = kOffW + a256((size_t)kNoAllocMaxTokens * kTopK * 4);
constexpr size_t kScratchBytes = kOffRank + a256((size_t)kNoAllocMaxTokens * kTopK * 4);  // 790,272 B
static_assert(kScratchBytes == 790272, "the size stated in include/moe_fp8_ds.h");

static __device__ __align__(256) unsigned char g_route_scratch[kScratchBytes];

// Device address of g_route_scratch, resolved once per device. In host code
// the symbol name is only a host-side stand-in, never a device address.
std::mutex g_na_mu;
void* g_na_ptr[64] = {nullptr};

int scratch_ptr(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOE_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (!g_na_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return MOE_ERR_CUDA;
    }
    g_na_ptr[dev] = p;
  }
  *out = g_na_ptr[dev];
  return MOE_OK;
}

}  // namespace

extern "C" int moe_fp8_ds_route_noalloc(const float* routing_logits, const void* routing_bias, int64_t seq_len,
                                        int64_t local_expert_offset, int64_t num_local_experts,
                                        double routed_scaling_factor, int32_t* topk_ids_out,
                                        float* topk_weights_out, int32_t* expert_counts_out, void* stream) {
  if (seq_len < 0 || seq_len > kNoAllocMaxTokens) return MOE_ERR_INVALID_ARG;
  if (!(num_local_experts == 32 || num_local_experts == 64 || num_local_experts == 128 ||
        num_local_experts == 256))
    return MOE_ERR_INVALID_ARG;
  if (local_expert_offset < -(int64_t(1) << 30) || local_expert_offset > (int64_t(1) << 30))
    return MOE_ERR_INVALID_ARG;
  // the device check comes first so that empty calls return the same codes as moe_fp8_ds_route
  int major = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
    return MOE_ERR_NO_DEVICE;
  if (seq_len == 0) return MOE_OK;
  if (!routing_logits || !routing_bias || !topk_ids_out || !topk_weights_out) return MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(routing_logits) & 15u) || (reinterpret_cast<uintptr_t>(routing_bias) & 15u))
    return MOE_ERR_ALIGNMENT;
  void* base = nullptr;
  int rc = scratch_ptr(&base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* b = static_cast<uint8_t*>(base);
  // the arrival counters must start at zero; clear them on the caller's stream
  if (cudaMemsetAsync(b, 0, kZeroBytes, s) != cudaSuccess) return MOE_ERR_CUDA;

  Workspace ws{};
  ws.t_cap = seq_len;
  ws.e_local = static_cast<int>(num_local_experts);
  ws.expert_fill = reinterpret_cast<int32_t*>(b + kOffFill);
  ws.done_ctas = reinterpret_cast<uint32_t*>(b + kOffDone);
  ws.status = reinterpret_cast<unsigned*>(b + kOffStatus);
  ws.plan = reinterpret_cast<Plan*>(b + kOffPlan);
  ws.topk_ids = reinterpret_cast<int32_t*>(b + kOffIds);
  ws.topk_w = reinterpret_cast<float*>(b + kOffW);
  ws.topk_rank = reinterpret_cast<int32_t*>(b + kOffRank);

  RouteArgs ra{};
  ra.logits = routing_logits;
  ra.bias = static_cast<const uint16_t*>(routing_bias);
  ra.T = static_cast<int>(seq_len);
  ra.offset = static_cast<int>(local_expert_offset);
  ra.e_local = static_cast<int>(num_local_experts);
  ra.scale = static_cast<float>(routed_scaling_factor);
  ra.tokens_per_cta = tokens_per_cta_for(ra.T, 1);
  ra.user_ids = topk_ids_out;
  ra.user_w = topk_weights_out;
  ra.user_counts = expert_counts_out;
  if (route_ctas_for(ra.T, 1) > kNoAllocMaxCtas) return MOE_ERR_INVALID_ARG;
  return launch_route(ws, ra, s) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
