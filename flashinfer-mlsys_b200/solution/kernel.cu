// kernel.cu — entry point of the packed contest solution (spec binding
// "torch", entry point "kernel.cu::kernel"). It is the operator
// moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048 as the
// reference's torch extension registers it: the 11-argument
// destination-passing-style `kernel` (solution/cuda/kernel.cu:134-146) exposed
// by a pybind11 module as `kernel` (solution/cuda/kernel.cu:296-298). It checks
// the tensors and forwards to the C ABI (moe_fp8_ds.h) on the current CUDA
// stream; the other .cu files of the solution are the library itself. No
// fallback: a nonzero status raises with the library's message.
//
// Build: every .cu of the solution directory with that directory on the
// include path, for sm_100a only (nvcc -gencode arch=compute_100a,code=sm_100a).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "moe_fp8_ds.h"

namespace {

void check_tensor(const at::Tensor& t, const char* name, at::ScalarType dtype, std::initializer_list<int64_t> shape,
                  const at::Device& dev) {
  TORCH_CHECK(t.is_cuda() && t.device() == dev, name, " must be a CUDA tensor on ", dev);
  TORCH_CHECK(t.scalar_type() == dtype, name, " must be ", dtype, ", got ", t.scalar_type());
  TORCH_CHECK(t.sizes().equals(shape), name, " must have shape ", at::IntArrayRef(shape), ", got ", t.sizes());
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace

void kernel(at::Tensor routing_logits, at::Tensor routing_bias, at::Tensor hidden_states,
            at::Tensor hidden_states_scale, at::Tensor gemm1_weights, at::Tensor gemm1_weights_scale,
            at::Tensor gemm2_weights, at::Tensor gemm2_weights_scale, int64_t local_expert_offset,
            double routed_scaling_factor, at::Tensor output) {
  TORCH_CHECK(routing_logits.dim() == 2, "routing_logits must be [seq_len, 256]");
  TORCH_CHECK(gemm1_weights.dim() == 3, "gemm1_weights must be [num_local_experts, 4096, 7168]");
  const int64_t T = routing_logits.size(0);
  const int64_t E = gemm1_weights.size(0);
  const at::Device dev = output.device();
  check_tensor(routing_logits, "routing_logits", at::kFloat, {T, 256}, dev);
  check_tensor(routing_bias, "routing_bias", at::kBFloat16, {256}, dev);
  check_tensor(hidden_states, "hidden_states", at::kFloat8_e4m3fn, {T, 7168}, dev);
  check_tensor(hidden_states_scale, "hidden_states_scale", at::kFloat, {56, T}, dev);
  check_tensor(gemm1_weights, "gemm1_weights", at::kFloat8_e4m3fn, {E, 4096, 7168}, dev);
  check_tensor(gemm1_weights_scale, "gemm1_weights_scale", at::kFloat, {E, 32, 56}, dev);
  check_tensor(gemm2_weights, "gemm2_weights", at::kFloat8_e4m3fn, {E, 7168, 2048}, dev);
  check_tensor(gemm2_weights_scale, "gemm2_weights_scale", at::kFloat, {E, 56, 16}, dev);
  check_tensor(output, "output", at::kBFloat16, {T, 7168}, dev);
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = moe_fp8_ds_kernel(
      routing_logits.data_ptr<float>(), routing_bias.data_ptr(), hidden_states.data_ptr(),
      hidden_states_scale.data_ptr<float>(), gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr<float>(),
      gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr<float>(), local_expert_offset, routed_scaling_factor,
      output.data_ptr(), T, E, at::cuda::getCurrentCUDAStream(dev.index()).stream());
  TORCH_CHECK(rc == 0, "moe_fp8_ds_kernel: ", moe_fp8_ds_status_string(rc));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("kernel", &kernel, "fused FP8 block-scale DeepSeek-V3 MoE layer (sm_100a)");
}
