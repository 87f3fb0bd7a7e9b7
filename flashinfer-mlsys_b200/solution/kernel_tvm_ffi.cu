// kernel_tvm_ffi.cu — entry point of the packed contest solution for the
// harness's default binding, TVM-FFI (spec binding "tvm-ffi", entry point
// "kernel_tvm_ffi.cu::kernel"). Same operator and argument list as the torch
// entry (kernel.cu here; reference solution/cuda/kernel.cu:134-146): the
// 11-argument destination-passing-style `kernel`, exported with
// TVM_FFI_DLL_EXPORT_TYPED_FUNC. Tensors arrive as DLPack views; the call
// runs on the FFI environment's current stream for the output's device (the
// caller's torch stream when called under tvm_ffi's torch stream context,
// else the legacy default stream) and forwards to the C ABI (moe_fp8_ds.h).
// A nonzero status raises with the library's message; there is no fallback.
//
// Build: every .cu of the solution directory except kernel.cu (the torch
// entry), with that directory on the include path, for sm_100a only.
#include <cuda_runtime.h>

#include <initializer_list>

#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include "moe_fp8_ds.h"

namespace {

using tvm::ffi::TensorView;

void* base_ptr(const TensorView& t) { return static_cast<char*>(t.data_ptr()) + t.byte_offset(); }

void check_tensor(const TensorView& t, const char* name, DLDataTypeCode code, int bits,
                  std::initializer_list<int64_t> shape, const DLDevice& dev) {
  TVM_FFI_ICHECK(t.device().device_type == kDLCUDA && t.device().device_id == dev.device_id)
      << name << " must be a CUDA tensor on device " << dev.device_id;
  TVM_FFI_ICHECK(t.dtype().code == code && t.dtype().bits == bits && t.dtype().lanes == 1)
      << name << " has the wrong dtype";
  TVM_FFI_ICHECK(t.ndim() == static_cast<int32_t>(shape.size())) << name << " has the wrong rank";
  int i = 0;
  for (int64_t d : shape) {
    TVM_FFI_ICHECK(t.shape()[i] == d) << name << " dimension " << i << " must be " << d;
    ++i;
  }
  // row-major contiguity (a DLPack tensor without strides is contiguous)
  int64_t expect = 1;
  for (int k = t.ndim() - 1; k >= 0; --k) {
    TVM_FFI_ICHECK(t.shape()[k] <= 1 || t.strides()[k] == expect) << name << " must be contiguous";
    expect *= t.shape()[k];
  }
}

void kernel_impl(TensorView routing_logits, TensorView routing_bias, TensorView hidden_states,
                 TensorView hidden_states_scale, TensorView gemm1_weights, TensorView gemm1_weights_scale,
                 TensorView gemm2_weights, TensorView gemm2_weights_scale, int64_t local_expert_offset,
                 double routed_scaling_factor, TensorView output) {
  TVM_FFI_ICHECK(routing_logits.ndim() == 2) << "routing_logits must be [seq_len, 256]";
  TVM_FFI_ICHECK(gemm1_weights.ndim() == 3) << "gemm1_weights must be [num_local_experts, 4096, 7168]";
  const int64_t T = routing_logits.shape()[0];
  const int64_t E = gemm1_weights.shape()[0];
  const DLDevice dev = output.device();
  check_tensor(routing_logits, "routing_logits", kDLFloat, 32, {T, 256}, dev);
  check_tensor(routing_bias, "routing_bias", kDLBfloat, 16, {256}, dev);
  check_tensor(hidden_states, "hidden_states", kDLFloat8_e4m3fn, 8, {T, 7168}, dev);
  check_tensor(hidden_states_scale, "hidden_states_scale", kDLFloat, 32, {56, T}, dev);
  check_tensor(gemm1_weights, "gemm1_weights", kDLFloat8_e4m3fn, 8, {E, 4096, 7168}, dev);
  check_tensor(gemm1_weights_scale, "gemm1_weights_scale", kDLFloat, 32, {E, 32, 56}, dev);
  check_tensor(gemm2_weights, "gemm2_weights", kDLFloat8_e4m3fn, 8, {E, 7168, 2048}, dev);
  check_tensor(gemm2_weights_scale, "gemm2_weights_scale", kDLFloat, 32, {E, 56, 16}, dev);
  check_tensor(output, "output", kDLBfloat, 16, {T, 7168}, dev);
  int prev = 0;
  TVM_FFI_ICHECK(cudaGetDevice(&prev) == cudaSuccess) << "no CUDA device";
  if (prev != dev.device_id) TVM_FFI_ICHECK(cudaSetDevice(dev.device_id) == cudaSuccess) << "cudaSetDevice failed";
  void* stream = TVMFFIEnvGetStream(kDLCUDA, dev.device_id);
  const int rc = moe_fp8_ds_kernel(
      static_cast<const float*>(base_ptr(routing_logits)), base_ptr(routing_bias), base_ptr(hidden_states),
      static_cast<const float*>(base_ptr(hidden_states_scale)), base_ptr(gemm1_weights),
      static_cast<const float*>(base_ptr(gemm1_weights_scale)), base_ptr(gemm2_weights),
      static_cast<const float*>(base_ptr(gemm2_weights_scale)), local_expert_offset, routed_scaling_factor,
      base_ptr(output), T, E, stream);
  if (prev != dev.device_id) cudaSetDevice(prev);
  TVM_FFI_ICHECK(rc == 0) << "moe_fp8_ds_kernel: " << moe_fp8_ds_status_string(rc);
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, kernel_impl);
