"""GPU: the packed contest solution, extracted and built the way the
harness's builders build it, runs the operator through its `kernel` entry and
matches the oracle:
- binding "tvm-ffi" (the harness default): tvm_ffi.cpp.load over every .cu of
  the directory with TVM_FFI_CUDA_ARCH_LIST=10.0a (seconds to build);
- binding "torch": torch.utils.cpp_extension with the sm_100a -gencode. The
  torch headers make this build take minutes, so it runs only with
  MOE_FP8_DS_TEST_PACKED=1."""
import importlib
import os

import pytest
import torch

from conftest import oracle, workloads
from parity import check_output
from test_gpu_moe import gpu_weights

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.skipif(os.environ.get("MOE_FP8_DS_TEST_PACKED") != "1",
                    reason="builds the packed solution (minutes): set MOE_FP8_DS_TEST_PACKED=1")
def test_packed_solution_builds_and_matches_the_oracle(gpu_available, tmp_path):
    from torch.utils.cpp_extension import load

    pack = importlib.import_module("flashinfer-mlsys_b200.pack_solution")
    src = tmp_path / "solution"
    cu = pack.extract(pack.pack(), str(src))
    (tmp_path / "build").mkdir()
    mod = load(name="moe_fp8_ds_packed_solution", sources=cu, extra_include_paths=[str(src)],
               extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17"],
               build_directory=str(tmp_path / "build"), verbose=False)
    w = gpu_weights()
    O = oracle()
    for T in (8, 64):
        acts = workloads().config_activations(T)
        a = acts.to(DEV)
        out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=DEV)
        mod.kernel(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, w.offset, 2.5, out)
        torch.cuda.synchronize()
        ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden),
                            acts.hidden_scale.numpy(), lambda le: w.expert_cpu(le), w.offset, 2.5, w.e_local)
        check_output(out, ref["out_f32"])
    with pytest.raises(RuntimeError):
        mod.kernel(a.logits.double(), a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, 0, 2.5, out)


def test_packed_tvm_ffi_solution_matches_the_oracle(gpu_available, tmp_path, monkeypatch):
    tvm_ffi = pytest.importorskip("tvm_ffi")
    import tvm_ffi.cpp

    monkeypatch.setenv("TVM_FFI_CUDA_ARCH_LIST", "10.0a")
    pack = importlib.import_module("flashinfer-mlsys_b200.pack_solution")
    src = tmp_path / "solution"
    cu = pack.extract(pack.pack(binding="tvm-ffi"), str(src))
    mod = tvm_ffi.cpp.load("moe_fp8_ds_packed_tvm_ffi", cuda_files=cu, extra_cuda_cflags=["-O3"],
                           extra_include_paths=[str(src)], build_directory=str(tmp_path / "build"))
    w = gpu_weights()
    O = oracle()
    for T in (8, 64):
        acts = workloads().config_activations(T)
        a = acts.to(DEV)
        out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=DEV)
        with tvm_ffi.use_torch_stream():
            mod.kernel(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, w.offset, 2.5, out)
        torch.cuda.synchronize()
        ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden),
                            acts.hidden_scale.numpy(), lambda le: w.expert_cpu(le), w.offset, 2.5, w.e_local)
        check_output(out, ref["out_f32"])
    with pytest.raises(Exception, match="dtype"):
        mod.kernel(a.logits.double(), a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, 0, 2.5, out)
