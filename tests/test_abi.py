"""CPU: the C-ABI library builds for sm_100a, loads, and exports every symbol
declared in include/*.h; the Python boundary rejects bad arguments before
any GPU work. No compute calls are made here."""
import glob
import os
import re

import pytest
import torch

from conftest import ROOT, pkg


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(moe_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = _declared_symbols()
    for n in ("moe_fp8_ds_kernel", "moe_fp8_ds_kernel_ex", "moe_fp8_ds_route", "moe_fp8_ds_experts"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = pkg().load()
    for n in _declared_symbols():
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"


def test_library_is_built_for_sm100a_only():
    """The build recipe names one target, sm_100a, and the kernels' common
    header refuses device compilation for any other (tested on the extracted
    sources in test_pack_cpu.py)."""
    import importlib

    build = importlib.import_module("flashinfer-mlsys_b200.build")
    archs = [f for f in build.NVCC_FLAGS if f.startswith("arch=")]
    assert archs == ["arch=compute_100a,code=sm_100a"]
    with open(os.path.join(build.CSRC, "moe_common.cuh")) as f:
        assert "__CUDA_ARCH_FEAT_SM100_ALL" in f.read()


def test_status_strings_and_version():
    lib = pkg().load()
    assert lib.moe_fp8_ds_status_string(0) == b"ok"
    for code in range(1, 7):
        assert lib.moe_fp8_ds_status_string(code) != b"unknown status"
    assert b"sm_100a" in lib.moe_fp8_ds_version()


def test_workspace_size_formula():
    lib = pkg().load()
    small = lib.moe_fp8_ds_workspace_bytes(8, 32)
    big = lib.moe_fp8_ds_workspace_bytes(16384, 32)
    assert 0 < small < big
    # the bf16 expert rows of the combine dominate: at least T*8 rows of
    # 7168 bf16 values, plus the permuted e4m3 rows
    assert big > 16384 * 8 * 7168 * 3
    assert lib.moe_fp8_ds_workspace_bytes(8, 33) == 0  # unsupported E_local


def test_binding_rejects_cpu_tensors():
    m = pkg()
    T = 2
    with pytest.raises(ValueError, match="CUDA"):
        m.kernel(torch.zeros(T, 256), torch.zeros(256, dtype=torch.bfloat16),
                 torch.zeros(T, 7168, dtype=torch.float8_e4m3fn), torch.zeros(56, T),
                 torch.zeros(32, 4096, 7168, dtype=torch.float8_e4m3fn), torch.zeros(32, 32, 56),
                 torch.zeros(32, 7168, 2048, dtype=torch.float8_e4m3fn), torch.zeros(32, 56, 16),
                 0, 2.5, torch.zeros(T, 7168, dtype=torch.bfloat16))


def test_c_abi_rejects_bad_arguments_without_gpu():
    """Argument checks run before any device call: a null pointer or an
    unsupported E_local returns MOE_ERR_INVALID_ARG (1)."""
    lib = pkg().load()
    assert lib.moe_fp8_ds_kernel(None, None, None, None, None, None, None, None, 0, 2.5, None, 8, 32, None) == 1
    assert lib.moe_fp8_ds_route(None, None, 8, 0, 32, 2.5, None, None, None, None) == 1
