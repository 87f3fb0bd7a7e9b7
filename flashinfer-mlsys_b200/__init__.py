"""B200 (sm_100a) fused FP8 DeepSeek-V3 MoE layer.

Drop-in for the reference's DPS entry point (solution/cuda/kernel.cu +
binding.py of vanshnawander/flashinfer-mlsys): ``kernel(...)`` with the same
11 arguments. The package directory name contains a hyphen, so import it
with ``importlib.import_module("flashinfer-mlsys_b200")``.
"""
from .binding import (  # noqa: F401
    BLOCK_Q,
    HIDDEN_SIZE,
    INTERMEDIATE_SIZE,
    NUM_EXPERTS,
    NUM_LOCAL_EXPERTS,
    TOP_K,
    device_status,
    experts,
    kernel,
    kernel_ex,
    kernel_shared,
    last_rows,
    quantize_activations,
    add_rmsnorm_quantize,
    route,
)
from . import workloads  # noqa: F401
from ._lib import MoeError, lib_path, load  # noqa: F401

__all__ = [
    "kernel", "kernel_ex", "kernel_shared", "route", "experts", "quantize_activations", "add_rmsnorm_quantize", "device_status", "last_rows", "workloads", "MoeError", "load", "lib_path",
]
