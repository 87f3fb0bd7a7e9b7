"""GPU test of the allocation-free router, moe_fp8_ds_route_noalloc.

That entry point serves callers that must not allocate device memory when
they route tokens — for example an engine whose memory is owned by a fixed
arena, or code that cannot take the CUDA allocator's locks on its hot path.
It keeps its scratch in a fixed array inside the library instead of the
workspace moe_fp8_ds_route() allocates. Here both are called through the C
ABI on the same inputs, twice in a row with different inputs (so the second
call runs on the array the first one left behind), and must agree.

This file is named so that pytest collects it last.
"""
import ctypes
import importlib

import pytest
import torch

from conftest import oracle, workloads
from parity import check_routing, check_weights

pytestmark = pytest.mark.gpu


def _route_both(lib, acts, offset, e_local, scale, stream):
    dev = acts.logits.device
    T = acts.logits.shape[0]
    outs = []
    for name in ("moe_fp8_ds_route", "moe_fp8_ds_route_noalloc"):
        ids = torch.full((T, 8), -9, dtype=torch.int32, device=dev)
        wts = torch.full((T, 8), -1.0, dtype=torch.float32, device=dev)
        cnt = torch.full((e_local,), -1, dtype=torch.int32, device=dev)
        rc = getattr(lib, name)(acts.logits.data_ptr(), acts.bias.data_ptr(), T, offset, e_local, scale,
                                ids.data_ptr(), wts.data_ptr(), cnt.data_ptr(), stream)
        assert rc == 0, f"{name} returned {rc}"
        outs.append((ids, wts, cnt))
    torch.cuda.synchronize()
    return outs


def test_route_noalloc_matches_route_twice(gpu_available):
    pkg = importlib.import_module("flashinfer-mlsys_b200")
    lib = pkg.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    # (tokens, seed, local_expert_offset, local experts); 8192 tokens is the
    # documented limit, where the id, weight and rank arrays fill the static
    # array, and 256 local experts is the largest expert table
    cases = [(300, 3, 64, 32), (37, 4, 0, 128), (8192, 5, 0, 256), (8192, 6, 128, 32)]
    O = oracle()
    for T, seed, offset, e_local in cases:
        cpu = workloads().make_activations(T, seed)
        acts = cpu.to(dev)
        (ids_a, w_a, c_a), (ids_b, w_b, c_b) = _route_both(lib, acts, offset, e_local, 2.5, stream)
        assert torch.equal(ids_a, ids_b)
        assert torch.equal(c_a, c_b)
        torch.testing.assert_close(w_b, w_a, rtol=1e-6, atol=1e-7)
        assert int(c_b.sum()) > 0
        if T == 8192:
            # at the limit, also against the CPU oracle: ids and counts exact
            # (near-ties reported), weights at the chosen ids
            routing = O.route(cpu.logits.numpy(), O.as_f32(cpu.bias), 2.5)
            check_routing(routing, ids_b, c_b, offset, e_local)
            check_weights(routing, ids_b, w_b)


def test_route_noalloc_rejects_oversize_without_launch(gpu_available):
    pkg = importlib.import_module("flashinfer-mlsys_b200")
    lib = pkg.load()
    # 8193 tokens is past the documented limit: MOE_ERR_INVALID_ARG (1),
    # checked before any pointer is touched
    rc = lib.moe_fp8_ds_route_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), 8193, 0, 32, 2.5,
                                      ctypes.c_void_p(16), ctypes.c_void_p(16), None, None)
    assert rc == 1
