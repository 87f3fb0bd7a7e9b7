"""GPU: the fused decode kernel (one persistent launch for calls with
1..64 tokens) against the kernel pipeline and the CPU oracle.

Both paths must route identically (ids, weights, counts bit-exact) and give
outputs within the parity tolerance of the oracle; the fused path's scratch
(split-unit partial sums, progress counters, the combine accumulator) must
come back clean, so repeated and resized calls agree."""
import numpy as np
import pytest
import torch

from conftest import oracle, pkg, workloads
from parity import check_output, check_routing, check_weights, run_gpu

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    return pkg().load()


class _Path:
    """Context manager selecting the fused decode kernel (1) or the pipeline (0)."""

    def __init__(self, on):
        self.on = on

    def __enter__(self):
        self.prev = _lib().moe_fp8_ds_set_fused_decode(self.on)

    def __exit__(self, *exc):
        _lib().moe_fp8_ds_set_fused_decode(self.prev)


_W = {}


def _weights(e_local=32, offset=0):
    key = (e_local, offset)
    if key not in _W:
        _W.clear()
        _W[key] = workloads().make_weights(e_local, offset, DEV, weight_seed=0)
    return _W[key]


def _oracle(acts, w, offset=None):
    O = oracle()
    off = w.offset if offset is None else offset
    return O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                         lambda le: w.expert_cpu(le), off, 2.5, w.e_local)


@pytest.mark.parametrize("T", [1, 3, 17, 40, 64])
def test_fused_matches_pipeline_and_oracle(gpu_available, T):
    acts = workloads().make_activations(T, seed=100 + T).to(DEV)
    w = _weights()
    with _Path(1):
        of, idf, wf, cf = run_gpu(acts, w)
    with _Path(0):
        op, idp, wp, cp = run_gpu(acts, w)
    assert torch.equal(idf, idp) and torch.equal(wf, wp) and torch.equal(cf, cp)
    ref = _oracle(acts.to("cpu"), w)
    check_routing(ref["routing"], idf, cf, 0, 32)
    check_weights(ref["routing"], idf, wf)
    check_output(of, ref["out_f32"])
    check_output(op, ref["out_f32"])


@pytest.mark.parametrize("e_local,offset,T", [(64, 64, 24), (128, 0, 9), (256, 0, 64)])
def test_fused_other_expert_ranges(gpu_available, e_local, offset, T):
    """More local experts (up to all 256: one GPU holding the whole layer)."""
    acts = workloads().make_activations(T, seed=7 * T + e_local)
    w = _weights(e_local, offset)
    with _Path(1):
        out, ids, wts, cnt = run_gpu(acts.to(DEV), w)
    ref = _oracle(acts, w)
    check_routing(ref["routing"], ids, cnt, offset, e_local)
    check_output(out, ref["out_f32"])


def test_fused_scratch_is_left_clean(gpu_available):
    """Alternating sizes through the fused path reproduce the first answers."""
    w = _weights()
    a64 = workloads().make_activations(64, seed=5).to(DEV)
    a1 = workloads().make_activations(1, seed=6).to(DEV)
    with _Path(1):
        o64, i64, _, _ = run_gpu(a64, w)
        o1, i1, _, _ = run_gpu(a1, w)
        for _ in range(3):
            p64, j64, _, _ = run_gpu(a64, w)
            p1, j1, _, _ = run_gpu(a1, w)
    assert torch.equal(i64, j64) and torch.equal(i1, j1)
    for a, b in ((o64, p64), (o1, p1)):
        # split-unit partials and the combine add in arrival order: equal up to
        # fp32 rounding of the sums, so compare with a tight tolerance
        diff = (a.float() - b.float()).abs().max().item()
        assert diff <= 1e-2 * max(1.0, a.float().abs().max().item())


def test_fused_profile_reports_one_kernel(gpu_available):
    lib = _lib()
    acts = workloads().make_activations(8, seed=1).to(DEV)
    w = _weights()
    buf = (__import__("ctypes").c_float * 5)()
    with _Path(1):
        lib.moe_fp8_ds_profile_enable(1)
        try:
            run_gpu(acts, w)
            n = lib.moe_fp8_ds_profile_last(buf, 5)
        finally:
            lib.moe_fp8_ds_profile_enable(0)
    assert n == 1 and buf[0] > 0.0
