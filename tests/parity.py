"""Parity checks of the CUDA path against the CPU oracle (test helpers)."""
from __future__ import annotations

import numpy as np
import torch

from conftest import oracle, pkg

ATOL = 1e-2          # bf16 output within atol=rtol=1e-2
RTOL = 1e-2
MIN_PASS = 0.999     # ... on >= 99.9% of elements


def run_gpu(acts_gpu, w_gpu, scale=2.5, offset=None):
    """One DPS call through the public binding, with the routing outputs."""
    m = pkg()
    T = acts_gpu.logits.shape[0]
    dev = acts_gpu.logits.device
    out = torch.full((T, 7168), float("nan"), dtype=torch.bfloat16, device=dev)
    ids = torch.full((T, 8), -7, dtype=torch.int32, device=dev)
    wts = torch.zeros((T, 8), dtype=torch.float32, device=dev)
    cnt = torch.full((w_gpu.e_local,), -1, dtype=torch.int32, device=dev)
    m.kernel_ex(acts_gpu.logits, acts_gpu.bias, acts_gpu.hidden, acts_gpu.hidden_scale, w_gpu.w13, w_gpu.s13,
                w_gpu.w2, w_gpu.s2, w_gpu.offset if offset is None else offset, scale, out, ids, wts, cnt)
    torch.cuda.synchronize()
    assert m.device_status() == 0
    return out, ids, wts, cnt


def check_routing(routing, ids_gpu, counts_gpu, offset, e_local):
    """Expert-id sets per token bit-exact (ties within 4 ulps reported, not
    failed); per-expert counts bit-exact when no tie flipped an id."""
    O = oracle()
    ids = np.sort(ids_gpu.cpu().numpy().astype(np.int64), axis=1)
    ref = np.sort(routing["topk_idx"].astype(np.int64), axis=1)
    mism = np.nonzero((ids != ref).any(axis=1))[0]
    ties = [int(t) for t in mism if O.routing_mismatch_is_tie(routing, int(t))]
    hard = sorted(set(int(t) for t in mism) - set(ties))
    assert not hard, f"routing differs at tokens {hard[:10]} without a near-tie"
    if not ties:
        np.testing.assert_array_equal(counts_gpu.cpu().numpy(), O.local_counts(routing["topk_idx"], offset, e_local))
    return ties


def check_weights(routing, ids_gpu, w_gpu):
    """Routing weights equal the reference's dense weights at the chosen ids."""
    ids = ids_gpu.cpu().numpy().astype(np.int64)
    w = w_gpu.cpu().numpy()
    ref = np.take_along_axis(routing["weights"], ids, axis=1)
    np.testing.assert_allclose(w, ref, rtol=2e-6, atol=1e-7)


def check_output(out_gpu_bf16, ref_f32, rows=None, min_pass=MIN_PASS):
    O = oracle()
    got = out_gpu_bf16.float().cpu().numpy()
    if rows is not None:
        got = got[rows]
    ref = O.bf16_bits_to_f32(O.f32_to_bf16_bits(ref_f32))
    assert np.isfinite(got).all(), "non-finite output"
    frac = O.allclose_fraction(got, ref, ATOL, RTOL)
    err = float(np.max(np.abs(got - ref))) if got.size else 0.0
    assert frac >= min_pass, f"only {frac:.5f} of elements within atol=rtol=1e-2 (max abs err {err:.4g})"
    return frac, err
