"""CPU: pin the numpy oracle to the reference's own outputs (golden fixtures
made by tests/golden/make_golden.py from ref_moe.run)."""
import hashlib

import numpy as np
import pytest
import torch

from conftest import cpu_weights, golden_activations, golden_cases, load_golden, oracle


def _sha(t):
    t = t.contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16):
        t = t.view(torch.uint8)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("name", golden_cases())
def test_inputs_regenerate_bit_identically(name):
    g = load_golden(name)
    a = golden_activations(g)
    assert _sha(a.logits) == str(g["sha_logits"])
    assert _sha(a.bias) == str(g["sha_bias"])
    assert _sha(a.hidden) == str(g["sha_hidden"])
    assert _sha(a.hidden_scale) == str(g["sha_hidden_scale"])


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_reference_golden(name):
    O = oracle()
    g = load_golden(name)
    a = golden_activations(g)
    w = cpu_weights(int(g["offset"]))
    res = O.moe_forward(a.logits.numpy(), O.as_f32(a.bias), O.as_u8(a.hidden), a.hidden_scale.numpy(),
                        lambda le: w.expert_cpu(le), int(g["offset"]), float(g["scale"]), 32)
    # routing: expert id sets per token and per-expert counts are bit-exact
    ids = np.sort(res["topk_idx"], axis=1)
    mism = np.nonzero((ids != g["topk_idx_sorted"]).any(axis=1))[0]
    for t in mism:
        assert O.routing_mismatch_is_tie(res["routing"], int(t)), f"token {t}: routing differs without a tie"
    if len(mism) == 0:
        np.testing.assert_array_equal(res["counts"], g["counts"])
    # output: same bf16 result up to fp32 summation order
    ref = O.bf16_bits_to_f32(g["out_bf16"])
    got = O.bf16_bits_to_f32(res["out_bf16"])
    frac = O.allclose_fraction(got, ref, atol=1e-2, rtol=1e-2)
    assert frac == 1.0, f"{name}: oracle/reference agreement {frac}"
    # and nearly always the very same bits
    same = float(np.mean(res["out_bf16"] == g["out_bf16"]))
    assert same > 0.99, f"{name}: only {same:.4f} of bf16 outputs bit-identical"


def test_routing_oracle_properties():
    """Structural invariants of ref_moe.py:95-126 on a random batch."""
    O = oracle()
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((512, 256)).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.1).astype(np.float32)
    r = O.route(logits, bias, 2.5)
    idx = r["topk_idx"]
    # 8 distinct experts drawn from exactly the 4 selected groups
    assert all(len(set(row)) == 8 for row in idx)
    for t in range(idx.shape[0]):
        assert set(idx[t] // 32) <= set(r["group_idx"][t])
    # weights: nonzero exactly at the selected experts, sum = scaling factor
    nz = (r["weights"] != 0).sum(axis=1)
    assert (nz == 8).all()
    np.testing.assert_allclose(r["weights"].sum(axis=1), 2.5, rtol=1e-5)


def test_bf16_rounding_matches_torch():
    O = oracle()
    x = torch.randn(10000) * 100
    ours = O.f32_to_bf16_bits(x.numpy())
    theirs = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, theirs)


def test_e4m3_table_matches_torch():
    O = oracle()
    b = torch.arange(256, dtype=torch.uint8)
    f = b.view(torch.float8_e4m3fn).float().numpy()
    ok = np.isnan(f) == np.isnan(O.E4M3)
    assert ok.all()
    np.testing.assert_array_equal(f[~np.isnan(f)], O.E4M3[~np.isnan(f)])
