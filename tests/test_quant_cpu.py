"""CPU: the oracle's BF16 -> FP8 1x128 activation quantiser (the layer's input
format) is bit-identical to the torch recipe that produced every benchmark
input (flashinfer-mlsys_b200/workloads.py:quant_rows_1x128)."""
import numpy as np
import torch

from conftest import oracle, workloads


def _inputs(T, seed):
    g = torch.Generator().manual_seed(seed)
    # wide dynamic range per row, plus blocks that exercise the edges
    x = torch.randn(T, 7168, generator=g) * torch.exp(torch.randn(T, 1, generator=g) * 4.0)
    x = x.to(torch.bfloat16)
    if T >= 4:
        x[0, :128] = 0.0                      # all-zero block: scale clamps to 1e-12
        x[1, 128:256] = -0.0                  # negative zeros keep their sign
        x[2, :] = (x[2, :].float() * 1e-35).to(torch.bfloat16)  # subnormal-range inputs
        x[3, 300] = 3.0e38                    # one huge element dominates its block
    return x


def test_oracle_quantiser_matches_torch_recipe():
    O, wl = oracle(), workloads()
    for T, seed in ((1, 1), (5, 2), (64, 3), (300, 4)):
        x = _inputs(T, seed)
        q_t, s_t = wl.quant_rows_1x128(x)
        q_o, s_o = O.quant_rows_1x128(O.as_f32(x))
        np.testing.assert_array_equal(q_o, q_t.view(torch.uint8).numpy())
        np.testing.assert_array_equal(s_o, s_t.numpy())


def test_e4m3_rounding_ties_and_saturation():
    O = oracle()
    # exact values, midpoints between neighbours (ties to the even code), saturation
    vals = O.E4M3[:0x7F].astype(np.float64)
    mids = (vals[:-1] + vals[1:]) / 2.0
    y = np.concatenate([vals, mids, [448.0001, 460.0]]).astype(np.float32)
    got = O.f32_to_e4m3_rne(y)
    want = torch.from_numpy(np.minimum(y, 448.0)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(got, want)
    assert O.f32_to_e4m3_rne(np.array([-0.0], np.float32))[0] == 0x80
