"""CPU: the oracle of the step after the layer (residual add + DeepSeek-V3
RMSNorm + 1x128 FP8 quantisation) against the model's own definition, HF
transformers' DeepseekV3RMSNorm run by torch on the CPU."""
import numpy as np
import torch

from conftest import oracle


def _hf_rmsnorm(h_bf16: torch.Tensor, w_bf16: torch.Tensor, eps: float) -> torch.Tensor:
    """DeepseekV3RMSNorm.forward (transformers, models/deepseek_v3), restated
    so that the test does not depend on the model class being importable."""
    hs = h_bf16.to(torch.float32)
    var = hs.pow(2).mean(-1, keepdim=True)
    hs = hs * torch.rsqrt(var + eps)
    return w_bf16 * hs.to(torch.bfloat16)


def add_norm_inputs(T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, 7168, generator=g).to(torch.bfloat16)                  # layer output
    res = (torch.randn(T, 7168, generator=g) * 4.0).to(torch.bfloat16)       # residual stream
    w = (1.0 + 0.1 * torch.randn(7168, generator=g)).to(torch.bfloat16)      # norm weight
    if T >= 3:
        x[0] = 0.0
        res[0] = 0.0                       # all-zero row: y = 0, every scale 1e-12
        res[1] = -x[1]                     # exact cancellation in the residual add
        x[2, :64] = 3.0e4                  # one dominant block
    return x, res, w


def test_residual_add_and_rmsnorm_match_the_model_definition():
    O = oracle()
    eps = 1e-6
    x, res, w = add_norm_inputs(64, 5)
    h_t = res + x                                          # bf16 add, as the decoder layer does
    y_t = _hf_rmsnorm(h_t, w, eps)
    h, q, s = O.add_rmsnorm_quant(O.as_f32(x), O.as_f32(res), O.as_f32(w), eps)
    np.testing.assert_array_equal(h, O.as_f32(h_t))
    # the oracle's y, recovered through its own quantisation, is the model's y
    # up to the order of a float32 sum and one rsqrt rounding: bf16 y values
    # may differ by one bf16 step on a few elements
    q_t, s_t = O.quant_rows_1x128(O.as_f32(y_t))
    same = np.mean(q == q_t)
    assert same >= 0.999, same
    np.testing.assert_allclose(s, s_t, rtol=2 ** -7, atol=0)


def test_without_weight_is_add_then_quantise_and_without_residual_is_x():
    O = oracle()
    x, res, _ = add_norm_inputs(8, 6)
    h, q, s = O.add_rmsnorm_quant(O.as_f32(x), O.as_f32(res), None)
    q2, s2 = O.quant_rows_1x128(O.as_f32(res + x))
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s, s2)
    h, q, s = O.add_rmsnorm_quant(O.as_f32(x), None, None)
    np.testing.assert_array_equal(h, O.as_f32(x))
