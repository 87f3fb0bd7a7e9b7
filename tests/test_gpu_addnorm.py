"""GPU: the step after the layer (moe_fp8_ds_add_norm_quant: residual add +
DeepSeek-V3 RMSNorm + 1x128 FP8 quantisation) against the oracle, bit-exact:
the residual written back, the e4m3 bytes and the scales."""
import numpy as np
import pytest
import torch

from conftest import oracle, pkg
from test_addnorm_cpu import add_norm_inputs

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("T,residual,weight", [(1, True, True), (3, True, True), (64, True, True),
                                               (1000, True, True), (64, False, True), (64, True, False),
                                               (9, False, False)])
def test_add_norm_quant_bit_exact(gpu_available, T, residual, weight):
    O = oracle()
    x, res, w = add_norm_inputs(T, 40 + T)
    eps = 1e-6
    res_d = res.to(DEV) if residual else None
    q, s = pkg().add_rmsnorm_quantize(x.to(DEV), res_d, w.to(DEV) if weight else None, eps)
    torch.cuda.synchronize()
    h, q_o, s_o = O.add_rmsnorm_quant(O.as_f32(x), O.as_f32(res) if residual else None,
                                      O.as_f32(w) if weight else None, eps)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), q_o)
    np.testing.assert_array_equal(s.cpu().numpy(), s_o)
    if residual:
        np.testing.assert_array_equal(O.as_f32(res_d.cpu()), h)


def test_add_norm_quant_after_the_layer_output(gpu_available):
    """The layer's bf16 output feeds the step; the residual update equals
    torch's bf16 add and the norm matches the oracle at eps = 1e-5."""
    O = oracle()
    T = 256
    g = torch.Generator().manual_seed(3)
    out = (torch.randn(T, 7168, generator=g) * 0.05).to(torch.bfloat16)
    res = torch.randn(T, 7168, generator=g).to(torch.bfloat16)
    w = torch.rand(7168, generator=g).to(torch.bfloat16)
    res_d = res.to(DEV)
    q, s = pkg().add_rmsnorm_quantize(out.to(DEV), res_d, w.to(DEV), 1e-5)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(res_d), _bits(res + out))
    _, q_o, s_o = O.add_rmsnorm_quant(O.as_f32(out), O.as_f32(res), O.as_f32(w), 1e-5)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), q_o)
    np.testing.assert_array_equal(s.cpu().numpy(), s_o)


def test_add_norm_quant_arguments(gpu_available):
    m = pkg()
    x = torch.randn(4, 7168, device=DEV).to(torch.bfloat16)
    e = torch.empty((0, 7168), dtype=torch.bfloat16, device=DEV)
    q0, s0 = m.add_rmsnorm_quantize(e, e.clone(), None)
    assert q0.shape == (0, 7168) and s0.shape == (56, 0)
    with pytest.raises(ValueError):
        m.add_rmsnorm_quantize(x, None, None, eps=-1.0)
    with pytest.raises(ValueError):
        m.add_rmsnorm_quantize(x, x.float(), None)
    with pytest.raises(ValueError):
        m.add_rmsnorm_quantize(x, None, torch.ones(7000, dtype=torch.bfloat16, device=DEV))
