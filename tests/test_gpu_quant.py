"""GPU: the BF16 -> FP8 1x128 activation quantiser (moe_fp8_ds_quantize_act)
against the oracle, bit-exact, and feeding the layer."""
import numpy as np
import pytest
import torch

from conftest import oracle, pkg, workloads
from parity import check_output, run_gpu
from test_quant_cpu import _inputs

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("T", [1, 3, 8, 64, 1000, 4096])
def test_quantiser_bit_exact(gpu_available, T):
    O = oracle()
    x = _inputs(T, 10 + T)
    q, s = pkg().quantize_activations(x.to(DEV))
    torch.cuda.synchronize()
    q_o, s_o = O.quant_rows_1x128(O.as_f32(x))
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), q_o)
    np.testing.assert_array_equal(s.cpu().numpy(), s_o)


def test_quantiser_writes_given_outputs_and_handles_empty(gpu_available):
    m = pkg()
    x = _inputs(5, 77).to(DEV)
    q = torch.empty((5, 7168), dtype=torch.float8_e4m3fn, device=DEV)
    s = torch.empty((56, 5), dtype=torch.float32, device=DEV)
    q2, s2 = m.quantize_activations(x, q, s)
    assert q2.data_ptr() == q.data_ptr() and s2.data_ptr() == s.data_ptr()
    e = torch.empty((0, 7168), dtype=torch.bfloat16, device=DEV)
    q0, s0 = m.quantize_activations(e)
    assert q0.shape == (0, 7168) and s0.shape == (56, 0)
    with pytest.raises(ValueError):
        m.quantize_activations(x.float())


def test_quantised_activations_feed_the_layer(gpu_available):
    """BF16 hidden states -> quantiser -> layer, against the oracle on the
    same quantised inputs."""
    T = 16
    acts = workloads().make_activations(T, seed=123)
    # BASELINE's hidden-state distribution (bf16 ~N(0,1)); the edge-case rows of
    # _inputs stress the quantiser, not the layer
    x = torch.randn(T, 7168, generator=torch.Generator().manual_seed(321)).to(torch.bfloat16)
    q, s = pkg().quantize_activations(x.to(DEV))
    acts.hidden, acts.hidden_scale = q.cpu(), s.cpu()
    w = workloads().make_weights(32, 0, DEV, weight_seed=0)
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w)
    O = oracle()
    ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                        lambda le: w.expert_cpu(le), 0, 2.5, 32)
    check_output(out, ref["out_f32"])
