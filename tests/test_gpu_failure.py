"""GPU: a device-side bounded wait that runs out, in an allowed form.

Calls with more than 8 tokens route in one cooperative kernel whose CTAs meet
at a grid barrier (a global-memory poll with a 2 s limit). A test-only hook
lowers the limit to 1 ms and keeps one CTA away from the barrier, so the
others give up: they set the library's device status bit and return. The host
must read MOE_ERR_DEVICE_TIMEOUT, the flag must clear, and the next normal
call must match the oracle. Nothing faults, traps or hangs: the wait that runs
out is a flag that nothing sets."""
import pytest
import torch

from conftest import oracle, pkg, workloads
from parity import check_output, check_routing, run_gpu

pytestmark = pytest.mark.gpu

DEV = "cuda"
MOE_ERR_DEVICE_TIMEOUT = 6


def test_route_barrier_timeout_is_reported_and_the_next_call_recovers(gpu_available):
    m = pkg()
    lib = m.load()
    wl = workloads()
    w = wl.make_weights(32, 0, DEV, weight_seed=0)
    acts = wl.make_activations(256, seed=7)
    a = acts.to(DEV)
    out = torch.empty((256, 7168), dtype=torch.bfloat16, device=DEV)
    assert m.device_status() == 0
    lib.moe_fp8_ds_test_route_barrier(1_000_000, 1)  # 1 ms limit, CTA 1 stays away
    try:
        m.kernel(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, 0, 2.5, out)
        rc = m.device_status()
    finally:
        lib.moe_fp8_ds_test_route_barrier(0, -1)
    assert rc == MOE_ERR_DEVICE_TIMEOUT
    assert m.device_status() == 0  # read once, then cleared
    # the same call again, normally: parity with the CPU oracle
    got, ids, wts, cnt = run_gpu(a, w)
    O = oracle()
    ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                        lambda le: w.expert_cpu(le), 0, 2.5, 32)
    check_routing(ref["routing"], ids, cnt, 0, 32)
    check_output(got, ref["out_f32"])
