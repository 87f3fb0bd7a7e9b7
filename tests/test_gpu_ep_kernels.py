"""GPU (one device, no NCCL): the expert-parallel row exchange kernels
(moe_fp8_ds_ep_pack / _unpack / _combine) against their torch restatement in
flashinfer-mlsys_b200/ep.py, bit-exact, for 2, 4 and 8 ranks."""
import importlib

import pytest
import torch

from conftest import ROOT  # noqa: F401  (puts the repository on sys.path)

pytestmark = pytest.mark.gpu


def _ep():
    return importlib.import_module("flashinfer-mlsys_b200.ep")


def _plan(ids, world):
    """dispatch_plan without the count exchange (one rank's view)."""
    ep = _ep()
    T = ids.shape[0]
    e_local = 256 // world
    dest = torch.zeros((world, T), dtype=torch.bool)
    dest.scatter_(0, (ids.long() // e_local).t().contiguous(), True)
    send_idx = torch.nonzero(dest.reshape(-1)).flatten() % T
    counts = dest.sum(dim=1).tolist()
    return ep.Plan(send_idx, counts, counts)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_pack_unpack_combine_match_torch(gpu_available, world):
    ep = _ep()
    g = torch.Generator().manual_seed(world)
    T = 333
    hidden = torch.randint(0, 256, (T, 7168), generator=g, dtype=torch.uint8)
    hidden[hidden == 0x7F] = 0  # no NaN codes
    hidden = hidden.view(torch.float8_e4m3fn)
    scale = torch.rand(56, T, generator=g)
    ids = torch.stack([torch.randperm(256, generator=g)[:8] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, 8, generator=g)
    plan = _plan(ids, world)
    dev = "cuda"
    buf_c = ep.pack_rows(hidden, scale, ids, w, plan.send_idx)
    buf_g = ep.pack_rows(hidden.to(dev), scale.to(dev), ids.to(dev), w.to(dev), plan.send_idx.to(dev))
    assert torch.equal(buf_g.cpu(), buf_c)
    parts_c = ep.unpack_rows(buf_c)
    parts_g = ep.unpack_rows(buf_g)
    for a, b in zip(parts_c, parts_g):
        assert torch.equal(a.view(torch.uint8) if a.dtype == torch.float8_e4m3fn else a,
                           (b.view(torch.uint8) if b.dtype == torch.float8_e4m3fn else b).cpu())
    S = plan.send_idx.numel()
    back = torch.randn(S, 7168, generator=g).to(torch.bfloat16)
    out_c = ep.combine_rows(back, plan, T, world)
    plan_g = ep.Plan(plan.send_idx.to(dev), plan.send_counts, plan.recv_counts)
    out_g = ep.combine_rows(back.to(dev), plan_g, T, world)
    torch.cuda.synchronize()
    assert torch.equal(out_g.cpu(), out_c)


def test_empty_exchange(gpu_available):
    ep = _ep()
    dev = "cuda"
    T = 4
    plan = ep.Plan(torch.empty(0, dtype=torch.int64, device=dev), [0, 0], [0, 0])
    out = ep.combine_rows(torch.empty((0, 7168), dtype=torch.bfloat16, device=dev), plan, T, 2)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out.float()).item() == 0


@pytest.mark.parametrize("world", [1, 2, 4, 8, 64])
@pytest.mark.parametrize("T", [1, 77, 1024, 3001])
def test_dispatch_plan_kernel_matches_restatement(gpu_available, world, T):
    """moe_fp8_ds_ep_plan (one CTA, ballot scan per rank) against the torch
    restatement: send order, per-rank counts and the combine's row map,
    bit-exact."""
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    g = torch.Generator().manual_seed(world * 10000 + T)
    ids = torch.stack([torch.randperm(256, generator=g)[:8] for _ in range(T)]).to(torch.int32)
    if T > 10:
        ids[3] = torch.arange(8, dtype=torch.int32)        # every expert on rank 0
        ids[5] = torch.arange(248, 256, dtype=torch.int32)  # every expert on the last rank
    o_ref, c_ref, r_ref = ep.plan_local(ids, world)
    o, c, r = ep.plan_cuda(ids.cuda(), world)
    torch.cuda.synchronize()
    n = int(c_ref.sum())
    assert torch.equal(c.cpu(), c_ref)
    assert torch.equal(o[:n].cpu(), o_ref[:n])
    assert torch.equal(r.cpu(), r_ref)
