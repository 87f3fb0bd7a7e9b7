"""CPU (gloo, 2 ranks): expert-parallel dispatch/combine bookkeeping.

The EP layer must give every token the same result as one process holding
all 256 experts. The expert computation here is a cheap deterministic
stand-in with a different linear map per expert, so every
routing/packing/permutation mistake shows up."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

H = 7168


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_route(logits, bias, scale):
    O = importlib.import_module("oracle.moe_oracle")
    r = O.route(logits.numpy(), O.as_f32(bias), scale)
    ids = torch.from_numpy(r["topk_idx"].astype(np.int32))
    w = torch.from_numpy(np.take_along_axis(r["weights"], r["topk_idx"], axis=1).astype(np.float32))
    return ids, w


def _fake_experts(hidden, scale, ids, w, offset, out, e_local):
    """out[r] = sum over local experts e of w * (e + 1) / 256 * dequant(hidden[r])
    (a per-expert linear map, summed in ascending expert id)."""
    O = importlib.import_module("oracle.moe_oracle")
    a = torch.from_numpy(O.dequant_rows(O.as_u8(hidden), scale.numpy()))
    acc = torch.zeros_like(a)
    order = torch.argsort(ids.long(), dim=1)
    for k in range(ids.shape[1]):
        e = torch.gather(ids.long(), 1, order[:, k:k + 1]).squeeze(1)
        wk = torch.gather(w, 1, order[:, k:k + 1]).squeeze(1)
        loc = (e >= offset) & (e < offset + e_local)
        f = torch.where(loc, wk * (e.float() + 1.0) / 256.0, torch.zeros_like(wk))
        acc += f[:, None] * a
    out.copy_(acc.to(out.dtype))


def _worker(rank, world, port, T, combine, skew_zero_rank, result_dir):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    acts = wl.make_activations(T, seed=rank * 1_000_000 + T)
    if skew_zero_rank:
        # no token may pick the last rank's experts: it receives nothing
        b = acts.bias.float()
        b[128:] -= 10.0
        acts.bias = b.to(torch.bfloat16)
    e_local = 256 // world
    dtype = torch.float32 if combine == "f32" else torch.bfloat16
    plans = []
    out = ep.ep_forward(acts.logits, acts.bias, acts.hidden, acts.hidden_scale, 2.5, _oracle_route,
                        lambda h, s, i, w, off, o: _fake_experts(h, s, i, w, off, o, e_local),
                        combine_dtype=dtype, plan_out=plans)
    # same tokens, one process holding all 256 experts
    ids, w = _oracle_route(acts.logits, acts.bias, 2.5)
    full = torch.empty((T, H), dtype=torch.float32)
    _fake_experts(acts.hidden, acts.hidden_scale, ids, w, 0, full, 256)
    torch.save({"out": out, "full": full, "send": plans[0].send_counts, "recv": plans[0].recv_counts},
               os.path.join(result_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _run(tmp_path, T, combine, skew_zero_rank=False, world=2):
    mp.start_processes(_worker, args=(world, _free_port(), T, combine, skew_zero_rank, str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    return [torch.load(os.path.join(tmp_path, f"r{r}.pt")) for r in range(world)]


@pytest.mark.timeout(300)
def test_ep_matches_single_process_f32(tmp_path):
    res = _run(tmp_path, 24, "f32")
    for r in res:
        ref = r["full"].to(torch.bfloat16).float()
        got = r["out"].float()
        torch.testing.assert_close(got, ref, rtol=1e-2, atol=1e-2)
        # the fp32 sum differs from the single-process order only by rounding
        assert (got == ref).float().mean().item() > 0.99
    # the row counts each rank sends are what the other receives
    assert res[0]["send"][1] == res[1]["recv"][0] and res[1]["send"][0] == res[0]["recv"][1]


@pytest.mark.timeout(300)
def test_ep_bf16_combine_and_empty_rank(tmp_path):
    res = _run(tmp_path, 16, "bf16", skew_zero_rank=True)
    for r in res:
        torch.testing.assert_close(r["out"].float(), r["full"].to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
    assert res[0]["send"][1] == 0 and res[1]["send"][1] == 0  # nobody routes to rank 1's experts


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [4, 8])
def test_ep_four_and_eight_ranks(tmp_path, world):
    """4 and 8 ranks (64 / 32 experts each): every rank's output equals the
    single-process layer, and the send/recv matrix is consistent."""
    res = _run(tmp_path, 20, "f32", world=world)
    for r in res:
        torch.testing.assert_close(r["out"].float(), r["full"].to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
    for a in range(world):
        for b in range(world):
            assert res[a]["send"][b] == res[b]["recv"][a]
    assert sum(sum(r["send"]) for r in res) > 0


def test_pack_unpack_round_trip():
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    a = wl.make_activations(10, seed=7)
    ids = torch.randint(0, 256, (10, 8), dtype=torch.int32)
    w = torch.rand(10, 8)
    idx = torch.tensor([3, 0, 9, 3])
    h, s, i, ww = ep.unpack_rows(ep.pack_rows(a.hidden, a.hidden_scale, ids, w, idx))
    assert torch.equal(h.view(torch.uint8), a.hidden.view(torch.uint8)[idx])
    assert torch.equal(s, a.hidden_scale[:, idx])
    assert torch.equal(i, ids[idx]) and torch.equal(ww, w[idx])


def test_plan_local_row_map_matches_send_order():
    """The torch restatement of the dispatch-plan kernel: row_of[t][q] is the
    position of token t in the send order for rank q, and the send order lists
    each rank's tokens ascending."""
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    g = torch.Generator().manual_seed(3)
    for world in (1, 2, 4, 8):
        ids = torch.stack([torch.randperm(256, generator=g)[:8] for _ in range(50)]).to(torch.int32)
        order, counts, row_of = ep.plan_local(ids, world)
        total = int(counts.sum())
        off = 0
        for q in range(world):
            n = int(counts[q])
            toks = order[off:off + n]
            assert torch.all(toks[1:] > toks[:-1])
            want = ((ids.long() // (256 // world)) == q).any(dim=1).nonzero().flatten()
            assert torch.equal(toks, want)
            assert torch.equal(row_of[toks, q].long(), torch.arange(off, off + n))
            off += n
        assert off == total and int((row_of >= 0).sum()) == total
