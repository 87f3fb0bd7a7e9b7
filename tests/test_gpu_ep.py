"""GPU, 2, 4 and 8 ranks over NCCL: the expert-parallel layer (routing on
each rank, all-to-all dispatch, moe_fp8_ds_experts on the owner, all-to-all
return, fp32 combine) against the CPU oracle of the full 256-expert layer, on
32 tokens of every rank. Each case is skipped when fewer GPUs are visible."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, n_rows, result_dir):
    import sys
    import datetime

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    O = importlib.import_module("oracle.moe_oracle")
    dev = torch.device("cuda", rank)
    e_local = 256 // world
    w = wl.make_weights(e_local, rank * e_local, dev)
    acts = wl.make_activations(T, seed=rank * 1_000_000 + T)
    a = acts.to(dev)
    out = ep.ep_forward(a.logits, a.bias, a.hidden, a.hidden_scale, 2.5, ep.cuda_route_fn,
                        ep.make_cuda_experts_fn(w.w13, w.s13, w.w2, w.s2))
    torch.cuda.synchronize()
    rows = np.linspace(0, T - 1, n_rows).astype(np.int64)
    got = out.float().cpu().numpy()[rows]
    del w
    dist.barrier()
    dist.destroy_process_group()
    # the oracle over all 256 experts for this rank's checked rows, after the
    # process group is gone (no collective waits while the host computes);
    # expert weights are generated on this GPU exactly as the ranks did
    torch.set_num_threads(max(1, (os.cpu_count() or 8) // world))

    def get_expert(g):
        q13, s13, q2, s2 = wl.expert_weights(g, dev, 0)
        return q13.cpu(), s13.cpu(), q2.cpu(), s2.cpu()

    ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                        get_expert, 0, 2.5, 256, token_subset=rows)
    refb = O.bf16_bits_to_f32(ref["out_bf16"])
    frac = O.allclose_fraction(got, refb, 1e-2, 1e-2)
    torch.save({"frac": frac, "rows": int(len(rows)), "finite": bool(np.isfinite(got).all())},
               os.path.join(result_dir, f"r{rank}.pt"))


@pytest.mark.timeout(1500)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_matches_oracle(gpu_available, tmp_path, world):
    """world NCCL ranks (one per GPU), 256/world experts each, 256 tokens per
    rank; 32 output rows of every rank against the 256-expert oracle."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_worker, args=(world, _free_port(), 256, 32, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        res = torch.load(os.path.join(tmp_path, f"r{r}.pt"))
        assert res["finite"] and res["rows"] == 32
        assert res["frac"] >= 0.999, (r, res)
