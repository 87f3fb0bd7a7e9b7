"""CPU: the benchmark's reference arm (the driver runs it at every round end)
prints one JSON line with the contract's keys, timing the oracle port on the
host cores."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT


@pytest.mark.timeout(600)
def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=580, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is False
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert "workload" in d["config"]


def test_reference_and_our_arm_share_the_config_keys():
    """The driver compares the two arms' `config`; both build it with the same
    function, for the default workload at every N and for the T sweep."""
    sys.path.insert(0, ROOT)
    import bench

    for world in (1, 2, 4, 8):
        c = bench._config("ep", world, (4096,))
        assert c["num_local_experts"] == 256 // world and c["T_per_gpu"] == 4096
        assert c["parallelism"] == f"ep{world}"
    for name in bench.SWEEP:
        assert bench._config(name, 1, bench.WORKLOADS[name][0])["T"] == list(bench.WORKLOADS[name][0])


@pytest.mark.parametrize("T", [1, 7, 64, 300])
def test_packed_end_to_end_inputs(monkeypatch, T):
    """The end-to-end step moves a call's inputs with one copy of a packed
    buffer: every input tensor is a contiguous view of it at a 16-byte-aligned
    offset, with its source's dtype, shape and bytes (checked here with a
    CPU 'device' buffer; page-locking needs a GPU)."""
    import torch

    sys.path.insert(0, ROOT)
    import bench
    from conftest import workloads

    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    a = workloads().make_activations(T, seed=T)
    host, buf, v = bench._packed_inputs(a, "cpu")
    assert host.dtype == torch.uint8 and host.numel() == buf.numel()
    buf.copy_(host)
    for got, ref in ((v.logits, a.logits), (v.bias, a.bias), (v.hidden, a.hidden), (v.hidden_scale, a.hidden_scale)):
        assert got.dtype == ref.dtype and tuple(got.shape) == tuple(ref.shape) and got.is_contiguous()
        assert (got.data_ptr() - buf.data_ptr()) % 16 == 0
        assert torch.equal(got.reshape(-1).view(torch.uint8), ref.reshape(-1).view(torch.uint8))
