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
