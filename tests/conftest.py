import functools
import glob
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running test")


def pkg():
    """The product package (its directory name has a hyphen)."""
    return importlib.import_module("flashinfer-mlsys_b200")


def workloads():
    return importlib.import_module("flashinfer-mlsys_b200.workloads")


def oracle():
    return importlib.import_module("oracle.moe_oracle")


@functools.lru_cache(maxsize=4)
def cpu_weights(offset: int, e_local: int = 32):
    """CPU-generated weights (the bytes the golden fixtures were made from)."""
    return workloads().make_weights(e_local, offset, "cpu", weight_seed=0)


def golden_cases():
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))


def golden_activations(g):
    wl = workloads()
    hot = tuple(int(h) for h in g["hot"]) or None
    return wl.make_activations(int(g["T"]), int(g["seed"]), skew_hot=hot)


@pytest.fixture(scope="session")
def gpu_available():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
