"""Generate the golden fixtures by running the REFERENCE implementation
(``reference moe/ref_moe.py:run`` of vanshnawander/flashinfer-mlsys) on CPU.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/reference [case ...]

(all cases by default; naming cases regenerates only those).

Inputs are regenerated from seeds by ``flashinfer-mlsys_b200/workloads.py``
(CPU generators, so the bytes are reproducible on any machine with the same
torch build); the fixture stores input checksums so a test can prove it
rebuilt the same bytes. Stored per case: the reference's bf16 output bits,
its top-8 expert ids (captured from the reference's own final torch.topk
call, ref_moe.py:119) and the per-local-expert token counts.
"""
from __future__ import annotations

import hashlib
import importlib
import importlib.util
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
wl = importlib.import_module("flashinfer-mlsys_b200.workloads")

# name: (T, activation seed, local_expert_offset, hot experts for skew or None)
CASES = {
    "cfg0_T8": (8, 8, 0, None),
    "decode_T1": (1, 1, 0, None),
    "decode_T64": (64, 64, 0, None),
    "skew_T32": (32, 32, 0, (0, 1, 2, 3)),
    "offset224_T16": (16, 16, 224, None),
    # token counts and expert offsets of the contest's workloads (T in
    # {1, 7, 14, 15, 16, 32, 52-59, 62, 80, ...}, offsets multiples of 32)
    "contest_T7_off96": (7, 7, 96, None),
    "contest_T15_off32": (15, 15, 32, None),
    "contest_T55_off160": (55, 55, 160, None),
    "contest_T80_off192": (80, 80, 192, None),
}
SCALE = 2.5
E_LOCAL = 32


def sha(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16):
        t = t.view(torch.uint8)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def weights_digest(w: "wl.Weights") -> str:
    h = hashlib.sha256()
    for le in range(w.e_local):
        h.update(w.w13[le, ::97].view(torch.uint8).numpy().tobytes())
        h.update(w.w2[le, ::97].view(torch.uint8).numpy().tobytes())
        h.update(w.s13[le].numpy().tobytes())
        h.update(w.s2[le].numpy().tobytes())
    return h.hexdigest()


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "reference moe", "ref_moe.py")
    spec = importlib.util.spec_from_file_location("ref_moe", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference(ref, a: "wl.Activations", w: "wl.Weights"):
    captured = []
    real_topk = torch.topk

    def spy(*args, **kw):
        res = real_topk(*args, **kw)
        captured.append(res.indices.clone())
        return res

    torch.topk = spy
    try:
        out = ref.run(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, w.offset, SCALE)
    finally:
        torch.topk = real_topk
    topk_idx = captured[-1]  # the final top-8 of ref_moe.py:119
    assert topk_idx.shape == (a.T, 8)
    return out, topk_idx


def main(ref_root: str, names=None) -> None:
    torch.set_num_threads(os.cpu_count() or 1)
    ref = load_reference(ref_root)
    weights = {}
    for name, (T, seed, offset, hot) in CASES.items():
        if names and name not in names:
            continue
        if offset not in weights:
            t0 = time.time()
            weights[offset] = wl.make_weights(E_LOCAL, offset, "cpu", weight_seed=0)
            print(f"weights offset={offset}: {time.time() - t0:.1f}s", flush=True)
        w = weights[offset]
        a = wl.make_activations(T, seed, skew_hot=hot)
        t0 = time.time()
        out, idx = run_reference(ref, a, w)
        dt = time.time() - t0
        idx_np = np.sort(idx.numpy(), axis=1).astype(np.int16)
        le = idx.numpy().astype(np.int64) - offset
        counts = np.bincount(le[(le >= 0) & (le < E_LOCAL)], minlength=E_LOCAL)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            T=T, seed=seed, offset=offset, scale=SCALE, e_local=E_LOCAL,
            hot=np.array(hot if hot else [], dtype=np.int64),
            out_bf16=out.view(torch.int16).numpy().view(np.uint16),
            topk_idx_sorted=idx_np, counts=counts.astype(np.int32),
            sha_logits=sha(a.logits), sha_bias=sha(a.bias), sha_hidden=sha(a.hidden),
            sha_hidden_scale=sha(a.hidden_scale), weights_digest=weights_digest(w),
            ref_seconds=dt, torch_version=torch.__version__,
        )
        print(f"{name}: T={T} offset={offset} local_assignments={int(counts.sum())} ref {dt:.1f}s", flush=True)


if __name__ == "__main__":
    if len(sys.argv) < 2 or not os.path.isdir(sys.argv[1]):
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout> [case ...]")
    main(sys.argv[1], sys.argv[2:])
