"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the contest workloads themselves are not
available; these stand in for them):

* routing_logits f32 [T, 256] ~ N(0, 1)
* routing_bias bf16 [256] ~ N(0, 0.1) (skewed configs: +2.0 on 4 hot experts)
* hidden bf16 [T, 7168] ~ N(0, 1), quantised to e4m3 per 1x128 block with
  scale = amax / 448; scales stored transposed as f32 [56, T]
* W13 [E_l, 4096, 7168] and W2 [E_l, 7168, 2048] ~ N(0, 0.02), quantised per
  128x128 block (scale = amax / 448) -> f32 [E_l, 32, 56] and [E_l, 56, 16]

Activations always come from a CPU ``torch.Generator`` seeded with ``seed``.
Weights of global expert ``g`` come from a generator seeded with
``weight_seed * 1_000_003 + g`` on ``weight_device``, so every rank layout
(1 GPU with experts 0..31, or EP shards) sees identical per-expert weights.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

H, I, E, BLK = 7168, 2048, 256, 128
FP8_MAX = 448.0
HOT_EXPERTS_LOCAL = (0, 1, 2, 3)


def quant_rows_1x128(x: torch.Tensor):
    """[T, K] float -> (e4m3 [T, K], f32 scales [K/128, T])."""
    T, K = x.shape
    xb = x.float().view(T, K // BLK, BLK)
    s = (xb.abs().amax(-1) / FP8_MAX).clamp_min(1e-12)
    q = (xb / s[..., None]).to(torch.float8_e4m3fn).view(T, K)
    return q, s.t().contiguous()


def quant_blocks_128x128(w: torch.Tensor):
    """[N, K] float -> (e4m3 [N, K], f32 scales [N/128, K/128])."""
    N, K = w.shape
    wb = w.float().view(N // BLK, BLK, K // BLK, BLK)
    s = (wb.abs().amax(dim=(1, 3)) / FP8_MAX).clamp_min(1e-12)
    q = (wb / s[:, None, :, None]).to(torch.float8_e4m3fn).view(N, K)
    return q, s.contiguous()


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


@dataclass
class Weights:
    w13: torch.Tensor   # e4m3 [E_l, 4096, 7168]
    s13: torch.Tensor   # f32  [E_l, 32, 56]
    w2: torch.Tensor    # e4m3 [E_l, 7168, 2048]
    s2: torch.Tensor    # f32  [E_l, 56, 16]
    offset: int

    @property
    def e_local(self) -> int:
        return self.w13.shape[0]

    def to(self, device) -> "Weights":
        return Weights(self.w13.to(device), self.s13.to(device), self.w2.to(device), self.s2.to(device), self.offset)

    def expert_cpu(self, le: int):
        """(w13, s13, w2, s2) of local expert ``le`` on the CPU."""
        return (self.w13[le].cpu(), self.s13[le].cpu(), self.w2[le].cpu(), self.s2[le].cpu())


def expert_weights(g: int, device="cpu", weight_seed: int = 0):
    """Quantised weights of global expert ``g``."""
    gen = _gen(weight_seed * 1_000_003 + g, device)
    w13 = torch.randn(2 * I, H, generator=gen, device=device) * 0.02
    q13, s13 = quant_blocks_128x128(w13)
    del w13
    w2 = torch.randn(H, I, generator=gen, device=device) * 0.02
    q2, s2 = quant_blocks_128x128(w2)
    return q13, s13, q2, s2


def make_weights(e_local: int = 32, offset: int = 0, device="cpu", weight_seed: int = 0) -> Weights:
    dev = torch.device(device)
    w13 = torch.empty((e_local, 2 * I, H), dtype=torch.float8_e4m3fn, device=dev)
    s13 = torch.empty((e_local, 2 * I // BLK, H // BLK), dtype=torch.float32, device=dev)
    w2 = torch.empty((e_local, H, I), dtype=torch.float8_e4m3fn, device=dev)
    s2 = torch.empty((e_local, H // BLK, I // BLK), dtype=torch.float32, device=dev)
    for le in range(e_local):
        q13, a13, q2, a2 = expert_weights(offset + le, dev, weight_seed)
        w13[le].copy_(q13)
        s13[le].copy_(a13)
        w2[le].copy_(q2)
        s2[le].copy_(a2)
    return Weights(w13, s13, w2, s2, offset)


@dataclass
class Activations:
    logits: torch.Tensor        # f32 [T, 256]
    bias: torch.Tensor          # bf16 [256]
    hidden: torch.Tensor        # e4m3 [T, 7168]
    hidden_scale: torch.Tensor  # f32 [56, T]

    @property
    def T(self) -> int:
        return self.logits.shape[0]

    def to(self, device) -> "Activations":
        return Activations(self.logits.to(device), self.bias.to(device), self.hidden.to(device),
                           self.hidden_scale.to(device))


def make_activations(T: int, seed: int, skew_hot: tuple | None = None, skew: float = 2.0) -> Activations:
    """CPU tensors. ``skew_hot``: global expert ids whose bias gets ``+skew``."""
    g = _gen(seed, "cpu")
    logits = torch.randn(T, E, generator=g)
    bias = torch.randn(E, generator=g) * 0.1
    if skew_hot:
        bias[list(skew_hot)] += skew
    bias = bias.to(torch.bfloat16)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    hidden, hscale = quant_rows_1x128(x) if T > 0 else (
        torch.empty((0, H), dtype=torch.float8_e4m3fn), torch.empty((H // BLK, 0)))
    return Activations(logits.contiguous(), bias.contiguous(), hidden.contiguous(), hscale.contiguous())


# Benchmark configurations (seed = T; skewed prefill puts the 4 hot experts in
# the first local group).
DECODE_T = (1, 2, 4, 8, 16, 32, 64)
MID_T = (256, 1024)
LARGE_T = (4096, 8192, 16384)


def config_activations(T: int, offset: int = 0, rank: int = 0) -> Activations:
    skew = tuple(offset + h for h in HOT_EXPERTS_LOCAL) if T in LARGE_T else None
    return make_activations(T, seed=rank * 1_000_000 + T, skew_hot=skew)


def moe_flops(n_assign: int) -> int:
    """Algorithmic FLOPs of one call: GEMM1 2*7168*4096 + GEMM2 2*2048*7168 per
    (token, local expert) pair (scripts/run_modal.py:67-81 uses the same
    per-pair figure with the expected pair count)."""
    return int(n_assign) * (2 * H * 2 * I + 2 * I * H)


def moe_bytes(T: int, e_touched: int) -> int:
    """Algorithmic HBM bytes of one call: every touched expert's e4m3 weights
    and scales once, plus per token its logits, e4m3 row, scales and bf16
    output, plus the bias."""
    per_expert = 2 * I * H + H * I + (2 * I // BLK) * (H // BLK) * 4 + (H // BLK) * (I // BLK) * 4
    per_token = E * 4 + H + (H // BLK) * 4 + H * 2
    return e_touched * per_expert + T * per_token + E * 2
