"""CPU oracle for the fused FP8 DeepSeek-V3 MoE layer — TEST INFRASTRUCTURE.

This is a numpy restatement of the reference implementation
``reference moe/ref_moe.py:run`` (vanshnawander/flashinfer-mlsys). It exists
only to check the CUDA path: it is imported by ``tests/``, by
``__graft_entry__.smoke()`` (as the checker) and by ``bench.py``'s CPU
baseline leg. The product path never calls it.

Pinned against golden vectors produced by running the reference's own
``ref_moe.run`` on CPU (``tests/golden/make_golden.py``; fixtures in
``tests/golden/*.npz``), see ``tests/test_oracle_golden.py``.

Every step cites the reference line it follows. One deliberate deviation in
cost, not in result: the reference dequantises all local experts up front
(ref_moe.py:80-92) but only ever uses the experts some token selected
(ref_moe.py:140-144); this oracle dequantises an expert only when it is used.
"""
from __future__ import annotations

import numpy as np

H, I, E, BLOCK = 7168, 2048, 256, 128
TOP_K, N_GROUP, TOPK_GROUP = 8, 8, 4
GROUP_SIZE = E // N_GROUP


def _e4m3_table() -> np.ndarray:
    """float32 value of every e4m3fn byte (sign, 4-bit exponent bias 7,
    3-bit mantissa; exponent 0 is subnormal; 0x7f/0xff are NaN)."""
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3 = _e4m3_table()


def as_u8(x) -> np.ndarray:
    """numpy uint8 view of an e4m3 tensor (torch float8 or uint8 array)."""
    if hasattr(x, "view") and hasattr(x, "dtype") and "float8" in str(x.dtype):
        import torch  # only for the dtype view of torch inputs

        return x.detach().cpu().view(torch.uint8).numpy()
    return np.asarray(x, dtype=np.uint8)


def as_f32(x) -> np.ndarray:
    if hasattr(x, "detach"):
        import torch

        x = x.detach().cpu()
        if x.dtype == torch.bfloat16:
            return bf16_bits_to_f32(x.view(torch.int16).numpy().view(np.uint16))
        return x.float().numpy()
    return np.asarray(x, dtype=np.float32)


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit pattern (what
    ``Tensor.to(torch.bfloat16)`` does for finite values)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    out = ((u + r) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def dequant_rows(q_u8: np.ndarray, scale_kt: np.ndarray) -> np.ndarray:
    """ref_moe.py:69-78: A[t, h] = fp8[t, h] * scale[h // 128, t] (scale is [H/128, T])."""
    T = q_u8.shape[0]
    a = E4M3[q_u8].reshape(T, H // BLOCK, BLOCK)
    return (a * scale_kt.T[:, :, None]).reshape(T, H)


def dequant_blocks(q_u8: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """ref_moe.py:80-92: W[n, k] = fp8[n, k] * S[n // 128, k // 128]."""
    n, k = q_u8.shape
    w = E4M3[q_u8].reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    return (w * scale[:, None, :, None]).reshape(n, k)


def _topk_desc(x: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries per row, best first; equal values go
    to the lower index (torch.topk leaves tie order unspecified)."""
    return np.argsort(-x, axis=1, kind="stable")[:, :k]


def route(logits: np.ndarray, bias: np.ndarray, routed_scaling_factor: float):
    """DeepSeek-V3 no-aux routing, ref_moe.py:95-126.

    Returns dict with topk_idx [T, 8] (best first), weights [T, 256] (the
    reference's dense weight matrix), s, s_with_bias, group_scores, group_idx.
    """
    logits = np.asarray(logits, dtype=np.float32)
    bias = np.asarray(bias, dtype=np.float32).reshape(-1)
    T = logits.shape[0]
    one = np.float32(1.0)
    s = one / (one + np.exp(-logits))                                   # :99
    sb = (s + bias).astype(np.float32)                                  # :100
    grouped = sb.reshape(T, N_GROUP, GROUP_SIZE)                        # :104
    top2 = -np.sort(-grouped, axis=2)[:, :, :2]                         # :107
    group_scores = (top2[:, :, 0] + top2[:, :, 1]).astype(np.float32)   # :108
    group_idx = _topk_desc(group_scores, TOPK_GROUP)                    # :111
    group_mask = np.zeros((T, N_GROUP), dtype=np.float32)               # :112
    np.put_along_axis(group_mask, group_idx, 1.0, axis=1)               # :113
    score_mask = np.repeat(group_mask, GROUP_SIZE, axis=1)              # :114
    neg = np.float32(np.finfo(np.float32).min)                          # :117
    pruned = np.where(score_mask == 0, neg, sb)                         # :118
    topk_idx = _topk_desc(pruned, TOP_K)                                # :119
    M = np.zeros_like(s)                                                # :122
    np.put_along_axis(M, topk_idx, 1.0, axis=1)                         # :123
    w = s * M                                                           # :124
    wsum = w.sum(axis=1, keepdims=True, dtype=np.float32) + np.float32(1e-20)  # :125
    w = (w / wsum) * np.float32(routed_scaling_factor)                 # :126
    return {
        "topk_idx": topk_idx, "weights": w.astype(np.float32), "s": s, "s_with_bias": sb,
        "group_scores": group_scores, "group_idx": group_idx, "pruned": pruned,
    }


def local_counts(topk_idx: np.ndarray, offset: int, e_local: int) -> np.ndarray:
    """Tokens per local expert (ref_moe.py:131-144 selection rule)."""
    le = topk_idx.astype(np.int64) - int(offset)
    le = le[(le >= 0) & (le < e_local)]
    return np.bincount(le, minlength=e_local).astype(np.int64)


def _expert_ffn(hidden_u8, hidden_scale, tok, w13, s13, w2, s2):
    """One expert on tokens `tok` (ref_moe.py:148-162): dequantise, GEMM1,
    SwiGLU (silu on the second half, the first half the multiplicand), GEMM2."""
    A_e = dequant_rows(hidden_u8[tok], hidden_scale[:, tok])            # :69-78, :148
    W13 = dequant_blocks(as_u8(w13), as_f32(s13))                       # :80-86
    G1 = A_e @ W13.T                                                    # :153
    X1, X2 = G1[:, :I], G1[:, I:]                                       # :156-157
    C = (X2 / (np.float32(1.0) + np.exp(-X2))) * X1                     # :158-159
    W2 = dequant_blocks(as_u8(w2), as_f32(s2))                          # :88-92
    return C @ W2.T                                                     # :162


def moe_forward(logits, bias, hidden_u8, hidden_scale, get_expert, offset: int, routed_scaling_factor: float,
                e_local: int = 32, token_subset=None, routing=None, shared=None):
    """The whole layer (ref_moe.py:5-167) on CPU.

    get_expert(le) -> (w13_u8 [4096, 7168], s13 [32, 56], w2_u8 [7168, 2048], s2 [56, 16])
    token_subset: optional token indices; only those output rows are computed
    (each output row depends only on its own token).
    shared: optional (w13, s13, w2, s2) of an always-on shared expert. The
    reference's operator has none; this follows DeepSeek-V3's MoE block, whose
    output is the routed sum plus the shared expert applied to every token with
    weight 1. It is added to the fp32 accumulator after the routed experts,
    before the single bf16 cast.
    Returns dict: out_f32 [n, 7168], out_bf16 (uint16 bits), rows, topk_idx, counts, routing.
    """
    r = routing if routing is not None else route(logits, bias, routed_scaling_factor)
    topk_idx, weights = r["topk_idx"], r["weights"]
    T = topk_idx.shape[0]
    rows = np.arange(T) if token_subset is None else np.asarray(token_subset, dtype=np.int64)
    pos = {int(t): i for i, t in enumerate(rows)}
    out = np.zeros((len(rows), H), dtype=np.float32)                   # :129
    hidden_u8 = np.asarray(hidden_u8)
    hidden_scale = np.asarray(hidden_scale, dtype=np.float32)
    for le in range(e_local):                                           # :134
        ge = int(offset) + le
        if ge < 0 or ge >= E:                                           # :136
            continue
        sel = (topk_idx[rows] == ge).any(axis=1)                        # :140
        if not sel.any():                                               # :141
            continue
        tok = rows[sel]                                                 # :144
        O = _expert_ffn(hidden_u8, hidden_scale, tok, *get_expert(le))
        w_tok = weights[tok, ge]                                        # :165
        idx = np.fromiter((pos[int(t)] for t in tok), dtype=np.int64, count=len(tok))
        out[idx] += O * w_tok[:, None]                                  # :166
    if shared is not None and len(rows):
        out += _expert_ffn(hidden_u8, hidden_scale, rows, *shared)
    return {
        "out_f32": out, "out_bf16": f32_to_bf16_bits(out), "rows": rows, "topk_idx": topk_idx,
        "counts": local_counts(topk_idx, offset, e_local), "routing": r,
    }


# ---------------------------------------------------------------------------
# Upstream step: BF16 activations -> the layer's FP8 input.
# ---------------------------------------------------------------------------
_E4M3_POS = E4M3[:0x7F].astype(np.float64)  # codes 0x00..0x7e, ascending finite values 0..448


def f32_to_e4m3_rne(y: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn byte, round to nearest (ties to the even code),
    magnitudes above 448 saturating to 448 (the inputs here never exceed 448
    by more than one rounding of a division). Sign kept, -0.0 -> 0x80."""
    y = np.asarray(y, dtype=np.float32)
    a = np.minimum(np.abs(y).astype(np.float64), 448.0)
    idx = np.clip(np.searchsorted(_E4M3_POS, a, side="left"), 1, 0x7E)
    lo, hi = _E4M3_POS[idx - 1], _E4M3_POS[idx]
    d_lo, d_hi = a - lo, hi - a
    code = np.where(d_lo < d_hi, idx - 1, np.where(d_hi < d_lo, idx, np.where((idx - 1) % 2 == 0, idx - 1, idx)))
    code = code.astype(np.uint8)
    return np.where(np.signbit(y), code | np.uint8(0x80), code).astype(np.uint8)


def quant_rows_1x128(x: np.ndarray):
    """[T, 7168] float32 (bf16 values) -> (e4m3 bytes [T, 7168], f32 scales [56, T]).

    The layer's input format (reference moe/ref_moe.json:57-80, hidden_states
    and the transposed hidden_states_scale): one scale per 1x128 block,
    s = max(amax|x| / 448, 1e-12), q = e4m3(x / s) with a float32 division;
    the same amax / 448 recipe the reference uses for its intermediate
    (solution/triton/dsl-temp1.py:479-481)."""
    x = np.asarray(x, dtype=np.float32)
    T = x.shape[0]
    xb = x.reshape(T, H // BLOCK, BLOCK)
    s = np.maximum(np.abs(xb).max(axis=-1) / np.float32(448.0), np.float32(1e-12)).astype(np.float32)
    q = f32_to_e4m3_rne((xb / s[..., None]).astype(np.float32))
    return q.reshape(T, H), np.ascontiguousarray(s.T)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def add_rmsnorm_quant(x, residual=None, weight=None, eps: float = 1e-6):
    """The step after the layer, as the CUDA kernel defines it (no counterpart
    in the reference, whose operator ends at the bf16 output, solution/cuda/
    kernel.cu:288-291). x, residual: [T, 7168] float32 holding bf16 values;
    weight: [7168] bf16 values or None; eps is taken as float32.

      h = bf16(residual + x)        (h = x without a residual)
      y = bf16(w * bf16(h * r)),  r = 1 / sqrt(sum(h^2) / 7168 + eps)
      (y = h without a weight), then quant_rows_1x128(y).

    The DeepSeek-V3 decoder's residual add and input RMSNorm (HF transformers
    DeepseekV3RMSNorm: float32 variance, rsqrt, cast to bf16, times the bf16
    weight). The float32 sum of squares follows the kernel's order: thread i
    of 128 owns 8-column chunks c = 128 j + i (j = 0..6) and sums its 56
    squares in column order; a warp reduces by xor-butterfly (offsets 16, 8,
    4, 2, 1); the 4 warp sums add as ((w0 + w1) + w2) + w3. r is
    RN(1 / RN(sqrt(RN(RN(ss / 7168) + eps)))).
    Returns (h, q bytes [T, 7168], scales [56, T])."""
    f32 = np.float32
    x = np.asarray(x, dtype=f32)
    T = x.shape[0]
    h = bf16_round(np.asarray(residual, dtype=f32) + x) if residual is not None else x.copy()
    if weight is None:
        y = h
    else:
        sq = (h * h).astype(f32)                                   # exact for bf16 values
        per_thread = sq.reshape(T, 7, 128, 8).transpose(0, 2, 1, 3).reshape(T, 128, 56)
        acc = np.zeros((T, 128), dtype=f32)
        for i in range(56):
            acc = (acc + per_thread[:, :, i]).astype(f32)
        v = acc.reshape(T, 4, 32)
        lanes = np.arange(32)
        for off in (16, 8, 4, 2, 1):
            v = (v + v[:, :, lanes ^ off]).astype(f32)
        tot = (((v[:, 0, 0] + v[:, 1, 0]).astype(f32) + v[:, 2, 0]).astype(f32) + v[:, 3, 0]).astype(f32)
        mean = (tot / f32(H)).astype(f32)
        r = (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32))).astype(f32)
        n = bf16_round(h * r[:, None])
        y = bf16_round(np.asarray(weight, dtype=f32)[None, :] * n)
    q, sc = quant_rows_1x128(y)
    return h, q, sc


# ---------------------------------------------------------------------------
# Comparison helpers used by the tests.
# ---------------------------------------------------------------------------
def routing_mismatch_is_tie(routing: dict, t: int, ulps: int = 4) -> bool:
    """True if token t's selection boundary is within ``ulps`` float32 ulps of a
    tie: the 8th vs 9th kept score, or the 4th vs 5th group score. A routing
    difference at such a token can come from a 1-ulp difference of exp()
    between libraries and is reported as a tie, not a failure."""
    sb = routing["pruned"][t]
    srt = np.sort(sb)[::-1]
    gs = np.sort(routing["group_scores"][t])[::-1]

    def close(a, b):
        tol = ulps * np.spacing(np.float32(max(abs(a), abs(b))))
        return abs(float(a) - float(b)) <= tol

    return close(srt[TOP_K - 1], srt[TOP_K]) or close(gs[TOPK_GROUP - 1], gs[TOPK_GROUP])


def allclose_fraction(y: np.ndarray, y_ref: np.ndarray, atol: float = 1e-2, rtol: float = 1e-2) -> float:
    """Fraction of elements with |y - y_ref| <= atol + rtol * |y_ref|."""
    y = np.asarray(y, dtype=np.float32)
    y_ref = np.asarray(y_ref, dtype=np.float32)
    if y.size == 0:
        return 1.0
    return float(np.mean(np.abs(y - y_ref) <= atol + rtol * np.abs(y_ref)))
