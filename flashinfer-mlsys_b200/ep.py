"""Expert parallelism for the full 256-expert layer: one process per GPU.

Rank r of N owns the contiguous experts [r*256/N, (r+1)*256/N), exactly the
slice the reference computes for ``local_expert_offset = r*256/N``
(reference moe/ref_moe.py:131-137). Every rank holds its own tokens. A layer
call:

1. routes its tokens over all 256 experts (DeepSeek-V3 no-aux routing);
2. sends every token row once to each rank that owns at least one of its 8
   experts. A row is packed as e4m3 hidden (7168 B) + 56 f32 block scales +
   8 int32 expert ids + 8 f32 routing weights = 7456 B. The exchange is one
   NCCL all-to-all-v over NVLink, after a small all-to-all of the row counts;
3. on the owner, runs the expert computation for what it received
   (``moe_fp8_ds_experts``: only that rank's experts contribute to a row);
4. returns each row's partial output (bf16) with the reverse all-to-all-v;
5. sums the partials of every token in fp32 (rank order = ascending expert
   id order) and casts once to bf16.

The route and expert functions are parameters, so the same bookkeeping runs
with the CUDA library on GPUs (NCCL) and with CPU functions under a gloo
process group in the tests.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

H = 7168
HB = H // 128          # 56 hidden scale blocks
TOPK = 8
E_GLOBAL = 256
ROW_BYTES = H + HB * 4 + TOPK * 4 + TOPK * 4  # 7456


def pack_rows(hidden: torch.Tensor, hidden_scale: torch.Tensor, ids: torch.Tensor, w: torch.Tensor,
              idx: torch.Tensor) -> torch.Tensor:
    """Rows ``idx`` of (hidden e4m3 [T,7168], scale f32 [56,T], ids int32 [T,8],
    weights f32 [T,8]) -> uint8 [len(idx), 7456]."""
    n = idx.numel()
    buf = torch.empty((n, ROW_BYTES), dtype=torch.uint8, device=hidden.device)
    buf[:, :H] = hidden.view(torch.uint8).index_select(0, idx)
    buf[:, H:H + HB * 4] = hidden_scale.t().index_select(0, idx).contiguous().view(torch.uint8)
    o = H + HB * 4
    buf[:, o:o + TOPK * 4] = ids.index_select(0, idx).contiguous().view(torch.uint8)
    buf[:, o + TOPK * 4:] = w.index_select(0, idx).contiguous().view(torch.uint8)
    return buf


def unpack_rows(buf: torch.Tensor):
    """uint8 [R, 7456] -> (hidden e4m3 [R,7168], scale f32 [56,R], ids int32 [R,8], weights f32 [R,8])."""
    R = buf.shape[0]
    hidden = buf[:, :H].contiguous().view(torch.float8_e4m3fn)
    scale = buf[:, H:H + HB * 4].contiguous().view(torch.float32).reshape(R, HB).t().contiguous()
    o = H + HB * 4
    ids = buf[:, o:o + TOPK * 4].contiguous().view(torch.int32).reshape(R, TOPK)
    w = buf[:, o + TOPK * 4:].contiguous().view(torch.float32).reshape(R, TOPK)
    return hidden, scale, ids, w


@dataclass
class Plan:
    send_idx: torch.Tensor      # token index of every sent row, grouped by destination rank
    send_counts: list           # rows sent to each rank
    recv_counts: list           # rows received from each rank


def dispatch_plan(ids: torch.Tensor, world: int, group=None) -> Plan:
    """Which tokens go to which rank (once per rank, ascending token order),
    and the exchange of the per-rank row counts."""
    e_local = E_GLOBAL // world
    T = ids.shape[0]
    dest = torch.zeros((T, world), dtype=torch.bool, device=ids.device)
    owner = (ids.long() // e_local).clamp_(0, world - 1)
    dest.scatter_(1, owner, True)
    send_idx = torch.cat([torch.nonzero(dest[:, r], as_tuple=False).flatten() for r in range(world)])
    send_counts_t = dest.sum(dim=0).to(torch.int64)
    recv_counts_t = torch.empty_like(send_counts_t)
    dist.all_to_all_single(recv_counts_t, send_counts_t, group=group)
    return Plan(send_idx, send_counts_t.tolist(), recv_counts_t.tolist())


def ep_forward(routing_logits: torch.Tensor, routing_bias: torch.Tensor, hidden: torch.Tensor,
               hidden_scale: torch.Tensor, routed_scaling_factor: float,
               route_fn: Callable, experts_fn: Callable, group=None,
               combine_dtype: torch.dtype = torch.bfloat16, plan_out: Optional[list] = None) -> torch.Tensor:
    """One expert-parallel MoE layer call on this rank's tokens; returns bf16 [T, 7168].

    route_fn(logits, bias, scale) -> (ids int32 [T,8], weights f32 [T,8]) over all 256 experts.
    experts_fn(hidden, scale, ids, weights, local_expert_offset, out) writes
    out [R,7168] (dtype ``combine_dtype``) = sum over this rank's experts.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    e_local = E_GLOBAL // world
    T = hidden.shape[0]
    ids, w = route_fn(routing_logits, routing_bias, routed_scaling_factor)
    plan = dispatch_plan(ids, world, group)
    if plan_out is not None:
        plan_out.append(plan)
    send_buf = pack_rows(hidden, hidden_scale, ids, w, plan.send_idx)
    R = sum(plan.recv_counts)
    recv_buf = torch.empty((R, ROW_BYTES), dtype=torch.uint8, device=hidden.device)
    dist.all_to_all_single(recv_buf, send_buf, output_split_sizes=plan.recv_counts,
                           input_split_sizes=plan.send_counts, group=group)
    h_r, s_r, ids_r, w_r = unpack_rows(recv_buf)
    out_r = torch.empty((R, H), dtype=combine_dtype, device=hidden.device)
    if R:
        experts_fn(h_r, s_r, ids_r, w_r, rank * e_local, out_r)
    back = torch.empty((plan.send_idx.numel(), H), dtype=combine_dtype, device=hidden.device)
    dist.all_to_all_single(back, out_r, output_split_sizes=plan.send_counts,
                           input_split_sizes=plan.recv_counts, group=group)
    out = torch.zeros((T, H), dtype=torch.float32, device=hidden.device)
    # rows come back grouped by source rank in rank order; adding rank by rank
    # sums a token's partials in ascending expert-id order
    off = 0
    for r in range(world):
        n = plan.send_counts[r]
        if n:
            out.index_add_(0, plan.send_idx[off:off + n], back[off:off + n].float())
        off += n
    return out.to(torch.bfloat16)


# ---------------------------------------------------------------------------
# CUDA-library bindings of the two callbacks (the product path on GPUs).
# ---------------------------------------------------------------------------
def cuda_route_fn(routing_logits, routing_bias, routed_scaling_factor):
    from .binding import route

    ids, w, _ = route(routing_logits, routing_bias, 0, 32, routed_scaling_factor)
    return ids, w


def make_cuda_experts_fn(w13, s13, w2, s2):
    """experts_fn running this rank's experts with ``moe_fp8_ds_experts``."""
    from .binding import experts

    def fn(h, s, ids, wts, offset, out):
        experts(h, s, ids, wts, w13, s13, w2, s2, offset, out)

    return fn
