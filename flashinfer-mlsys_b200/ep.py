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
process group in the tests. On CUDA tensors the row packing, unpacking and
the combine, and the dispatch plan, are the library's kernels
(moe_fp8_ds_ep_pack / _unpack / _combine / _plan); the torch expressions
below are their CPU restatement for the gloo tests.
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


def _lib_call(name, dev, *args):
    from . import _lib
    from .binding import _call, _stream

    rc = _call(dev, getattr(_lib.load(), name), *args, _stream(dev))
    _lib.check(rc, name)


def pack_rows(hidden: torch.Tensor, hidden_scale: torch.Tensor, ids: torch.Tensor, w: torch.Tensor,
              idx: torch.Tensor) -> torch.Tensor:
    """Rows ``idx`` of (hidden e4m3 [T,7168], scale f32 [56,T], ids int32 [T,8],
    weights f32 [T,8]) -> uint8 [len(idx), 7456]."""
    n = idx.numel()
    buf = torch.empty((n, ROW_BYTES), dtype=torch.uint8, device=hidden.device)
    if hidden.is_cuda:
        idx64 = idx.to(torch.int64).contiguous()
        hidden, hidden_scale = hidden.contiguous(), hidden_scale.contiguous()
        _lib_call("moe_fp8_ds_ep_pack", hidden.device, hidden.data_ptr(), hidden_scale.data_ptr(),
                  ids.contiguous().data_ptr(), w.contiguous().data_ptr(), hidden.shape[0], idx64.data_ptr(), n,
                  buf.data_ptr())
        return buf
    buf[:, :H] = hidden.view(torch.uint8).index_select(0, idx)
    buf[:, H:H + HB * 4] = hidden_scale.t().index_select(0, idx).contiguous().view(torch.uint8)
    o = H + HB * 4
    buf[:, o:o + TOPK * 4] = ids.index_select(0, idx).contiguous().view(torch.uint8)
    buf[:, o + TOPK * 4:] = w.index_select(0, idx).contiguous().view(torch.uint8)
    return buf


def unpack_rows(buf: torch.Tensor):
    """uint8 [R, 7456] -> (hidden e4m3 [R,7168], scale f32 [56,R], ids int32 [R,8], weights f32 [R,8])."""
    R = buf.shape[0]
    if buf.is_cuda:
        dev = buf.device
        hidden = torch.empty((R, H), dtype=torch.float8_e4m3fn, device=dev)
        scale = torch.empty((HB, R), dtype=torch.float32, device=dev)
        ids = torch.empty((R, TOPK), dtype=torch.int32, device=dev)
        w = torch.empty((R, TOPK), dtype=torch.float32, device=dev)
        _lib_call("moe_fp8_ds_ep_unpack", dev, buf.data_ptr(), R, hidden.data_ptr(), scale.data_ptr(),
                  ids.data_ptr(), w.data_ptr())
        return hidden, scale, ids, w
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
    row_of: Optional[torch.Tensor] = None  # int32 [T, world]: row of token t in send_idx for rank q, -1 if none


def plan_local(ids: torch.Tensor, world: int):
    """The local half of the dispatch plan in torch (the restatement of the
    moe_fp8_ds_ep_plan kernel): (send order int64 [world*T] with the first
    sum(counts) valid, counts int64 [world], row_of int32 [T, world])."""
    e_local = E_GLOBAL // world
    T = ids.shape[0]
    dest = torch.zeros((world, T), dtype=torch.bool, device=ids.device)
    owner = (ids.long() // e_local).clamp_(0, world - 1)
    dest.scatter_(0, owner.t().contiguous(), True)
    # rank-major flat order: tokens grouped by destination rank, ascending
    # within a rank; positions from a running count (no size-dependent op, so
    # no host synchronisation before the count exchange)
    flat = dest.reshape(-1)
    n = flat.numel()
    pos = torch.where(flat, torch.cumsum(flat, 0) - 1, torch.full_like(flat, n, dtype=torch.int64))
    order = torch.empty(n + 1, dtype=torch.int64, device=ids.device)
    order.scatter_(0, pos, torch.arange(n, device=ids.device) % T)
    counts = dest.sum(dim=1).to(torch.int64)
    row_of = torch.full((T, world), -1, dtype=torch.int32, device=ids.device)
    rows = torch.where(flat, torch.cumsum(flat, 0) - 1, torch.full_like(flat, -1, dtype=torch.int64))
    row_of.copy_(rows.view(world, T).t().to(torch.int32))
    return order[:n], counts, row_of


def plan_cuda(ids: torch.Tensor, world: int):
    """plan_local's triple from the moe_fp8_ds_ep_plan kernel (one launch)."""
    dev = ids.device
    T = ids.shape[0]
    order = torch.empty(max(world * T, 1), dtype=torch.int64, device=dev)
    counts = torch.empty(world, dtype=torch.int64, device=dev)
    row_of = torch.empty((T, world), dtype=torch.int32, device=dev)
    ids32 = ids.to(torch.int32).contiguous()
    _lib_call("moe_fp8_ds_ep_plan", dev, ids32.data_ptr() if T else None, T, world, order.data_ptr(),
              counts.data_ptr(), row_of.data_ptr() if T else None)
    return order, counts, row_of


def dispatch_plan(ids: torch.Tensor, world: int, group=None) -> Plan:
    """Which tokens go to which rank (once per rank, ascending token order),
    and the exchange of the per-rank row counts. One host synchronisation:
    NCCL's all-to-all-v takes its split sizes on the host."""
    order, send_counts_t, row_of = plan_cuda(ids, world) if ids.is_cuda else plan_local(ids, world)
    recv_counts_t = torch.empty_like(send_counts_t)
    dist.all_to_all_single(recv_counts_t, send_counts_t, group=group)
    both = torch.cat([send_counts_t, recv_counts_t]).tolist()
    send_counts, recv_counts = both[:world], both[world:]
    return Plan(order[:sum(send_counts)], send_counts, recv_counts, row_of)


# Phases of one expert-parallel call, in order (ep_forward's `marks`).
PHASES = ("route", "plan+counts", "pack", "dispatch", "unpack", "experts", "return", "combine")


def ep_forward(routing_logits: torch.Tensor, routing_bias: torch.Tensor, hidden: torch.Tensor,
               hidden_scale: torch.Tensor, routed_scaling_factor: float,
               route_fn: Callable, experts_fn: Callable, group=None,
               combine_dtype: torch.dtype = torch.bfloat16, plan_out: Optional[list] = None,
               marks: Optional[Callable] = None) -> torch.Tensor:
    """One expert-parallel MoE layer call on this rank's tokens; returns bf16 [T, 7168].

    route_fn(logits, bias, scale) -> (ids int32 [T,8], weights f32 [T,8]) over all 256 experts.
    experts_fn(hidden, scale, ids, weights, local_expert_offset, out) writes
    out [R,7168] (dtype ``combine_dtype``) = sum over this rank's experts.
    marks(i): called before phase i of PHASES and once more at the end
    (i = len(PHASES)); the benchmark records CUDA events there.
    """
    mark = marks if marks is not None else (lambda i: None)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    e_local = E_GLOBAL // world
    T = hidden.shape[0]
    mark(0)
    ids, w = route_fn(routing_logits, routing_bias, routed_scaling_factor)
    mark(1)
    plan = dispatch_plan(ids, world, group)
    if plan_out is not None:
        plan_out.append(plan)
    mark(2)
    send_buf = pack_rows(hidden, hidden_scale, ids, w, plan.send_idx)
    R = sum(plan.recv_counts)
    recv_buf = torch.empty((R, ROW_BYTES), dtype=torch.uint8, device=hidden.device)
    mark(3)
    dist.all_to_all_single(recv_buf, send_buf, output_split_sizes=plan.recv_counts,
                           input_split_sizes=plan.send_counts, group=group)
    mark(4)
    h_r, s_r, ids_r, w_r = unpack_rows(recv_buf)
    out_r = torch.empty((R, H), dtype=combine_dtype, device=hidden.device)
    mark(5)
    if R:
        experts_fn(h_r, s_r, ids_r, w_r, rank * e_local, out_r)
    back = torch.empty((plan.send_idx.numel(), H), dtype=combine_dtype, device=hidden.device)
    mark(6)
    dist.all_to_all_single(back, out_r, output_split_sizes=plan.send_counts,
                           input_split_sizes=plan.recv_counts, group=group)
    mark(7)
    out = combine_rows(back, plan, T, world)
    mark(8)
    return out


def combine_rows(back: torch.Tensor, plan: Plan, T: int, world: int) -> torch.Tensor:
    """Sum each token's returned partial rows in fp32 in rank order (= ascending
    expert-id order) and cast once to bf16. Rows come back grouped by rank, in
    the order they were sent."""
    if back.is_cuda and back.dtype == torch.bfloat16:
        dev = back.device
        # row_of[t][q]: the row of token t in the block returned by rank q, -1 if none
        row_of = plan.row_of
        if row_of is None:
            row_of = torch.full((T, world), -1, dtype=torch.int32, device=dev)
            if plan.send_idx.numel():
                q = torch.repeat_interleave(torch.arange(world, device=dev),
                                            torch.tensor(plan.send_counts, device=dev))
                row_of[plan.send_idx, q] = torch.arange(plan.send_idx.numel(), dtype=torch.int32, device=dev)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        _lib_call("moe_fp8_ds_ep_combine", dev, back.data_ptr() if back.numel() else None, row_of.data_ptr(), T,
                  world, out.data_ptr())
        return out
    out = torch.zeros((T, H), dtype=torch.float32, device=back.device)
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
