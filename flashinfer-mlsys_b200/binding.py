"""Python drop-in for the reference's destination-passing MoE entry point.

``kernel(...)`` has the 11 parameters, order and meaning of
solution/cuda/binding.py:149-161 and solution/cuda/kernel.cu:134-146
(definition: reference moe/ref_moe.json:57-145): it writes the bf16 MoE
output of one expert-parallel rank into the caller's ``output`` tensor.

Everything runs in the sm_100a library ``libmoe_fp8_ds.so`` on the caller's
current CUDA stream; this module only checks arguments and passes pointers.
There is no PyTorch or CPU fallback: a missing library or a failing call
raises.
"""
from __future__ import annotations

import torch

from . import _lib

HIDDEN_SIZE = 7168
INTERMEDIATE_SIZE = 2048
NUM_EXPERTS = 256
NUM_LOCAL_EXPERTS = 32
BLOCK_Q = 128
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4

_E4M3 = torch.float8_e4m3fn


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _tensor(t: torch.Tensor, name: str, dtype: torch.dtype, shape: tuple) -> None:
    _need(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _need(tuple(t.shape) == tuple(shape), f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    _need(t.is_contiguous(), f"{name} must be contiguous")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _chk(t, name, dtype, shape, dev):
    """Fast-path check of one tensor (dtype, shape, device, contiguity)."""
    if t.dtype != dtype or t.shape != shape or t.device != dev or not t.is_contiguous():
        _tensor(t, name, dtype, shape)
        _need(t.device == dev, f"{name} must be on {dev}")


try:  # raw current-stream handle without constructing a Stream object
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover
    _raw_stream = None


def _stream(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


# Weight tensors are the same objects call after call; remember the ones
# already validated (keyed by identity and data pointer).
_VALID_WEIGHTS: dict = {}


def _weights_ok(w1, s1, w2, s2, e_local, dev):
    key = (id(w1), id(s1), id(w2), id(s2))
    sig = (e_local, dev) + tuple((t.data_ptr(), t.dtype, tuple(t.shape), t.stride()) for t in (w1, s1, w2, s2))
    if _VALID_WEIGHTS.get(key) == sig:
        return
    _check_weights(w1, s1, w2, s2, e_local)
    for t in (w1, s1, w2, s2):
        _need(t.device == dev, "all tensors must be on the same device")
    if len(_VALID_WEIGHTS) > 64:
        _VALID_WEIGHTS.clear()
    _VALID_WEIGHTS[key] = sig


def _call(dev, fn, *args):
    """Run a C-ABI call with `dev` current (no device switch in the common case)."""
    if dev.index == torch.cuda.current_device():
        return fn(*args)
    with torch.cuda.device(dev):
        return fn(*args)


def _check_weights(w1, s1, w2, s2, e_local):
    _tensor(w1, "gemm1_weights", _E4M3, (e_local, 2 * INTERMEDIATE_SIZE, HIDDEN_SIZE))
    _tensor(s1, "gemm1_weights_scale", torch.float32, (e_local, 2 * INTERMEDIATE_SIZE // BLOCK_Q, HIDDEN_SIZE // BLOCK_Q))
    _tensor(w2, "gemm2_weights", _E4M3, (e_local, HIDDEN_SIZE, INTERMEDIATE_SIZE))
    _tensor(s2, "gemm2_weights_scale", torch.float32, (e_local, HIDDEN_SIZE // BLOCK_Q, INTERMEDIATE_SIZE // BLOCK_Q))


def kernel_ex(
    routing_logits: torch.Tensor,
    routing_bias: torch.Tensor,
    hidden_states: torch.Tensor,
    hidden_states_scale: torch.Tensor,
    gemm1_weights: torch.Tensor,
    gemm1_weights_scale: torch.Tensor,
    gemm2_weights: torch.Tensor,
    gemm2_weights_scale: torch.Tensor,
    local_expert_offset: int,
    routed_scaling_factor: float,
    output: torch.Tensor,
    topk_ids: torch.Tensor | None = None,
    topk_weights: torch.Tensor | None = None,
    expert_counts: torch.Tensor | None = None,
) -> None:
    """``kernel`` plus optional device outputs of this call's routing decision
    (int32 [T, 8] ids, f32 [T, 8] weights, int32 [E_local] per-expert counts)."""
    if routing_logits.dim() != 2:
        raise ValueError("routing_logits must be 2-D [seq_len, 256]")
    T = routing_logits.shape[0]
    e_local = gemm1_weights.shape[0]
    dev = hidden_states.device
    _need(dev.type == "cuda", "hidden_states must be a CUDA tensor")
    _chk(routing_logits, "routing_logits", torch.float32, (T, NUM_EXPERTS), dev)
    _chk(routing_bias, "routing_bias", torch.bfloat16, (NUM_EXPERTS,), dev)
    _chk(hidden_states, "hidden_states", _E4M3, (T, HIDDEN_SIZE), dev)
    _chk(hidden_states_scale, "hidden_states_scale", torch.float32, (HIDDEN_SIZE // BLOCK_Q, T), dev)
    _chk(output, "output", torch.bfloat16, (T, HIDDEN_SIZE), dev)
    _weights_ok(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, e_local, dev)
    if topk_ids is not None:
        _chk(topk_ids, "topk_ids", torch.int32, (T, TOP_K), dev)
    if topk_weights is not None:
        _chk(topk_weights, "topk_weights", torch.float32, (T, TOP_K), dev)
    if expert_counts is not None:
        _chk(expert_counts, "expert_counts", torch.int32, (e_local,), dev)
    lib = _lib.load()
    rc = _call(dev, lib.moe_fp8_ds_kernel_ex,
               routing_logits.data_ptr(), routing_bias.data_ptr(), hidden_states.data_ptr(),
               hidden_states_scale.data_ptr(), gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(),
               gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr(), int(local_expert_offset),
               float(routed_scaling_factor), output.data_ptr(), T, e_local,
               _ptr(topk_ids), _ptr(topk_weights), _ptr(expert_counts), _stream(dev))
    if rc:
        _lib.check(rc, "moe_fp8_ds_kernel_ex")


def kernel(
    routing_logits: torch.Tensor,
    routing_bias: torch.Tensor,
    hidden_states: torch.Tensor,
    hidden_states_scale: torch.Tensor,
    gemm1_weights: torch.Tensor,
    gemm1_weights_scale: torch.Tensor,
    gemm2_weights: torch.Tensor,
    gemm2_weights_scale: torch.Tensor,
    local_expert_offset: int,
    routed_scaling_factor: float,
    output: torch.Tensor,
) -> None:
    """DPS MoE layer: routing, per-expert GEMM1 -> SwiGLU -> GEMM2 and the
    weighted combine, written to ``output`` (bf16 [seq_len, 7168])."""
    kernel_ex(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
              routed_scaling_factor, output)


@torch.no_grad()
def kernel_shared(
    routing_logits: torch.Tensor,
    routing_bias: torch.Tensor,
    hidden_states: torch.Tensor,
    hidden_states_scale: torch.Tensor,
    gemm1_weights: torch.Tensor,
    gemm1_weights_scale: torch.Tensor,
    gemm2_weights: torch.Tensor,
    gemm2_weights_scale: torch.Tensor,
    local_expert_offset: int,
    routed_scaling_factor: float,
    shared_gemm1_weights: torch.Tensor,
    shared_gemm1_weights_scale: torch.Tensor,
    shared_gemm2_weights: torch.Tensor,
    shared_gemm2_weights_scale: torch.Tensor,
    output: torch.Tensor,
) -> None:
    """``kernel`` plus DeepSeek-V3's shared expert (weights of one expert:
    e4m3 [4096, 7168] + f32 [32, 56], e4m3 [7168, 2048] + f32 [56, 16]) applied
    to every token with weight 1 and added to the routed sum, in the same
    launches (no counterpart in the reference's operator)."""
    _need(routing_logits.dim() == 2, "routing_logits must be 2-D [seq_len, 256]")
    T = routing_logits.shape[0]
    e_local = gemm1_weights.shape[0]
    dev = hidden_states.device
    _need(dev.type == "cuda", "hidden_states must be a CUDA tensor")
    _need(e_local in (32, 64, 128), "the shared expert needs 32, 64 or 128 local experts")
    _chk(routing_logits, "routing_logits", torch.float32, (T, NUM_EXPERTS), dev)
    _chk(routing_bias, "routing_bias", torch.bfloat16, (NUM_EXPERTS,), dev)
    _chk(hidden_states, "hidden_states", _E4M3, (T, HIDDEN_SIZE), dev)
    _chk(hidden_states_scale, "hidden_states_scale", torch.float32, (HIDDEN_SIZE // BLOCK_Q, T), dev)
    _chk(output, "output", torch.bfloat16, (T, HIDDEN_SIZE), dev)
    _weights_ok(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, e_local, dev)
    _chk(shared_gemm1_weights, "shared_gemm1_weights", _E4M3, (2 * INTERMEDIATE_SIZE, HIDDEN_SIZE), dev)
    _chk(shared_gemm1_weights_scale, "shared_gemm1_weights_scale", torch.float32,
         (2 * INTERMEDIATE_SIZE // BLOCK_Q, HIDDEN_SIZE // BLOCK_Q), dev)
    _chk(shared_gemm2_weights, "shared_gemm2_weights", _E4M3, (HIDDEN_SIZE, INTERMEDIATE_SIZE), dev)
    _chk(shared_gemm2_weights_scale, "shared_gemm2_weights_scale", torch.float32,
         (HIDDEN_SIZE // BLOCK_Q, INTERMEDIATE_SIZE // BLOCK_Q), dev)
    lib = _lib.load()
    rc = _call(dev, lib.moe_fp8_ds_kernel_shared,
               routing_logits.data_ptr(), routing_bias.data_ptr(), hidden_states.data_ptr(),
               hidden_states_scale.data_ptr(), gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(),
               gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr(), int(local_expert_offset),
               float(routed_scaling_factor), shared_gemm1_weights.data_ptr(), shared_gemm1_weights_scale.data_ptr(),
               shared_gemm2_weights.data_ptr(), shared_gemm2_weights_scale.data_ptr(), output.data_ptr(), T,
               e_local, _stream(dev))
    _lib.check(rc, "moe_fp8_ds_kernel_shared")


@torch.no_grad()
def route(
    routing_logits: torch.Tensor,
    routing_bias: torch.Tensor,
    local_expert_offset: int = 0,
    num_local_experts: int = NUM_LOCAL_EXPERTS,
    routed_scaling_factor: float = 2.5,
):
    """DeepSeek-V3 no-aux routing only. Returns (ids int32 [T,8], weights f32
    [T,8], local per-expert counts int32 [num_local_experts])."""
    _need(routing_logits.dim() == 2, "routing_logits must be 2-D [seq_len, 256]")
    T = routing_logits.shape[0]
    _tensor(routing_logits, "routing_logits", torch.float32, (T, NUM_EXPERTS))
    _tensor(routing_bias, "routing_bias", torch.bfloat16, (NUM_EXPERTS,))
    dev = routing_logits.device
    ids = torch.empty((T, TOP_K), dtype=torch.int32, device=dev)
    w = torch.empty((T, TOP_K), dtype=torch.float32, device=dev)
    counts = torch.zeros((num_local_experts,), dtype=torch.int32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.moe_fp8_ds_route(routing_logits.data_ptr(), routing_bias.data_ptr(), T, int(local_expert_offset),
                                  int(num_local_experts), float(routed_scaling_factor), ids.data_ptr(),
                                  w.data_ptr(), counts.data_ptr(), _stream(dev))
    _lib.check(rc, "moe_fp8_ds_route")
    return ids, w, counts


@torch.no_grad()
def experts(
    hidden_states: torch.Tensor,
    hidden_states_scale: torch.Tensor,
    topk_ids: torch.Tensor,
    topk_weights: torch.Tensor,
    gemm1_weights: torch.Tensor,
    gemm1_weights_scale: torch.Tensor,
    gemm2_weights: torch.Tensor,
    gemm2_weights_scale: torch.Tensor,
    local_expert_offset: int,
    output: torch.Tensor,
) -> None:
    """Expert computation of pre-routed rows: output[r] = sum over the row's
    local experts of weight * expert(row). ``output`` is f32 or bf16
    [num_rows, 7168]."""
    R = hidden_states.shape[0]
    e_local = gemm1_weights.shape[0]
    _tensor(hidden_states, "hidden_states", _E4M3, (R, HIDDEN_SIZE))
    _tensor(hidden_states_scale, "hidden_states_scale", torch.float32, (HIDDEN_SIZE // BLOCK_Q, R))
    _tensor(topk_ids, "topk_ids", torch.int32, (R, TOP_K))
    _tensor(topk_weights, "topk_weights", torch.float32, (R, TOP_K))
    _check_weights(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, e_local)
    _need(output.dtype in (torch.float32, torch.bfloat16), "output must be float32 or bfloat16")
    _tensor(output, "output", output.dtype, (R, HIDDEN_SIZE))
    dev = hidden_states.device
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.moe_fp8_ds_experts(
            hidden_states.data_ptr(), hidden_states_scale.data_ptr(), topk_ids.data_ptr(), topk_weights.data_ptr(),
            gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(), gemm2_weights.data_ptr(),
            gemm2_weights_scale.data_ptr(), int(local_expert_offset), R, e_local, output.data_ptr(),
            1 if output.dtype == torch.float32 else 0, _stream(dev))
    _lib.check(rc, "moe_fp8_ds_experts")


@torch.no_grad()
def quantize_activations(hidden_bf16: torch.Tensor, hidden_states: torch.Tensor | None = None,
                         hidden_states_scale: torch.Tensor | None = None):
    """BF16 hidden states [seq_len, 7168] -> the layer's FP8 input: e4m3
    [seq_len, 7168] and transposed f32 scales [56, seq_len], one scale
    max(amax / 448, 1e-12) per 1x128 block, round to nearest even. Writes the
    given output tensors (allocated if None) and returns them."""
    _need(hidden_bf16.dim() == 2, "hidden_bf16 must be 2-D [seq_len, 7168]")
    T = hidden_bf16.shape[0]
    _tensor(hidden_bf16, "hidden_bf16", torch.bfloat16, (T, HIDDEN_SIZE))
    dev = hidden_bf16.device
    if hidden_states is None:
        hidden_states = torch.empty((T, HIDDEN_SIZE), dtype=_E4M3, device=dev)
    if hidden_states_scale is None:
        hidden_states_scale = torch.empty((HIDDEN_SIZE // BLOCK_Q, T), dtype=torch.float32, device=dev)
    _tensor(hidden_states, "hidden_states", _E4M3, (T, HIDDEN_SIZE))
    _tensor(hidden_states_scale, "hidden_states_scale", torch.float32, (HIDDEN_SIZE // BLOCK_Q, T))
    lib = _lib.load()
    rc = _call(dev, lib.moe_fp8_ds_quantize_act, hidden_bf16.data_ptr(), T, hidden_states.data_ptr(),
               hidden_states_scale.data_ptr(), _stream(dev))
    _lib.check(rc, "moe_fp8_ds_quantize_act")
    return hidden_states, hidden_states_scale


@torch.no_grad()
def add_rmsnorm_quantize(x: torch.Tensor, residual: torch.Tensor | None = None,
                         norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                         out: torch.Tensor | None = None, out_scale: torch.Tensor | None = None):
    """The step after the layer: h = bf16(residual + x) (written back into
    ``residual``), y = DeepSeek-V3 RMSNorm of h with ``norm_weight`` and
    ``eps``, then the 1x128 FP8 quantisation of y (the next layer's input
    format, as ``quantize_activations``). ``residual`` None: h = x;
    ``norm_weight`` None: y = h. Returns (e4m3 [seq_len, 7168], f32 scales
    [56, seq_len])."""
    _need(x.dim() == 2, "x must be 2-D [seq_len, 7168]")
    T = x.shape[0]
    _tensor(x, "x", torch.bfloat16, (T, HIDDEN_SIZE))
    dev = x.device
    if residual is not None:
        _tensor(residual, "residual", torch.bfloat16, (T, HIDDEN_SIZE))
        _need(residual.device == dev, "residual must be on the same device as x")
    if norm_weight is not None:
        _tensor(norm_weight, "norm_weight", torch.bfloat16, (HIDDEN_SIZE,))
        _need(norm_weight.device == dev, "norm_weight must be on the same device as x")
    _need(float(eps) >= 0.0, "eps must be >= 0")
    if out is None:
        out = torch.empty((T, HIDDEN_SIZE), dtype=_E4M3, device=dev)
    if out_scale is None:
        out_scale = torch.empty((HIDDEN_SIZE // BLOCK_Q, T), dtype=torch.float32, device=dev)
    _tensor(out, "out", _E4M3, (T, HIDDEN_SIZE))
    _tensor(out_scale, "out_scale", torch.float32, (HIDDEN_SIZE // BLOCK_Q, T))
    lib = _lib.load()
    rc = _call(dev, lib.moe_fp8_ds_add_norm_quant, x.data_ptr(),
               None if residual is None else residual.data_ptr(),
               None if norm_weight is None else norm_weight.data_ptr(), float(eps), T, out.data_ptr(),
               out_scale.data_ptr(), _stream(dev))
    _lib.check(rc, "moe_fp8_ds_add_norm_quant")
    return out, out_scale


def last_rows(seq_len: int, num_local_experts: int, device=None):
    """Where the last layer call with ``num_local_experts`` on ``device`` put
    each token's expert rows: int32 [seq_len, 8], the padded-layout row of the
    token's j-th local expert (ascending id, -1 padded); row r lies in m-tile
    r // 128, and each m-tile belongs to one expert. A diagnostic for tests."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    rows = torch.empty((seq_len, TOP_K), dtype=torch.int32, device=dev)
    rc = _call(dev, _lib.load().moe_fp8_ds_last_rows, int(seq_len), int(num_local_experts), rows.data_ptr(),
               _stream(dev))
    _lib.check(rc, "moe_fp8_ds_last_rows")
    return rows


def device_status(stream=None) -> int:
    """Synchronise and return the library's device status (0 = ok)."""
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    return _lib.load().moe_fp8_ds_device_status(s)
