"""Benchmark of the sm_100a fused FP8 DeepSeek-V3 MoE layer.

Default (N=1): BASELINE configs[1], the decode sweep T in {1,2,4,8,16,32,64}
on one B200 with 32 local experts (offset 0, scaling 2.5). One step = one
layer call at every T of the sweep; `value` = mean microseconds per call
(device time from CUDA events around each call, the L2 flushed with a 256 MB
write before every call, outside the events). Other workloads:
- `--workload mid|large`: configs[2] / configs[3];
- `--workload ep` (the default under torchrun with N > 1): configs[4], the full
  256-expert layer with expert parallelism, 4096 tokens per GPU;
- `--workload quant|addnorm`: the steps either side of the layer.

`--impl reference` times the reference algorithm on the host CPU cores (the
numpy restatement in oracle/, because the reference is Python/PyTorch and
cannot be compiled into oracle/_ref), one sweep point per step.
`--impl flashinfer` times FlashInfer's fused FP8 block-scale MoE on the same
inputs (a library comparator, not the reference).
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "us/call & TFLOP/s for FP8 DS-V3 MoE layer over T sweep; % of HBM/FP8 roofline"
WORKLOADS = {
    "decode_sweep": ((1, 2, 4, 8, 16, 32, 64), "BASELINE configs[1]: decode sweep, 32 local experts, offset 0"),
    "mid": ((256, 1024), "BASELINE configs[2]: mid prefill, near-uniform routing"),
    "large": ((4096, 8192, 16384), "BASELINE configs[3]: large prefill, +2.0 bias on 4 hot local experts"),
    "ep": ((4096,), "BASELINE configs[4]: full 256-expert layer, expert parallel, 4096 tokens per GPU, "
                    "NCCL all-to-all dispatch/combine"),
    "quant": ((1, 64, 4096, 16384), "upstream step: BF16 -> FP8 1x128 activation quantisation "
                                    "(moe_fp8_ds_quantize_act), bf16 ~N(0,1) hidden states"),
    "addnorm": ((1, 64, 4096, 16384), "downstream step: residual add + DeepSeek-V3 RMSNorm + FP8 1x128 "
                                      "quantisation of the layer output (moe_fp8_ds_add_norm_quant), bf16 "
                                      "~N(0,1) output and residual, eps 1e-6"),
}
L2_FLUSH_BYTES = 256 << 20


def _host_info() -> dict:
    """The host the CPU arms ran on: CPU model and the numerics libraries."""
    import numpy as np

    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "numpy": np.__version__}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _fp8_peak_cublas(dev):
    """Dense FP8 peak measured here, as MEASURED_PEAKS.json measures bf16: a
    library GEMM (cuBLASLt e4m3 x e4m3 -> bf16 through torch._scaled_mm,
    8192^3, per-tensor scales, random operands), best of 10. None if the
    call is unavailable."""
    import torch

    n = 8192
    try:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(n, n, generator=g, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, generator=g, device=dev).to(torch.float8_e4m3fn)
        one = torch.ones((), dtype=torch.float32, device=dev)
        for _ in range(3):
            torch._scaled_mm(a, b.t(), one, one, out_dtype=torch.bfloat16)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b.t(), one, one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except (RuntimeError, TypeError, AttributeError):
        return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML reads every ~2 ms from a background thread (read-only
    queries), so that even a region of a few milliseconds gets samples;
    nvidia-smi at 200 ms when NVML is unavailable."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.proc = None
        self.thread = None
        self.gpu = gpu_index
        self.path = os.path.join("/tmp", f"moe_clocks_{os.getpid()}.csv")
        self.sm, self.smax, self.reasons = [], None, set()

    def _nvml_loop(self, nv, h, bits):
        import time as _t
        while not self.stop:
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, b in bits.items():
                    if r & b:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001 - sampling is best effort
                break
            _t.sleep(0.002)

    def __enter__(self):
        try:
            import threading

            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.smax = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            self.stop = False
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h, bits), daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.thread = None
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop = True
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.thread is None and self.proc is not None and os.path.exists(self.path):
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    self.sm.append(float(f[1]))
                    self.smax = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(self.NAMES, f[5:9]):
                    if v.lower() == "active":
                        self.reasons.add(n)
        if not self.sm:
            return None
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.smax, "reasons": sorted(self.reasons),
                "samples": len(self.sm), "source": "nvml" if self.thread is not None else "nvidia-smi"}


def _dist():
    import torch.distributed as dist

    n = int(os.environ.get("WORLD_SIZE", "1"))
    if n > 1 and not dist.is_initialized():
        import datetime

        backend = "nccl"
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return int(os.environ.get("RANK", "0")), n


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def bench_ours(args):
    import numpy as np
    import torch

    rank, world = _dist()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pkg = importlib.import_module("flashinfer-mlsys_b200")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    lib = pkg.load()
    Ts, wdesc = WORKLOADS[args.workload]
    if args.T:
        Ts = tuple(int(t) for t in args.T.split(","))
    offset = 0
    w = wl.make_weights(32, offset, dev)
    acts = {T: wl.config_activations(T, offset) for T in Ts}
    acts_gpu = {T: acts[T].to(dev) for T in Ts}
    outs = {T: torch.empty((T, 7168), dtype=torch.bfloat16, device=dev) for T in Ts}
    counts = {T: torch.zeros((32,), dtype=torch.int32, device=dev) for T in Ts}
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def call(T, cnt=None):
        a = acts_gpu[T]
        pkg.kernel_ex(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, offset, 2.5, outs[T],
                      None, None, cnt)

    # routing statistics for the algorithmic FLOP/byte counts
    stats = {}
    for T in Ts:
        call(T, counts[T])
    torch.cuda.synchronize()
    for T in Ts:
        c = counts[T].cpu().numpy()
        stats[T] = {"n_assign": int(c.sum()), "e_touched": int((c > 0).sum())}

    for _ in range(args.warmup):
        for T in Ts:
            flush.zero_()
            call(T)
    torch.cuda.synchronize()

    ev = {T: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)] for T in Ts}
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for s in range(args.steps):
            for T in Ts:
                flush.zero_()
                ev[T][s][0].record(stream)
                call(T)
                ev[T][s][1].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
    per_T_ms = {T: statistics.mean(a.elapsed_time(b) for a, b in ev[T]) for T in Ts}
    if pkg.device_status() != 0:
        raise RuntimeError("device-side wait timed out during the benchmark")
    step_ms = sum(per_T_ms.values())
    if world > 1:
        t = torch.tensor([step_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        step_ms = float(t.item())

    # per-kernel device times (CUDA events recorded by the library on this stream)
    lib.moe_fp8_ds_profile_enable(1)
    kern = {T: np.zeros(3) for T in Ts}
    nkern = {T: 3 for T in Ts}  # 1 when the call is served by the fused decode kernel
    buf = (ctypes.c_float * 3)()
    for s in range(args.steps):
        for T in Ts:
            flush.zero_()
            call(T)
            n = lib.moe_fp8_ds_profile_last(buf, 3)
            nkern[T] = n
            kern[T][:n] += np.array(buf[:n])
    lib.moe_fp8_ds_profile_enable(0)
    for T in Ts:
        kern[T] /= args.steps

    # host-side enqueue cost of one call (argument checks, ctypes, launches)
    host_us = {}
    for T in Ts:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(20):
            call(T)
        host_us[T] = (time.perf_counter() - t0) / 20 * 1e6
        torch.cuda.synchronize()

    # end to end through the public API with host buffers (pinned), H2D of the
    # call's inputs and D2H of its output inside the events
    host_in = {T: [acts[T].logits.pin_memory(), acts[T].bias.pin_memory(),
                   acts[T].hidden.view(torch.uint8).pin_memory(), acts[T].hidden_scale.pin_memory()] for T in Ts}
    host_out = {T: torch.empty((T, 7168), dtype=torch.bfloat16).pin_memory() for T in Ts}
    e2e_ev = {T: [] for T in Ts}
    for s in range(args.warmup + args.steps):
        for T in Ts:
            a = acts_gpu[T]
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            a.logits.copy_(host_in[T][0], non_blocking=True)
            a.bias.copy_(host_in[T][1], non_blocking=True)
            a.hidden.view(torch.uint8).copy_(host_in[T][2], non_blocking=True)
            a.hidden_scale.copy_(host_in[T][3], non_blocking=True)
            call(T)
            host_out[T].copy_(outs[T], non_blocking=True)
            e1.record(stream)
            if s >= args.warmup:
                e2e_ev[T].append((e0, e1))
    torch.cuda.synchronize()
    e2e_ms = {T: statistics.mean(a.elapsed_time(b) for a, b in e2e_ev[T]) for T in Ts}
    h2d = sum(int(sum(x.numel() * x.element_size() for x in host_in[T])) for T in Ts)
    d2h = sum(T * 7168 * 2 for T in Ts)

    hbm_peak, bf16_peak, peak_src = _peaks()
    fp8_peak = 2 * bf16_peak
    sweep = {}
    tot_flops = tot_bytes = 0
    g1_bytes = g1_flops = g1_ms = 0.0
    fused_bytes = fused_ms = 0.0
    for T in Ts:
        st = stats[T]
        flops = wl.moe_flops(st["n_assign"])
        byts = wl.moe_bytes(T, st["e_touched"])
        ms = per_T_ms[T]
        t_roof_ms = max(byts / (hbm_peak * 1e9), flops / (fp8_peak * 1e12)) * 1e3
        sweep[str(T)] = {
            "us": round(ms * 1e3, 2), "e2e_us": round(e2e_ms[T] * 1e3, 2), "host_enqueue_us": round(host_us[T], 1),
            **st,
            "tflops": round(flops / (ms * 1e-3) / 1e12, 3), "gbs": round(byts / (ms * 1e-3) / 1e9, 1),
            "roofline_frac": round(t_roof_ms / ms, 4),
            "kernel_us": ({"fused_decode": round(kern[T][0] * 1e3, 2)} if nkern[T] == 1 else
                          {k: round(v * 1e3, 2) for k, v in zip(
                              ["route", "gemm1", "gemm2"], kern[T])}),
        }
        tot_flops += flops
        tot_bytes += byts
        # GEMM1 algorithmic bytes: touched W13 + scales, permuted rows in, intermediate out
        if nkern[T] == 1:
            # fused decode kernel: the whole layer's algorithmic bytes
            fused_bytes += byts
            fused_ms += kern[T][0]
        else:
            g1_bytes += st["e_touched"] * (4096 * 7168 + 32 * 56 * 4) + st["n_assign"] * (7168 + 56 * 4 + 4096 + 64)
            g1_flops += st["n_assign"] * 2 * 7168 * 4096
            g1_ms += kern[T][1]
    tot_ms = sum(per_T_ms.values())
    n_calls = len(Ts)
    value = tot_ms * 1e3 / n_calls
    if fused_ms > 0 and fused_ms >= g1_ms:
        roof_kernel = "moe_decode_kernel (whole layer in one launch)"
        achieved = fused_bytes / (fused_ms * 1e-3) / 1e9
        traffic = _ncu_traffic("decode_dram_bytes_per_launch")
    else:
        roof_kernel = "moe_gemm_kernel<1> (GEMM1 + SwiGLU)"
        achieved = g1_bytes / (g1_ms * 1e-3) / 1e9 if g1_ms > 0 else 0.0
        traffic = _ncu_traffic("gemm1_dram_bytes_per_launch")
    # GEMM1 is HBM-bound while its weight bytes take longer than its FLOPs
    # (decode, mid); past the ridge (large prefill) it is tensor-bound
    tensor_bound = g1_ms > 0 and g1_flops / (fp8_peak * 1e12) > g1_bytes / (hbm_peak * 1e9)
    if tensor_bound:
        g1_tflops = g1_flops / (g1_ms * 1e-3) / 1e12
        fp8_meas = _fp8_peak_cublas(dev)
        peak = fp8_meas if fp8_meas else fp8_peak
        src = ("measured here: cuBLASLt FP8 GEMM (torch._scaled_mm 8192^3, random e4m3), best of 10" if fp8_meas
               else f"{peak_src}: dense FP8 taken as 2x the bf16 GEMM figure")
        roofline = {"bound": "tensor", "kernel": roof_kernel, "achieved": round(g1_tflops, 1),
                    "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(g1_tflops / peak, 4),
                    "peak_source": src, "fp8_2x_bf16": round(fp8_peak, 1), "traffic": None}
    else:
        roofline = {"bound": "hbm", "kernel": roof_kernel, "achieved": round(achieved, 1),
                    "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                    "peak_source": peak_src, "traffic": traffic}
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "us/call", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (tcgen05 kind::f8f6f4)",
        "data": "synthetic, seeded (BASELINE value distributions; contest dataset unavailable)",
        "config": {"workload": f"{args.workload}: {wdesc}", "T": list(Ts), "num_local_experts": 32,
                   "local_expert_offset": offset, "routed_scaling_factor": 2.5,
                   "l2": "256 MB L2 flush before every call, outside the timed events",
                   "parallelism": "ep1" if world == 1 else f"replicas{world}"},
        "tflops": round(tot_flops / (tot_ms * 1e-3) / 1e12, 3),
        "hbm_gbs_algorithmic": round(tot_bytes / (tot_ms * 1e-3) / 1e9, 1),
        "sweep": sweep,
        "roofline": roofline,
        "e2e": {"value": round(sum(e2e_ms.values()) * 1e3 / n_calls, 3), "unit": "us/call",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": sum(nkern[T] for T in Ts) * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(Ts, acts, w)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def _ncu_traffic(key):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get(key)
        except (OSError, ValueError):
            return None
    return None


# ---------------------------------------------------------------------------
# CPU arms (oracle = numpy restatement of reference moe/ref_moe.py)
# ---------------------------------------------------------------------------
def _oracle_call(O, acts, get_expert, offset=0):
    return O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden),
                         acts.hidden_scale.numpy(), get_expert, offset, 2.5, 32)


def cpu_baseline(Ts, acts, w):
    O = importlib.import_module("oracle.moe_oracle")
    sample = [T for T in Ts if T <= 8] or [min(Ts)]
    cache = {}

    def get_expert(le):
        if le not in cache:
            cache[le] = w.expert_cpu(le)
        return cache[le]

    for T in sample:  # fetch the touched experts to host memory first (not timed)
        r = O.route(acts[T].logits.numpy(), O.as_f32(acts[T].bias), 2.5)
        for le in set(int(x) for x in r["topk_idx"].ravel() if 0 <= x < 32):
            get_expert(le)
    times = []
    for T in sample:
        t0 = time.perf_counter()
        _oracle_call(O, acts[T], get_expert)
        times.append(time.perf_counter() - t0)
    return {"value": round(statistics.mean(times) * 1e6, 1), "unit": "us/call", "cores": os.cpu_count(),
            "kind": "port", "sample": f"one oracle call at each T in {sample} (numpy, BLAS on all cores)",
            **_host_info()}


def bench_reference(args):
    """The reference algorithm on the host CPU (oracle port, BLAS on all cores).
    One step = one oracle call on a bounded token sample of one workload point:
    the whole batch when T <= 64, else 64 of its tokens with the time scaled by
    T / 64 (each output row depends only on its own token)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    O = importlib.import_module("oracle.moe_oracle")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    Ts, wdesc = WORKLOADS[args.workload]
    if args.T:
        Ts = tuple(int(t) for t in args.T.split(","))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    e_local = 256 if args.workload == "ep" else 32
    cache = {}

    def get_expert(le):
        if le not in cache:
            cache[le] = wl.expert_weights(le, "cpu", 0)
        return cache[le]

    SAMPLE = 64
    acts, subset = {}, {}
    for T in Ts:
        acts[T] = (wl.make_activations(T, seed=T) if args.workload == "ep" else wl.config_activations(T))
        subset[T] = None if T <= SAMPLE else list(range(0, T, T // SAMPLE))[:SAMPLE]
    seq = [Ts[i % len(Ts)] for i in range(args.warmup + args.steps)]
    # weight generation is setup, not the reference's work
    for T in set(seq):
        r = O.route(acts[T].logits.numpy(), O.as_f32(acts[T].bias), 2.5)
        rows = r["topk_idx"] if subset[T] is None else r["topk_idx"][subset[T]]
        for le in set(int(x) for x in rows.ravel() if 0 <= x < e_local):
            get_expert(le)
    times = []
    for i, T in enumerate(seq):
        t0 = time.perf_counter()
        O.moe_forward(acts[T].logits.numpy(), O.as_f32(acts[T].bias), O.as_u8(acts[T].hidden),
                      acts[T].hidden_scale.numpy(), get_expert, 0, 2.5, e_local, token_subset=subset[T])
        dt = time.perf_counter() - t0
        if subset[T] is not None:
            dt *= T / len(subset[T])
        if i >= args.warmup:
            times.append(dt)
    us = statistics.mean(times) * 1e6
    sample = ("one oracle call per step, T cycling through " + str(list(Ts)) +
              ("; T > 64 runs 64 of its tokens, time scaled by T/64" if max(Ts) > SAMPLE else ""))
    line = {
        "metric": METRIC, "value": round(us, 1), "unit": "us/call", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantised)", "data": "synthetic, seeded",
        "config": {"workload": f"{args.workload}: {wdesc}", "T": list(Ts), "num_local_experts": e_local,
                   "local_expert_offset": 0, "routed_scaling_factor": 2.5},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/call", "cores": os.cpu_count(), "kind": "port",
                         "sample": sample, **_host_info()},
        "e2e": {"value": round(us, 1), "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_ep(args):
    """every GPU holds 256/N experts and 4096 tokens of its
    own; one step = one expert-parallel layer call on every rank (routing,
    all-to-all dispatch, expert compute, all-to-all combine, fp32 sum)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world = _dist()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pkg = importlib.import_module("flashinfer-mlsys_b200")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    T = int(args.T) if args.T else 4096
    e_local = 256 // world
    offset = rank * e_local
    w = wl.make_weights(e_local, offset, dev)
    acts = wl.make_activations(T, seed=rank * 1_000_000 + T)
    a = acts.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        experts_fn = ep.make_cuda_experts_fn(w.w13, w.s13, w.w2, w.s2)

        def call(x):
            return ep.ep_forward(x.logits, x.bias, x.hidden, x.hidden_scale, 2.5, ep.cuda_route_fn, experts_fn)
    else:
        out1 = torch.empty((T, 7168), dtype=torch.bfloat16, device=dev)

        def call(x):
            pkg.kernel(x.logits, x.bias, x.hidden, x.hidden_scale, w.w13, w.s13, w.w2, w.s2, 0, 2.5, out1)
            return out1

    # routing statistics of this rank's share (local pairs over all ranks' tokens)
    ids, _, cnt = pkg.route(a.logits, a.bias, 0, 256, 2.5)
    own = torch.zeros(1, dtype=torch.int64, device=dev)
    pairs = torch.tensor([ids.numel()], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(pairs)
    n_assign_total = int(pairs.item())  # 8 pairs per token over the whole job
    for _ in range(args.warmup):
        flush.zero_()
        call(a)
    torch.cuda.synchronize()
    evs = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call(a)
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = statistics.mean(x.elapsed_time(y) for x, y in evs)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # end to end: H2D of this rank's inputs, the call, D2H of the output
    host = [acts.logits.pin_memory(), acts.bias.pin_memory(), acts.hidden.view(torch.uint8).pin_memory(),
            acts.hidden_scale.pin_memory()]
    host_out = torch.empty((T, 7168), dtype=torch.bfloat16).pin_memory()
    e2e = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        a.logits.copy_(host[0], non_blocking=True)
        a.bias.copy_(host[1], non_blocking=True)
        a.hidden.view(torch.uint8).copy_(host[2], non_blocking=True)
        a.hidden_scale.copy_(host[3], non_blocking=True)
        o = call(a)
        host_out.copy_(o, non_blocking=True)
        e1.record(stream)
        if i >= args.warmup:
            e2e.append((e0, e1))
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([statistics.mean(x.elapsed_time(y) for x, y in e2e)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    flops = wl.moe_flops(n_assign_total)
    hbm_peak, bf16_peak, peak_src = _peaks()
    line = {
        "metric": METRIC, "value": round(ms * 1e3, 2), "unit": "us/call", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (tcgen05 kind::f8f6f4)",
        "data": "synthetic, seeded (BASELINE value distributions)",
        "config": {"workload": f"ep: {WORKLOADS['ep'][1]}", "T_per_gpu": T, "num_local_experts": e_local,
                   "local_expert_offset": "rank*256/N", "routed_scaling_factor": 2.5,
                   "combine": "bf16 partials, fp32 sum", "l2": "256 MB L2 flush before every call, outside events",
                   "parallelism": f"ep{world}"},
        "tflops": round(flops / (ms * 1e-3) / 1e12, 3),
        "e2e": {"value": round(float(e2e_ms.item()) * 1e3, 2), "unit": "us/call",
                "h2d_bytes_per_step": int(sum(x.numel() * x.element_size() for x in host)),
                "d2h_bytes_per_step": T * 7168 * 2},
        "gpu_launches": 6 * args.steps if world > 1 else 5 * args.steps,
        "clocks": clk.summary(),
        "peak_source": peak_src,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_flashinfer(args):
    """Comparator (not the reference): FlashInfer's fused FP8 block-scale MoE,
    flashinfer.fused_moe.trtllm_fp8_block_scale_moe, called as a library on
    the same inputs, with DeepSeek-V3 routing (routing_method_type=2). The
    reference wires this call in solution/triton/dsl-temp1.py:226-263. Its
    first call JIT-compiles the launcher (minutes on a fresh machine); the
    line also reports its parity against the CPU oracle on the first T."""
    import numpy as np
    import torch
    from flashinfer.fused_moe import trtllm_fp8_block_scale_moe

    dev = torch.device("cuda", 0)
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    O = importlib.import_module("oracle.moe_oracle")
    Ts, wdesc = WORKLOADS[args.workload if args.workload != "ep" else "decode_sweep"]
    if args.T:
        Ts = tuple(int(t) for t in args.T.split(","))
    w = wl.make_weights(32, 0, dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    per_T, parity = {}, None
    for T in Ts:
        acts = wl.config_activations(T)
        a = acts.to(dev)

        def fn():
            return trtllm_fp8_block_scale_moe(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2,
                                              256, 8, 8, 4, 2048, 0, 32, 2.5, routing_method_type=2)

        out = fn()
        torch.cuda.synchronize()
        if parity is None:
            ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden),
                                acts.hidden_scale.numpy(), lambda le: w.expert_cpu(le), 0, 2.5, 32)
            parity = {"T": T, "frac_within_1e-2": O.allclose_fraction(
                out.float().cpu().numpy(), O.bf16_bits_to_f32(ref["out_bf16"]), 1e-2, 1e-2)}
        for _ in range(args.warmup):
            flush.zero_()
            fn()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        per_T[str(T)] = round(statistics.mean(x.elapsed_time(y) for x, y in evs) * 1e3, 2)
    value = statistics.mean(per_T.values())
    print(json.dumps({"metric": METRIC, "value": round(value, 3), "unit": "us/call", "impl": "flashinfer",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                      "config": {"workload": f"{args.workload}: {wdesc}", "T": list(Ts)}, "sweep_us": per_T,
                      "parity_vs_oracle": parity}), flush=True)


def bench_quant(args):
    """The steps either side of the layer alone, µs per call and achieved GB/s
    against the measured HBM peak:
    - quant: the upstream activation quantiser, 14,336 B read + 7,392 B
      written per token;
    - addnorm: residual add + RMSNorm + quantisation of the layer output,
      28,672 B read (output, residual) + 21,728 B written (residual, e4m3,
      scales) per token."""
    import torch

    pkg = importlib.import_module("flashinfer-mlsys_b200")
    dev = torch.device("cuda", 0)
    addnorm = args.workload == "addnorm"
    Ts = tuple(int(t) for t in args.T.split(",")) if args.T else WORKLOADS[args.workload][0]
    hbm_peak, _, peak_src = _peaks()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    g = torch.Generator(device="cpu").manual_seed(0)
    xs = {T: torch.randn(T, 7168, generator=g).to(torch.bfloat16).to(dev) for T in Ts}
    res = {T: torch.randn(T, 7168, generator=g).to(torch.bfloat16).to(dev) for T in Ts} if addnorm else {}
    norm_w = (1.0 + 0.1 * torch.randn(7168, generator=g)).to(torch.bfloat16).to(dev)
    outs = {T: (torch.empty((T, 7168), dtype=torch.float8_e4m3fn, device=dev),
                torch.empty((56, T), dtype=torch.float32, device=dev)) for T in Ts}

    def call(T):
        if addnorm:
            pkg.add_rmsnorm_quantize(xs[T], res[T], norm_w, 1e-6, *outs[T])
        else:
            pkg.quantize_activations(xs[T], *outs[T])

    for _ in range(args.warmup):
        for T in Ts:
            call(T)
    torch.cuda.synchronize()
    sweep = {}
    with ClockSampler(0) as clk:
        for T in Ts:
            ms = []
            for _ in range(args.steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                call(T)
                e1.record()
                ms.append((e0, e1))
            torch.cuda.synchronize()
            t = statistics.mean(a.elapsed_time(b) for a, b in ms)
            byts = T * ((7168 * 4 + 7168 * 2 + 7168 + 56 * 4) if addnorm else (7168 * 2 + 7168 + 56 * 4))
            sweep[str(T)] = {"us": round(t * 1e3, 2), "gbs": round(byts / (t * 1e-3) / 1e9, 1),
                             "hbm_frac": round(byts / (t * 1e-3) / 1e9 / hbm_peak, 4)}
    big = str(max(Ts))
    what = ("residual add + RMSNorm + FP8 1x128 quantisation of the layer output" if addnorm
            else "BF16 -> FP8 1x128 activation quantiser")
    line = {"metric": f"us/call and GB/s of the {what}", "value": sweep[big]["us"],
            "unit": f"us/call at T={big}", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "dtype": "bf16 -> e4m3", "data": "synthetic ~N(0,1)",
            "config": {"workload": f"{args.workload}: {WORKLOADS[args.workload][1]}", "T": list(Ts),
                       "l2": "256 MB L2 flush before every call, outside the timed events"},
            "sweep": sweep,
            "roofline": {"bound": "hbm", "kernel": "add_norm_quant_kernel" if addnorm else "quant_rows_kernel",
                         "achieved": sweep[big]["gbs"],
                         "peak": hbm_peak, "unit": "GB/s", "frac": sweep[big]["hbm_frac"],
                         "peak_source": peak_src},
            "gpu_launches": len(Ts) * args.steps, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "flashinfer"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="default: decode_sweep on 1 GPU, ep on N>1 GPUs")
    ap.add_argument("--T", default="", help="comma-separated token counts overriding the workload's sweep")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload is None:
        args.workload = "ep" if world > 1 else "decode_sweep"
    if args.impl == "reference":
        bench_reference(args)
    elif args.impl == "flashinfer":
        bench_flashinfer(args)
    elif args.workload == "ep":
        bench_ep(args)
    elif args.workload in ("quant", "addnorm"):
        bench_quant(args)
    else:
        bench_ours(args)


if __name__ == "__main__":
    main()
