"""Benchmark of the sm_100a fused FP8 DeepSeek-V3 MoE layer.

Default at every N (one process per GPU; torchrun for N > 1): the shape of
BASELINE configs[4]. Every GPU holds 256/N experts and 4096 tokens of its
own. N = 1 holds all 256 experts and runs the layer as one call of the
library; N > 1 runs the expert-parallel layer (routing, NCCL all-to-all
dispatch, the expert GEMMs, all-to-all return, fp32 combine). One step = one
layer call on every rank; `value` = mean microseconds per call, max over
ranks. The workload is the same at every N, so the driver's 1 -> N efficiency
compares like with like (weak scaling: tokens per GPU fixed).

The N = 1 line also carries the metric's T sweep on one expert-parallel rank
(32 local experts, offset 0), under "sweeps": BASELINE configs[1] (decode, T in
1..64), configs[2] (mid, T in {256, 1024}) and configs[3] (large, T in {4096,
8192, 16384}, 4 hot local experts). Every T has its µs/call, TFLOP/s,
whole-call roofline fraction, per-kernel times and end-to-end time; every
workload has the roofline of its dominant kernel.

Timing: CUDA events on the launching stream around each call; a 256 MB write
flushes L2 before every call, outside the events; at least 3 warm-up calls;
SM clocks and throttle reasons sampled through NVML during the timed region.

Other arms: `--impl reference` (the reference algorithm on the host CPU
cores: the numpy restatement in oracle/, because the reference is
Python/PyTorch and cannot be compiled into oracle/_ref), `--impl flashinfer`
(FlashInfer's fused FP8 block-scale MoE as a library comparator, not the
reference). `--workload NAME` runs one workload alone: ep, decode_sweep, mid,
large, quant (the upstream activation quantiser), addnorm (the downstream
residual add + RMSNorm + quantisation).
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
EP_T = 4096
WORKLOADS = {
    "ep": ((EP_T,), "BASELINE configs[4] shape: 4096 tokens and 256/N experts per GPU (N = 1: all 256 experts "
                    "on one GPU, one library call; N > 1: NCCL all-to-all dispatch and return over NVLink)"),
    "decode_sweep": ((1, 2, 4, 8, 16, 32, 64), "BASELINE configs[1]: decode sweep, 32 local experts, offset 0"),
    "mid": ((256, 1024), "BASELINE configs[2]: mid prefill, near-uniform routing"),
    "large": ((4096, 8192, 16384), "BASELINE configs[3]: large prefill, +2.0 bias on 4 hot local experts"),
    "shared": ((1, 8, 64, 1024, 4096), "DeepSeek-V3's shared expert fused into the layer (moe_fp8_ds_kernel_shared, "
                                       "32 local experts) against the routed layer plus a separate shared-expert call"),
    "quant": ((1, 64, 4096, 16384), "upstream step: BF16 -> FP8 1x128 activation quantisation "
                                    "(moe_fp8_ds_quantize_act), bf16 ~N(0,1) hidden states"),
    "addnorm": ((1, 64, 4096, 16384), "downstream step: residual add + DeepSeek-V3 RMSNorm + FP8 1x128 "
                                      "quantisation of the layer output (moe_fp8_ds_add_norm_quant), bf16 "
                                      "~N(0,1) output and residual, eps 1e-6"),
}
SWEEP = ("decode_sweep", "mid", "large")
L2_FLUSH_BYTES = 256 << 20
# The CPU arms time the reference algorithm on a sample of experts with all
# their tokens (the reference loops over experts, ref_moe.py:134-166) and scale
# by experts / sample.
CPU_SAMPLE_EXPERTS = 4
CPU_SAMPLE_GROUPS = ((0, 4), (100, 4), (200, 4))
L2_NOTE = "256 MB L2 flush before every call, outside the timed events"


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


def _config(workload, world, Ts):
    """The `config` object of every arm (ours, reference) for a workload."""
    if workload == "ep":
        return {"workload": f"ep: {WORKLOADS['ep'][1]}", "T_per_gpu": Ts[0], "num_local_experts": 256 // world,
                "local_expert_offset": "rank*256/N", "routed_scaling_factor": 2.5, "l2": L2_NOTE,
                "parallelism": f"ep{world}"}
    return {"workload": f"{workload}: {WORKLOADS[workload][1]}", "T": list(Ts), "num_local_experts": 32,
            "local_expert_offset": 0, "routed_scaling_factor": 2.5, "l2": L2_NOTE,
            "parallelism": "one expert-parallel rank of 8"}


def _gemm1_bytes(e_touched, n_assign):
    """GEMM1's algorithmic HBM bytes: every touched expert's W13 and its block
    scales once, each assignment's gathered e4m3 row and 56 scales in, its
    two-term intermediate row and 16 scales out."""
    return e_touched * (4096 * 7168 + 32 * 56 * 4) + n_assign * (7168 + 56 * 4 + 4096 + 16 * 4)


def _gemm1_flops(n_assign):
    return n_assign * 2 * 7168 * 4096


class _Fp8Peak:
    """Dense FP8 peak measured once per run (cuBLASLt), else 2x the bf16 figure."""

    def __init__(self, dev, bf16_peak, peak_src):
        self.dev, self.bf16, self.src, self.val = dev, bf16_peak, peak_src, None

    def get(self):
        if self.val is None:
            m = _fp8_peak_cublas(self.dev)
            self.val = (m, "measured here: cuBLASLt FP8 GEMM (torch._scaled_mm 8192^3, random e4m3), best of 10") \
                if m else (2 * self.bf16, f"{self.src}: dense FP8 taken as 2x the bf16 GEMM figure")
        return self.val


def _roofline_gemm1(stats, g1_ms, hbm_peak, peak_src, fp8, fp8_2x_sustained, traffic_key):
    """Roofline of GEMM1 (the dominant kernel) over a set of calls: HBM-bound
    while its weight bytes take longer than its FLOPs at the FP8 rate, else
    tensor-bound (TFLOP/s against the FP8 GEMM measured in this run)."""
    byts = sum(_gemm1_bytes(s["e_touched"], s["n_assign"]) for s in stats)
    flops = sum(_gemm1_flops(s["n_assign"]) for s in stats)
    if g1_ms <= 0:
        return None
    traffic = _ncu_traffic(traffic_key, byts / max(1, len(stats)))
    fp8_nominal = 2 * _peaks()[1]
    if flops / (fp8_nominal * 1e12) > byts / (hbm_peak * 1e9):
        peak, src = fp8.get()
        ach = flops / (g1_ms * 1e-3) / 1e12
        return {"bound": "tensor", "kernel": "moe_gemm_kernel<1> (GEMM1 + SwiGLU + requant)", "achieved": round(ach, 1),
                "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(ach / peak, 4), "peak_source": src,
                "frac_of_2x_bf16_sustained": round(ach / fp8_2x_sustained, 4),
                "traffic": traffic["bytes"] if traffic else None, "traffic_detail": traffic,
                "algorithmic_flops": flops}
    ach = byts / (g1_ms * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": "moe_gemm_kernel<1> (GEMM1 + SwiGLU + requant)", "achieved": round(ach, 1),
            "peak": hbm_peak, "unit": "GB/s", "frac": round(ach / hbm_peak, 4),
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
            "traffic": traffic["bytes"] if traffic else None, "traffic_detail": traffic,
            "algorithmic_bytes_per_launch": int(byts / max(1, len(stats)))}


def _packed_inputs(acts_cpu, dev):
    """One pinned host buffer holding a call's inputs (logits | bias | hidden |
    hidden_scale, each at a 16-byte-aligned offset) and a device buffer of the
    same layout with the layer's input tensors as views into it, so that the
    end-to-end step moves its inputs with one host-to-device copy."""
    import torch

    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    T = acts_cpu.T
    parts = [t.contiguous().reshape(-1).view(torch.uint8)
             for t in (acts_cpu.logits, acts_cpu.bias, acts_cpu.hidden, acts_cpu.hidden_scale)]
    offs, n = [], 0
    for t in parts:
        offs.append(n)
        n += (t.numel() + 15) // 16 * 16
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    for o, t in zip(offs, parts):
        host[o:o + t.numel()].copy_(t)
    buf = torch.empty(n, dtype=torch.uint8, device=dev)

    def view(i, dtype, shape):
        nbytes = parts[i].numel()
        return buf[offs[i]:offs[i] + nbytes].view(dtype).view(shape)

    acts = wl.Activations(view(0, torch.float32, (T, 256)), view(1, torch.bfloat16, (256,)),
                          view(2, torch.float8_e4m3fn, (T, 7168)), view(3, torch.float32, (56, T)))
    return host, buf, acts


def _measure_layer(pkg, lib, dev, stream, flush, w, acts_cpu, e_local, steps, warmup, kernels=True, e2e=True):
    """Per-T device time, per-kernel times, host enqueue and end-to-end time of
    the layer (one library call per T per step) on weights `w`."""
    import numpy as np
    import torch

    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    Ts = list(acts_cpu)
    acts = {T: acts_cpu[T].to(dev) for T in Ts}
    outs = {T: torch.empty((T, 7168), dtype=torch.bfloat16, device=dev) for T in Ts}
    counts = {T: torch.zeros((e_local,), dtype=torch.int32, device=dev) for T in Ts}

    def call(T, cnt=None):
        a = acts[T]
        pkg.kernel_ex(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, w.offset, 2.5, outs[T],
                      None, None, cnt)

    stats = {}
    for T in Ts:
        call(T, counts[T])
    torch.cuda.synchronize()
    for T in Ts:
        c = counts[T].cpu().numpy()
        stats[T] = {"n_assign": int(c.sum()), "e_touched": int((c > 0).sum())}
    for _ in range(warmup):
        for T in Ts:
            flush.zero_()
            call(T)
    torch.cuda.synchronize()
    ev = {T: [] for T in Ts}
    for _ in range(steps):
        for T in Ts:
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call(T)
            e1.record(stream)
            ev[T].append((e0, e1))
    torch.cuda.synchronize()
    ms = {T: statistics.mean(a.elapsed_time(b) for a, b in ev[T]) for T in Ts}
    if pkg.device_status() != 0:
        raise RuntimeError("device-side wait timed out during the benchmark")
    res = {"ms": ms, "stats": stats}
    if kernels:
        # per-kernel device times (CUDA events recorded by the library on this stream)
        lib.moe_fp8_ds_profile_enable(1)
        kern = {T: np.zeros(5) for T in Ts}
        nk = {T: 5 for T in Ts}
        buf = (ctypes.c_float * 5)()
        for _ in range(steps):
            for T in Ts:
                flush.zero_()
                call(T)
                n = lib.moe_fp8_ds_profile_last(buf, 5)
                nk[T] = n
                kern[T][:n] += np.array(buf[:n])
        lib.moe_fp8_ds_profile_enable(0)
        res["kernel_ms"] = {T: kern[T] / steps for T in Ts}
        res["nkern"] = nk
        # host-side enqueue cost of one call (argument checks, ctypes, launches)
        host = {}
        for T in Ts:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(20):
                call(T)
            host[T] = (time.perf_counter() - t0) / 20 * 1e6
            torch.cuda.synchronize()
        res["host_us"] = host
    if e2e:
        # end to end through the public API with host buffers (pinned): the
        # H2D copy of the call's inputs (one packed buffer) and the D2H of its
        # output inside the events
        packed = {T: _packed_inputs(acts_cpu[T], dev) for T in Ts}
        host_out = {T: torch.empty((T, 7168), dtype=torch.bfloat16).pin_memory() for T in Ts}
        e2e_ev = {T: [] for T in Ts}
        for i in range(warmup + steps):
            for T in Ts:
                host_in, dev_in, a = packed[T]
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                dev_in.copy_(host_in, non_blocking=True)
                pkg.kernel(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2, w.offset, 2.5,
                           outs[T])
                host_out[T].copy_(outs[T], non_blocking=True)
                e1.record(stream)
                if i >= warmup:
                    e2e_ev[T].append((e0, e1))
        torch.cuda.synchronize()
        for T in Ts:  # the packed inputs reached the device intact
            if not torch.equal(packed[T][1].cpu(), packed[T][0]):
                raise RuntimeError("packed input copy mismatch")
        res["e2e_ms"] = {T: statistics.mean(a.elapsed_time(b) for a, b in e2e_ev[T]) for T in Ts}
        res["h2d"] = {T: int(packed[T][0].numel()) for T in Ts}
        res["d2h"] = {T: T * 7168 * 2 for T in Ts}
    return res


# Intervals moe_fp8_ds_profile_last reports, by their number.
KERNEL_NAMES = {5: ("route", "permute", "gemm1", "gemm2", "finalize"), 4: ("route+permute", "gemm1", "gemm2", "finalize"),
                3: ("route+permute", "gemm1", "gemm2+combine"), 1: ("fused_decode",)}


def _gemm1_ms(m, T):
    """GEMM1's event time of a call (0 when the call ran the fused decode kernel)."""
    names = KERNEL_NAMES[m["nkern"][T]]
    return float(m["kernel_ms"][T][names.index("gemm1")]) if "gemm1" in names else 0.0


def _sweep_entry(wl, T, m, hbm_peak, fp8_nominal):
    st = m["stats"][T]
    ms = m["ms"][T]
    flops = wl.moe_flops(st["n_assign"])
    byts = wl.moe_bytes(T, st["e_touched"])
    t_roof = max(byts / (hbm_peak * 1e9), flops / (fp8_nominal * 1e12)) * 1e3
    e = {"us": round(ms * 1e3, 2), **st, "tflops": round(flops / (ms * 1e-3) / 1e12, 3),
         "gbs": round(byts / (ms * 1e-3) / 1e9, 1), "roofline_frac": round(t_roof / ms, 4)}
    if "e2e_ms" in m:
        e["e2e_us"] = round(m["e2e_ms"][T] * 1e3, 2)
    if "host_us" in m:
        e["host_enqueue_us"] = round(m["host_us"][T], 1)
    if "kernel_ms" in m:
        k = m["kernel_ms"][T]
        e["kernel_us"] = {n: round(v * 1e3, 2) for n, v in zip(KERNEL_NAMES[m["nkern"][T]], k)}
    return e


def _run_sweep(pkg, lib, wl, dev, stream, flush, w32, name, steps, warmup, fp8, Ts=None):
    """One workload of the metric's T sweep on one rank (32 local experts)."""
    Ts = Ts or WORKLOADS[name][0]
    acts = {T: wl.config_activations(T) for T in Ts}
    hbm_peak, bf16_peak, peak_src = _peaks()
    m = _measure_layer(pkg, lib, dev, stream, flush, w32, acts, 32, steps, warmup)
    entries = {str(T): _sweep_entry(wl, T, m, hbm_peak, 2 * bf16_peak) for T in Ts}
    g1_ms = sum(_gemm1_ms(m, T) for T in Ts if _gemm1_ms(m, T) > 0)
    roof = _roofline_gemm1([m["stats"][T] for T in Ts if _gemm1_ms(m, T) > 0], g1_ms, hbm_peak, peak_src, fp8,
                           2 * _sustained_bf16(), f"gemm1_{name}")
    tot_ms = sum(m["ms"].values())
    return {"T": list(Ts), "us_mean": round(tot_ms * 1e3 / len(Ts), 3),
            "e2e_us_mean": round(sum(m["e2e_ms"].values()) * 1e3 / len(Ts), 3),
            "h2d_bytes": sum(m["h2d"].values()), "d2h_bytes": sum(m["d2h"].values()),
            "tflops": round(sum(wl.moe_flops(m["stats"][T]["n_assign"]) for T in Ts) / (tot_ms * 1e-3) / 1e12, 3),
            "roofline": roof, "per_T": entries}


def _sustained_bf16():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))
    return 1400.0


def _ncu_traffic(key, algorithmic_per_launch):
    """DRAM bytes per launch of GEMM1 for this run's calls, from the committed
    ncu capture of the same workload (ncu cannot run inside the benchmark):
    the capture's DRAM/algorithmic ratio times this run's algorithmic bytes
    per launch (exact where the capture covered the same calls). None when
    there is no capture."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        d = json.load(open(p)).get(key)
    except (OSError, ValueError):
        return None
    if not isinstance(d, dict) or not d.get("algorithmic_bytes"):
        return None
    ratio = d["dram_bytes"] / d["algorithmic_bytes"]
    return {"bytes": int(ratio * algorithmic_per_launch), "ratio_to_algorithmic": round(ratio, 3),
            "source": f"profiles/traffic.json[{key}]: {d.get('case')}"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def bench_ours(args):
    import torch

    rank, world = _dist()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.workload == "ep" or world > 1:
        return bench_ep(args, rank, world, local, dev)
    pkg = importlib.import_module("flashinfer-mlsys_b200")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    lib = pkg.load()
    w = wl.make_weights(32, 0, dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    hbm_peak, bf16_peak, peak_src = _peaks()
    fp8 = _Fp8Peak(dev, bf16_peak, peak_src)
    Ts = tuple(int(t) for t in args.T.split(",")) if args.T else WORKLOADS[args.workload][0]
    with ClockSampler(local) as clk:
        sw = _run_sweep(pkg, lib, wl, dev, stream, flush, w, args.workload, args.steps, args.warmup, fp8, Ts)
    line = {
        "metric": METRIC, "value": sw["us_mean"], "unit": "us/call", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(sw["us_mean"] * len(Ts) / 1e3, 4), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (tcgen05 kind::f8f6f4)",
        "data": "synthetic, seeded (BASELINE value distributions; contest dataset unavailable)",
        "config": _config(args.workload, 1, Ts), "tflops": sw["tflops"], "sweep": sw["per_T"],
        "roofline": sw["roofline"],
        "e2e": {"value": sw["e2e_us_mean"], "unit": "us/call", "h2d_bytes_per_step": sw["h2d_bytes"],
                "d2h_bytes_per_step": sw["d2h_bytes"]},
        "gpu_launches": 3 * args.steps * len(Ts), "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def bench_ep(args, rank, world, local, dev):
    """The default workload (configs[4] shape) at N GPUs; at N = 1 also the
    metric's T sweep."""
    import numpy as np
    import torch
    import torch.distributed as dist

    pkg = importlib.import_module("flashinfer-mlsys_b200")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    ep = importlib.import_module("flashinfer-mlsys_b200.ep")
    lib = pkg.load()
    T = int(args.T) if args.T else EP_T
    e_local = 256 // world
    offset = rank * e_local
    w = wl.make_weights(e_local, offset, dev)
    acts = wl.make_activations(T, seed=rank * 1_000_000 + T)
    a = acts.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    hbm_peak, bf16_peak, peak_src = _peaks()
    fp8 = _Fp8Peak(dev, bf16_peak, peak_src)
    line = {"metric": METRIC, "unit": "us/call", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> f32 (tcgen05 kind::f8f6f4)",
            "data": "synthetic, seeded (BASELINE value distributions; contest dataset unavailable)",
            "config": _config("ep", world, (T,))}

    if world == 1:
        # all 256 experts on one GPU: one library call per step
        with ClockSampler(local) as clk:
            m = _measure_layer(pkg, lib, dev, stream, flush, w, {T: acts}, 256, args.steps, args.warmup)
        ms = m["ms"][T]
        st = m["stats"][T]
        entry = _sweep_entry(wl, T, m, hbm_peak, 2 * bf16_peak)
        roof = _roofline_gemm1([st], _gemm1_ms(m, T), hbm_peak, peak_src, fp8, 2 * _sustained_bf16(),
                               "gemm1_ep1")
        line.update({"value": round(ms * 1e3, 2), "ms_per_step": round(ms, 4), "tflops": entry["tflops"],
                     "detail": entry, "roofline": roof,
                     "e2e": {"value": round(m["e2e_ms"][T] * 1e3, 2), "unit": "us/call",
                             "h2d_bytes_per_step": m["h2d"][T], "d2h_bytes_per_step": m["d2h"][T]},
                     "gpu_launches": 3 * args.steps, "clocks": clk.summary()})
    else:
        experts_fn = ep.make_cuda_experts_fn(w.w13, w.s13, w.w2, w.s2)

        def call(x, marks=None, plan_out=None):
            return ep.ep_forward(x.logits, x.bias, x.hidden, x.hidden_scale, 2.5, ep.cuda_route_fn, experts_fn,
                                 marks=marks, plan_out=plan_out)

        plans = []
        call(a, plan_out=plans)
        for _ in range(args.warmup):
            flush.zero_()
            call(a)
        torch.cuda.synchronize()
        evs = []
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
            dist.barrier()
        ms_t = torch.tensor([statistics.mean(x.elapsed_time(y) for x, y in evs)], device=dev)
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t.item())
        # per-phase device times (events between phases; a separate pass)
        nph = len(ep.PHASES)
        ph = np.zeros(nph)
        for _ in range(args.steps):
            flush.zero_()
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(nph + 1)]
            call(a, marks=lambda i: marks[i].record(stream))
            torch.cuda.synchronize()
            ph += np.array([marks[i].elapsed_time(marks[i + 1]) for i in range(nph)])
        ph_t = torch.tensor(ph / args.steps, device=dev)
        dist.all_reduce(ph_t, op=dist.ReduceOp.MAX)
        # end to end: H2D of this rank's inputs (one packed buffer), the call,
        # D2H of the output
        host_in, dev_in, a_e2e = _packed_inputs(acts, dev)
        host_out = torch.empty((T, 7168), dtype=torch.bfloat16).pin_memory()
        e2e = []
        for i in range(args.warmup + args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            dev_in.copy_(host_in, non_blocking=True)
            o = call(a_e2e)
            host_out.copy_(o, non_blocking=True)
            e1.record(stream)
            if i >= args.warmup:
                e2e.append((e0, e1))
        torch.cuda.synchronize()
        e2e_t = torch.tensor([statistics.mean(x.elapsed_time(y) for x, y in e2e)], device=dev)
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        # work and exchange volume of every rank
        p = plans[0]
        recv_rows = sum(p.recv_counts)
        send_rows = sum(p.send_counts)
        own = p.send_counts[rank]
        # bytes that cross NVLink (rows a rank sends to itself do not):
        # dispatch of packed rows out, expert rows (bf16) back
        vol = torch.tensor([[(send_rows - own) * ep.ROW_BYTES + (recv_rows - own) * 7168 * 2,
                             (recv_rows - own) * ep.ROW_BYTES + (send_rows - own) * 7168 * 2]],
                           dtype=torch.float64, device=dev)
        vols = [torch.zeros_like(vol) for _ in range(world)]
        dist.all_gather(vols, vol)
        vols = torch.cat(vols).cpu().numpy()
        n_assign_total = int(T * 8 * world)  # every token has 8 experts, all present over the job
        per_gpu_flops = wl.moe_flops(n_assign_total) / world
        per_gpu_wbytes = e_local * 44_050_944
        link_out = float(vols[:, 0].max())
        link_in = float(vols[:, 1].max())
        t_link = max(link_out, link_in) / 770e9 * 1e3
        fp8_peak, fp8_src = fp8.get()
        t_flop = per_gpu_flops / (fp8_peak * 1e12) * 1e3
        t_hbm = per_gpu_wbytes / (hbm_peak * 1e9) * 1e3
        bound = max((t_link, "nvlink"), (t_flop, "tensor"), (t_hbm, "hbm"))
        phases = {n: round(float(v) * 1e3, 1) for n, v in zip(ep.PHASES, ph_t.cpu().numpy())}
        line.update({
            "value": round(ms * 1e3, 2), "ms_per_step": round(ms, 4),
            "tflops": round(wl.moe_flops(n_assign_total) / (ms * 1e-3) / 1e12, 3),
            "phases_us_max_over_ranks": phases,
            "roofline": {"bound": bound[1], "kernel": "whole expert-parallel call (per GPU)",
                         "achieved": round(bound[0] / ms, 4), "peak": 1.0, "unit": "fraction of t_roof",
                         "frac": round(bound[0] / ms, 4), "t_roof_ms": round(bound[0], 4),
                         "t_nvlink_ms": round(t_link, 4), "t_tensor_ms": round(t_flop, 4),
                         "t_hbm_ms": round(t_hbm, 4), "nvlink_gbs_per_direction_assumed": 770.0,
                         "fp8_peak_tflops": round(fp8_peak, 1), "fp8_peak_source": fp8_src,
                         "nvlink_bytes_out_per_call_max_rank": int(link_out),
                         "nvlink_bytes_in_per_call_max_rank": int(link_in),
                         "nccl_achieved_gbs": round(max(link_out, link_in) / ((phases["dispatch"] + phases["return"])
                                                                               * 1e-6) / 1e9, 1),
                         "traffic": None},
            "e2e": {"value": round(float(e2e_t.item()) * 1e3, 2), "unit": "us/call",
                    "h2d_bytes_per_step": int(host_in.numel()),
                    "d2h_bytes_per_step": T * 7168 * 2},
            "gpu_launches": 8 * args.steps, "clocks": clk.summary(),
        })
    if world == 1 and not args.no_sweep:
        w32 = wl.Weights(w.w13[:32], w.s13[:32], w.w2[:32], w.s2[:32], 0)
        sweeps = {}
        with ClockSampler(local) as clk2:
            for name in SWEEP:
                sweeps[name] = _run_sweep(pkg, lib, wl, dev, stream, flush, w32, name, args.steps, args.warmup, fp8)
        line["sweeps"] = sweeps
        line["sweeps_clocks"] = clk2.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(T, acts)
    if rank == 0:
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# CPU arms (oracle = numpy restatement of reference moe/ref_moe.py)
# ---------------------------------------------------------------------------
def _cpu_sample(O, wl, acts, r, groups, cache):
    """Seconds of the reference algorithm for one rank's call (T tokens over
    all 256 experts), from the routing plus samples of experts with all their
    tokens scaled by 256 / sample size (the expert loop dominates)."""
    t0 = time.perf_counter()
    r2 = O.route(acts.logits.numpy(), O.as_f32(acts.bias), 2.5)
    t_route = time.perf_counter() - t0
    tot = 0.0
    for off, n in groups:
        def get_expert(le, off=off):
            return cache[off + le]
        t0 = time.perf_counter()
        O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                      get_expert, off, 2.5, n, routing=r2)
        tot += (time.perf_counter() - t0) * 256 / n
    return t_route + tot / len(groups)


def _cpu_setup(T, acts, groups):
    O = importlib.import_module("oracle.moe_oracle")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    cache = {}
    for off, n in groups:  # expert weights are setup, not the reference's work
        for g in range(off, off + n):
            cache[g] = wl.expert_weights(g, "cpu", 0)
    r = O.route(acts.logits.numpy(), O.as_f32(acts.bias), 2.5)
    return O, wl, r, cache


def _sample_text(T):
    return (f"one rank's call, {T} tokens over 256 experts: the routing plus {len(CPU_SAMPLE_GROUPS)} samples of "
            f"{CPU_SAMPLE_EXPERTS} experts with all their tokens (experts "
            + ", ".join(f"{o}-{o + n - 1}" for o, n in CPU_SAMPLE_GROUPS)
            + f"), each scaled by 256/{CPU_SAMPLE_EXPERTS}; numpy with BLAS on all host cores")


def cpu_baseline(T, acts):
    O, wl, r, cache = _cpu_setup(T, acts, CPU_SAMPLE_GROUPS)
    s = _cpu_sample(O, wl, acts, r, CPU_SAMPLE_GROUPS, cache)
    return {"value": round(s * 1e6, 1), "unit": "us/call", "cores": os.cpu_count(), "kind": "port",
            "sample": _sample_text(T), **_host_info()}


def bench_reference(args):
    """The reference algorithm on the host CPU (oracle port, BLAS on all cores)
    for our default workload: one step = one rank's call (4096 tokens over 256
    experts), measured by the expert sampling of cpu_baseline. Under torchrun
    only rank 0 runs; the others exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    if args.workload not in (None, "ep"):
        raise SystemExit("--impl reference times the default workload (ep)")
    T = int(args.T) if args.T else EP_T
    acts = wl.make_activations(T, seed=T)
    O, wl, r, cache = _cpu_setup(T, acts, CPU_SAMPLE_GROUPS)
    times = []
    for i in range(args.warmup + args.steps):
        g = (CPU_SAMPLE_GROUPS[i % len(CPU_SAMPLE_GROUPS)],)
        dt = _cpu_sample(O, wl, acts, r, g, cache)
        if i >= args.warmup:
            times.append(dt)
    us = statistics.mean(times) * 1e6
    sample = _sample_text(T).replace(f"{len(CPU_SAMPLE_GROUPS)} samples", "one sample per step (cycling through")
    line = {
        "metric": METRIC, "value": round(us, 1), "unit": "us/call", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantised)", "data": "synthetic, seeded",
        "config": _config("ep", world, (T,)),
        "cpu_baseline": {"value": round(us, 1), "unit": "us/call", "cores": os.cpu_count(), "kind": "port",
                         "sample": sample, **_host_info()},
        "e2e": {"value": round(us, 1), "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_flashinfer(args):
    """Comparator (not the reference): FlashInfer's fused FP8 block-scale MoE,
    flashinfer.fused_moe.trtllm_fp8_block_scale_moe, called as a library on
    the same inputs with DeepSeek-V3 routing (routing_method_type=2). The
    reference wires this call in solution/triton/dsl-temp1.py:226-263. Its
    first call JIT-compiles the launcher (minutes on a fresh machine); every
    T gets one tuning pass under flashinfer's autotuner before timing. The
    line reports, per T, the µs/call and the parity against the CPU oracle on
    up to 64 tokens (fraction of elements within atol = rtol = 1e-2)."""
    import numpy as np
    import torch
    from flashinfer.fused_moe import trtllm_fp8_block_scale_moe

    try:
        from flashinfer.autotuner import autotune
    except ImportError:  # pragma: no cover
        autotune = None
    dev = torch.device("cuda", 0)
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    O = importlib.import_module("oracle.moe_oracle")
    name = args.workload if args.workload in SWEEP else "decode_sweep"
    Ts, wdesc = WORKLOADS[name]
    if args.T:
        Ts = tuple(int(t) for t in args.T.split(","))
    w = wl.make_weights(32, 0, dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    per_T = {}
    for T in Ts:
        acts = wl.config_activations(T)
        a = acts.to(dev)

        def fn():
            return trtllm_fp8_block_scale_moe(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2,
                                              256, 8, 8, 4, 2048, 0, 32, 2.5, routing_method_type=2,
                                              tune_max_num_tokens=max(T, 8192))

        if autotune is not None:
            with autotune(True):
                fn()
        out = fn()
        torch.cuda.synchronize()
        rows = np.arange(T) if T <= 64 else np.linspace(0, T - 1, 64).astype(np.int64)
        ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden),
                            acts.hidden_scale.numpy(), lambda le: w.expert_cpu(le), 0, 2.5, 32, token_subset=rows)
        frac = O.allclose_fraction(out.float().cpu().numpy()[rows], O.bf16_bits_to_f32(ref["out_bf16"]), 1e-2, 1e-2)
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
        per_T[str(T)] = {"us": round(statistics.mean(x.elapsed_time(y) for x, y in evs) * 1e3, 2),
                         "parity_frac_within_1e-2": round(frac, 4), "parity_rows": int(len(rows))}
    value = statistics.mean(v["us"] for v in per_T.values())
    print(json.dumps({"metric": METRIC, "value": round(value, 3), "unit": "us/call", "impl": "flashinfer",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                      "config": _config(name, 1, Ts), "sweep": per_T}), flush=True)


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


def bench_shared(args):
    """The shared expert fused into the layer's persistent GEMMs, against the
    routed-only layer and against running it separately: per T, µs of
    (a) the routed layer, (b) the fused call, (c) a shared-expert-only call of
    the same entry (a routing bias that sends no token to a local expert), so
    that a separate launch costs a + c and the fused one b."""
    import torch

    pkg = importlib.import_module("flashinfer-mlsys_b200")
    wl = importlib.import_module("flashinfer-mlsys_b200.workloads")
    dev = torch.device("cuda", 0)
    Ts = tuple(int(t) for t in args.T.split(",")) if args.T else WORKLOADS["shared"][0]
    w = wl.make_weights(32, 0, dev)
    sh = tuple(t.to(dev) for t in wl.expert_weights(300, dev, 0))
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
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
        return statistics.mean(a.elapsed_time(b) for a, b in evs) * 1e3

    sweep = {}
    with ClockSampler(0) as clk:
        for T in Ts:
            a = wl.config_activations(T).to(dev)
            none_bias = a.bias.float().clone()
            none_bias[:32] -= 10.0  # no token picks a local expert
            none_bias = none_bias.to(torch.bfloat16)
            out = torch.empty((T, 7168), dtype=torch.bfloat16, device=dev)
            routed = timed(lambda: pkg.kernel(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2, w.s2,
                                              0, 2.5, out))
            fused = timed(lambda: pkg.kernel_shared(a.logits, a.bias, a.hidden, a.hidden_scale, w.w13, w.s13, w.w2,
                                                    w.s2, 0, 2.5, *sh, out))
            alone = timed(lambda: pkg.kernel_shared(a.logits, none_bias, a.hidden, a.hidden_scale, w.w13, w.s13,
                                                    w.w2, w.s2, 0, 2.5, *sh, out))
            sweep[str(T)] = {"routed_us": round(routed, 2), "fused_us": round(fused, 2),
                             "shared_alone_us": round(alone, 2), "added_by_fusion_us": round(fused - routed, 2),
                             "separate_total_us": round(routed + alone, 2)}
    if pkg.device_status() != 0:
        raise RuntimeError("device-side wait timed out during the benchmark")
    line = {"metric": "us/call of the MoE layer with DeepSeek-V3's shared expert, fused vs separate",
            "value": statistics.mean(v["fused_us"] for v in sweep.values()), "unit": "us/call (mean over T)",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "dtype": "e4m3 x e4m3 -> f32 (tcgen05 kind::f8f6f4)", "data": "synthetic, seeded",
            "config": {"workload": f"shared: {WORKLOADS['shared'][1]}", "T": list(Ts), "l2": L2_NOTE},
            "sweep": sweep, "gpu_launches": 4 * 3 * (args.steps + args.warmup) * len(Ts), "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "flashinfer"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="default: ep (the configs[4] shape) at every N, with the T sweep at N = 1")
    ap.add_argument("--T", default="", help="comma-separated token counts overriding the workload's sweep")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="N = 1: skip the T sweep")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        bench_reference(args)
    elif args.impl == "flashinfer":
        bench_flashinfer(args)
    elif args.workload in ("quant", "addnorm"):
        bench_quant(args)
    elif args.workload == "shared":
        bench_shared(args)
    else:
        if args.workload is None:
            args.workload = "ep"
        bench_ours(args)


if __name__ == "__main__":
    main()
