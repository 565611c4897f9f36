#!/usr/bin/env python
"""Headline benchmark: GQA flash-attention TFLOPS/s on B200.

One GPU (the default): BASELINE config 2, the north-star shape: Gemma-4-E2B
global layer, B=1, H_Q=32, H_KV=4, D=512, causal, N=16384, bf16, inputs seeded
N(0,1)*0.5. One step = one forward + backward through the public autograd API
(FlashAttnGQAFunction: 1 forward launch, then the materialised backward's dQ +
P/dS launch and dK + dV launch). FLOPs are charged by the reference's
convention (fwd+bwd = 7*B*H*N^2*D, window-limited for a sliding window).

N > 1 GPUs (torchrun, one rank per GPU): BASELINE config 4 as one fixed
problem (strong scaling): B=4, H_Q=16, H_KV=2, D=512, causal, N=16384, bf16.
Its 8 (batch, KV-head) units are spread over the ranks in equal blocks, each
rank computes whole units, and NCCL all-gathers reassemble O, LSE, dQ, dK and
dV on every rank inside the timed step (sharding.UnitShardedAttention; the O
gather overlaps the backward kernels, the dQ gather the dK/dV kernels).
`--scaling weak` instead runs config 2 with one batch element per rank and no
collective. The one-GPU line carries config 4 on one GPU (`cfg4_1gpu`) as the
strong-scaling reference.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Timing: W warm-up steps, then K steps between barrier + synchronize, CUDA
events on the launching stream, max over ranks. Q/dO are 512 MiB each (1 GiB
at config 4), larger than the 126 MB L2, so no flush is needed between steps.

CPU legs (`cpu_baseline`, `--impl reference`): the reference's own CPU path
for this math, its eager `attention_gqa_ref` (expand KV heads + torch SDPA in
fp32, autograd backward; restated in oracle/eager_ref.py), on all host cores,
on a bounded sample of the same workload (2 query heads of one KV group at the
full N=16384), plus BASELINE config 1 whole (B=1, 32/4, N=512, D=512, fp32).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "gemma-triton-flash-attn_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "attn TFLOPS/s fwd & fwd+bwd (D=512 causal, D=256 SWA) at 1/2/4/8 B200"
WORKLOADS = {
    "cfg2": dict(name="gemma4-e2b global layer: GQA 32/4, D=512, causal, N=16384, bf16, fwd+bwd",
                 B=1, Hq=32, Hkv=4, N=16384, D=512, causal=True, W=0, dtype=torch.bfloat16, factor=0.5),
    "cfg3": dict(name="MoE sliding layer: GQA 16/8, D=256, causal SWA W=1024, N=16384, fp16, fwd+bwd",
                 B=1, Hq=16, Hkv=8, N=16384, D=256, causal=True, W=1024, dtype=torch.float16, factor=1.0),
    "cfg5": dict(name="config 5: random-init Gemma-4-E2B-shaped decoder (35 layers: 7 global D=512 32/4, "
                      "28 sliding W=512 D=256 16/8), forward through hf_integration, N=16384, bf16",
                 B=1, Hq=32, Hkv=4, N=16384, D=512, causal=True, W=0, dtype=torch.bfloat16, factor=1.0),
    "cfg4": dict(name="MoE global layer: GQA 16/2, D=512, causal, N=16384, bf16, fwd+bwd (B=4 total)",
                 B=4, Hq=16, Hkv=2, N=16384, D=512, causal=True, W=0, dtype=torch.bfloat16, factor=1.0),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="default: cfg2 on one GPU, cfg4 (strong scaling) on several")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="N > 1: strong = one config-4 problem over the GPUs with all-gathers (default); "
                         "weak = config 2 per GPU, no collective")
    ap.add_argument("--gather", choices=["nccl", "ce"], default="ce",
                    help="N > 1 strong scaling: all-gathers by NCCL, or copy-engine pushes into symmetric memory")
    ap.add_argument("--seqlen", type=int, default=None, help="override N (not the headline)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-config sweep of the one-GPU line")
    ap.add_argument("--only", choices=["fwd", "dq", "dk", "dv", "dqps", "dkv"], default=None,
                    help="profiling mode: run only this kernel, warmup + steps launches, print nothing")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return dict(tflops_burst=d.get("bf16_tflops"), tflops_sustained=d.get("bf16_tflops_sustained"),
                    hbm_gbs=d.get("hbm_gbs"), source="measured")
    return dict(tflops_burst=1590.0, tflops_sustained=1400.0, hbm_gbs=6650.0, source="fallback")


class ClockSampler:
    """SM clocks and throttle reasons sampled while the timed steps run.

    NVML (read-only queries) from a background thread every 20 ms, so even a
    timed region of a few hundred ms gets samples; the first sample is taken
    before __enter__ returns. Falls back to `nvidia-smi -lms 200` without NVML."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, uuids, period_s=0.02):
        self.uuids = list(uuids)
        self.period = period_s
        self.proc = None
        self.thread = None
        self.samples = []  # (sm_mhz, max_mhz, reason bits)
        self.path = os.path.join("/tmp", f"gqafa_clocks_{os.getpid()}.csv")

    def _nvml_start(self):
        import threading

        import pynvml
        pynvml.nvmlInit()
        handles = [pynvml.nvmlDeviceGetHandleByUUID(u) for u in self.uuids]
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

        def sample():
            for h in handles:
                self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                     pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM),
                                     int(get_reasons(h))))

        self.stop = threading.Event()

        def loop():
            while not self.stop.wait(self.period):
                sample()

        sample()
        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def __enter__(self):
        try:
            self._nvml_start()
            return self
        except Exception:  # no NVML: nvidia-smi
            self.thread = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()
        return False

    def summary(self):
        if self.thread is not None:
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
            bits = 0
            for _, _, r in self.samples:
                bits |= r
            reasons = sorted(n for n, b in self.REASON_BITS.items() if bits & b)
            return {"sm_mhz": statistics.median(x[0] for x in self.samples),
                    "sm_max_mhz": max(x[1] for x in self.samples), "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml, 20 ms"}
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        mhz, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            if self.uuids and parts[0] not in self.uuids:
                continue
            try:
                mhz.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for n, flag in zip(names, parts[4:8]):
                if flag.lower().startswith("active"):
                    reasons.add(n)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(mhz), "source": "nvidia-smi, 200 ms"}


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


# ------------------------------------------------------------------ CPU legs
CPU_SAMPLE_HEADS = 1


def cpu_eager_sample(wl, seed=0, warmup=1, reps=3):
    """The reference's eager CPU path (oracle/eager_ref.py) on a bounded sample
    of `wl`: query heads 0 .. CPU_SAMPLE_HEADS-1 of batch 0 (both in KV group
    0) with their KV head, at the full sequence length, fp32 forward +
    autograd backward. Returns (median seconds, charged FLOPs, threads, text)."""
    from gemma_triton_flash_attn.flops import attn_flops
    from oracle.eager_ref import time_fwd_bwd, use_all_cores

    threads = use_all_cores()
    N, D, causal = wl["N"], wl["D"], wl["causal"]
    window = wl["W"] if (causal and 0 < wl["W"] < N) else 0
    hq = min(CPU_SAMPLE_HEADS, wl["Hq"] // wl["Hkv"])
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g) * wl["factor"]).to(wl["dtype"]).float()  # noqa: E731
    q, k, v, do = mk(1, hq, N, D), mk(1, 1, N, D), mk(1, 1, N, D), mk(1, hq, N, D)
    t = time_fwd_bwd(q, k, v, do, causal, window, warmup=warmup, reps=reps)
    fl = attn_flops(1, hq, N, D, causal, window, bwd=True)
    text = (f"reference eager path (KV heads repeated + torch SDPA, fp32, autograd backward; oracle/eager_ref.py) "
            f"on {threads} threads: fwd+bwd of query heads 0-{hq - 1} of KV group 0 at N={N}, D={D}"
            + (f", window {window}" if window else "") + f"; median of {reps} after {warmup} warm-up")
    return t, fl, threads, text


def cpu_config1(warmup=3, reps=9):
    """BASELINE config 1 whole: fp32, B=1, H_Q=32, H_KV=4, N=512, D=512, causal,
    N(0,1) inputs; fwd and fwd+bwd medians of the reference's eager path."""
    from oracle.eager_ref import time_fwd_bwd, use_all_cores

    threads = use_all_cores()
    g = torch.Generator().manual_seed(0)
    q, k, v, do = (torch.randn(s, generator=g) for s in ((1, 32, 512, 512), (1, 4, 512, 512), (1, 4, 512, 512),
                                                         (1, 32, 512, 512)))
    t_fwd = time_fwd_bwd(q, k, v, do, True, warmup=warmup, reps=reps, fwd_only=True)
    t_all = time_fwd_bwd(q, k, v, do, True, warmup=warmup, reps=reps)
    fl = 32 * 512 * 512 * 512
    return dict(fwd_ms=round(t_fwd * 1e3, 2), fwd_tflops=round(2 * fl / t_fwd / 1e12, 4),
                fwd_bwd_ms=round(t_all * 1e3, 2), fwd_bwd_tflops=round(7 * fl / t_all / 1e12, 4),
                threads=threads, cpu=_cpu_model(), method=f"median of {reps} after {warmup} warm-up")


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_baseline(wl):
    t, fl, threads, text = cpu_eager_sample(wl)
    return dict(value=round(fl / t / 1e12, 5), unit="TFLOPS/s", cores=threads, kind="port", sample=text,
                ms_per_sample=round(t * 1e3, 1), config1=cpu_config1())


# ------------------------------------------------------------------ GPU helpers
def make_inputs(wl, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    B, Hq, Hkv, N, D = wl["B"], wl["Hq"], wl["Hkv"], wl["N"], wl["D"]
    out = []
    for shp in ((B, Hq, N, D), (B, Hkv, N, D), (B, Hkv, N, D), (B, Hq, N, D)):
        x = torch.randn(shp, generator=g, device=device, dtype=torch.float32) * wl["factor"]
        out.append(x.to(wl["dtype"]))
        del x
    return out


def time_loop(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def _window(wl):
    return wl["W"] if (wl["causal"] and 0 < wl["W"] < wl["N"]) else 0


def _uuid(device):
    u = str(torch.cuda.get_device_properties(device).uuid)
    return [u if u.startswith("GPU-") else "GPU-" + u]


def train_step_fn(q, k, v, do, causal, W):
    from gemma_triton_flash_attn import FlashAttnGQAFunction

    qg, kg, vg = (t.detach().requires_grad_(True) for t in (q, k, v))

    def step():
        qg.grad = kg.grad = vg.grad = None
        out = FlashAttnGQAFunction.apply(qg, kg, vg, causal, W)
        out.backward(do)

    return step


def measure_config(wl, device, stream, warmup=2, steps=3, seed=1234):
    """fwd and fwd+bwd of one workload through the public API: ms and TFLOPS/s."""
    from gemma_triton_flash_attn.attention import _fwd
    from gemma_triton_flash_attn.flops import attn_flops

    q, k, v, do = make_inputs(wl, seed, device)
    causal, W, window = wl["causal"], wl["W"], _window(wl)
    scale = 1.0 / math.sqrt(wl["D"])
    step = train_step_fn(q, k, v, do, causal, W)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ms = time_loop(step, steps, stream)
    f = lambda: _fwd(q, k, v, causal, window, scale, True)  # noqa: E731
    f()
    torch.cuda.synchronize()
    ms_f = time_loop(f, max(steps, 5), stream)
    B, Hq, N, D = wl["B"], wl["Hq"], wl["N"], wl["D"]
    res = dict(N=N, D=D, H_Q=Hq, H_KV=wl["Hkv"], B=B, window=window,
               dtype="bf16" if wl["dtype"] == torch.bfloat16 else "fp16",
               fwd_ms=round(ms_f, 3), fwd_tflops=round(attn_flops(B, Hq, N, D, causal, window) / ms_f / 1e9, 1),
               fwd_bwd_ms=round(ms, 3),
               fwd_bwd_tflops=round(attn_flops(B, Hq, N, D, causal, window, bwd=True) / ms / 1e9, 1))
    del q, k, v, do, step
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------ profiling mode
def run_only(args, wl, local):
    """Run one kernel (warmup + steps launches) for ncu; prints nothing."""
    from gemma_triton_flash_attn import _lib
    from gemma_triton_flash_attn.attention import _alloc_workspace, _bwd, _fwd, bwd_workspace_size

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    B, Hq, Hkv, N, D, causal = (wl[x] for x in ("B", "Hq", "Hkv", "N", "D", "causal"))
    window = _window(wl)
    scale = 1.0 / math.sqrt(D)
    q, k, v, do = make_inputs(wl, 1234, device)
    o, lse = _fwd(q, k, v, causal, window, scale, True)
    bufs = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
            torch.empty((B, Hq, N), dtype=torch.float32, device=device))
    ws = None
    if args.only in ("dqps", "dkv"):
        ws = _alloc_workspace(bwd_workspace_size(B, Hq, Hkv, N, D, causal, window), device)
        if ws is None:
            raise SystemExit("--only %s: no materialised backward for this workload" % args.only)
        _bwd(q, k, v, o, lse, do, causal, window, scale, stage=0, out=bufs, workspace=ws)
    elif args.only != "fwd":
        _bwd(q, k, v, o, lse, do, causal, window, scale, stage=0, out=bufs)  # delta for dK
    torch.cuda.synchronize()
    stage = {"dq": 0, "dk": 1, "dv": 2, "dqps": 0, "dkv": 1}.get(args.only)
    for _ in range(args.warmup + args.steps):
        if stage is None:
            _fwd(q, k, v, causal, window, scale, True)
        else:
            _bwd(q, k, v, o, lse, do, causal, window, scale, stage=stage, out=bufs, workspace=ws)
    torch.cuda.synchronize()
    if _lib.device_status(local) != 0:
        raise RuntimeError("kernel status word set")


# ------------------------------------------------------------------ one GPU (and weak scaling)
def run_single(args, wl, world, rank, local):
    from gemma_triton_flash_attn import FlashAttnGQAFunction, _lib
    from gemma_triton_flash_attn.attention import _alloc_workspace, _bwd, _fwd, bwd_workspace_size
    from gemma_triton_flash_attn.flops import attn_flops, kernel_flops

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    B, Hq, Hkv, N, D, causal, W = (wl[x] for x in ("B", "Hq", "Hkv", "N", "D", "causal", "W"))
    window = _window(wl)
    scale = 1.0 / math.sqrt(D)
    q, k, v, do = make_inputs(wl, 1234 + rank, device)
    step = train_step_fn(q, k, v, do, causal, W)
    flops_step = attn_flops(B, Hq, N, D, causal, window, bwd=True)
    flops_fwd = attn_flops(B, Hq, N, D, causal, window)

    torch.cuda.reset_peak_memory_stats(device)
    base_mem = torch.cuda.memory_allocated(device)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(_uuid(device)) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        ms = time_loop(step, args.steps, stream)
        barrier(world)
    peak_gb = (torch.cuda.max_memory_allocated(device) - base_mem) / 1e9
    ms_max = max_over_ranks(ms, world, device)
    value = world * flops_step / (ms_max * 1e-3) / 1e12

    # forward alone (same launch as inside the step)
    for _ in range(2):
        _fwd(q, k, v, causal, window, scale, True)
    torch.cuda.synchronize()
    barrier(world)
    ms_fwd = max_over_ranks(time_loop(lambda: _fwd(q, k, v, causal, window, scale, True), args.steps, stream),
                            world, device)

    ws_bytes = bwd_workspace_size(B, Hq, Hkv, N, D, causal, window)
    # per-kernel timing for the roofline: the kernels the step above ran
    o, lse = _fwd(q, k, v, causal, window, scale, True)
    bufs = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
            torch.empty((B, Hq, N), dtype=torch.float32, device=device))
    kernels = {"fwd": ms_fwd}
    ws = _alloc_workspace(ws_bytes, device)
    if ws is not None:  # materialised backward: dQ (+ P, dS stores), then dK + dV
        names = ("dqps", "dkv")
        mk = lambda st: (lambda: _bwd(q, k, v, o, lse, do, causal, window, scale, stage=st, out=bufs,  # noqa: E731
                                      workspace=ws))
    else:
        names = ("dq", "dk", "dv")
        mk = lambda st: (lambda: _bwd(q, k, v, o, lse, do, causal, window, scale, stage=st, out=bufs))  # noqa: E731
    for stage, name in enumerate(names):
        fn = mk(stage)
        fn()
        torch.cuda.synchronize()
        kernels[name] = time_loop(fn, args.steps, stream)
    del ws
    status = _lib.device_status(local)
    dom = max(kernels, key=kernels.get)
    peaks = measured_peaks()
    kflops = kernel_flops(dom, B, Hq, N, D, causal, window)
    achieved = kflops / (kernels[dom] * 1e-3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get(f"{args.workload}:{dom}")
    burst, sust = peaks["tflops_burst"], peaks["tflops_sustained"]
    roofline = dict(bound="tensor", kernel=dom, achieved=round(achieved, 1), peak=burst, unit="TFLOP/s",
                    frac=round(achieved / burst, 4), traffic=traffic,
                    peak_kind=f"bf16_tflops burst ({peaks['source']}): the kernel is timed alone in a sub-second loop",
                    frac_of_sustained=round(achieved / sust, 4), sustained_peak=sust,
                    step_frac=round(value / world / burst, 4),
                    flops_per_launch=kflops, ms_per_launch=round(kernels[dom], 3),
                    kernel_ms={k_: round(v_, 3) for k_, v_ in kernels.items()},
                    kernel_share={k_: round(v_ / sum(kernels.values()), 3) for k_, v_ in kernels.items()})

    # the recomputing backward (no workspace): what the memory fallback runs
    recompute = None
    if world == 1 and not args.no_sweep:
        os.environ["GQAFA_BWD_WORKSPACE_LIMIT"] = "0"
        try:
            torch.cuda.reset_peak_memory_stats(device)
            base = torch.cuda.memory_allocated(device)
            step()
            torch.cuda.synchronize()
            ms_r = time_loop(step, 3, stream)
            recompute = dict(value=round(flops_step / (ms_r * 1e-3) / 1e12, 2), unit="TFLOPS/s",
                             ms_per_step=round(ms_r, 3),
                             peak_mem_gb=round((torch.cuda.max_memory_allocated(device) - base) / 1e9, 3),
                             kernels="fwd + dQ(+delta) + dK + dV, recomputing S and dP")
        finally:
            del os.environ["GQAFA_BWD_WORKSPACE_LIMIT"]

    # end to end through the public API with host buffers. Every step uploads
    # its own q, k, v, dO from pinned host memory and downloads dQ, dK, dV;
    # the copies run on their own streams, step s+1's upload (into the other
    # of two input buffer sets) overlapping step s's kernels and step s's
    # download overlapping step s+1's, as a prefetching input pipeline would.
    e2e = None
    if not args.no_e2e:
        host_in = [t.cpu().pin_memory() for t in (q, k, v, do)]
        host_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, k, v)]
        dev_in = [[torch.empty_like(t) for t in (q, k, v, do)] for _ in range(2)]
        up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_free = [torch.cuda.Event() for _ in range(2)]

        def upload(s):
            buf = dev_in[s % 2]
            with torch.cuda.stream(up):
                if s >= 2:
                    up.wait_event(ev_free[s % 2])
                for d_, h_ in zip(buf, host_in):
                    d_.copy_(h_, non_blocking=True)
                ev_in[s % 2].record(up)

        def e2e_run(nsteps):
            up.wait_stream(stream)  # uploads start inside the timed region
            upload(0)
            for s_ in range(nsteps):
                if s_ + 1 < nsteps:
                    upload(s_ + 1)
                stream.wait_event(ev_in[s_ % 2])
                xq, xk, xv, xdo = dev_in[s_ % 2]
                qq, kk, vv = (t.detach().requires_grad_(True) for t in (xq, xk, xv))
                out = FlashAttnGQAFunction.apply(qq, kk, vv, causal, W)
                out.backward(xdo)
                ev_free[s_ % 2].record(stream)
                grads = (qq.grad, kk.grad, vv.grad)
                down.wait_stream(stream)
                with torch.cuda.stream(down):
                    for h_, g_ in zip(host_out, grads):
                        g_.record_stream(down)
                        h_.copy_(g_, non_blocking=True)
            stream.wait_stream(down)

        e2e_run(2)
        torch.cuda.synchronize()
        barrier(world)
        ms_e2e = max_over_ranks(time_loop(lambda: e2e_run(args.steps), 1, stream) / args.steps, world, device)
        h2d = sum(t.numel() * t.element_size() for t in host_in)
        d2h = sum(t.numel() * t.element_size() for t in host_out)
        e2e = dict(value=round(world * flops_step / (ms_e2e * 1e-3) / 1e12, 2), unit="TFLOPS/s",
                   ms_per_step=round(ms_e2e, 3), h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                   pipeline="copy streams; step s+1 upload and step s download overlap kernels")
        del host_in, host_out, dev_in

    del q, k, v, do, step, o, lse, bufs
    torch.cuda.empty_cache()

    # the other configurations of the reference's sweep, through the same API
    sweep, cfg4, cfg5, host = None, None, None, None
    if world == 1 and not args.no_sweep and args.workload == "cfg2" and args.seqlen is None:
        sweep = []
        variants = [("cfg2", dict(N=1024), 20), ("cfg2", dict(N=4096), 5), ("cfg2", dict(N=32768), 2),
                    ("cfg2", dict(dtype=torch.float16), 3), ("cfg3", dict(), 10), ("cfg3", dict(N=32768), 5)]
        for name, over, nsteps in variants:
            w = dict(WORKLOADS[name])
            w.update(over)
            r = measure_config(w, device, stream, steps=nsteps)
            r["workload"] = name
            sweep.append(r)
        cfg4 = run_cfg4_one_gpu(device, stream, steps=3)
        host = host_overhead(device, stream)
        cfg5 = run_decoder_once(device, stream, steps=2)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(wl)

    if rank == 0:
        line = dict(
            metric=METRIC, value=round(value, 2), unit="TFLOPS/s", n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=round(ms_max, 3), higher_is_better=True, scaling="weak",
            vs_baseline=None, dtype="bf16" if wl["dtype"] == torch.bfloat16 else "fp16",
            data="synthetic (seeded N(0,1)*%g, per-rank seed)" % wl["factor"],
            config=dict(workload=wl["name"], B_per_gpu=B, H_Q=Hq, H_KV=Hkv, N=N, D=D, causal=causal,
                        window=window, global_batch=B * world, seq_len=N,
                        parallelism=f"(b,kv-group) units, dp{world}, no collective",
                        l2="inputs larger than L2 (Q, dO 512 MiB each); no flush"),
            fwd=dict(value=round(world * flops_fwd / (ms_fwd * 1e-3) / 1e12, 2), unit="TFLOPS/s",
                     ms=round(ms_fwd, 3)),
            roofline=roofline, cpu_baseline=cpu, e2e=e2e, clocks=clocks.summary(),
            gpu_launches=(1 + len(names)) * args.steps, kernel_status=status,
            bwd_path="materialised (workspace %d bytes)" % ws_bytes if len(names) == 2 else "recompute",
            peak_mem_gb=round(peak_gb, 3), recompute_bwd=recompute, sweep=sweep, cfg4_1gpu=cfg4,
            cfg5_decoder_1gpu=cfg5, host_overhead=host,
        )
        print(json.dumps(line), flush=True)


def host_overhead(device, stream, n=1024, calls=30):
    """Host (CPU) cost of one fwd+bwd through the public autograd API at a short
    sequence, where the GPU work per call is smallest: wall time per call of
    a loop that only enqueues (the GPU queue absorbs the launches), against
    the GPU time per call from CUDA events."""
    wl = dict(WORKLOADS["cfg2"])
    wl["N"] = n
    q, k, v, do = make_inputs(wl, 7, device)
    step = train_step_fn(q, k, v, do, True, 0)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(calls):
        step()
    host_ms = (time.perf_counter() - t0) * 1e3 / calls
    torch.cuda.synchronize()
    gpu_ms = time_loop(step, calls, stream)
    return dict(N=n, host_ms_per_call=round(host_ms, 4), gpu_ms_per_call=round(gpu_ms, 4),
                note="config-2 shape at N=1024; host = enqueue-only wall time per public-API fwd+bwd "
                     "(autograd, torch operators over the C ABI, tensor-map encoding, allocations); 3 kernels per call")


def run_cfg4_one_gpu(device, stream, steps=3, warmup=2):
    """Config 4 on one GPU through the same UnitShardedAttention step the
    multi-GPU line runs (no collective at world size 1): the strong-scaling
    reference."""
    from gemma_triton_flash_attn.flops import attn_flops
    from gemma_triton_flash_attn.sharding import UnitShardedAttention

    wl = WORKLOADS["cfg4"]
    B, Hq, Hkv, N, D = wl["B"], wl["Hq"], wl["Hkv"], wl["N"], wl["D"]
    q, k, v, do = make_inputs(wl, 1234, device)
    att = UnitShardedAttention(B, Hq, Hkv, N, D, wl["dtype"], device, causal=True)
    for _ in range(warmup):
        att.step(q, k, v, do)
    torch.cuda.synchronize()
    ms = time_loop(lambda: att.step(q, k, v, do), steps, stream)
    res = dict(value=round(attn_flops(B, Hq, N, D, True, 0, bwd=True) / (ms * 1e-3) / 1e12, 2), unit="TFLOPS/s",
               ms_per_step=round(ms, 3), workload=wl["name"])
    del att, q, k, v, do
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------ N GPUs, one problem
def run_strong(args, wl, world, rank, local):
    """Strong scaling: one config-4 problem over all ranks in (batch, KV-head)
    unit blocks; O, LSE, dQ, dK, dV all-gathered on every rank inside the step."""
    from gemma_triton_flash_attn import _lib
    from gemma_triton_flash_attn.flops import attn_flops, kernel_flops
    from gemma_triton_flash_attn.sharding import UnitShardedAttention

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    B, Hq, Hkv, N, D, causal = (wl[x] for x in ("B", "Hq", "Hkv", "N", "D", "causal"))
    window = _window(wl)
    q, k, v, do = make_inputs(wl, 1234, device)  # the same problem on every rank
    att = UnitShardedAttention(B, Hq, Hkv, N, D, wl["dtype"], device, causal=causal, slide_size=wl["W"],
                               gather=args.gather)
    step = lambda: att.step(q, k, v, do)  # noqa: E731
    total = attn_flops(B, Hq, N, D, causal, window, bwd=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(_uuid(device)) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        ms = time_loop(step, args.steps, stream)
        barrier(world)
    ms_max = max_over_ranks(ms, world, device)
    value = total / (ms_max * 1e-3) / 1e12

    # the same kernels with the collectives left out: the exposed share of the
    # all-gathers is the difference
    def compute_only():
        w = att.world
        att.world = 1
        try:
            att.forward(q, k, v)
            att.backward(q, k, v, do)
        finally:
            att.world = w

    compute_only()
    torch.cuda.synchronize()
    barrier(world)
    ms_c = max_over_ranks(time_loop(compute_only, args.steps, stream), world, device)
    status = _lib.device_status(local)
    gathered = sum(t.numel() * t.element_size() for t in (att.o, att.lse, att.dq, att.dk, att.dv))

    # end to end: each rank uploads its own units' q, k, v, dO from pinned host
    # memory and downloads its own units' dQ, dK, dV; the all-gathers still
    # reassemble every output on every rank inside the step. Two device input
    # sets: step s+1's upload (copy stream) overlaps step s's kernels, and step
    # s's download (another copy stream) overlaps step s+1's.
    e2e = None
    if not args.no_e2e:
        nr = len(att.runs)
        host_q = [[att._qv(i, t).cpu().pin_memory() for t in (q, do)] for i in range(nr)]
        host_k = [[att._kvv(i, t).cpu().pin_memory() for t in (k, v)] for i in range(nr)]
        outs = [[torch.empty(att._qv(i, att.dq).shape, dtype=q.dtype).pin_memory(),
                 torch.empty(att._kvv(i, att.dk).shape, dtype=k.dtype).pin_memory(),
                 torch.empty(att._kvv(i, att.dv).shape, dtype=v.dtype).pin_memory()] for i in range(nr)]
        sets = [[q, k, v, do], [torch.empty_like(t) for t in (q, k, v, do)]]
        up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_free = [torch.cuda.Event() for _ in range(2)]
        ev_out = torch.cuda.Event()

        def upload(s_):
            xq, xk, xv, xdo = sets[s_ % 2]
            with torch.cuda.stream(up):
                if s_ >= 2:
                    up.wait_event(ev_free[s_ % 2])
                for i in range(nr):
                    att._qv(i, xq).copy_(host_q[i][0], non_blocking=True)
                    att._qv(i, xdo).copy_(host_q[i][1], non_blocking=True)
                    att._kvv(i, xk).copy_(host_k[i][0], non_blocking=True)
                    att._kvv(i, xv).copy_(host_k[i][1], non_blocking=True)
                ev_in[s_ % 2].record(up)

        def e2e_run(nsteps):
            up.wait_stream(stream)  # uploads start inside the timed region
            upload(0)
            for s_ in range(nsteps):
                if s_ + 1 < nsteps:
                    upload(s_ + 1)
                stream.wait_event(ev_in[s_ % 2])
                xq, xk, xv, xdo = sets[s_ % 2]
                att.forward(xq, xk, xv)
                if s_ > 0:  # this step's backward overwrites dQ / dK / dV: after the last download
                    stream.wait_event(ev_out)
                att.backward(xq, xk, xv, xdo)
                att.wait()
                ev_free[s_ % 2].record(stream)
                down.wait_stream(stream)
                with torch.cuda.stream(down):
                    for i in range(nr):
                        outs[i][0].copy_(att._qv(i, att.dq), non_blocking=True)
                        outs[i][1].copy_(att._kvv(i, att.dk), non_blocking=True)
                        outs[i][2].copy_(att._kvv(i, att.dv), non_blocking=True)
                    ev_out.record(down)
            stream.wait_stream(down)

        e2e_run(2)
        torch.cuda.synchronize()
        barrier(world)
        ms_e = max_over_ranks(time_loop(lambda: e2e_run(args.steps), 1, stream) / args.steps, world, device)
        h2d = sum(t.numel() * t.element_size() for r in host_q + host_k for t in r)
        d2h = sum(t.numel() * t.element_size() for r in outs for t in r)
        e2e = dict(value=round(total / (ms_e * 1e-3) / 1e12, 2), unit="TFLOPS/s", ms_per_step=round(ms_e, 3),
                   h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                   pipeline="each rank copies only its own units in and out on copy streams (step s+1 upload "
                            "overlaps step s); all-gathers inside the step")

    gather_kind, n_runs = att.gather, len(att.runs)
    del att, q, k, v, do
    torch.cuda.empty_cache()
    try:
        cfg2 = cfg2_over_gpus(args, world, device, stream)
    except Exception as e:  # a secondary key must not take the headline down
        cfg2 = dict(error=f"{type(e).__name__}: {e}"[:300])

    peaks = measured_peaks()
    per_rank = total / world
    if rank == 0:
        line = dict(
            metric=METRIC, value=round(value, 2), unit="TFLOPS/s", n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=round(ms_max, 3), higher_is_better=True, scaling="strong",
            vs_baseline=None, dtype="bf16" if wl["dtype"] == torch.bfloat16 else "fp16",
            data="synthetic (seeded N(0,1)*%g, the same problem on every rank)" % wl["factor"],
            config=dict(workload=wl["name"], global_batch=B, H_Q=Hq, H_KV=Hkv, N=N, D=D, causal=causal,
                        seq_len=N, units=B * Hkv, units_per_gpu=B * Hkv // world,
                        parallelism=f"{B * Hkv} (b,kv-group) units in equal blocks over {world} GPUs; "
                                    f"O/LSE/dQ/dK/dV all-gathered ({gather_kind}) inside the step",
                        l2="inputs larger than L2 (Q, dO 1 GiB each); no flush"),
            collective=dict(ms_compute_only=round(ms_c, 3), exposed_ms=round(ms_max - ms_c, 3),
                            exposed_share=round(max(0.0, ms_max - ms_c) / ms_max, 4),
                            bytes_gathered_per_rank=round(gathered * (world - 1) / world),
                            op=("all_gather_into_tensor x5 (NCCL, in place)" if gather_kind == "nccl" else
                                "copy-engine pushes of each rank's slice into every peer's symmetric buffer x5, "
                                "one-element NCCL all-reduce to close the step")
                            + ", overlapped with the next kernels"),
            roofline=dict(bound="tensor", kernel="whole step per rank", achieved=round(per_rank / ms_max / 1e9, 1),
                          peak=peaks["tflops_burst"], unit="TFLOP/s",
                          frac=round(per_rank / ms_max / 1e9 / peaks["tflops_burst"], 4), traffic=None),
            e2e=e2e, clocks=clocks.summary(), kernel_status=status,
            gpu_launches=3 * n_runs * args.steps, cfg2_over_gpus=cfg2,
            gpu_launches_note="per rank and step: per run of units 1 forward, 1 dQ+P/dS, 1 dK+dV kernel "
                              "(plus 5 NCCL all-gathers, not counted)",
        )
        print(json.dumps(line), flush=True)


def run_decoder_once(device, stream, steps=2, warmup=1):
    """Config 5 on one GPU: forward tokens/s of the synthetic 35-layer decoder
    with every attention layer through hf_integration (one N=16384 sequence)."""
    from gemma_triton_flash_attn import register_triton_attention
    from gemma_triton_flash_attn.gemma4_synthetic import Gemma4SyntheticConfig, Gemma4SyntheticDecoder

    register_triton_attention()
    cfg = Gemma4SyntheticConfig()
    model = Gemma4SyntheticDecoder(cfg).to(device=device, dtype=torch.bfloat16).init_weights(seed=0)
    N = WORKLOADS["cfg5"]["N"]
    g = torch.Generator().manual_seed(1000)
    ids = torch.randint(0, cfg.vocab_size, (1, N), generator=g).to(device)

    def step():
        with torch.no_grad():
            model(ids)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ms = time_loop(step, steps, stream)
    del model
    torch.cuda.empty_cache()
    return dict(value=round(N / (ms * 1e-3), 1), unit="tokens/s", ms_per_step=round(ms, 3),
                workload=WORKLOADS["cfg5"]["name"])


def cfg2_over_gpus(args, world, device, stream, steps=5, warmup=2):
    """Config 2 (B=1, 4 (batch, KV-head) units) as one problem over the ranks:
    unit blocks with all-gathers when the ranks divide the 4 units, else the
    head split (the query heads of each unit over world/4 ranks, fp32 dK/dV
    partials summed within the unit's ranks). A secondary key of the
    multi-GPU line."""
    from gemma_triton_flash_attn.flops import attn_flops
    from gemma_triton_flash_attn.sharding import UnitShardedAttention

    wl = WORKLOADS["cfg2"]
    B, Hq, Hkv, N, D = wl["B"], wl["Hq"], wl["Hkv"], wl["N"], wl["D"]
    units = B * Hkv
    if units % world != 0 and (world % units != 0 or (Hq // Hkv) % (world // units) != 0):
        return None
    q, k, v, do = make_inputs(wl, 1234, device)
    att = UnitShardedAttention(B, Hq, Hkv, N, D, wl["dtype"], device, causal=True, gather=args.gather)
    step = lambda: att.step(q, k, v, do)  # noqa: E731
    if att.split == 1:
        how = f"(b, kv-group) units, {units // world} per GPU, all-gathers ({args.gather})"
    else:
        how = (f"head split: {Hq // Hkv // att.split} query heads per GPU, fp32 dK/dV partials all-reduced within "
               f"each unit's {att.split} GPUs; O/LSE/dQ all-gathers ({args.gather})")
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(time_loop(step, steps, stream), world, device)
    total = attn_flops(B, Hq, N, D, True, 0, bwd=True)
    res = dict(value=round(total / (ms * 1e-3) / 1e12, 2), unit="TFLOPS/s", ms_per_step=round(ms, 3),
               workload=wl["name"], parallelism=how)
    del q, k, v, do, step, att
    torch.cuda.empty_cache()
    return res


def run_decoder(args, wl, world, rank, local):
    """Config 5: one sequence per GPU (weak scaling), forward tokens/s through
    register_triton_attention() + the synthetic decoder."""
    from gemma_triton_flash_attn import register_triton_attention
    from gemma_triton_flash_attn.flops import attn_flops
    from gemma_triton_flash_attn.gemma4_synthetic import Gemma4SyntheticConfig, Gemma4SyntheticDecoder

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    register_triton_attention()
    cfg = Gemma4SyntheticConfig()
    model = Gemma4SyntheticDecoder(cfg).to(device=device, dtype=torch.bfloat16).init_weights(seed=0)
    N = wl["N"]
    g = torch.Generator().manual_seed(1000 + rank)
    ids_h = torch.randint(0, cfg.vocab_size, (1, N), generator=g).pin_memory()
    ids = torch.empty_like(ids_h, device=device)
    out_h = torch.empty((1,), dtype=torch.int64).pin_memory()

    def step():
        ids.copy_(ids_h, non_blocking=True)
        with torch.no_grad():
            logits = model(ids)
        out_h.copy_(logits[0, -1].argmax().view(1), non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(_uuid(device)) as clocks:
        ms = max_over_ranks(time_loop(step, args.steps, stream), world, device)
    n_glob = sum(cfg.is_global(i) for i in range(cfg.num_layers))
    attn_fl = n_glob * attn_flops(1, cfg.global_heads, N, cfg.global_head_dim, True) + \
        (cfg.num_layers - n_glob) * attn_flops(1, cfg.local_heads, N, cfg.local_head_dim, True, cfg.sliding_window)
    if rank == 0:
        line = dict(metric="config-5 decoder forward tokens/s (attention through hf_integration)",
                    value=round(world * N / (ms * 1e-3), 1), unit="tokens/s", n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=round(ms, 3), higher_is_better=True, scaling="weak",
                    vs_baseline=None, dtype="bf16", data="synthetic (seeded uniform token ids, random-init weights)",
                    config=dict(workload=wl["name"], global_batch=world, seq_len=N,
                                parallelism=f"one sequence per GPU, dp{world}"),
                    attention_tflops_in_step=round(attn_fl / (ms * 1e-3) / 1e12, 1),
                    e2e=dict(value=round(world * N / (ms * 1e-3), 1), unit="tokens/s",
                             h2d_bytes_per_step=ids_h.numel() * 8, d2h_bytes_per_step=8),
                    clocks=clocks.summary(), gpu_launches=35 * args.steps)
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ reference arm
def run_reference(args, wl, world, rank):
    """The reference's eager CPU path (oracle/eager_ref.py) on the host cores:
    each step is one fp32 fwd+bwd of the bounded sample of `wl` that
    cpu_eager_sample describes. Rank 0 only; other ranks exit without work."""
    if rank != 0:
        return
    from gemma_triton_flash_attn.flops import attn_flops
    from oracle.eager_ref import time_fwd_bwd, use_all_cores

    threads = use_all_cores()
    N, D, causal = wl["N"], wl["D"], wl["causal"]
    window = _window(wl)
    hq = min(CPU_SAMPLE_HEADS, wl["Hq"] // wl["Hkv"])
    g = torch.Generator().manual_seed(0)
    mk = lambda *s: (torch.randn(*s, generator=g) * wl["factor"]).to(wl["dtype"]).float()  # noqa: E731
    q, k, v, do = mk(1, hq, N, D), mk(1, 1, N, D), mk(1, 1, N, D), mk(1, hq, N, D)
    t = time_fwd_bwd(q, k, v, do, causal, window, warmup=args.warmup, reps=args.steps)
    value = attn_flops(1, hq, N, D, causal, window, bwd=True) / t / 1e12
    sample = (f"reference eager path (KV heads repeated + torch SDPA, fp32, autograd backward; oracle/eager_ref.py) "
              f"on {threads} threads: fwd+bwd of query heads 0-{hq - 1} of KV group 0 at N={N}, D={D} per step")
    line = dict(
        metric=METRIC, value=round(value, 5), unit="TFLOPS/s", n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(t * 1e3, 1), higher_is_better=True,
        scaling="strong" if args.workload == "cfg4" else "weak",
        vs_baseline=None, dtype="f32", data="synthetic", impl="reference",
        config=dict(workload=wl["name"], B=wl["B"], H_Q=wl["Hq"], H_KV=wl["Hkv"], N=N, D=D, causal=causal,
                    window=window, global_batch=wl["B"], seq_len=N, parallelism="host cores"),
        cpu_baseline=dict(value=round(value, 5), unit="TFLOPS/s", cores=threads, kind="port", sample=sample),
        e2e=dict(value=round(value, 5), unit="TFLOPS/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
        config1=cpu_config1(),
    )
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world, rank, local = setup_dist()
    if args.workload is None:
        args.workload = "cfg4" if (world > 1 and args.scaling == "strong") else "cfg2"
    wl = WORKLOADS[args.workload]
    if args.seqlen:
        wl = dict(wl)
        wl["N"] = args.seqlen
        wl["name"] = wl["name"].replace("N=16384", f"N={args.seqlen}")
    try:
        if args.impl == "reference":
            run_reference(args, wl, world, rank)
        elif args.only:
            run_only(args, wl, local)
        elif args.workload == "cfg5":
            run_decoder(args, wl, world, rank, local)
        elif args.workload == "cfg4":
            run_strong(args, wl, world, rank, local)
        else:
            run_single(args, wl, world, rank, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
