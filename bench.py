#!/usr/bin/env python
"""Headline benchmark: GQA flash-attention TFLOPS/s on B200.

Workload (the north-star shape): Gemma-4-E2B global layer,
B=1 per GPU, H_Q=32, H_KV=4, D=512, causal, N=16384, bf16, inputs seeded
N(0,1)*0.5. One step = one forward + backward through the public autograd API
(FlashAttnGQAFunction: 1 forward launch + 3 backward launches). FLOPs are
charged by the reference's convention (fwd+bwd = 7*B*H*N^2*D).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU: weak scaling, each rank owns one
batch element, i.e. the (b, kv-head-group) units of b = rank; there is no
collective on the data path (the units are independent), so the timed region
holds no communication. Timing: CUDA events on the launching stream, barrier +
synchronize around the K timed steps, max over ranks. Q/dO are 512 MiB each,
larger than the 126 MB L2, so no flush is needed between steps.

`--impl reference` times the reference algorithm's CPU restatement (the
oracle port; the reference itself is Python + Triton and has no native CPU
path of its own beyond PyTorch eager) on this host's cores, on bounded
samples of the same workload.
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
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2")
    ap.add_argument("--seqlen", type=int, default=None, help="override N (not the headline)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="target CPU seconds per sample")
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: one config-2 problem (B=1) split over the GPUs by (batch, KV-group) units, "
                         "and by sequence blocks when there are more GPUs than units; outputs all-gathered")
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


# ------------------------------------------------------------------ CPU leg
def cpu_sample_run(wl, rows, seed=0):
    """fwd+bwd of the oracle port on query head 0 of batch 0, query rows
    [N-rows, N) against all keys (the heaviest causal rows). Returns
    (seconds, charged FLOPs of the sample)."""
    import numpy as np

    from oracle.attention_oracle import attention_bwd, attention_fwd

    N, D = wl["N"], wl["D"]
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g) * wl["factor"]).to(wl["dtype"]).float().numpy()  # noqa: E731
    q = mk(1, 1, rows, D)
    k = mk(1, 1, N, D)
    v = mk(1, 1, N, D)
    do = mk(1, 1, rows, D)
    off = N - rows
    t0 = time.perf_counter()
    o, lse = attention_fwd(q, k, v, wl["causal"], wl["W"], q_offset=off, chunk=256)
    attention_bwd(q, k, v, o, lse, do, wl["causal"], wl["W"], q_offset=off, chunk=256)
    dt = time.perf_counter() - t0
    W = wl["W"]
    pairs = 0
    for qpos in range(off, N):
        lo = max(0, qpos - W + 1) if (wl["causal"] and W) else 0
        hi = qpos + 1 if wl["causal"] else N
        pairs += hi - lo
    del np
    return dt, 14 * D * pairs


def cpu_calibrate(wl, target_s):
    cpu_sample_run(wl, 256)  # warm the BLAS thread pool and allocator
    t, _ = cpu_sample_run(wl, 256)
    rows = int(256 * target_s / max(t, 1e-3))
    rows = max(64, min(wl["N"], rows // 64 * 64))
    return rows


def cpu_baseline(wl, target_s, steps=1):
    rows = cpu_calibrate(wl, target_s)
    vals = []
    for s in range(steps):
        dt, fl = cpu_sample_run(wl, rows, seed=s)
        vals.append(fl / dt / 1e12)
    cores = os.cpu_count()
    return dict(value=statistics.median(vals), unit="TFLOPS/s", cores=cores, kind="port",
                sample=(f"oracle port (numpy fp32, {cores} BLAS threads): fwd+bwd of query head 0, "
                        f"the last {rows} query rows of N={wl['N']} (D={wl['D']}) against all keys; "
                        f"FLOPs charged 14*D*attended pairs"),
                values=vals, rows=rows)


# ------------------------------------------------------------------ GPU leg
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


def run_ours(args, wl, world, rank, local):
    from gemma_triton_flash_attn import FlashAttnGQAFunction, _lib
    from gemma_triton_flash_attn.attention import _alloc_workspace, _bwd, _fwd, bwd_workspace_size
    from gemma_triton_flash_attn.flops import attn_flops, kernel_flops

    def _bwd_workspace(*shape_args):
        # the same workspace decision the public API's backward makes
        return _alloc_workspace(bwd_workspace_size(*shape_args[:-1]), shape_args[-1])

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    B, Hq, Hkv, N, D, causal, W = (wl[x] for x in ("B", "Hq", "Hkv", "N", "D", "causal", "W"))
    window = W if (causal and 0 < W < N) else 0
    scale = 1.0 / math.sqrt(D)
    q, k, v, do = make_inputs(wl, 1234 + rank, device)
    qg, kg, vg = (t.detach().requires_grad_(True) for t in (q, k, v))
    if args.only:
        o, lse = _fwd(q, k, v, causal, window, scale, True)
        bufs = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
                torch.empty((B, Hq, N), dtype=torch.float32, device=device))
        ws = None
        if args.only in ("dqps", "dkv"):
            ws = _bwd_workspace(B, Hq, Hkv, N, D, causal, window, device)
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
        return

    def step():
        qg.grad = kg.grad = vg.grad = None
        out = FlashAttnGQAFunction.apply(qg, kg, vg, causal, W)
        out.backward(do)

    flops_step = attn_flops(B, Hq, N, D, causal, window, bwd=True)
    flops_fwd = attn_flops(B, Hq, N, D, causal, window)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    uuids = [uuid if uuid.startswith("GPU-") else "GPU-" + uuid]
    with ClockSampler(uuids) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        ms = time_loop(step, args.steps, stream)
        barrier(world)
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
    ws = _bwd_workspace(B, Hq, Hkv, N, D, causal, window, device)
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
    roofline = dict(bound="tensor", kernel=dom, achieved=round(achieved, 1), peak=peaks["tflops_sustained"],
                    unit="TFLOP/s", frac=round(achieved / peaks["tflops_sustained"], 4), traffic=traffic,
                    peak_kind=f"bf16_tflops_sustained ({peaks['source']}); burst {peaks['tflops_burst']}",
                    flops_per_launch=kflops, ms_per_launch=round(kernels[dom], 3),
                    kernel_ms={k_: round(v_, 3) for k_, v_ in kernels.items()},
                    kernel_share={k_: round(v_ / sum(kernels.values()), 3) for k_, v_ in kernels.items()})

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

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(wl, args.cpu_seconds, steps=1)
        cpu.pop("values", None)

    if rank == 0:
        line = dict(
            metric=METRIC, value=round(value, 2), unit="TFLOPS/s", n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=round(ms_max, 3), higher_is_better=True, scaling="weak",
            vs_baseline=None, dtype="bf16" if wl["dtype"] == torch.bfloat16 else "fp16",
            data="synthetic (seeded N(0,1)*%g, per-rank seed)" % wl["factor"],
            config=dict(workload=wl["name"], B_per_gpu=B, H_Q=Hq, H_KV=Hkv, N=N, D=D, causal=causal,
                        window=window, global_batch=B * world, seq_len=N, parallelism=f"(b,kv-group) units, dp{world}",
                        l2="inputs larger than L2 (Q, dO 512 MiB each); no flush"),
            fwd=dict(value=round(world * flops_fwd / (ms_fwd * 1e-3) / 1e12, 2), unit="TFLOPS/s",
                     ms=round(ms_fwd, 3)),
            roofline=roofline, cpu_baseline=cpu, e2e=e2e, clocks=clocks.summary(),
            gpu_launches=(1 + len(names)) * args.steps, kernel_status=status,
            bwd_path="materialised (workspace %d bytes)" % ws_bytes if len(names) == 2 else "recompute",
        )
        print(json.dumps(line), flush=True)


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
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    with ClockSampler([uuid if uuid.startswith("GPU-") else "GPU-" + uuid]) as clocks:
        ms = max_over_ranks(time_loop(step, args.steps, stream), world, device)
    n_glob = sum(cfg.is_global(i) for i in range(cfg.num_layers))
    attn_fl = n_glob * attn_flops(1, cfg.global_heads, N, cfg.global_head_dim, True) + \
        (cfg.num_layers - n_glob) * attn_flops(1, cfg.local_heads, N, cfg.local_head_dim, True, cfg.sliding_window)
    if rank == 0:
        line = dict(metric="config-5 decoder forward tokens/s (attention through hf_integration)",
                    value=round(world * N / (ms * 1e-3), 1), unit="tokens/s", n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=round(ms, 3), higher_is_better=True, scaling="weak",
                    vs_baseline=None, dtype="bf16", data="synthetic (seeded uniform token ids, random-init weights)",
                    config=dict(workload=wl["name"], global_batch=world, seq_len=N, parallelism=f"one sequence per GPU, dp{world}"),
                    attention_tflops_in_step=round(attn_fl / (ms * 1e-3) / 1e12, 1),
                    e2e=dict(value=round(world * N / (ms * 1e-3), 1), unit="tokens/s", h2d_bytes_per_step=ids_h.numel() * 8,
                             d2h_bytes_per_step=8),
                    clocks=clocks.summary(), gpu_launches=35 * args.steps)
        print(json.dumps(line), flush=True)


def run_strong(args, wl, world, rank, local):
    """Strong scaling: the whole job is one problem; every rank ends with the
    complete O, LSE, dQ, dK, dV (the all-gathers are inside the timed step)."""
    from gemma_triton_flash_attn.flops import attn_flops
    from gemma_triton_flash_attn.sharding import (head_split_backward, head_split_forward, sharded_backward,
                                                  sharded_forward)

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    B, Hq, Hkv, N, D, causal, W = (wl[x] for x in ("B", "Hq", "Hkv", "N", "D", "causal", "W"))
    q, k, v, do = make_inputs(wl, 1234, device)  # same problem on every rank
    split = world > B * Hkv
    fwd, bwd = (head_split_forward, head_split_backward) if split else (sharded_forward, sharded_backward)

    def step():
        o, lse = fwd(q, k, v, causal, W)
        bwd(q, k, v, o, lse, do, causal, W)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    with ClockSampler([uuid if uuid.startswith("GPU-") else "GPU-" + uuid]) as clocks:
        ms = max_over_ranks(time_loop(step, args.steps, stream), world, device)
    window = W if (causal and 0 < W < N) else 0
    total = attn_flops(B, Hq, N, D, causal, window, bwd=True)
    if rank == 0:
        line = dict(metric=METRIC + " (strong scaling)", value=round(total / (ms * 1e-3) / 1e12, 2), unit="TFLOPS/s",
                    n_gpus=world, steps=args.steps, warmup=args.warmup, ms_per_step=round(ms, 3),
                    higher_is_better=True, scaling="strong", vs_baseline=None,
                    dtype="bf16" if wl["dtype"] == torch.bfloat16 else "fp16", data="synthetic",
                    config=dict(workload=wl["name"], global_batch=B, seq_len=N,
                                parallelism=("query heads of each (b, kv-group) unit split, dK/dV all-reduced"
                                             if split else "(b, kv-group) units")
                                + f" over {world} GPUs, outputs all-gathered"),
                    clocks=clocks.summary(), gpu_launches=4 * args.steps)
        print(json.dumps(line), flush=True)


def run_reference(args, wl, world, rank):
    if rank != 0:
        return
    cores = os.cpu_count()
    rows = cpu_calibrate(wl, args.cpu_seconds)
    for s in range(args.warmup):
        cpu_sample_run(wl, max(64, rows // 8), seed=100 + s)
    times, fl = [], None
    for s in range(args.steps):
        dt, fl = cpu_sample_run(wl, rows, seed=s)
        times.append(dt)
    t = statistics.mean(times)
    value = fl / t / 1e12
    sample = (f"oracle port (numpy fp32, {cores} BLAS threads): fwd+bwd of query head 0, the last {rows} "
              f"query rows of N={wl['N']} (D={wl['D']}) against all keys per step")
    line = dict(
        metric=METRIC, value=round(value, 5), unit="TFLOPS/s", n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(t * 1e3, 1), higher_is_better=True, scaling="weak",
        vs_baseline=None, dtype="f32", data="synthetic", impl="reference",
        config=dict(workload=wl["name"], B_per_gpu=wl["B"], H_Q=wl["Hq"], H_KV=wl["Hkv"], N=wl["N"], D=wl["D"],
                    causal=wl["causal"], window=wl["W"], global_batch=wl["B"] * world, seq_len=wl["N"],
                    parallelism="host cores"),
        cpu_baseline=dict(value=round(value, 5), unit="TFLOPS/s", cores=cores, kind="port", sample=sample),
        e2e=dict(value=round(value, 5), unit="TFLOPS/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
    )
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    wl = dict(WORKLOADS[args.workload])
    if args.seqlen:
        wl["N"] = args.seqlen
        wl["name"] = wl["name"].replace("N=16384", f"N={args.seqlen}")
    world, rank, local = setup_dist()
    try:
        if args.impl == "reference":
            run_reference(args, wl, world, rank)
        elif args.workload == "cfg5":
            run_decoder(args, wl, world, rank, local)
        elif args.strong:
            run_strong(args, wl, world, rank, local)
        else:
            run_ours(args, wl, world, rank, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
