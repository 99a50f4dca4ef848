#!/usr/bin/env python
"""Benchmark of the B200 recurrent operators (one JSON line on rank 0).

Headline workload: SelectiveScanFn, benchmark configuration 1 (batch 8,
d_inner 4096, d_state 16, seqlen 2048, bfloat16 I/O with FP32 state, z
gating, D skip, delta_softplus), synthetic seeded inputs. A step is one
operator call over one batch. With --gpus N (one process per GPU under
torchrun) the configuration's one global call is sharded over the ranks
(batch rows when N divides the batch, else channels / heads), each rank
running its shard on its own GPU with no collective: strong scaling, value =
the global call's tokens / max-over-ranks time. `--scaling weak` instead
gives every rank a full call of its own (per-rank seeds).

  value       device-resident throughput, tokens (B*L) per second, CUDA events
              on the launching stream over exactly --steps calls
  e2e         the same metric through the public API with pinned HOST buffers:
              every step copies the inputs host->device, runs the op and
              copies the output back, pipelined per batch block over two copy
              streams (the op is independent per batch row)
  roofline    the binding unit of the headline kernel (MUFU operations for the
              selective scan) against its issue rate, plus the HBM fraction:
              algorithmic bytes per launch / average launch time against the
              measured copy bandwidth (MEASURED_PEAKS.json)
  cpu_baseline  the FP32 sequential CPU recurrence (oracle port) on a sample of
              the workload, all host cores (rank 0, N=1 only)

`--impl reference` prints the reference arm: the same metric for the
reference path's CPU restatement on the host cores (the reference has no CPU
implementation of these ops), plus, as extra fields, the reference's own CUDA
ops rebuilt for sm_100a timed on this GPU, for the headline and for every
other configuration (`ref_cuda_op`, `ref_cuda_other`).
"""

from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG = "xmetai_onnx_plugins_b200"


def load_package():
    if PKG in sys.modules:
        return sys.modules[PKG]
    pkg_dir = ROOT / "xmetai-onnx-plugins_b200"
    spec = importlib.util.spec_from_file_location(PKG, pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[PKG] = mod
    spec.loader.exec_module(mod)
    return mod


# ---------------------------------------------------------------- environment


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def sm_clock_mhz():
    """Maximum SM clock for issue-rate peaks (MEASURED_PEAKS.json, else the B200's 1965 MHz)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if d.get("sm_max_mhz"):
            return float(d["sm_max_mhz"])
    return 1965.0


def measured_bf16_tflops():
    """Dense bf16 tensor peak (MEASURED_PEAKS.json burst figure, else the pool's earlier 1590)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if d.get("bf16_tflops"):
            return float(d["bf16_tflops"])
    return 1590.0


def gdn_tensor_core_path(cfg):
    """Whether GatedDeltaNet2Fn takes the chunked tensor-core form for this
    config under the default (automatic) path: keys up to 512 and sequences
    of 512 tokens or more (the library's rule)."""
    return cfg["K"] <= 512 and cfg["T"] >= 512


# Issue rates per SM and clock on sm_100 (148 SMs): MUFU (ex2 / tanh / rcp)
# 16 operations, FP32 FMA 128 lanes.
MUFU_PER_SM_CLK = 16
FMA_PER_SM_CLK = 128


def profiled_traffic(workload):
    """DRAM bytes per launch of the workload's kernel from the committed ncu summary."""
    p = ROOT / "profiles" / f"{workload}_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples taken while the benchmark runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.samples = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.samples.append((time.time(), float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        window = "timed"
        if not inside:
            inside, window = self.samples, "run"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for s in inside for n, v in zip(names, s[3]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": max(s[2] for s in inside),
                "reasons": reasons, "samples": len(inside), "window": window}


class NvmlSampler:
    """SM clock and clock-event reasons polled through NVML every ~2 ms while
    running, so that even a timed region of a few milliseconds is sampled."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_index):
        self.samples = []
        self.handle = None
        self.running = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            idx = int(gpu_index)
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 -- sampling is best effort
            self.handle = None

    def _poll(self):
        nv = self.nvml
        masks = [(name, getattr(nv, attr)) for name, attr in self.REASONS]
        while self.running:
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((mhz, [n for n, m in masks if bits & m]))
            except Exception:  # noqa: BLE001
                break
            time.sleep(0.002)

    def start(self):
        if self.handle is None:
            return
        self.running = True
        self.thread = threading.Thread(target=self._poll, daemon=True)
        self.thread.start()

    def stop(self):
        if self.handle is None or not self.running:
            return
        self.running = False
        self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted({r for _, rs in self.samples for r in rs}), "samples": len(self.samples),
                "window": "timed (NVML, every ~2 ms)"}


# ---------------------------------------------------------------- workloads


class Workload:
    """Device-resident inputs of one configuration and a closure running one step.

    world / scaling: with "strong" the configuration's global call (seed 0) is
    split over `world` ranks and this object holds rank `rank`'s shard; with
    "weak" every rank holds a full call drawn from its own seed."""

    def __init__(self, name, rank, device, batch=None, world=1, scaling="strong"):
        import numpy as np
        import torch

        xm = load_package()
        from xmetai_onnx_plugins_b200 import shard
        from xmetai_onnx_plugins_b200 import workloads as W

        self.name = name
        c = dict(W.CONFIGS[name])
        if batch:  # reduced case for profiling captures
            c["batch" if c["op"] == "ss" else "B"] = batch
        self.cfg = c
        bf16 = c.get("dtype") == "bfloat16"
        io = torch.bfloat16 if bf16 else torch.float32
        seed = shard.rank_seed(0, rank) if scaling == "weak" else 0
        f32 = torch.float32
        if c["op"] == "ss":
            x = W.ss_inputs(seed=seed, **c)
            if bf16 or c.get("round_bf16"):
                x = W.bf16_rounded(x, W.SS_BF16)
            order, io_names = W.SS_ORDER, W.SS_BF16
            gate = int(c.get("gate", False))
            self.kwargs = dict(delta_softplus=1, apply_z_gate=gate)
            self.fn = xm.SelectiveScanFn
            self.out_like = "u"
        elif c["op"] == "gdn":
            x = W.gdn_inputs(seed=seed, **c)
            order, io_names = W.GDN_ORDER, ()
            self.kwargs = dict(scale=x["scale"], use_qk_l2norm_in_kernel=1)
            self.fn = xm.GatedDeltaNet2Fn
            self.out_like = "v"
        else:
            x = W.m3_inputs(seed=seed, **c)
            if bf16:
                x = W.bf16_rounded(x, W.M3_BF16)
            order, io_names = W.M3_ORDER, W.M3_BF16
            self.kwargs = {}
            self.fn = xm.Mamba3SisoFn
            self.out_like = "V"
        self.shard_axis = "none"
        if scaling == "strong" and world > 1:
            x, self.shard_axis = shard.shard_units(c["op"], x, world, rank,
                                                   prefer="batch" if c.get("shard", "batch") == "batch" else "unit")
        # this rank's tokens (B*L) and independent units, from its shard's shapes
        lead = x[{"ss": "u", "gdn": "q", "m3": "V"}[c["op"]]]
        if c["op"] == "ss":
            self.batch, self.units = lead.shape[0], lead.shape[0] * lead.shape[1]
            self.tokens = lead.shape[0] * lead.shape[2]
            self.unit_frac = lead.shape[1] / c["dim"]
        else:
            self.batch, self.units = lead.shape[0], lead.shape[0] * lead.shape[2]
            self.tokens = lead.shape[0] * lead.shape[1]
            self.unit_frac = lead.shape[2] / c["H"]
        self.host_np = x
        self.order = order
        self.dtypes = [io if k in io_names else f32 for k in order]
        self.host = []
        self.dev = []
        for k, dt in zip(order, self.dtypes):
            a = x.get(k)
            if a is None:
                self.host.append(None)
                self.dev.append(None)
                continue
            h = torch.from_numpy(np.ascontiguousarray(a)).to(dt).pin_memory()
            self.host.append(h)
            self.dev.append(h.to(device))
        ref = self.dev[order.index(self.out_like)]
        self.out = torch.empty_like(ref)
        self.out_host = torch.empty(ref.shape, dtype=ref.dtype).pin_memory()
        self.in_bytes = sum(t.numel() * t.element_size() for t in self.host if t is not None)
        self.out_bytes = self.out.numel() * self.out.element_size()
        self.algo_bytes = self.algorithmic_bytes()
        self.dtype_name = {torch.bfloat16: "bf16", torch.float32: "fp32"}[self.out.dtype]

    def binding(self, ms):
        """The unit that bounds this workload's kernel, its algorithmic work per
        call, the rate achieved in `ms` and the unit's issue-rate peak:
          SelectiveScanFn: MUFU operations -- per (row, token) one ex2 per state
            (the decay), one ex2 for the softplus, and for the gate one tanh
            (2-byte I/O) or an ex2 and a reciprocal (float32 I/O);
          GatedDeltaNet2Fn, register-state recurrence (K > 512 or sequences
            under 512 tokens): FP32 FMA, 3 K V per token-head (decay-free state
            update and the two projections);
          GatedDeltaNet2Fn, chunked tensor-core form (K <= 512, 512 tokens or
            more): bf16 tensor-core FLOPs of the split products (3 MMAs per
            product) per 128-token chunk and head -- Lh, Ph (2 C^2 KP), PT (C^3),
            KT (KP C^2), X and qr R0 (2 C V KP), PT X (C^2 V), KT X (KP C V), C = 128,
            KP = K padded to 128 -- against the measured bf16 burst peak;
          Mamba3SisoFn: HBM (the chunk kernel is latency bound; its bytes are
            the roofline reported)."""
        clk = sm_clock_mhz() * 1e6
        sms = 148
        c = self.cfg
        if c["op"] == "ss":
            gate_ops = 0 if not self.kwargs.get("apply_z_gate") else (1 if self.dtype_name != "fp32" else 2)
            ops = self.units * c["seqlen"] * (c["dstate"] + 1 + gate_ops)
            peak = sms * MUFU_PER_SM_CLK * clk
            return {"unit": "mufu", "ops_per_call": ops, "achieved": ops / (ms * 1e-3) / 1e9,
                    "peak": peak / 1e9, "rate_unit": "Gop/s", "frac": ops / (ms * 1e-3) / peak,
                    "peak_source": f"148 SMs x {MUFU_PER_SM_CLK}/clk x {clk / 1e6:.0f} MHz"}
        if c["op"] == "gdn" and gdn_tensor_core_path(c):
            C, KP, V = 128, -(-c["K"] // 128) * 128, c["V"]
            chunk_heads = -(-c["T"] // C) * self.units  # units: batch rows x heads
            per = 6 * (2 * C * C * KP + C ** 3 + KP * C * C + 2 * C * V * KP + C * C * V + KP * C * V)
            flops = chunk_heads * per
            peak = measured_bf16_tflops() * 1e12
            return {"unit": "tensor_bf16", "ops_per_call": flops, "achieved": flops / (ms * 1e-3) / 1e12,
                    "peak": peak / 1e12, "rate_unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / peak,
                    "peak_source": "MEASURED_PEAKS.json bf16_tflops (cuBLAS burst)"}
        if c["op"] == "gdn":
            fma = self.tokens * (self.units // max(self.batch, 1)) * 3 * c["K"] * c["V"]
            peak = sms * FMA_PER_SM_CLK * clk
            return {"unit": "fp32_fma", "ops_per_call": fma, "achieved": fma / (ms * 1e-3) / 1e9,
                    "peak": peak / 1e9, "rate_unit": "GFMA/s", "frac": fma / (ms * 1e-3) / peak,
                    "peak_source": f"148 SMs x {FMA_PER_SM_CLK}/clk x {clk / 1e6:.0f} MHz"}
        return None

    def algorithmic_bytes(self):
        """Bytes the operator must move: each input it reads once, the output once."""
        skip = set()
        if self.cfg["op"] == "ss" and not self.kwargs.get("apply_z_gate"):
            skip.add("z")  # the ungated op does not read z
        total = self.out_bytes
        for k, t in zip(self.order, self.host):
            if t is not None and k not in skip:
                total += t.numel() * t.element_size()
        return total

    def step(self):
        self.fn(*self.dev, out=self.out, **self.kwargs)

    def setup_e2e(self, device):
        """Streams and batch blocks for the end-to-end step. The operators are
        independent per batch row, so the step pipelines per block: upload block
        i+1 (host->device copy engine) while block i computes and block i-1
        downloads (device->host copy engine)."""
        import torch

        from xmetai_onnx_plugins_b200 import shard

        batch = self.host[0].shape[0]
        axes = shard._BATCH_AXIS[self.cfg["op"]]
        self.batched = [h is not None and k in axes and h.dim() >= 3 and h.shape[0] == batch
                        for k, h in zip(self.order, self.host)]
        nblk = min(batch, 8)
        self.blocks = [shard.block_range(batch, nblk, i) for i in range(nblk)]
        self.s_up = torch.cuda.Stream(device)
        self.s_down = torch.cuda.Stream(device)

    def step_e2e(self):
        import torch

        cur = torch.cuda.current_stream()
        self.s_up.wait_stream(cur)
        self.s_down.wait_stream(cur)
        with torch.cuda.stream(self.s_up):
            for h, d, bat in zip(self.host, self.dev, self.batched):
                if h is not None and not bat:
                    d.copy_(h, non_blocking=True)  # shared per-channel / per-head parameters
        for b0, b1 in self.blocks:
            with torch.cuda.stream(self.s_up):
                for h, d, bat in zip(self.host, self.dev, self.batched):
                    if bat:
                        d[b0:b1].copy_(h[b0:b1], non_blocking=True)
            cur.wait_stream(self.s_up)
            args = [d[b0:b1] if bat else d for d, bat in zip(self.dev, self.batched)]
            self.fn(*args, out=self.out[b0:b1], **self.kwargs)
            self.s_down.wait_stream(cur)
            with torch.cuda.stream(self.s_down):
                self.out_host[b0:b1].copy_(self.out[b0:b1], non_blocking=True)
        cur.wait_stream(self.s_down)


def timed(fn, steps, warmup, dist_on, device, sampler=None):
    """Run warmup untimed steps then exactly `steps` timed ones; return (ms per step, host t0, host t1).
    `sampler` (start / stop) runs from just before the first timed launch until the GPU has finished."""
    import torch
    import torch.distributed as dist

    load_package()
    from xmetai_onnx_plugins_b200 import shard

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler is not None:
        sampler.start()
    t0 = time.time()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize(device)
    t1 = time.time()
    if sampler is not None:
        sampler.stop()
    if dist_on:
        dist.barrier()
    ms = start.elapsed_time(end)
    if dist_on:
        ms = shard.max_over_ranks(ms, device)
    return ms / steps, t0, t1


# ---------------------------------------------------------------- CPU restatement


def cpu_sample_run(wl, units_fraction, nthreads):
    """Run the FP32 sequential CPU recurrence on a leading slice of the workload's
    independent units; returns (seconds, fraction of units actually run)."""
    import numpy as np

    import oracle

    x, c = wl.host_np, wl.cfg
    if c["op"] == "ss":
        B, D = c["batch"], c["dim"]
        nb = max(1, int(round(B * units_fraction))) if units_fraction >= 1.0 / B else 1
        nd = D if nb > 1 else max(1, int(D * units_fraction * B))
        sl = lambda a: None if a is None else np.ascontiguousarray(a[:nb, :nd])  # noqa: E731
        args = [sl(x["u"]), sl(x["delta"]), x["A"][:nd], x["B"][:nb], x["C"][:nb],
                None if x["D"] is None else x["D"][:nd], sl(x["z"]),
                None if x["delta_bias"] is None else x["delta_bias"][:nd]]
        t = time.perf_counter()
        oracle.ss(*args, softplus=True, gate=bool(wl.kwargs.get("apply_z_gate")), precision="f32",
                  nthreads=nthreads)
        return time.perf_counter() - t, (nb * nd) / (B * D)
    if c["op"] == "gdn":
        B, H = c["B"], c["H"]
        nh = max(1, int(round(B * H * units_fraction)))
        nb, nh = (1, min(nh, H)) if nh < H else (max(1, nh // H), H)
        sl = lambda a: None if a is None else np.ascontiguousarray(a[:nb, :, :nh])  # noqa: E731
        s0 = None if x["initial_state"] is None else np.ascontiguousarray(x["initial_state"][:nb, :nh])
        t = time.perf_counter()
        oracle.gdn(sl(x["q"]), sl(x["k"]), sl(x["v"]), sl(x["g"]), sl(x["beta"]), sl(x["w"]), s0,
                   scale=x["scale"], precision="f32", nthreads=nthreads)
        return time.perf_counter() - t, (nb * nh) / (B * H)
    B, H = c["B"], c["H"]
    nh = max(1, int(round(B * H * units_fraction)))
    nb, nh = (1, min(nh, H)) if nh < H else (max(1, nh // H), H)
    sl = lambda a: None if a is None else np.ascontiguousarray(a[:nb, :, :nh])  # noqa: E731
    slh = lambda a: None if a is None else np.ascontiguousarray(a[:nb, :nh])  # noqa: E731
    t = time.perf_counter()
    oracle.m3(x["Q"][:nb], x["K"][:nb], sl(x["V"]), slh(x["ADT"]), slh(x["DT"]), slh(x["Trap"]),
              x["Q_bias"][:nh], x["K_bias"][:nh], sl(x["Angles"]), None if x["D"] is None else x["D"][:nh],
              sl(x["Z"]), precision="f32", nthreads=nthreads)
    return time.perf_counter() - t, (nb * nh) / (B * H)


def cpu_baseline(wl, budget_s=10.0):
    """Throughput of the CPU restatement, scaled from a sample sized to ~budget_s."""
    nthreads = os.cpu_count() or 1
    frac = 1.0 / 512
    secs, got = cpu_sample_run(wl, frac, nthreads)
    while secs < budget_s / 4 and got < 1.0:
        frac = min(1.0, frac * max(2.0, budget_s / 2 / max(secs, 1e-3)))
        secs, got = cpu_sample_run(wl, frac, nthreads)
    full_time = secs / got
    return {"value": wl.tokens / full_time, "unit": "tokens/s", "cores": nthreads, "kind": "port",
            "sample": f"{got * 100:.3g}% of the (batch, channel/head) units of {wl.name}, "
                      f"{secs:.2f} s on {nthreads} threads, FP32 sequential recurrence"}


# ---------------------------------------------------------------- arms


def run_xm(args, rank, world, local_rank, device, dist_on):
    import torch

    peak, peak_kind = measured_peaks()
    wl = Workload(args.workload, rank, device, args.batch, world=world, scaling=args.scaling)
    gpu_index = local_rank
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids):
            gpu_index = ids[local_rank]
    sampler = ClockSampler(gpu_index) if rank == 0 else None
    nvml = NvmlSampler(gpu_index) if rank == 0 else None
    ms, t0, t1 = timed(wl.step, args.steps, args.warmup, dist_on, device, sampler=nvml)
    wl.setup_e2e(device)
    e2e_ms, _, _ = timed(wl.step_e2e, max(3, min(args.steps, 50)), 3, dist_on, device)
    # the pipelined end-to-end result agrees with the device-resident call's.
    # Each block is a call over fewer batch rows, for which the launcher may pick
    # another kernel of the op (SelectiveScanFn: four lanes per channel for one
    # row) that sums in another order, so the check is normwise against the
    # parity tolerance of the I/O type rather than bit-equality.
    wl.step()
    torch.cuda.synchronize(device)
    ref_out = wl.out.cpu().double()
    e2e_err = float((wl.out_host.double() - ref_out).abs().max() / ref_out.abs().max().clamp_min(1e-30))
    e2e_tol = 2e-2 if wl.out.dtype in (torch.bfloat16, torch.float16) else 1e-4
    e2e_check = {"max_rel_err": e2e_err, "tol": e2e_tol, "ok": e2e_err <= e2e_tol,
                 "bit_identical": bool(torch.equal(wl.out_host, wl.out.cpu()))}
    if sampler:
        sampler.stop()
    clocks = None
    if rank == 0:
        clocks = nvml.summary() if nvml is not None else None
        if clocks is None:
            clocks = sampler.summary(t0, t1)
        else:
            smi = sampler.summary(t0, t1)
            clocks["nvidia_smi"] = smi
    # whole-job tokens: the global call (strong) or one call per rank (weak)
    tokens_total = wl.tokens * world if args.scaling == "weak" else \
        wl.cfg.get("batch", wl.cfg.get("B")) * wl.cfg.get("seqlen", wl.cfg.get("T"))
    line = None
    if rank == 0:
        hbm_achieved = wl.algo_bytes / (ms * 1e-3) / 1e9
        c = wl.cfg
        hbm = {"bound": "hbm", "achieved": hbm_achieved, "peak": peak, "unit": "GB/s", "frac": hbm_achieved / peak,
               "traffic": profiled_traffic(wl.name) if world == 1 else None,
               "peak_source": f"{peak_kind} (hbm_gbs)", "algorithmic_bytes": wl.algo_bytes}
        b = wl.binding(ms)
        if b is not None:
            roofline = {"bound": b["unit"], "achieved": b["achieved"], "peak": b["peak"], "unit": b["rate_unit"],
                        "frac": b["frac"], "traffic": hbm["traffic"], "peak_source": b["peak_source"],
                        "ops_per_launch": b["ops_per_call"], "hbm": hbm}
        else:
            roofline = hbm
        gb = c.get("batch", c.get("B"))
        line = {
            "metric": "tokens/s (B*L) per SelectiveScanFn call" if c["op"] == "ss" else
                      f"tokens/s (B*L) per {wl.fn.__name__} call",
            "value": tokens_total / (ms * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": args.scaling if world > 1 else "strong",
            "vs_baseline": None,
            "dtype": wl.dtype_name,
            "data": "synthetic (seeded; shapes and distributions of the benchmark configuration)",
            "config": dict(workload=f"{wl.name}: {json.dumps(c)}",
                           per_gpu_batch=wl.batch, per_gpu_unit_fraction=wl.unit_frac,
                           global_batch=gb if args.scaling == "strong" else gb * world,
                           seq_len=c.get("seqlen", c.get("T")),
                           parallelism=(f"{world} ranks, each a shard of one global call split over "
                                        f"{wl.shard_axis if world > 1 else 'batch'}, no collective"
                                        if args.scaling == "strong" else
                                        f"{world} ranks, each a full call of its own, no collective"),
                           l2="inputs larger than L2 (%.0f MB per step)" % (wl.algo_bytes / 1e6)
                           if wl.algo_bytes > 126e6 else "inputs smaller than L2 (%.0f MB per step)"
                           % (wl.algo_bytes / 1e6)),
            "roofline": roofline,
            "e2e": {"value": tokens_total / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": wl.in_bytes, "d2h_bytes_per_step": wl.out_bytes,
                    "ms_per_step": e2e_ms,
                    "pipeline": f"{len(wl.blocks)} batch blocks: upload, compute and download overlapped",
                    "output_vs_device_call": e2e_check},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
    del wl
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_other:
        others = {}
        for name in args.other:
            w2 = Workload(name, 0, device)
            reps = 50 if w2.algo_bytes < 1.5e9 else 20
            m2, _, _ = timed(w2.step, reps, 5, False, device)
            ach = w2.algo_bytes / (m2 * 1e-3) / 1e9
            others[name] = {"tokens_per_s": w2.tokens / (m2 * 1e-3), "ms_per_step": m2, "hbm_gbs": ach,
                            "hbm_frac": ach / peak, "dtype": w2.dtype_name}
            b2 = w2.binding(m2)
            if b2 is not None:
                others[name]["binding"] = {k: b2[k] for k in ("unit", "achieved", "peak", "rate_unit", "frac")}
            del w2
            torch.cuda.empty_cache()
        line["other_configs"] = others
    if rank == 0 and world == 1 and not args.no_cpu:
        wl = Workload(args.workload, 0, device)
        line["cpu_baseline"] = cpu_baseline(wl)
    return line


def ref_cuda_time(wl, device, reps):
    """Kernel-level time (ms) of the reference's own CUDA op for this workload,
    rebuilt for sm_100a, with caller-provided scratch, on fp32 tensors holding
    the workload's values."""
    import torch

    import oracle

    f32 = [None if t is None else t.float() for t in wl.dev]
    c = wl.cfg
    if c["op"] == "ss":
        out = torch.empty_like(f32[0])
        out_z = torch.empty_like(f32[0]) if f32[6] is not None and wl.kwargs.get("apply_z_gate") else None
        xs = torch.empty(oracle.ref_ss_scratch_floats(c["batch"], c["dim"], c["seqlen"], c["dstate"]),
                         dtype=torch.float32, device=device)
        fn = lambda: oracle.ref_ss(*f32, softplus=True, out=out, out_z=out_z, x_scratch=xs)  # noqa: E731
    elif c["op"] == "gdn":
        out = torch.empty_like(f32[2])
        scr = torch.empty(oracle.ref_gdn_scratch_floats(c["B"], c["T"], c["H"], c["K"], c["V"]),
                          dtype=torch.float32, device=device)
        fn = lambda: oracle.ref_gdn(*f32, scale=wl.kwargs["scale"], l2norm=True, scratch=scr,  # noqa: E731
                                    out=out)
    else:
        out = torch.empty_like(f32[2])
        fn = lambda: oracle.ref_m3(*f32, out=out)  # noqa: E731
    ms, _, _ = timed(fn, reps, 1, False, device)
    return ms


def run_reference(args, rank, world, device):
    """Reference arm: the CPU restatement of the reference path on the host cores,
    plus the reference CUDA op (rebuilt for sm_100a) as extra fields."""
    import torch

    import oracle

    if rank != 0:
        return None
    wl = Workload(args.workload, 0, device)
    nthreads = os.cpu_count() or 1
    # size one step's sample so the whole run stays within ~2 minutes
    per_step = max(0.05, 120.0 / (args.steps + args.warmup))
    frac = 1.0 / 512
    secs, got = cpu_sample_run(wl, frac, nthreads)
    while secs < per_step / 2 and got < 1.0:
        frac = min(1.0, frac * max(2.0, per_step / max(secs, 1e-3)))
        secs, got = cpu_sample_run(wl, frac, nthreads)
    for _ in range(args.warmup):
        cpu_sample_run(wl, frac, nthreads)
    times = []
    for _ in range(args.steps):
        s, got = cpu_sample_run(wl, frac, nthreads)
        times.append(s / got)
    full = statistics.mean(times)
    value = wl.tokens / full
    line = {
        "metric": "tokens/s (B*L) per SelectiveScanFn call" if wl.cfg["op"] == "ss" else "tokens/s (B*L)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": full * 1e3, "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic (same seeded inputs as the xm arm)", "impl": "reference",
        "config": {"workload": f"{wl.name}: {json.dumps(wl.cfg)}"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                         "sample": f"{got * 100:.3g}% of the units per step, FP32 sequential recurrence "
                                   f"(the reference has no CPU implementation of this op)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if oracle.ref_available() and wl.cfg["op"] == "ss":
        f32 = [None if t is None else t.float() for t in wl.dev]
        out = torch.empty_like(f32[0])
        op = lambda: oracle.ref_ss(*f32, softplus=True, out=out, op_level=True)  # noqa: E731
        k_ms = ref_cuda_time(wl, device, 10)
        o_ms, _, _ = timed(op, 10, 2, False, device)
        line["ref_cuda_op"] = {
            "what": "reference SelectiveScanFn CUDA kernels rebuilt for sm_100a, fp32 tensors holding the "
                    "bf16-rounded inputs, on this B200",
            "op_tokens_per_s": wl.tokens / (o_ms * 1e-3), "op_ms": o_ms,
            "kernel_tokens_per_s": wl.tokens / (k_ms * 1e-3), "kernel_ms": k_ms,
        }
    if oracle.ref_available() and not args.no_other:
        del wl
        torch.cuda.empty_cache()
        other = {}
        for name in args.other:
            w2 = Workload(name, 0, device)
            slow = w2.cfg["op"] == "gdn" and w2.cfg["K"] > 256  # the generic path takes seconds per call
            k_ms = ref_cuda_time(w2, device, 2 if slow else 10)
            other[name] = {"kernel_ms": k_ms, "kernel_tokens_per_s": w2.tokens / (k_ms * 1e-3),
                           "io": "fp32 tensors holding the workload's values"}
            del w2
            torch.cuda.empty_cache()
        line["ref_cuda_other"] = other
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["xm", "reference"], default="xm")
    ap.add_argument("--workload", default="ss_cfg1")
    ap.add_argument("--other", nargs="*",
                    default=["ss_cfg0", "ss_cfg1_f32", "gdn_cfg2", "gdn_cfg3", "m3_cfg4", "m3_cfg4_b32"])
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="N>1: shard one global call (strong) or run a full call per rank (weak)")
    ap.add_argument("--no-other", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (reduced cases for ncu captures only)")
    args = ap.parse_args()

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist_on = world > 1
    if dist_on:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        if args.impl == "reference":
            line = run_reference(args, rank, world, device)
        else:
            line = run_xm(args, rank, world, local_rank, device, dist_on)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist_on:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
