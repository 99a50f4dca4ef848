#!/usr/bin/env python
"""Benchmark of the B200 recurrent operators (one JSON line on rank 0).

Headline workload: SelectiveScanFn, benchmark configuration 1 (batch 8,
d_inner 4096, d_state 16, seqlen 2048, bfloat16 I/O with FP32 state, z
gating, D skip, delta_softplus), synthetic seeded inputs. A step is one
operator call over one batch. With --gpus N (one process per GPU under
torchrun) every rank runs its own batch of the same shape on its own GPU
(the op shards over (batch, channel) with no collective): weak scaling,
value = all ranks' tokens / max-over-ranks time.

  value       device-resident throughput, tokens (B*L) per second, CUDA events
              on the launching stream over exactly --steps calls
  e2e         the same metric through the public API with pinned HOST buffers:
              every step copies the inputs host->device, runs the op and
              copies the output back, pipelined per batch block over two copy
              streams (the op is independent per batch row)
  roofline    algorithmic HBM bytes per launch / average launch time against
              the measured copy bandwidth (MEASURED_PEAKS.json)
  cpu_baseline  the FP32 sequential CPU recurrence (oracle port) on a sample of
              the workload, all host cores (rank 0, N=1 only)

`--impl reference` prints the reference arm: the same metric for the
reference path's CPU restatement on the host cores (the reference has no CPU
implementation of these ops), plus, as extra fields, the reference's own CUDA
op rebuilt for sm_100a timed on this GPU.
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


# ---------------------------------------------------------------- workloads


class Workload:
    """Device-resident inputs of one configuration and a closure running one step."""

    def __init__(self, name, rank, device, batch=None):
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
        seed = shard.rank_seed(0, rank)
        f32 = torch.float32
        if c["op"] == "ss":
            x = W.ss_inputs(seed=seed, **c)
            if bf16:
                x = W.bf16_rounded(x, W.SS_BF16)
            order, io_names = W.SS_ORDER, W.SS_BF16
            self.tokens = c["batch"] * c["seqlen"]
            gate = int(c.get("gate", False))
            self.kwargs = dict(delta_softplus=1, apply_z_gate=gate)
            self.fn = xm.SelectiveScanFn
            self.out_like = "u"
        elif c["op"] == "gdn":
            x = W.gdn_inputs(seed=seed, **c)
            order, io_names = W.GDN_ORDER, ()
            self.tokens = c["B"] * c["T"]
            self.kwargs = dict(scale=x["scale"], use_qk_l2norm_in_kernel=1)
            self.fn = xm.GatedDeltaNet2Fn
            self.out_like = "v"
        else:
            x = W.m3_inputs(seed=seed, **c)
            if bf16:
                x = W.bf16_rounded(x, W.M3_BF16)
            order, io_names = W.M3_ORDER, W.M3_BF16
            self.tokens = c["B"] * c["T"]
            self.kwargs = {}
            self.fn = xm.Mamba3SisoFn
            self.out_like = "V"
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


def timed(fn, steps, warmup, dist_on, device):
    """Run warmup untimed steps then exactly `steps` timed ones; return (ms per step, host t0, host t1)."""
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
    t0 = time.time()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize(device)
    t1 = time.time()
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
    wl = Workload(args.workload, rank, device, args.batch)
    gpu_index = local_rank
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids):
            gpu_index = ids[local_rank]
    sampler = ClockSampler(gpu_index) if rank == 0 else None
    ms, t0, t1 = timed(wl.step, args.steps, args.warmup, dist_on, device)
    wl.setup_e2e(device)
    e2e_ms, _, _ = timed(wl.step_e2e, max(3, min(args.steps, 50)), 2, dist_on, device)
    # the pipelined end-to-end result equals the device-resident call's
    wl.step()
    torch.cuda.synchronize(device)
    e2e_ok = bool(torch.equal(wl.out_host, wl.out.cpu()))
    if sampler:
        sampler.stop()
    clocks = sampler.summary(t0, t1) if sampler else None
    tokens_total = wl.tokens * world
    line = None
    if rank == 0:
        achieved = wl.algo_bytes / (ms * 1e-3) / 1e9
        c = wl.cfg
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
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": wl.dtype_name,
            "data": "synthetic (seeded; shapes and distributions of the benchmark configuration)",
            "config": dict(workload=f"{wl.name}: {json.dumps(c)}", per_gpu_batch=c.get("batch", c.get("B")),
                           global_batch=c.get("batch", c.get("B")) * world,
                           seq_len=c.get("seqlen", c.get("T")),
                           parallelism=f"shard (batch, channel) x{world}, no collective",
                           l2="inputs larger than L2 (%.0f MB per step)" % (wl.algo_bytes / 1e6)),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(wl.name),
                         "peak_source": f"{peak_kind} (hbm_gbs)", "algorithmic_bytes": wl.algo_bytes},
            "e2e": {"value": tokens_total / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": wl.in_bytes, "d2h_bytes_per_step": wl.out_bytes,
                    "ms_per_step": e2e_ms,
                    "pipeline": f"{len(wl.blocks)} batch blocks: upload, compute and download overlapped",
                    "output_matches_device_call": e2e_ok},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
    del wl
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_other:
        others = {}
        for name in args.other:
            w2 = Workload(name, 0, device)
            m2, _, _ = timed(w2.step, 50, 5, False, device)
            ach = w2.algo_bytes / (m2 * 1e-3) / 1e9
            others[name] = {"tokens_per_s": w2.tokens / (m2 * 1e-3), "ms_per_step": m2, "hbm_gbs": ach,
                            "hbm_frac": ach / peak, "dtype": w2.dtype_name}
            del w2
            torch.cuda.empty_cache()
        line["other_configs"] = others
    if rank == 0 and world == 1 and not args.no_cpu:
        wl = Workload(args.workload, 0, device)
        line["cpu_baseline"] = cpu_baseline(wl)
    return line


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
        "ms_per_step": full * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
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
        out_z = torch.empty_like(f32[0]) if f32[6] is not None else None
        c = wl.cfg
        xs = torch.empty(oracle.ref_ss_scratch_floats(c["batch"], c["dim"], c["seqlen"], c["dstate"]),
                         dtype=torch.float32, device=device)
        kernel = lambda: oracle.ref_ss(*f32, softplus=True, out=out, out_z=out_z, x_scratch=xs)  # noqa: E731
        op = lambda: oracle.ref_ss(*f32, softplus=True, out=out, op_level=True)  # noqa: E731
        k_ms, _, _ = timed(kernel, 10, 2, False, device)
        o_ms, _, _ = timed(op, 10, 2, False, device)
        line["ref_cuda_op"] = {
            "what": "reference SelectiveScanFn CUDA kernels rebuilt for sm_100a, fp32 tensors holding the "
                    "bf16-rounded inputs, on this B200",
            "op_tokens_per_s": wl.tokens / (o_ms * 1e-3), "op_ms": o_ms,
            "kernel_tokens_per_s": wl.tokens / (k_ms * 1e-3), "kernel_ms": k_ms,
        }
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["xm", "reference"], default="xm")
    ap.add_argument("--workload", default="ss_cfg1")
    ap.add_argument("--other", nargs="*", default=["ss_cfg0", "gdn_cfg2", "gdn_cfg3", "m3_cfg4"])
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
