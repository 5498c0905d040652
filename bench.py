#!/usr/bin/env python3
"""Benchmark of the cuButterfly hot path on B200 (one process per GPU).

Headline workload: FWHT online rotation of a bf16
16384 x 4096 activation matrix -- pass A: H_4096 per row x 1/64, pass B: the
same rows as 128-element heads, H_128 x 1/sqrt(128); FP32 compute, one final
bf16 rounding.  A step is pass A + pass B over one batch; inputs live in HBM
(two rotating input buffers, each larger than L2).  `value` is transform HBM
GB/s (algorithmic bytes: each pass reads and writes the matrix once) summed
over all GPUs; every rank transforms its own full batch (weak scaling, no
data-path collective).  `e2e` repeats the step through the public C ABI with
host buffers (pinned host -> device copy of the input and device -> host copy
of both outputs inside the timed region).  `ops` reports the other hot-path
configurations (FFT, RNS NTT, subset zeta) on the same GPU; `strong_scaling` splits configs 2, 3 and 4 over the ranks
(limbs 32/P, transforms 16/P, 2^20 FFTs / P, the 2^30 FFT as a four-step
with its per-phase times, exchanges by peer-store kernels over NVLink and by
NCCL send/recv), each the max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MIB = 1 << 20


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default: 4000 for the FWHT workload and --only, 20 for fft4step / fftbatch)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--no-ops", action="store_true", help="skip the per-op table (FFT, NTT, zeta)")
    p.add_argument("--cpu-baseline", choices=["auto", "skip"], default="auto")
    p.add_argument("--no-strong", action="store_true",
                   help="skip the strong-scaled configurations (limbs, zeta transforms, FFT batch, 2^30 FFT)")
    p.add_argument("--only", choices=["fwht4096", "fwht128", "fft", "zeta", "ntt", "fft1g"],
                   help="run just this operator's launches (profiling driver; prints a short JSON line)")
    p.add_argument("--inventory", action="store_true",
                   help="time every other kernel family once per operator on moderate sizes (one JSON line each)")
    p.add_argument("--workload", choices=["fwht", "fft4step", "fftbatch"], default="fwht",
                   help="fwht: configs[1] (default, weak scaling); fft4step: config 4, one 2^30-point FFT "
                        "split over all ranks (strong scaling); fftbatch: config 4's batch sweep, 2^20 "
                        "transforms of 4096 points split over the ranks (strong scaling)")
    p.add_argument("--log-batch", type=int, default=20, help="fftbatch total batch (log2)")
    p.add_argument("--log-n", type=int, default=30, help="fft4step transform length (log2)")
    p.add_argument("--transport", choices=["peer", "nccl"], default="peer",
                   help="fft4step exchanges on 2+ GPUs: peer-store kernels over NVLink or NCCL send/recv")
    p.add_argument("--mapping", default="",
                   help="explicit mapping for --only fwht4096 / fft1g and --workload fft4step (1 GPU), "
                        "e.g. 'fwht-tcgen05[6+6]' for the tensor-core FWHT")
    args = p.parse_args()
    if args.steps is None:
        args.steps = 20 if (args.workload in ("fft4step", "fftbatch") and not args.only) or args.inventory else 4000
    return args


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        j = json.loads(f.read_text())
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_summary():
    f = ROOT / "profiles" / "traffic.json"
    return json.loads(f.read_text()) if f.exists() else {}


# ---- workload definition -------------------------------------------------------------
ROWS, COLS, HEAD = 16384, 4096, 128
PASS_BYTES = 2 * ROWS * COLS * 2          # one pass: read + write of the bf16 matrix
STEP_BYTES = 2 * PASS_BYTES               # pass A + pass B
E2E_CHUNKS, E2E_STREAMS = 8, 3            # end-to-end pipeline: row chunks over streams


def fwht_transform(cb, n, rows, scale):
    return cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[n],
                        batch=rows, output_scale=scale, output_rounding=cb.OutputRounding.FINAL_STORAGE)


# ---- clocks during the timed region ---------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = str(device_index)
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", self.dev, f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                row = [x.strip() for x in out.stdout.strip().split(",")]
                if len(row) == 7:
                    self.samples.append(row)
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---- reference arm: the reference's own CPU implementation ------------------------------------
def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from cubutterfly_b200 import workloads as w
    from oracle.oracle import Reference, build as build_oracle

    import numpy as np

    if not Reference.available():
        try:
            build_oracle()
        except Exception:
            pass
    threads = os.cpu_count() or 1
    if Reference.available():
        ref, kind = Reference(), "reference"
        fa = lambda x, s: ref.fwht_bf16_final(x, s, threads=threads)  # noqa: E731
    else:
        from oracle.oracle import Oracle
        ref, kind = Oracle(), "port"
        fa = lambda x, s: ref.fwht_bf16_final(x, s)  # noqa: E731
    # bounded sample of the workload: each step transforms `sample_rows` of the
    # 16384 rows (both passes), sized so all steps take about a minute;
    # throughput in the same algorithmic bytes per second
    bits = w.fwht_input_bits(2048, COLS, seed=0)
    t0 = time.perf_counter()
    fa(bits[:256], 1 / 64)
    fa(bits[:256].reshape(-1, HEAD), 1 / math.sqrt(HEAD))
    per_row = (time.perf_counter() - t0) / 256
    budget = 60.0 / max(1, args.steps + args.warmup)
    sample_rows = int(max(16, min(2048, budget / max(per_row, 1e-9))))
    bits = np.ascontiguousarray(bits[:sample_rows])
    blocks = bits.reshape(-1, HEAD)
    for _ in range(args.warmup):
        fa(bits, 1 / 64)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fa(bits, 1 / 64)
        fa(blocks, 1 / math.sqrt(HEAD))
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    sample_bytes = 2 * 2 * sample_rows * COLS * 2
    gbs = sample_bytes / t / 1e9
    line = {
        "impl": "reference", "metric": "transform HBM GB/s (FWHT bf16 16384x4096, H_4096 + H_128 passes)",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3 * (ROWS / sample_rows), 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "fwht_bf16_16384x4096_h4096_h128", "sample_rows_per_step": sample_rows},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{sample_rows} of {ROWS} rows per step, both passes, median of {args.steps}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- kernel inventory ----------------------------------------------------------------------------
def inventory(args):
    """One line per operator outside the headline and per-op table: device
    time per execution (CUDA events over `steps` executions after `warmup`)
    and algorithmic bytes (input + output once) per execution.  Sizes are
    moderate (a few hundred MiB at most) so that the same command can run
    under an ncu launch list."""
    import torch

    import cubutterfly_b200 as cb

    dev = torch.device("cuda", 0)
    lib = cb.Library()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    steps = args.steps
    g = torch.Generator(device=dev).manual_seed(7)

    def fill(nbytes):
        return torch.randint(0, 1 << 20, (nbytes // 4,), dtype=torch.int32, device=dev, generator=g)

    def case(label, t, in_bytes, out_bytes, make_input=None):
        with cb.Plan(lib, t, stream=sp) as p:
            x = make_input() if make_input else fill(p.input_size())
            y = x if t.in_place else torch.empty(p.output_size() // 4 + 1, dtype=torch.int32, device=dev)
            ws = torch.empty(max(p.workspace_size(), 16), dtype=torch.uint8, device=dev)
            if p.workspace_size():
                p.set_workspace(ws.data_ptr(), ws.numel())
            ms = time_launches(lambda i: p.execute(x.data_ptr(), y.data_ptr()), stream, steps, args.warmup)
            nbytes = in_bytes + out_bytes
            print(json.dumps({"inventory": label, "algorithm": p.algorithm_name(), "us": round(ms * 1e3, 2),
                              "gbs": round(nbytes / ms / 1e6, 1), "bytes": nbytes}), flush=True)

    n, b = 1 << 20, 64
    mats = [[(0.6, 0.8, -0.8, 0.6)]]
    case("structured_2x2_f32_2^20x64",
         cb.Transform(op=cb.Operator.STRUCTURED_2X2, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32,
                      extents=[n], batch=b, stage_matrices=mats), 4 * n * b, 4 * n * b,
         lambda: torch.randn(n * b, dtype=torch.float32, device=dev))
    case("fwht_native_bf16_16384x4096",
         cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.NATIVE, extents=[4096],
                      batch=16384), 2 * 4096 * 16384, 2 * 4096 * 16384,
         lambda: torch.randn(4096 * 16384, dtype=torch.float32, device=dev).to(torch.bfloat16))
    case("fft_c128_2^16x256",
         cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP64, compute=cb.ComputeType.FP64,
                      extents=[1 << 16], batch=256), 16 * (1 << 16) * 256, 16 * (1 << 16) * 256,
         lambda: torch.randn(2 * (1 << 16) * 256, dtype=torch.float64, device=dev))
    q = 576460756061519873
    case("ntt_cyclic_u64_2^16x32_natural",
         cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[1 << 16], batch=32, modulus=q),
         8 * (1 << 16) * 32, 8 * (1 << 16) * 32)
    case("fft_r2c_f32_2^20x64",
         cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[n], batch=b,
                      fft_type=cb.FftType.R2C), 4 * n * b, 8 * (n // 2 + 1) * b,
         lambda: torch.randn(n * b, dtype=torch.float32, device=dev))
    case("fft_c64_4096x1024_strided_in",
         cb.Transform(op=cb.Operator.FFT, extents=[4096], batch=1024, input_strides=[2], output_strides=[1],
                      input_batch_stride=8192, output_batch_stride=4096), 8 * 4096 * 1024, 8 * 4096 * 1024,
         lambda: torch.randn(2 * 8192 * 1024, dtype=torch.float32, device=dev))
    case("fft_c64_bluestein_4095x1024",
         cb.Transform(op=cb.Operator.FFT, extents=[4095], batch=1024), 8 * 4095 * 1024, 8 * 4095 * 1024,
         lambda: torch.randn(2 * 4095 * 1024, dtype=torch.float32, device=dev))
    case("ntt_u64_bluestein_5419x64",
         cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[5419], batch=64,
                      modulus=1152921504606584833), 8 * 5419 * 64, 8 * 5419 * 64)
    case("fft_c64_rank2_1024x1024",
         cb.Transform(op=cb.Operator.FFT, extents=[1024, 1024], batch=16), 8 * (1 << 20) * 16, 8 * (1 << 20) * 16,
         lambda: torch.randn(2 * (1 << 20) * 16, dtype=torch.float32, device=dev))
    return 0


# ---- B200 arm ------------------------------------------------------------------------------------
def only_op(args):
    """Launch one operator `steps` times after `warmup` launches (ncu driver)."""
    import torch

    import cubutterfly_b200 as cb
    from cubutterfly_b200 import rns
    from cubutterfly_b200 import workloads as w

    dev = torch.device("cuda", 0)
    lib = cb.Library()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    if args.only in ("fwht4096", "fwht128"):
        x = w.torch_fwht_input(ROWS, COLS, dev)
        y = torch.empty_like(x)
        n = COLS if args.only == "fwht4096" else HEAD
        opts = cb.PlanOptions(mapping=args.mapping) if args.mapping else None
        p = cb.Plan(lib, fwht_transform(cb, n, ROWS * COLS // n, 1 / math.sqrt(n)), options=opts, stream=sp)
        fn, nbytes = (lambda i: p.execute(x.data_ptr(), y.data_ptr())), PASS_BYTES
    elif args.only == "fft":
        x = w.torch_fft_input(w.FFT_N, w.FFT_BATCH, dev)
        y = torch.empty_like(x)
        p = cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[w.FFT_N], batch=w.FFT_BATCH), stream=sp)
        fn, nbytes = (lambda i: p.execute(x.data_ptr(), y.data_ptr())), 2 * w.FFT_N * w.FFT_BATCH * 8
    elif args.only == "fft1g":
        n = 1 << args.log_n
        x = w.torch_fft_input(n, 1, dev)
        y = torch.empty_like(x)
        opts = cb.PlanOptions(mapping=args.mapping) if args.mapping else None
        p = cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[n], batch=1), options=opts, stream=sp)
        ws = torch.empty(p.workspace_size(), dtype=torch.uint8, device=dev)
        p.set_workspace(ws.data_ptr(), ws.numel())
        fn, nbytes = (lambda i: p.execute(x.data_ptr(), y.data_ptr())), 2 * n * 8
    elif args.only == "zeta":
        z = w.torch_zeta_input(w.ZETA_LOG_N, w.ZETA_BATCH, dev)
        t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << w.ZETA_LOG_N],
                         batch=w.ZETA_BATCH, in_place=True)
        p = cb.Plan(lib, t, stream=sp)
        fn, nbytes = (lambda i: p.execute(z.data_ptr(), z.data_ptr())), 2 * (1 << w.ZETA_LOG_N) * w.ZETA_BATCH * 4
    else:
        cfg = w.rns_config()
        qs = [d["modulus"] for d in cfg["domains"]]
        x = w.torch_ntt_input(qs, w.NTT_LOG_N, dev)
        y = torch.empty_like(x)
        p = rns.Plan(rns.Library(), cfg)
        p.prepare(stream=sp, repetitions=1)
        fn, nbytes = (lambda i: p.execute(x.data_ptr(), y.data_ptr(), stream=sp)), 2 * w.NTT_LIMBS * (1 << w.NTT_LOG_N) * 8
    ms = time_launches(fn, stream, args.steps, args.warmup)
    name = p.algorithm_name() if hasattr(p, "algorithm_name") else args.only
    print(json.dumps({"only": args.only, "algorithm": name, "ms_per_launch": round(ms, 5),
                      "gbs": round(nbytes / ms / 1e6, 1)}))
    p.close()
    return 0


def fft4step(args):
    """Config 4: one complex fp32 FFT of 2^log_n points; on one GPU the
    multi-pass plan, on P GPUs the four-step decomposition (exchanges by
    --transport).  Strong scaling; algorithmic bytes = input + output once."""
    import torch
    import torch.distributed as dist

    import cubutterfly_b200 as cb
    from cubutterfly_b200 import workloads as w
    from cubutterfly_b200.distributed import FourStepFFT

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    n = 1 << args.log_n
    shard = n // world
    stream = torch.cuda.current_stream()
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.rand((shard, 2), generator=g, device=dev, dtype=torch.float32) * 2 - 1
    if world == 1:
        lib = cb.load()
        plan = cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[n], batch=1), stream=stream.cuda_stream)
        ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=dev)
        plan.set_workspace(ws.data_ptr(), ws.numel())
        y = torch.empty_like(x)
        step = lambda: plan.execute(x.data_ptr(), y.data_ptr())  # noqa: E731
        algo = plan.algorithm_name()
    else:
        fs = FourStepFFT(n, device=dev, transport=args.transport)
        step = lambda: fs(x)  # noqa: E731
        how = {"peer": "peer-store exchange kernels over NVLink", "nccl": "NCCL grouped send/recv"}
        algo = f"four-step {fs.shape.n1}x{fs.shape.n2} over {world} ranks ({how[args.transport]}, 3 exchanges)"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if rank == 0:
        gbs = 2 * n * 8 / (ms * 1e-3) / 1e9
        peak, kind = peaks()
        print(json.dumps({
            "metric": f"transform HBM GB/s (complex fp32 FFT, N=2^{args.log_n}, one transform)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"fft_c64_2^{args.log_n}_four_step", "algorithm": algo,
                       "bytes_per_step": 2 * n * 8},
            "frac_of_single_gpu_hbm_peak": round(gbs / peak, 4), "peak_kind": kind}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def fftbatch(args):
    """Config 4's batch sweep: 2^log_batch independent 4096-point complex fp32
    FFTs (config 0's shape), the total batch split over the ranks with no
    communication (strong scaling).  At 2^20 the input is 32 GiB: far larger
    than L2, so every step streams from HBM."""
    import torch
    import torch.distributed as dist

    import cubutterfly_b200 as cb
    from cubutterfly_b200.distributed import shard_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    n, total = 4096, 1 << args.log_batch
    _, count = shard_range(total, world, rank)
    stream = torch.cuda.current_stream()
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.rand((count, n, 2), generator=g, device=dev, dtype=torch.float32)
    x.mul_(2).sub_(1)
    y = torch.empty_like(x)
    plan = cb.Plan(cb.load(), cb.Transform(op=cb.Operator.FFT, extents=[n], batch=count), stream=stream.cuda_stream)
    step = lambda: plan.execute(x.data_ptr(), y.data_ptr())  # noqa: E731
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if rank == 0:
        step_bytes = 2 * total * n * 8
        gbs = step_bytes / (ms * 1e-3) / 1e9
        peak, kind = peaks()
        print(json.dumps({
            "metric": f"transform HBM GB/s (complex fp32 FFT, N=4096, batch 2^{args.log_batch} split over ranks)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"fft_c64_4096_batch_2^{args.log_batch}", "algorithm": plan.algorithm_name(),
                       "bytes_per_step": step_bytes, "parallelism": f"batch-sharded x{world}",
                       "l2": "input larger than L2 (32 GiB at batch 2^20)"},
            "frac_of_aggregate_hbm_peak": round(gbs / (peak * world), 4), "peak_kind": kind,
            "clocks": clocks.summary()}), flush=True)
    plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.only:
        return only_op(args)
    if args.inventory:
        return inventory(args)
    if args.workload == "fft4step":
        return fft4step(args)
    if args.workload == "fftbatch":
        return fftbatch(args)
    import numpy as np
    import torch
    import torch.distributed as dist

    import cubutterfly_b200 as cb
    from cubutterfly_b200 import workloads as w

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    lib = cb.Library()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    # inputs: two rotating bf16 matrices (each 128 MiB > L2), generated on device
    xs = [w.torch_fwht_input(ROWS, COLS, dev, seed=s) for s in (0, 1)]
    ya = torch.empty_like(xs[0])
    yb = torch.empty_like(xs[0])
    plan_a = cb.Plan(lib, fwht_transform(cb, COLS, ROWS, 1 / 64), stream=sp)
    plan_b = cb.Plan(lib, fwht_transform(cb, HEAD, ROWS * COLS // HEAD, 1 / math.sqrt(HEAD)), stream=sp)
    launches_per_step = 2

    def step(i, ev=None):
        x = xs[i & 1]
        if ev is not None:
            ev[0].record(stream)
        plan_a.execute(x.data_ptr(), ya.data_ptr())
        if ev is not None:
            ev[1].record(stream)
        plan_b.execute(x.data_ptr(), yb.data_ptr())

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for i in range(args.steps):
            step(i, evs[i])
        t1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    pass_a_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * STEP_BYTES / (ms * 1e-3) / 1e9

    # e2e through the public API with host buffers: the rows run as E2E_CHUNKS
    # chunks round-robin over E2E_STREAMS streams (each with its own plans), so
    # a chunk's upload, both passes and its two read-backs overlap the other
    # chunks' copies in the opposite direction (PCIe is full duplex).
    host_in = torch.empty((ROWS, COLS), dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(xs[0])
    host_a = torch.empty_like(host_in, pin_memory=True)
    host_b = torch.empty_like(host_in, pin_memory=True)
    dev_in = torch.empty_like(xs[0])
    crows = ROWS // E2E_CHUNKS
    lanes = [torch.cuda.Stream(device=dev) for _ in range(E2E_STREAMS)]
    lane_plans = [(cb.Plan(lib, fwht_transform(cb, COLS, crows, 1 / 64), stream=l.cuda_stream),
                   cb.Plan(lib, fwht_transform(cb, HEAD, crows * COLS // HEAD, 1 / math.sqrt(HEAD)),
                           stream=l.cuda_stream)) for l in lanes]
    fork = torch.cuda.Event()

    def e2e_step():
        fork.record(stream)
        for l in lanes:
            l.wait_event(fork)
        for c in range(E2E_CHUNKS):
            k = c % E2E_STREAMS
            rows = slice(c * crows, (c + 1) * crows)
            pa, pb = lane_plans[k]
            with torch.cuda.stream(lanes[k]):
                dev_in[rows].copy_(host_in[rows], non_blocking=True)
                pa.execute(dev_in[rows].data_ptr(), ya[rows].data_ptr())
                pb.execute(dev_in[rows].data_ptr(), yb[rows].data_ptr())
                host_a[rows].copy_(ya[rows], non_blocking=True)
                host_b[rows].copy_(yb[rows], non_blocking=True)
        for l in lanes:
            stream.wait_stream(l)

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * STEP_BYTES / (e2e_ms * 1e-3) / 1e9

    peak, peak_kind = peaks()
    achieved = PASS_BYTES / (pass_a_ms * 1e-3) / 1e9
    traffic = traffic_summary().get("fwht_bf16_4096", {}).get("dram_bytes_per_launch")
    ops = {} if args.no_ops else measure_ops(cb, lib, dev, stream, peak, max(5, args.steps // 2), args.warmup)

    strong = None if args.no_strong else strong_scaling(world, rank, dev, lib, stream)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_baseline == "auto":
        cpu = cpu_baseline()
        for name, base in op_cpu_baselines().items():
            if name in ops:
                ops[name]["cpu_baseline"] = base

    if world > 1:
        dist.barrier()
    plan_a.close()
    plan_b.close()
    for pa, pb in lane_plans:
        pa.close()
        pb.close()
    if rank == 0:
        line = {
            "metric": "transform HBM GB/s (FWHT bf16 16384x4096, H_4096 + H_128 passes)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 storage, f32 compute", "data": "synthetic",
            "config": {"workload": "fwht_bf16_16384x4096_h4096_h128", "rows": ROWS, "cols": COLS, "head": HEAD,
                       "bytes_per_step": STEP_BYTES, "parallelism": f"batch-sharded x{world} (every rank its own batch)",
                       "l2": "inputs larger than L2 (2 rotating 128 MiB input buffers)"},
            "roofline": {"bound": "hbm", "kernel": "fwht_tile_kernel<bf16,LOGH=12,LOGE=6>",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": PASS_BYTES,
                         "kernel_ms": round(pass_a_ms, 5)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": ROWS * COLS * 2,
                    "d2h_bytes_per_step": 2 * ROWS * COLS * 2, "ms_per_step": round(e2e_ms, 4),
                    "pipeline": f"{E2E_CHUNKS} row chunks over {E2E_STREAMS} streams"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "ops": ops,
            "strong_scaling": strong,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def strong_scaling(world, rank, dev, lib, stream):
    """Strong-scaled configurations at this world size, every rank its share
    of a fixed total, no collective on the data path except the four-step's
    exchanges: config 2's 32 limbs (each rank only its domains' tables),
    config 3's 16 transforms, config 4's batch sweep (2^20 transforms of 4096
    points) and config 4's single 2^30-point transform (the single-GPU plan at
    one rank, the four-step over NCCL beyond).  Times are CUDA events around
    a few executions after warm-up, the max over ranks; GB/s count the whole
    job's input + output once."""
    import torch
    import torch.distributed as dist

    import cubutterfly_b200 as cb
    from cubutterfly_b200 import rns
    from cubutterfly_b200 import workloads as w
    from cubutterfly_b200.distributed import FourStepFFT, shard_range, shard_rns_config

    sp = stream.cuda_stream
    out = {}

    def timed(fn, steps, warmup=2):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # config 2: 32 limbs of 2^16, limbs 32/P per rank
    cfg = w.rns_config()
    shard, first, count = shard_rns_config(cfg, world, rank)
    qs = [d["modulus"] for d in shard["domains"]] if count else []
    x = w.torch_ntt_input([shard["domains"][p["domain"]]["modulus"] for p in shard["polynomials"]], w.NTT_LOG_N,
                          dev) if count else None
    y = torch.empty_like(x) if count else None
    plan = rns.Plan(rns.Library(), shard) if count else None
    if plan:
        plan.prepare(stream=sp, repetitions=1)
    ms = timed(lambda: plan.execute(x.data_ptr(), y.data_ptr(), stream=sp) if plan else None, 50)
    total = 2 * w.NTT_LIMBS * (1 << w.NTT_LOG_N) * 8
    out["rns_ntt_u64_32x2^16"] = {"ms": round(ms, 5), "gbs": round(total / ms / 1e6, 1),
                                  "per_rank": f"{count} limbs, {len(qs)} domains' tables"}
    if plan:
        plan.close()
    del x, y
    # config 3: 16 transforms of 2^24, 16/P per rank
    zs, zc = shard_range(w.ZETA_BATCH, world, rank)
    z = w.torch_zeta_input(w.ZETA_LOG_N, zc, dev) if zc else None
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << w.ZETA_LOG_N],
                     batch=max(zc, 1), in_place=True)
    zp = cb.Plan(lib, t, stream=sp) if zc else None
    ms = timed(lambda: zp.execute(z.data_ptr(), z.data_ptr()) if zp else None, 5)
    total = 2 * w.ZETA_BATCH * (1 << w.ZETA_LOG_N) * 4
    out["zeta_u32_2^24x16"] = {"ms": round(ms, 4), "gbs": round(total / ms / 1e6, 1), "per_rank": f"{zc} transforms"}
    if zp:
        zp.close()
    del z
    # config 4 batch sweep: 2^20 transforms of 4096 points
    fs, fc = shard_range(1 << 20, world, rank)
    xb = w.torch_fft_input(4096, fc, dev, seed=rank)
    yb = torch.empty_like(xb)
    fp = cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[4096], batch=fc), stream=sp)
    ms = timed(lambda: fp.execute(xb.data_ptr(), yb.data_ptr()), 3)
    total = 2 * (1 << 20) * 4096 * 8
    out["fft_c64_4096x2^20"] = {"ms": round(ms, 4), "gbs": round(total / ms / 1e6, 1), "per_rank": f"{fc} transforms"}
    fp.close()
    del xb, yb
    torch.cuda.empty_cache()
    # config 4: one 2^30-point transform
    n = 1 << 30
    if world == 1:
        xs = w.torch_fft_input(n, 1, dev, seed=4).reshape(n, 2)
        ys = torch.empty_like(xs)
        sp1 = cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[n], batch=1), stream=sp)
        ws = torch.empty(sp1.workspace_size(), dtype=torch.uint8, device=dev)
        sp1.set_workspace(ws.data_ptr(), ws.numel())
        ms = timed(lambda: sp1.execute(xs.data_ptr(), ys.data_ptr()), 3, warmup=1)
        entry = {"algorithm": sp1.algorithm_name()}
        sp1.close()
        del xs, ys, ws
    else:
        # both exchange transports; the line reports the faster, with the other beside it
        g = torch.Generator(device=dev).manual_seed(rank)
        xs = torch.rand((n // world, 2), generator=g, device=dev, dtype=torch.float32)
        runs, failed = {}, {}
        for transport in ("peer", "nccl"):
            try:
                four = FourStepFFT(n, device=dev, transport=transport)
            except Exception as e:  # e.g. no CUDA IPC between these devices: keep the other transport
                failed[transport] = str(e)[:200]
                continue
            t_ms = timed(lambda: four(xs), 3, warmup=1)
            four.record_phases = True
            four(xs)
            phases = four.phase_ms()
            four.record_phases = False
            keys = sorted(phases)
            t = torch.tensor([phases[k] for k in keys], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            phases = dict(zip(keys, (float(v) for v in t.tolist())))
            four.close()
            runs[transport] = (t_ms, phases)
        best = min(runs, key=lambda k: runs[k][0])
        ms, phases = runs[best]
        how = {"peer": "peer-store exchange kernels over NVLink", "nccl": "NCCL grouped send/recv"}
        # the limiting phase over phase kinds (the three exchanges together)
        kinds = {}
        for k, v in phases.items():
            kind = "exchange" if k.startswith("exchange") else k
            kinds[kind] = kinds.get(kind, 0.0) + v
        entry = {"algorithm": f"four-step 32768x32768 over {world} ranks ({how[best]})",
                 "phases_ms": {k: round(v, 3) for k, v in phases.items()},
                 "limiting_phase": max(kinds, key=kinds.get) if kinds else None,
                 "other_transport": {k: round(v[0], 3) for k, v in runs.items() if k != best}}
        if failed:
            entry["unavailable_transport"] = failed
        del xs
    torch.cuda.empty_cache()
    entry.update(ms=round(ms, 3), gbs=round(2 * n * 8 / ms / 1e6, 1))
    out["fft_c64_2^30"] = entry
    return out


def time_launches(fn, stream, steps, warmup):
    import torch

    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        fn(i)
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def measure_ops(cb, lib, dev, stream, peak, steps, warmup):
    """Per-op throughput of the other hot-path configurations (device-resident
    inputs, two rotating buffers each larger than L2 where the data allows)."""
    import torch

    from cubutterfly_b200 import rns
    from cubutterfly_b200 import workloads as w

    sp = stream.cuda_stream
    ops = {}
    # config 1 pass A on the tensor cores (tcgen05 mapping, H_64 (x) H_64): two rotating 128 MiB inputs
    xa = w.torch_fwht_input(ROWS, COLS, dev, seed=0)
    xb = w.torch_fwht_input(ROWS, COLS, dev, seed=1)
    y = torch.empty_like(xa)
    with cb.Plan(lib, fwht_transform(cb, COLS, ROWS, 1 / 64), options=cb.PlanOptions(mapping="fwht-tcgen05[6+6]"),
                 stream=sp) as p:
        ms = time_launches(lambda i: p.execute((xb if i % 2 else xa).data_ptr(), y.data_ptr()), stream, steps,
                           warmup)
        ops["fwht_tcgen05_bf16_16384x4096"] = {"gbs": round(PASS_BYTES / ms / 1e6, 1),
                                               "frac": round(PASS_BYTES / ms / 1e6 / peak, 4),
                                               "us": round(ms * 1e3, 2), "algorithm": p.algorithm_name()}
    del xa, xb, y
    # config 0: FFT c64 4096 x 1024 (32 MiB: rotate 8 buffers so each step reads cold data)
    xs = [w.torch_fft_input(w.FFT_N, w.FFT_BATCH, dev, seed=s) for s in range(8)]
    y = torch.empty_like(xs[0])
    with cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[w.FFT_N], batch=w.FFT_BATCH), stream=sp) as p:
        ms = time_launches(lambda i: p.execute(xs[i % 8].data_ptr(), y.data_ptr()), stream, steps * 4, warmup)
        b = 2 * w.FFT_N * w.FFT_BATCH * 8
        ops["fft_c64_4096x1024"] = {"gbs": round(b / ms / 1e6, 1), "frac": round(b / ms / 1e6 / peak, 4),
                                    "us": round(ms * 1e3, 2), "algorithm": p.algorithm_name()}
    del xs, y
    # config 3: subset zeta u32 2^24 x 16 (1 GiB), in place
    z = w.torch_zeta_input(w.ZETA_LOG_N, w.ZETA_BATCH, dev)
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << w.ZETA_LOG_N],
                     batch=w.ZETA_BATCH, in_place=True)
    with cb.Plan(lib, t, stream=sp) as p:
        ms = time_launches(lambda i: p.execute(z.data_ptr(), z.data_ptr()), stream, steps, warmup)
        b = 2 * (1 << w.ZETA_LOG_N) * w.ZETA_BATCH * 4
        ops["zeta_u32_2^24x16"] = {"gbs": round(b / ms / 1e6, 1), "frac": round(b / ms / 1e6 / peak, 4),
                                   "us": round(ms * 1e3, 2), "algorithm": p.algorithm_name()}
    del z
    # config 2: RNS negacyclic NTT 32 x 2^16 (16 MiB; rotate 16 inputs)
    cfg = w.rns_config()
    qs = [d["modulus"] for d in cfg["domains"]]
    ins = [w.torch_ntt_input(qs, w.NTT_LOG_N, dev, seed=s) for s in range(16)]
    out = torch.empty_like(ins[0])
    with rns.Plan(rns.Library(), cfg) as p:
        p.prepare(stream=sp, repetitions=3)
        ms = time_launches(lambda i: p.execute(ins[i % 16].data_ptr(), out.data_ptr(), stream=sp), stream,
                           steps * 4, warmup)
        b = 2 * w.NTT_LIMBS * (1 << w.NTT_LOG_N) * 8
        ops["rns_ntt_u64_32x2^16"] = {"gbs": round(b / ms / 1e6, 1), "frac": round(b / ms / 1e6 / peak, 4),
                                      "us": round(ms * 1e3, 2), "algorithm": "b200_two_pass_tile"}
        # integer roof: the measured rate of the same lazy butterfly from registers
        import ctypes as ct
        rate = ct.c_double()
        lib.invoke("B200NttButterflyPeak", max(qs), ct.byref(rate))
        butterflies = w.NTT_LIMBS * (1 << (w.NTT_LOG_N - 1)) * w.NTT_LOG_N
        ops["rns_ntt_u64_32x2^16"].update(
            butterflies_per_s=round(butterflies / (ms * 1e-3), 1), butterfly_peak_per_s=round(rate.value, 1),
            imad_frac=round(butterflies / (ms * 1e-3) / rate.value, 4) if rate.value else None,
            imad_peak_kind="measured: cubutterflyB200NttButterflyPeak (the pass's lazy butterfly from registers)")
    # the same shape as one cyclic single-modulus NTT plan of the main ABI:
    # natural -> bit-reversed (two passes) and natural -> natural (a
    # bit-reversal permutation first)
    q = 576460756061519873
    for tag, out_order in (("nr", cb.LogicalOrder.BIT_REVERSED), ("nn", cb.LogicalOrder.NATURAL)):
        t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[1 << w.NTT_LOG_N],
                         batch=w.NTT_LIMBS, modulus=q, output_orders=[out_order])
        with cb.Plan(lib, t, stream=sp) as p:
            ms = time_launches(lambda i: p.execute(ins[i % 16].data_ptr(), out.data_ptr()), stream, steps * 4,
                               warmup)
            ops[f"ntt_cyclic_u64_32x2^16_{tag}"] = {"gbs": round(b / ms / 1e6, 1),
                                                    "frac": round(b / ms / 1e6 / peak, 4),
                                                    "us": round(ms * 1e3, 2), "algorithm": p.algorithm_name()}
    del ins, out
    # config 4 on one GPU: one 2^30-point FFT (8 GiB in, 8 GiB out, 8 GiB workspace), multi-pass plan
    n = 1 << 30
    x = w.torch_fft_input(n, 1, dev, seed=4)
    y = torch.empty_like(x)
    with cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[n], batch=1), stream=sp) as p:
        ws = torch.empty(p.workspace_size(), dtype=torch.uint8, device=dev)
        p.set_workspace(ws.data_ptr(), ws.numel())
        ms = time_launches(lambda i: p.execute(x.data_ptr(), y.data_ptr()), stream, 3, 1)
        b = 2 * n * 8
        ops["fft_c64_2^30"] = {"gbs": round(b / ms / 1e6, 1), "frac": round(b / ms / 1e6 / peak, 4),
                               "us": round(ms * 1e3, 2), "algorithm": p.algorithm_name()}
    del x, y, ws
    return ops


def op_cpu_baselines():
    """The reference's own CPU code (oracle/_ref) on the other configurations,
    all host threads, each a bounded sample of a second or two: config 0
    reference_fft<Complex32> over the 1024 transforms; config 2 twist +
    reference_ntt + bit reversal per limb; config 3 reference_subset_zeta over
    the 16 transforms; config 4 one 2^24-point reference_fft<Complex32>
    (the reference runs one transform on one thread), scaled to 2^30 by
    N log N.  Reported beside each op, never required."""
    try:
        import numpy as np

        from cubutterfly_b200 import workloads as w
        from oracle.oracle import Reference

        if not Reference.available():
            return {}
        ref = Reference()
        threads = os.cpu_count() or 1

        def timed(fn, budget=1.5):
            fn()
            t0, reps = time.perf_counter(), 0
            while reps < 1 or time.perf_counter() - t0 < budget:
                fn()
                reps += 1
            return (time.perf_counter() - t0) / reps, reps

        def entry(nbytes, t, reps, sample, cores=threads):
            return {"value": round(nbytes / t / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "reference",
                    "sample": f"{sample}; {reps} repetitions"}

        out = {}
        x = w.fft_input(w.FFT_N, w.FFT_BATCH, seed=0)
        t, r = timed(lambda: ref.fft_c32(x, threads=threads))
        out["fft_c64_4096x1024"] = entry(2 * x.nbytes, t, r, "reference_fft<Complex32>, all 1024 transforms")
        cfg = w.rns_config()
        qs = [d["modulus"] for d in cfg["domains"]]
        v = w.ntt_input(qs, seed=0)
        t, r = timed(lambda: ref.negacyclic_ntt(v, qs, threads=threads))
        out["rns_ntt_u64_32x2^16"] = entry(2 * v.nbytes, t, r, "twist + reference_ntt + bit reversal, all 32 limbs")
        q = 576460756061519873
        t, r = timed(lambda: ref.ntt_cyclic(v, q, threads=threads))
        for tag in ("nr", "nn"):
            out[f"ntt_cyclic_u64_32x2^16_{tag}"] = entry(2 * v.nbytes, t, r, "reference_ntt (natural order), 32 rows")
        z = w.zeta_input(w.ZETA_LOG_N, w.ZETA_BATCH, seed=0)
        t, r = timed(lambda: ref.zeta_u32(z, threads=threads), budget=2.0)
        out["zeta_u32_2^24x16"] = entry(2 * z.nbytes, t, r, "reference_subset_zeta, all 16 transforms")
        del z
        big = w.fft_input(1 << 24, 1, seed=4)
        t, r = timed(lambda: ref.fft_c32(big, threads=1), budget=2.0)
        t30 = t * (2 ** 30 * 30) / (2 ** 24 * 24)
        out["fft_c64_2^30"] = entry(2 * 8 * 2 ** 30, t30, r, "one 2^24-point reference_fft<Complex32>, time "
                                    "scaled by N log N to 2^30", cores=1)
        return out
    except Exception as e:  # the baselines are reported, never required
        return {"error": {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "unavailable",
                          "sample": str(e)}}


def cpu_baseline():
    """The reference's own CPU FWHT (oracle/_ref) on a bounded sample, all host threads."""
    try:
        import numpy as np

        from cubutterfly_b200 import workloads as w
        from oracle.oracle import Reference, Oracle

        threads = os.cpu_count() or 1
        if Reference.available():
            ref, kind = Reference(), "reference"
            run = lambda x, s: ref.fwht_bf16_final(x, s, threads=threads)  # noqa: E731
        else:
            ref, kind = Oracle(), "port"
            run = lambda x, s: ref.fwht_bf16_final(x, s)  # noqa: E731
        rows = 2048
        bits = w.fwht_input_bits(rows, COLS, seed=0)
        run(bits[:128], 1 / 64)
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 8.0 or reps < 1:
            run(bits, 1 / 64)
            run(bits.reshape(-1, HEAD), 1 / math.sqrt(HEAD))
            reps += 1
        t = (time.perf_counter() - t0) / reps
        gbs = 2 * 2 * rows * COLS * 2 / t / 1e9
        return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                "sample": f"{rows} of {ROWS} rows, both passes, {reps} repetitions (~8 s)"}
    except Exception as e:  # the baseline is reported, never required
        return {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "unavailable", "sample": str(e)}


if __name__ == "__main__":
    sys.exit(main())
