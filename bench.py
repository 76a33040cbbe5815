"""Benchmark of the batched fp32 GEMM behind tl::matmul (libtl_cuda) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode tf32|3xtf32|exact]
                    [--workload batched|square8192|...] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run.  Prints ONE
JSON line on rank 0.

Workload (default "batched"): per GPU the batched GEMM
C[64,2048,2048] = A[64,2048,2048] . B[64,2048,2048], fp32 row-major,
A, B ~ U[-1,1] (seed 4), the batch-sharded case of the scaling sweep: rank r
owns its own 64 batch entries (weak scaling: the job at N GPUs is the
batch-sharded GEMM of 64*N entries, no data-path collective).  A step is one
call of tl::matmul's GEMM over that batch; each operand is 1 GiB, larger than
the 126 MB L2, so no flush is needed between steps.

Metric: GEMM TFLOP/s = 2*batch*M*N*K / time, whole job.  `value` times the
device-resident call (CUDA events on the launching stream, max over ranks);
`e2e` times tlc_matmul_host (the host-buffer C entry point): page-locked host
A, B in, host C out, copies inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "torchlite-cpp_b200")
sys.path.insert(0, PKG)

WORKLOADS = {
    # name: (batch, M, N, K)
    "batched": (64, 2048, 2048, 2048),
    "square8192": (1, 8192, 8192, 8192),
    "square4096": (1, 4096, 4096, 4096),
    "square16384": (1, 16384, 16384, 16384),
    "square512": (1, 512, 512, 512),
}
METRIC = "GEMM TFLOP/s (fp32-exact, TF32, 3xTF32) at 1/2/4/8 B200, % of peak"


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0}, "fallback"


def peak_for(mode, peaks, src, sms, clock_mhz):
    """Roofline denominator for a mode."""
    if mode == "exact":
        # FP32 FFMA: 128 lanes x 2 FLOP per SM per clock at the max SM clock.
        # MEASURED_PEAKS.json has no FP32 figure, so this one is nominal.
        return sms * 128 * 2 * clock_mhz * 1e6 / 1e12, "nominal FP32 FFMA at max SM clock"
    tf32 = peaks["bf16_tflops"] / 2.0  # dense TF32 issues at half the dense bf16 rate
    if mode == "tf32":
        return tf32, f"TF32 = 1/2 of {src} bf16 ({peaks['bf16_tflops']} TFLOP/s)"
    return tf32 / 3.0, f"3xTF32 = 1/3 of TF32 = 1/6 of {src} bf16 ({peaks['bf16_tflops']} TFLOP/s)"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, max_mhz_default):
        if not self.proc or not self.f:
            return {"sm_mhz": None, "sm_max_mhz": max_mhz_default, "reasons": ["unsampled"]}
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": max_mhz_default, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else max_mhz_default,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(wl, rank, device):
    import torch
    batch, M, N, K = WORKLOADS[wl]
    g = torch.Generator(device=device).manual_seed(4 + 1000 * rank)
    shp_a = (batch, M, K) if batch > 1 else (M, K)
    shp_b = (batch, K, N) if batch > 1 else (K, N)
    A = torch.rand(shp_a, generator=g, device=device, dtype=torch.float32) * 2 - 1
    B = torch.rand(shp_b, generator=g, device=device, dtype=torch.float32) * 2 - 1
    return A, B


def time_device(fn, steps, warmup, world, stream):
    """Per-step device time (ms): W warm-ups, then K steps between CUDA events
    on `stream`, bracketed by barrier + synchronize; max over ranks."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1) / steps
    return max_over_ranks(ms, world)


def cpu_reference_sample(wl, reps=3):
    """The reference's own tl::matmul (oracle/_ref, compiled from its sources)
    on a bounded sample of the workload: one 2048^3 batch entry (or a 256-row
    slab of a square GEMM), min over reps (time_best, bench/bench_matmul.cpp:27-39)."""
    import numpy as np
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    R = O.tlref()
    batch, M, N, K = WORKLOADS[wl]
    rows = M if batch > 1 else min(M, 256)
    rng = np.random.default_rng(4)
    a = rng.uniform(-1, 1, (rows, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        R.matmul(a, b)
        best = min(best, time.perf_counter() - t0)
    flops = 2.0 * rows * N * K
    return {"value": flops / best / 1e12, "unit": "TFLOP/s", "cores": R.hardware_threads(),
            "kind": "reference",
            "sample": f"tl::matmul [{rows},{K}]x[{K},{N}] fp32 "
                      f"({flops / 1e9:.1f} GFLOP), best of {reps}, "
                      f"{os.path.basename(R.path)} with std::thread::hardware_concurrency() threads"}


def run_reference_arm(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = args.workload
    import numpy as np
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    try:
        R = O.tlref()
    except FileNotFoundError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"oracle/_ref not built: {e}"}))
        return 0
    batch, M, N, K = WORKLOADS[wl]
    rows = M if batch > 1 else min(M, 256)
    rng = np.random.default_rng(4)
    a = rng.uniform(-1, 1, (rows, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    for _ in range(args.warmup):
        R.matmul(a, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        R.matmul(a, b)
    dt = (time.perf_counter() - t0) / args.steps
    flops = 2.0 * rows * N * K
    val = flops / dt / 1e12
    sample = (f"each step: reference tl::matmul on [{rows},{K}]x[{K},{N}] fp32 "
              f"({flops / 1e9:.1f} GFLOP), one {'batch entry' if batch > 1 else 'row slab'} "
              f"of the workload, host wall clock")
    line = {"metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic U[-1,1] seed 4", "impl": "reference",
            "config": {"workload": wl, "batch": batch, "M": M, "N": N, "K": K,
                       "sampled_rows": rows},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": R.hardware_threads(),
                             "kind": "reference", "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def traffic_for(mode, wl):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            t = json.load(f)
        return t.get(f"{wl}:{mode}")
    except OSError:
        return None


def run_ours(args):
    import torch
    import tlcuda
    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    wl = args.workload
    batch, M, N, K = WORKLOADS[wl]
    flops = 2.0 * batch * M * N * K
    A, B = make_inputs(wl, rank, device)
    C = torch.empty((batch, M, N) if batch > 1 else (M, N), device=device, dtype=torch.float32)
    stream = torch.cuda.current_stream()
    modes = [args.mode] + [m for m in ("tf32", "3xtf32", "exact") if m != args.mode and args.all_modes]
    peaks, psrc = load_peaks()
    sms = torch.cuda.get_device_properties(device).multi_processor_count

    results = {}
    launches = None
    clocks = None
    for mode in modes:
        fn = lambda: tlcuda.matmul(A, B, mode=mode, out=C)  # noqa: E731
        if mode == args.mode:
            l0 = tlcuda.launch_count()
            with ClockSampler(local) as cs:
                ms = time_device(fn, args.steps, args.warmup, world, stream)
            clocks = cs.summary(peaks.get("sm_max_mhz", 1965.0))
            launches = (tlcuda.launch_count() - l0)
            launches = launches * args.steps // (args.steps + args.warmup)
        else:
            ms = time_device(fn, max(3, args.steps // 2), 3, world, stream)
        peak, pdesc = peak_for(mode, peaks, psrc, sms, peaks.get("sm_max_mhz", 1965.0))
        per_gpu = flops / (ms * 1e-3) / 1e12
        results[mode] = {"ms_per_step": ms, "tflops_per_gpu": per_gpu,
                         "value": per_gpu * world, "roofline_frac": per_gpu / peak,
                         "peak_tflops": peak, "peak_source": pdesc}

    head = results[args.mode]
    peak = head["peak_tflops"]
    roofline = {"bound": "hbm" if False else "tensor", "achieved": head["tflops_per_gpu"],
                "peak": peak, "unit": "TFLOP/s", "frac": head["tflops_per_gpu"] / peak,
                "traffic": traffic_for(args.mode, wl), "peak_source": head["peak_source"],
                "kernel_ms": head["ms_per_step"],
                "algorithmic_flop_per_launch": flops}

    # End to end through the host-buffer C entry point (page-locked host memory).
    e2e = None
    if not args.no_e2e:
        ha = torch.empty(A.shape, dtype=torch.float32, pin_memory=True)
        hb = torch.empty(B.shape, dtype=torch.float32, pin_memory=True)
        hc = torch.empty(C.shape, dtype=torch.float32, pin_memory=True)
        ha.copy_(A)
        hb.copy_(B)
        es = torch.cuda.Stream(device)
        fn = lambda: tlcuda.matmul_host(ha, hb, mode=args.mode, out=hc, stream=es)  # noqa: E731
        e_steps = max(3, min(args.steps, 10))
        ms_e2e = time_device(fn, e_steps, 2, world, es)
        e2e = {"value": flops * world / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": int((A.numel() + B.numel()) * 4),
               "d2h_bytes_per_step": int(C.numel() * 4), "ms_per_step": ms_e2e,
               "api": "tlc_matmul_host"}
        del ha, hb, hc

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_reference_sample(wl)
        except Exception as e:  # the oracle/_ref build is optional on a user's host
            cpu = {"value": None, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"unavailable: {e}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic U[-1,1], torch.Generator seed 4 + 1000*rank",
            "mode": args.mode,
            "config": {"workload": wl, "batch_per_gpu": batch, "global_batch": batch * world,
                       "M": M, "N": N, "K": K, "layout": "row-major A, B, C",
                       "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (1 GiB per operand), no flush"},
            "roofline": roofline,
            "modes": results,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--mode", default=os.environ.get("TL_BENCH_MODE", "tf32"),
                    choices=["exact", "tf32", "3xtf32"])
    ap.add_argument("--workload", default="batched", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--all-modes", dest="all_modes", action="store_true", default=True)
    ap.add_argument("--head-only", dest="all_modes", action="store_false")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
