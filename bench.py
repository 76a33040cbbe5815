"""Benchmark of the batched fp32 GEMM behind tl::matmul (libtl_cuda) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode tf32|3xtf32|exact]
                    [--workload batched|square8192|...] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run.  Prints ONE
JSON line on rank 0.

Default workload "batched": per GPU the batched GEMM
C[64,2048,2048] = A[64,2048,2048] . B[64,2048,2048], fp32 row-major,
A, B ~ U[-1,1] (seed 4), the batch-sharded case of the scaling sweep: each
rank owns 64 batch entries of its own (weak scaling: the job at N GPUs is the
batch-sharded GEMM of 64*N entries; no data-path collective).  Square
workloads (square4096/8192/16384) are column-block sharded at N > 1 (strong
scaling: every rank holds A and B, computes C[:, its block]; the NCCL
all-gather that assembles C on every rank is timed separately as
`gather_ms`).  linear / attention / broadcast time the other configurations
(forward + backward where they have one) for reference.

A step is one call of the GEMM entry point over the workload; every operand is
at least 64 MiB and the batched operands are 1 GiB, above the 126 MB L2,
so no flush runs between steps.

Metric: GEMM TFLOP/s = useful FLOPs / time (2*batch*M*N*K per GEMM), whole
job.  `value` times the device-resident call (CUDA events on the launching
stream, max over ranks); `e2e` times tlc_matmul_host, the host-buffer C entry
point: page-locked host A, B in, host C out, copies inside the timed region.
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

# name: (batch, M, N, K) for the plain GEMM workloads
GEMMS = {
    "batched": (64, 2048, 2048, 2048),
    # 8 entries of the same shape (384 MiB of operands): the profiling stand-in
    # for "batched", whose DRAM traffic per launch is 8x this one's
    "batched8": (8, 2048, 2048, 2048),
    "square4096": (1, 4096, 4096, 4096),
    "square8192": (1, 8192, 8192, 8192),
    "square16384": (1, 16384, 16384, 16384),
    "square512": (1, 512, 512, 512),
}
OTHER = ("linear", "attention", "broadcast", "flash", "flash4", "conv")
METRIC = "GEMM TFLOP/s (fp32-exact, TF32, 3xTF32) at 1/2/4/8 B200, % of peak"


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0}, "fallback"


def peak_for(mode, peaks, src, sms, clock_mhz):
    """Roofline denominator (TFLOP/s) for a mode, with where it comes from."""
    if mode == "exact":
        # FP32 FFMA: 128 lanes x 2 FLOP per SM per clock at the max SM clock.
        # MEASURED_PEAKS.json has no FP32 figure, so this one is nominal.
        return sms * 128 * 2 * clock_mhz * 1e6 / 1e12, "nominal FP32 FFMA at max SM clock"
    tf32 = peaks["bf16_tflops"] / 2.0  # dense TF32 issues at half the dense bf16 rate
    if mode == "tf32":
        return tf32, f"TF32 = 1/2 of {src} bf16 ({peaks['bf16_tflops']} TFLOP/s)"
    return tf32 / 3.0, f"3xTF32 = 1/3 of TF32 = 1/6 of {src} bf16 ({peaks['bf16_tflops']} TFLOP/s)"


class ClockSampler:
    """SM clock, power and clock-event reasons sampled DURING the timed region.

    NVML (pynvml) is polled every 5 ms from a thread; only the samples taken
    between window_start() (just before the timed steps are enqueued) and
    window_end() (after the closing synchronize) count, so a short timed
    region is not drowned by idle samples around it.  Without pynvml,
    nvidia-smi is polled every 50 ms with host timestamps instead."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}
    Q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []  # (host time, sm MHz, max MHz, power W, set of reasons)
        self.t0 = self.t1 = None
        self.thread = None
        self.proc = None
        self.f = None

    def _nvml_handle(self, nv):
        """The NVML device of CUDA device `index` (by UUID: NVML numbers GPUs
        without regard to CUDA_VISIBLE_DEVICES)."""
        try:
            import torch
            u = str(torch.cuda.get_device_properties(self.index).uuid)
            return nv.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:  # noqa: BLE001
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def _nvml_sample(self):
        nv, h = self.nv, self.h
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.samples.append((time.time(), sm, self.mx, pw,
                             {n for b, n in self.REASONS.items() if bits & b}))

    def _nvml_loop(self, stop):
        while not stop.is_set():
            try:
                self._nvml_sample()
            except Exception:  # noqa: BLE001 - a failed query ends sampling
                return
            time.sleep(0.005)

    def __enter__(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            self.nv, self.h = nv, self._nvml_handle(nv)
            self.mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(self.stop,), daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001 - no NVML binding or device: nvidia-smi below
            self.thread = None
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # let the sampler start before the timed region
        except OSError:
            self.proc = None
        return self

    def window_start(self):
        self.t0 = time.time()

    def window_end(self):
        self.t1 = time.time()
        # A region shorter than the polling interval: one sample right at its end.
        if self.thread and not any(r[0] >= self.t0 for r in list(self.samples)):
            try:
                self._nvml_sample()
            except Exception:  # noqa: BLE001
                pass

    def __exit__(self, *a):
        if self.thread:
            self.stop.set()
            self.thread.join(2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._read_smi()

    def _read_smi(self):
        import datetime

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        with open(self.f.name) as fh:
            for line in fh:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 8:
                    continue
                try:
                    t = datetime.datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
                self.samples.append((t, num(p[1]), num(p[2]), num(p[3]),
                                     {n for n, v in zip(names, p[4:8]) if v.lower() == "active"}))
        os.unlink(self.f.name)

    def summary(self, max_mhz_default):
        rows = self.samples
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
            if not inside:  # region shorter than one sampling interval: the next sample
                after = [r for r in rows if r[0] >= self.t0]
                inside = after[:1]
            rows = inside
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": max_mhz_default, "reasons": ["unsampled"]}
        sm = [r[1] for r in rows if r[1] is not None]
        mx = [r[2] for r in rows if r[2] is not None]
        pw = [r[3] for r in rows if r[3] is not None]
        reasons = set().union(*(r[4] for r in rows))
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else max_mhz_default,
                "power_w_max": max(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(rows),
                "source": "nvml" if self.thread else "nvidia-smi",
                "window_ms": round((self.t1 - self.t0) * 1e3, 1) if self.t0 and self.t1 else None}


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
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


def time_device(fn, steps, warmup, world, stream, count=None, clocks=None):
    """Per-step device time (ms): W warm-ups, then K steps between CUDA events
    on `stream`, bracketed by barrier + synchronize; max over ranks.  With
    `count` (a function returning a launch counter) also returns the number of
    launches inside the timed region; `clocks` (a ClockSampler) is told where
    the timed region starts and ends."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = count() if count else 0
    if clocks:
        clocks.window_start()
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.window_end()
    l1 = count() if count else 0
    barrier(world)
    ms = e0.elapsed_time(e1) / steps
    return max_over_ranks(ms, world), l1 - l0


def time_graph(fn, steps, world):
    """Per-step device time (ms) of `fn` captured once into a CUDA graph and
    replayed `steps` times between CUDA events (max over ranks): the launch
    cost of the kernels without the Python binding's per-call host work."""
    import torch
    fn()  # set-up work (kernel attributes, checks) stays outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        g.replay()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del g
    return max_over_ranks(ms, world)


# Workloads whose per-step kernels are short enough that the Python binding's
# host work per call rivals them (a few microseconds per GEMM; the conv step's
# dozen launches in ~0.2 ms): also timed as CUDA-graph replays.
GRAPH_WORKLOADS = ("square512", "broadcast", "conv")


# ---- workloads -------------------------------------------------------------------------

class Work:
    """One workload on one rank: step(mode) runs it once; flops = useful FLOPs
    of one step on this rank; job_flops = of the whole job."""
    name = ""
    scaling = "weak"
    config = {}
    flops = 0.0
    job_flops = 0.0

    def step(self, mode):
        raise NotImplementedError


def gemm_config(name, world):
    """The `config` of a GEMM workload at `world` GPUs (both arms print it)."""
    batch, M, N, K = GEMMS[name]
    if batch > 1:
        par = f"batch-sharded x{world}" if world > 1 else "single GPU"
    else:
        par = f"output-column-block sharded x{world}" if world > 1 else "single GPU"
    return {"workload": name, "batch_per_gpu": batch,
            "global_batch": batch * world if batch > 1 else 1,
            "M": M, "N": N, "K": K, "layout": "row-major A, B, C",
            "parallelism": par,
            "l2": "operands larger than L2 (126 MB), no flush"}


class GemmWork(Work):
    def __init__(self, name, world, rank, device):
        import torch
        import tldist
        batch, M, N, K = GEMMS[name]
        self.name = name
        self.batch, self.M, self.N, self.K = batch, M, N, K
        if batch > 1:
            # batch-sharded, weak: every rank owns `batch` entries of its own
            g = torch.Generator(device=device).manual_seed(4 + 1000 * rank)
            self.A = torch.rand((batch, M, K), generator=g, device=device) * 2 - 1
            self.B = torch.rand((batch, K, N), generator=g, device=device) * 2 - 1
            self.C = torch.empty((batch, M, N), device=device)
            self.Bv = self.B
            self.scaling = "weak"
            self.flops = 2.0 * batch * M * N * K
            self.job_flops = self.flops * world
        else:
            # column-block sharded, strong: same A, B on every rank
            g = torch.Generator(device=device).manual_seed(4)
            self.A = torch.rand((M, K), generator=g, device=device) * 2 - 1
            self.B = torch.rand((K, N), generator=g, device=device) * 2 - 1
            self.edges = tldist.col_blocks(N, world, 256)
            c0, c1 = self.edges[rank], self.edges[rank + 1]
            self.Bv = self.B[:, c0:c1]  # read in place, row stride N
            self.C = torch.empty((M, c1 - c0), device=device)
            self.scaling = "strong" if world > 1 else "weak"
            self.flops = 2.0 * M * (c1 - c0) * K
            self.job_flops = 2.0 * M * N * K
        self.config = gemm_config(name, world)

    def step(self, mode):
        import tlcuda
        tlcuda.matmul(self.A, self.Bv, mode=mode, out=self.C)

    def gather_ms(self, world, stream, iters=5):
        """Square workloads at N > 1: the all-gather + reassembly of C."""
        if self.batch > 1 or world == 1:
            return None
        import torch
        import torch.distributed as dist
        import tlcuda
        M, N = self.M, self.N
        w = self.edges[1] - self.edges[0]
        if any(self.edges[q + 1] - self.edges[q] != w for q in range(world)):
            return None
        gathered = torch.empty((world * M * w,), device=self.C.device)
        out = torch.empty((M, N), device=self.C.device)

        def fn():
            dist.all_gather_into_tensor(gathered, self.C.reshape(-1))
            tlcuda.gather_colblocks(gathered, out, M, N, self.edges)
        ms, _ = time_device(fn, iters, 2, world, stream)
        return ms

    def e2e(self, mode, stream):
        """tlc_matmul_host on page-locked host buffers (this rank's share)."""
        import torch
        import tlcuda
        ha = torch.empty(self.A.shape, dtype=torch.float32, pin_memory=True)
        hb = torch.empty(self.Bv.shape, dtype=torch.float32, pin_memory=True)
        hc = torch.empty(self.C.shape, dtype=torch.float32, pin_memory=True)
        ha.copy_(self.A)
        hb.copy_(self.Bv)

        def fn():
            tlcuda.matmul_host(ha, hb, mode=mode, out=hc, stream=stream)
        return fn, int((ha.numel() + hb.numel()) * 4), int(hc.numel() * 4), (ha, hb, hc)


class LinearWork(Work):
    """Y = X.W^T + b fwd + bwd: X[4096,1024] ~ N(0,1), W[4096,1024] ~ U(-1/32,1/32),
    b = 0, dY ~ N(0,1).  Forward: one GEMM with the bias add fused into its
    epilogue; backward: dX = dY.W, dW^T = X^T.dY (MatmulBackward) and
    db = sum_to(dY, [4096]) (AddBackward).  FLOPs count the three GEMMs."""
    name = "linear"

    def __init__(self, world, rank, device):
        import torch
        g = torch.Generator(device=device).manual_seed(2)
        self.X = torch.randn((4096, 1024), generator=g, device=device)
        self.W = (torch.rand((4096, 1024), generator=g, device=device) * 2 - 1) / 32
        self.dY = torch.randn((4096, 4096), generator=g, device=device)
        self.Y = torch.empty((4096, 4096), device=device)
        self.dX = torch.empty((4096, 1024), device=device)
        self.dWt = torch.empty((1024, 4096), device=device)
        self.b = torch.zeros((4096,), device=device)
        self.db = torch.empty((4096,), device=device)
        self.flops = 3 * 2.0 * 4096 * 4096 * 1024
        self.job_flops = self.flops * world
        self.config = {"workload": "linear", "X": [4096, 1024], "W": [4096, 1024],
                       "gemms": "Y=X.W^T+b (bias fused), dX=dY.W, dW^T=X^T.dY; db=sum_to(dY)",
                       "parallelism": "replicas"}

    def step(self, mode):
        import tlcuda
        tlcuda.matmul_fused(self.X, self.W.t(), 1.0, self.b, mode=mode, out=self.Y)
        tlcuda.matmul_backward(self.dY, self.X, self.W.t(), mode=mode, da=self.dX, db=self.dWt)
        tlcuda.sum_to(self.dY, (4096,), out=self.db)


class AttentionWork(Work):
    """Encoder attention: batch 16, seq 512, d_model 768, 12 heads of 64:
    QKV [8192,768].[768,2304], scores [192,512,64].[192,64,512] (K^T read in
    place, the 1/8 scale fused into the GEMM epilogue), P = softmax(scores)
    (device kernel), context P.[192,512,64], out-proj [8192,768].[768,768];
    activations ~ N(0,1), weights ~ N(0,0.02).  FLOPs count the four GEMMs."""
    name = "attention"

    def __init__(self, world, rank, device):
        import torch
        import tlcuda
        g = torch.Generator(device=device).manual_seed(3)
        self.x = torch.randn((8192, 768), generator=g, device=device)
        self.Wqkv = torch.randn((768, 2304), generator=g, device=device) * 0.02
        self.Wo = torch.randn((768, 768), generator=g, device=device) * 0.02
        self.q = torch.randn((192, 512, 64), generator=g, device=device)
        self.k = torch.randn((192, 512, 64), generator=g, device=device)
        self.v = torch.randn((192, 512, 64), generator=g, device=device)
        self.P = torch.empty((192, 512, 512), device=device)
        self.qkv = torch.empty((8192, 2304), device=device)
        self.sc = torch.empty((192, 512, 512), device=device)
        self.ctx = torch.empty((192, 512, 64), device=device)
        self.o = torch.empty((8192, 768), device=device)
        self.flops = 2.0 * (8192 * 768 * 2304 + 2 * 192 * 512 * 512 * 64 + 8192 * 768 * 768)
        self.job_flops = self.flops * world
        self.config = {"workload": "attention", "batch": 16, "seq": 512, "d_model": 768,
                       "heads": 12, "glue": "scores scaled in the GEMM epilogue, softmax kernel",
                       "parallelism": "replicas"}

    def step(self, mode):
        import tlcuda
        tlcuda.matmul(self.x, self.Wqkv, mode=mode, out=self.qkv)
        tlcuda.matmul_fused(self.q, self.k.transpose(1, 2), 0.125, None, mode=mode, out=self.sc)
        tlcuda.softmax(self.sc, out=self.P)
        tlcuda.matmul(self.P, self.v, mode=mode, out=self.ctx)
        tlcuda.matmul(self.x, self.Wo, mode=mode, out=self.o)


class BroadcastWork(Work):
    """A[32,128,64] . B[64,128] (B broadcast) fwd + MatmulBackward, N(0,1) seed 1."""
    name = "broadcast"

    def __init__(self, world, rank, device):
        import torch
        g = torch.Generator(device=device).manual_seed(1)
        self.A = torch.randn((32, 128, 64), generator=g, device=device)
        self.B = torch.randn((64, 128), generator=g, device=device)
        self.dC = torch.randn((32, 128, 128), generator=g, device=device)
        self.C = torch.empty((32, 128, 128), device=device)
        self.dA = torch.empty_like(self.A)
        self.dB = torch.empty_like(self.B)
        self.flops = 3 * 2.0 * 32 * 128 * 128 * 64
        self.job_flops = self.flops * world
        self.config = {"workload": "broadcast", "A": [32, 128, 64], "B": [64, 128],
                       "parallelism": "replicas"}

    def step(self, mode):
        import tlcuda
        tlcuda.matmul(self.A, self.B, mode=mode, out=self.C)
        tlcuda.matmul_backward(self.dC, self.A, self.B, mode=mode, da=self.dA, db=self.dB)


class FlashWork(Work):
    """flash_attention forward + FlashAttentionBackward on batch 16 x 12 heads,
    S = 2048, d = 64 ([16,12,2048,64] Q, K, V, dO ~ N(0,1), seed 5), scale 1/8.
    TF32 mode: the tcgen05 forward, then the fused tcgen05 backward (prep,
    dK/dV, dQ kernels); exact / 3xTF32: the FFMA forward, then five batched
    GEMMs in the mode and elementwise kernels.  FLOPs: forward 4*S*S*d per
    head (Q.K^T and P.V), backward 10*S*S*d (Q.K^T recomputed, dV, dP, dQ, dK;
    the fused dQ kernel recomputes S and dP once more, not counted)."""
    name = "flash"

    def __init__(self, world, rank, device, batch=16):
        import torch
        g = torch.Generator(device=device).manual_seed(5)
        shape = (batch, 12, 2048, 64)
        self.q, self.k, self.v, self.dO = (torch.randn(shape, generator=g, device=device)
                                           for _ in range(4))
        self.o = torch.empty(shape, device=device)
        self.lse = torch.empty(shape[:-1], device=device)
        self.dq, self.dk, self.dv = (torch.empty(shape, device=device) for _ in range(3))
        heads, S, d = batch * 12, 2048, 64
        self.fwd_flops = 4.0 * heads * S * S * d
        self.flops = self.fwd_flops + 10.0 * heads * S * S * d
        self.job_flops = self.flops * world
        self.name = "flash" if batch == 16 else f"flash{batch}"
        self.config = {"workload": self.name, "batch": batch, "heads": 12, "S": 2048, "d": 64,
                       "sm_scale": 0.125,
                       "forward": "fused kernel: tcgen05 TF32 in tf32 mode, FFMA otherwise",
                       "backward": "tf32: fused tcgen05 dK/dV and dQ kernels; exact, 3xtf32: 5 batched GEMMs in the mode + elementwise kernels",
                       "parallelism": "replicas"}

    def forward(self, mode):
        import tlcuda
        tlcuda.flash_attention(self.q, self.k, self.v, 0.125, out=self.o, lse=self.lse, mode=mode)

    def step(self, mode):
        import tlcuda
        self.forward(mode)
        tlcuda.flash_attention_backward(self.dO, self.q, self.k, self.v, self.o, self.lse, 0.125,
                                        mode=mode, dq=self.dq, dk=self.dk, dv=self.dv)

    def forward_roofline(self, world, stream, mode, peak, steps=10):
        """The forward kernel alone against its peak: tf32 the tensor-core
        kernel (flash_tc_kernel) against TF32, else the FFMA kernel
        (flash_fwd_kernel<64>) against the FP32 FFMA peak."""
        ms, _ = time_device(lambda: self.forward(mode), steps, 3, world, stream)
        ach = self.fwd_flops / (ms * 1e-3) / 1e12
        tc = mode == "tf32"
        return {"kernel": "flash_tc_kernel" if tc else "flash_fwd_kernel<64>", "mode": mode,
                "ms": ms, "achieved": ach, "peak": peak[0], "unit": "TFLOP/s",
                "frac": ach / peak[0], "bound": "tensor" if tc else "fp32-fma",
                "peak_source": peak[1], "algorithmic_flop_per_launch": self.fwd_flops}


class ConvWork(Work):
    """conv2d forward + Conv2dBackward, a ResNet-style 3x3 layer: x [32,64,56,56],
    W [64,64,3,3], b [64], stride 1, padding 1 (x, dO ~ N(0,1), W ~ N(0,0.05^2),
    b ~ N(0,1), seed 6).  TF32 / 3xTF32: the forward, the input gradient and the
    weight gradient as implicit GEMMs over TMA boxes of NHWC copies; exact:
    im2col, the batched GEMMs, col2im.  FLOPs: 2*N*C_out*H*W*C_in*k*k forward,
    twice that backward (dW and dX)."""
    name = "conv"

    def __init__(self, world, rank, device):
        import torch
        g = torch.Generator(device=device).manual_seed(6)
        self.x = torch.randn((32, 64, 56, 56), generator=g, device=device)
        self.w = torch.randn((64, 64, 3, 3), generator=g, device=device) * 0.05
        self.b = torch.randn((64,), generator=g, device=device)
        self.go = torch.randn((32, 64, 56, 56), generator=g, device=device)
        self.y = torch.empty((32, 64, 56, 56), device=device)
        fwd = 2.0 * 32 * 64 * 56 * 56 * 64 * 9
        self.flops = 3 * fwd
        self.job_flops = self.flops * world
        self.config = {"workload": "conv", "x": [32, 64, 56, 56], "W": [64, 64, 3, 3], "stride": 1,
                       "padding": 1, "groups": 1, "parallelism": "replicas"}

    def step(self, mode):
        import tlcuda
        tlcuda.conv2d(self.x, self.w, self.b, 1, 1, 1, mode=mode, out=self.y)
        tlcuda.conv2d_backward(self.go, self.x, self.w, 1, 1, 1, mode=mode)


def make_work(name, world, rank, device):
    if name in GEMMS:
        return GemmWork(name, world, rank, device)
    if name == "flash4":  # the profiling stand-in for "flash": batch 4 instead of 16
        return FlashWork(world, rank, device, batch=4)
    return {"linear": LinearWork, "attention": AttentionWork, "broadcast": BroadcastWork,
            "flash": FlashWork, "conv": ConvWork}[name](world, rank, device)


# ---- the reference's CPU path ----------------------------------------------------------

def ref_sample(name):
    """A bounded sample of the workload for the reference CPU matmul:
    (a, b, useful FLOPs, description)."""
    import numpy as np
    rng = np.random.default_rng(4)
    if name in GEMMS:
        batch, M, N, K = GEMMS[name]
        rows = M if batch > 1 else min(M, 256)
        what = "one batch entry" if batch > 1 else f"a {rows}-row slab"
    elif name == "linear":
        rows, K, N = 256, 1024, 4096
        what = "a 256-row slab of Y = X.W^T"
    elif name == "attention":
        rows, K, N = 256, 768, 2304
        what = "a 256-row slab of the QKV projection"
    else:
        rows, K, N = 128, 64, 128
        what = "one batch entry of the broadcast forward"
    a = rng.uniform(-1, 1, (rows, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    return a, b, 2.0 * rows * N * K, f"tl::matmul [{rows},{K}]x[{K},{N}] fp32, {what} of the workload"


def ref_job(name, R):
    """(callable, useful FLOPs, description) of one bounded sample on the
    reference library R: tl::matmul for the GEMM workloads; for "flash" one
    head of the workload (S = 2048, d = 64) through tl::flash_attention and
    FlashAttentionBackward (bench/bench_attention.cpp's single-head call)."""
    if name.startswith("flash"):
        import numpy as np
        rng = np.random.default_rng(5)
        q, k, v, g = (rng.standard_normal((2048, 64)).astype(np.float32) for _ in range(4))
        flops = 14.0 * 2048 * 2048 * 64
        return (lambda: R.flash_attention(q, k, v, 0.125, grad=g), flops,
                f"tl::flash_attention + backward on one head [2048,64] of the workload "
                f"({flops / 1e9:.2f} GFLOP)")
    if name == "conv":
        import numpy as np
        rng = np.random.default_rng(6)
        x = rng.standard_normal((2, 64, 56, 56)).astype(np.float32)
        w = (rng.standard_normal((64, 64, 3, 3)) * 0.05).astype(np.float32)
        b = rng.standard_normal((64,)).astype(np.float32)
        g = rng.standard_normal((2, 64, 56, 56)).astype(np.float32)
        flops = 3 * 2.0 * 2 * 64 * 56 * 56 * 64 * 9
        return (lambda: R.conv2d(x, w, b, 1, 1, 1, grad=g), flops,
                f"tl::conv2d + Conv2dBackward on 2 of the 32 images ({flops / 1e9:.2f} GFLOP)")
    a, b, flops, what = ref_sample(name)
    return lambda: R.matmul(a, b), flops, f"{what} ({flops / 1e9:.2f} GFLOP)"


def cpu_reference_sample(name, reps=3):
    """The reference's own CPU path (oracle/_ref, compiled from its sources),
    min over reps (time_best, bench/bench_matmul.cpp:27-39)."""
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    R = O.tlref()
    fn, flops, what = ref_job(name, R)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    cores = 1 if name.startswith("flash") else R.hardware_threads()
    return {"value": flops / best / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
            "sample": f"{what}, best of {reps}, {os.path.basename(R.path)}"
                      + (" (single-threaded code path)" if name.startswith("flash")
                         else " with std::thread::hardware_concurrency() threads")}


def reference_full_workload(name):
    """The whole per-GPU workload for the reference's tl::matmul, when one step
    of it fits a bounded CPU run: the batched GEMM (64 entries of 2048^3, about
    6 s per step on 16 host threads).  None for the rest (they are sampled)."""
    if name not in GEMMS or GEMMS[name][0] <= 1:
        return None
    import numpy as np
    batch, M, N, K = GEMMS[name]
    rng = np.random.default_rng(4)
    a = inputs_uniform(rng, (batch, M, K))
    b = inputs_uniform(rng, (batch, K, N))
    return a, b, 2.0 * batch * M * N * K


def inputs_uniform(rng, shape):
    """U[-1,1] float32 in chunks of 16 Mi values (bounded float64 temporaries)."""
    import numpy as np
    out = np.empty(shape, np.float32)
    flat = out.reshape(-1)
    step = 1 << 24
    for i in range(0, flat.size, step):
        flat[i:i + step] = rng.uniform(-1.0, 1.0, size=min(step, flat.size - i))
    return out


def run_reference_arm(args, out_fd):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    try:
        R = O.tlref()
    except FileNotFoundError as e:
        emit({"impl": "reference", "unavailable": f"oracle/_ref not built: {e}"}, out_fd)
        return 0
    cores = 1 if args.workload.startswith("flash") else R.hardware_threads()
    full = reference_full_workload(args.workload)
    if full is not None:
        # the reference's own tl::matmul over this GPU's whole share of the workload
        a, b, flops = full
        dt = R.matmul_timed(a, b, args.warmup, args.steps)
        cfg = gemm_config(args.workload, world)
        what = (f"tl::matmul {list(a.shape)}x{list(b.shape)} fp32, the whole per-GPU workload "
                f"({flops / 1e12:.2f} TFLOP)")
        if world > 1:
            cfg = dict(cfg, reference_sample=f"one GPU's share ({a.shape[0]} of "
                                            f"{a.shape[0] * world} entries) per step")
        sample = (f"each step: {what}, steady_clock around tl::matmul alone, "
                  f"{os.path.basename(R.path)}, std::thread::hardware_concurrency() threads")
    else:
        fn, flops, what = ref_job(args.workload, R)
        for _ in range(args.warmup):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        dt = (time.perf_counter() - t0) / args.steps
        cfg = {"workload": args.workload}
        if args.workload in GEMMS:
            batch, M, N, K = GEMMS[args.workload]
            cfg.update({"batch": batch, "M": M, "N": N, "K": K,
                        "sampled_rows": M if batch > 1 else min(M, 256)})
        sample = f"each step: {what}, host wall clock"
    val = flops / dt / 1e12
    line = {"metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": ("synthetic N(0,1) seed 5" if args.workload.startswith("flash")
                     else "synthetic U[-1,1] seed 4"),
            "impl": "reference", "config": cfg,
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    emit(line, out_fd)
    return 0


def traffic_for(mode, wl):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            t = json.load(f)
        return t.get(f"{wl}:{mode}")
    except OSError:
        return None


def e2e_record(work, mode, world, device, steps):
    """`mode` end to end through tlc_matmul_host (page-locked host A, B in,
    host C out, copies inside the timed region)."""
    import torch
    try:
        es = torch.cuda.Stream(device)
        fn, hbytes, dbytes, keep = work.e2e(mode, es)
        ms, _ = time_device(fn, steps, 2, world, es)
        del keep
        return {"value": work.job_flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": hbytes, "d2h_bytes_per_step": dbytes,
                "ms_per_step": ms, "api": "tlc_matmul_host", "mode": mode}
    except Exception as e:  # e.g. not enough page-locked host memory
        return {"value": None, "unavailable": repr(e)[:200], "mode": mode}


def square8192_record(world, rank, device, stream, peaks, psrc, sms, steps):
    """The 8192^3 GEMM of the scaling sweep on one GPU, every mode, each with
    its own CUDA-event timing; TF32 (the target of 0.70 of dense TF32 peak)
    with the SM clock sampled inside its timed region."""
    import tlcuda
    w = GemmWork("square8192", 1, 0, device)
    out = {"config": {"M": 8192, "N": 8192, "K": 8192, "layout": "row-major A, B, C"}}
    mx = peaks.get("sm_max_mhz", 1965.0)
    for mode in ("tf32", "3xtf32", "exact"):
        n = steps if mode != "exact" else max(3, steps // 3)
        if mode == "tf32":
            with ClockSampler(device.index) as cs:
                ms, launches = time_device(lambda: w.step(mode), n, 3, world, stream,
                                           tlcuda.launch_count, clocks=cs)
            clocks = cs.summary(mx)
        else:
            ms, launches = time_device(lambda: w.step(mode), n, 3, world, stream, tlcuda.launch_count)
            clocks = None
        peak, pdesc = peak_for(mode, peaks, psrc, sms, mx)
        tf = w.flops / (ms * 1e-3) / 1e12
        rec = {"ms": ms, "tflops": tf, "frac": tf / peak, "peak": peak, "peak_source": pdesc,
               "launches_per_step": launches / n}
        if clocks:
            rec["clocks"] = clocks
        out[mode] = rec
    del w
    return out


def sustained_record(work, mode, world, stream, peaks, device, seconds=1.5):
    """The headline step back to back for about `seconds` (long enough to reach
    the 1000 W power cap), against the sustained TF32 peak (1/2 of the
    measured sustained bf16 figure), with the SM clock sampled inside."""
    import tlcuda
    probe, _ = time_device(lambda: work.step(mode), 3, 3, world, stream)
    n = max(10, int(seconds * 1e3 / max(probe, 1e-3)))
    with ClockSampler(device.index) as cs:
        ms, _ = time_device(lambda: work.step(mode), n, 3, world, stream, tlcuda.launch_count,
                            clocks=cs)
    tf = work.flops / (ms * 1e-3) / 1e12
    sus = peaks.get("bf16_tflops_sustained")
    peak = sus / 2.0 if (sus and mode == "tf32") else None
    return {"mode": mode, "steps": n, "seconds": n * ms * 1e-3, "ms_per_step": ms,
            "tflops_per_gpu": tf, "peak": peak,
            "peak_source": "TF32 = 1/2 of measured sustained bf16" if peak else None,
            "frac": tf / peak if peak else None, "clocks": cs.summary(peaks.get("sm_max_mhz", 1965.0))}


def scaling_records(args, world, rank, device, stream, peaks, psrc, sms):
    """At N > 1: what the weak-scaled headline does not show.
      strong          the fixed 64 x 2048^3 batch split over the N GPUs (64/N
                      entries each): compute alone, and compute + the NCCL
                      all-gather that puts the whole C on every GPU;
      square8192      one 8192^3 GEMM over output column blocks (A and B
                      replicated, each GPU reads its block of B in place):
                      compute, and the all-gather + reassembly of C;
      exact_db_chain  the broadcast workload's MatmulBackward in exact mode,
                      dB reduced by the rank-to-rank chain in batch order."""
    import torch
    import torch.distributed as dist
    import tldist
    import tlcuda
    out = {}
    mode = args.mode
    # strong scaling of the batched workload
    batch, M, N, K = GEMMS["batched"]
    b0, b1 = tldist.batch_shard(batch, world, rank)
    g = torch.Generator(device=device).manual_seed(4)
    A = torch.rand((b1 - b0, M, K), generator=g, device=device) * 2 - 1
    B = torch.rand((b1 - b0, K, N), generator=g, device=device) * 2 - 1
    C = torch.empty((b1 - b0, M, N), device=device)
    flops = 2.0 * batch * M * N * K
    ms, _ = time_device(lambda: tlcuda.matmul(A, B, mode=mode, out=C), 10, 3, world, stream)
    rec = {"entries_per_gpu": b1 - b0, "compute_ms": ms, "tflops": flops / (ms * 1e-3) / 1e12}
    if batch % world == 0:
        full = torch.empty((batch, M, N), device=device)

        def both():
            tlcuda.matmul(A, B, mode=mode, out=C)
            dist.all_gather_into_tensor(full, C)
        ms_g, _ = time_device(both, 10, 3, world, stream)
        rec.update({"with_allgather_ms": ms_g, "with_allgather_tflops": flops / (ms_g * 1e-3) / 1e12,
                    "allgather_bytes_per_gpu": 4 * M * N * (batch - (b1 - b0)),
                    "collective": "ncclAllGather of C (every GPU receives the other GPUs' shards)"})
    out["strong_batched"] = rec
    del A, B, C
    torch.cuda.empty_cache()
    # column-block sharded square
    w = GemmWork("square8192", world, rank, device)
    ms, _ = time_device(lambda: w.step(mode), 10, 3, world, stream)
    gms = w.gather_ms(world, stream)
    rec = {"compute_ms": ms, "tflops": w.job_flops / (ms * 1e-3) / 1e12, "gather_ms": gms,
           "collective": "ncclAllGather of the column blocks + tlc_gather_colblocks"}
    if gms:
        rec["with_gather_tflops"] = w.job_flops / ((ms + gms) * 1e-3) / 1e12
    out["square8192_colblock"] = rec
    del w
    torch.cuda.empty_cache()
    # exact-mode dB chain of the broadcast workload
    gb = torch.Generator(device=device).manual_seed(1)
    a = torch.randn((32, 128, 64), generator=gb, device=device)
    b = torch.randn((64, 128), generator=gb, device=device)
    c0, c1 = tldist.batch_shard(32, world, rank)
    dc = torch.randn((32, 128, 128), generator=gb, device=device)[c0:c1].contiguous()
    ms, _ = time_device(lambda: tldist.batch_sharded_matmul_backward(dc, a, b, mode="exact"),
                        10, 3, world, stream)
    out["exact_db_chain"] = {"workload": "A[32,128,64].B[64,128] backward, batch-sharded",
                             "ms": ms, "hops": world - 1,
                             "collective": "rank-to-rank send/recv chain + broadcast"}
    out["device_group"] = device_group_record(args, world, rank, device)
    return out


def device_group_record(args, world, rank, device):
    """The drop-in's own multi-GPU path: rank 0 alone drives all N GPUs from
    one host thread through a device group (tlc_group_matmul_host) on the
    batched workload from page-locked host buffers (64 x 2048^3 in total, each
    GPU copying in and computing its 64/N entries); the other ranks wait.  The
    call is synchronous (it returns when every GPU's share of C is back in host
    memory), so it is timed by the host clock around whole calls."""
    import torch
    import tlcuda
    rec = None
    if rank == 0:
        try:
            batch, M, N, K = GEMMS["batched"]
            g = torch.Generator().manual_seed(4)
            ha = (torch.rand((batch, M, K), generator=g) * 2 - 1).pin_memory()
            hb = (torch.rand((batch, K, N), generator=g) * 2 - 1).pin_memory()
            hc = torch.empty((batch, M, N)).pin_memory()
            flops = 2.0 * batch * M * N * K
            with tlcuda.Group(list(range(world))) as grp:
                members, uses_nccl = grp.size()
                for _ in range(2):
                    grp.matmul_host(ha, hb, mode=args.mode, out=hc)
                reps = 5
                t0 = time.perf_counter()
                for _ in range(reps):
                    grp.matmul_host(ha, hb, mode=args.mode, out=hc)
                dt = (time.perf_counter() - t0) / reps
            rec = {"api": "tlc_group_matmul_host", "gpus": members, "mode": args.mode,
                   "ms_per_call": dt * 1e3, "tflops": flops / dt / 1e12,
                   "h2d_bytes_per_call": 4 * (ha.numel() + hb.numel()),
                   "d2h_bytes_per_call": 4 * hc.numel(), "nccl": uses_nccl,
                   "timer": "host clock around synchronous calls"}
            del ha, hb, hc
        except Exception as e:  # noqa: BLE001 - reported, not fatal to the bench line
            rec = {"unavailable": repr(e)[:200]}
    barrier(world)
    return rec


def run_ours(args, out_fd):
    import torch
    import tlcuda
    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    work = make_work(args.workload, world, rank, device)
    stream = torch.cuda.current_stream()
    modes = [args.mode] + [m for m in ("tf32", "3xtf32", "exact") if m != args.mode and args.all_modes]
    peaks, psrc = load_peaks()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    mx = peaks.get("sm_max_mhz", 1965.0)

    results = {}
    launches = None
    clocks = None
    for mode in modes:
        fn = lambda: work.step(mode)  # noqa: E731
        if mode == args.mode:
            with ClockSampler(local) as cs:
                ms, launches = time_device(fn, args.steps, args.warmup, world, stream,
                                           tlcuda.launch_count, clocks=cs)
            clocks = cs.summary(mx)
        else:
            ms, _ = time_device(fn, max(3, args.steps // 2), 3, world, stream)
        peak, pdesc = peak_for(mode, peaks, psrc, sms, mx)
        per_gpu = work.flops / (ms * 1e-3) / 1e12
        results[mode] = {"ms_per_step": ms, "tflops_per_gpu": per_gpu,
                         "value": work.job_flops / (ms * 1e-3) / 1e12,
                         "roofline_frac": per_gpu / peak, "peak_tflops": peak,
                         "peak_source": pdesc}
        if args.workload in GRAPH_WORKLOADS:
            gms = time_graph(fn, max(args.steps, 50), world)
            results[mode].update({"graph_ms_per_step": gms,
                                  "graph_tflops_per_gpu": work.flops / (gms * 1e-3) / 1e12})

    head = results[args.mode]
    roofline = {"bound": "tensor" if args.mode != "exact" else "fp32-fma",
                "achieved": head["tflops_per_gpu"], "peak": head["peak_tflops"],
                "unit": "TFLOP/s", "frac": head["roofline_frac"],
                "traffic": traffic_for(args.mode, args.workload),
                "peak_source": head["peak_source"], "kernel_ms": head["ms_per_step"],
                "algorithmic_flop_per_launch": work.flops}

    gather = work.gather_ms(world, stream) if isinstance(work, GemmWork) else None
    fwd = None
    if isinstance(work, FlashWork):
        fmode = args.mode if args.mode == "tf32" else "exact"
        fwd = [work.forward_roofline(world, stream, m, peak_for(m, peaks, psrc, sms, mx))
               for m in dict.fromkeys((fmode, "exact"))]

    # End to end through the host-buffer C entry point (page-locked host memory),
    # every mode; the head mode's record is the line's `e2e`.
    e2e = None
    if not args.no_e2e and isinstance(work, GemmWork):
        for mode in modes:
            rec = e2e_record(work, mode, world, device,
                             max(3, min(args.steps, 10)) if mode == args.mode else 3)
            results[mode]["e2e"] = rec
            if mode == args.mode:
                e2e = rec

    extras = {}
    if not args.no_extras and args.workload == "batched":
        if world == 1:
            extras["square8192"] = square8192_record(world, rank, device, stream, peaks, psrc,
                                                     sms, max(5, min(args.steps, 20)))
            extras["sustained"] = sustained_record(work, args.mode, world, stream, peaks, device)
        else:
            extras["scaling"] = scaling_records(args, world, rank, device, stream, peaks, psrc, sms)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_reference_sample(args.workload)
        except Exception as e:  # the oracle/_ref build is optional on a user's host
            cpu = {"value": None, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"unavailable: {e}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": work.scaling, "vs_baseline": None,
            "dtype": "f32", "data": "synthetic, seeded torch.Generator (see config)",
            "mode": args.mode, "config": work.config, "roofline": roofline, "modes": results,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
        }
        if gather is not None:
            line["gather_ms"] = gather
        if fwd is not None:
            line["forward"] = fwd
        line.update(extras)
        emit(line, out_fd)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def emit(line, fd):
    """The one JSON line, written to the original standard output."""
    os.write(fd, (json.dumps(line) + "\n").encode())


def main():
    # Libraries (NCCL's version banner, for one) may print on standard output;
    # everything but the result line goes to standard error instead.
    sys.stdout.flush()
    out_fd = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--mode", default=os.environ.get("TL_BENCH_MODE", "tf32"),
                    choices=["exact", "tf32", "3xtf32"])
    ap.add_argument("--workload", default="batched", choices=sorted(GEMMS) + list(OTHER))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--all-modes", dest="all_modes", action="store_true", default=True)
    ap.add_argument("--head-only", dest="all_modes", action="store_false")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the 8192^3 / sustained (N=1) and scaling (N>1) sub-records")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args, out_fd)
    return run_ours(args, out_fd)


if __name__ == "__main__":
    sys.exit(main())
