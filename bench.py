"""Benchmark of the MXFP8 x BF16 GEMM path (D = A*B + C) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload dense_projection|long_k|tall_skinny|wide|square|codec]
                    [--scaling strong|weak] [--no-gather]

One step is one pass of the hot path over one batch of synthetic input: one
D = A*B + C at the workload's shape (default: the dense projection M=4096,
N=12288, K=4096), inputs resident in HBM.  The JSON line's ``value`` is
whole-job TFLOP/s (2*M*N*K per GEMM, the reference's formula,
include/gemm_common.h:30-37) over all ranks; ``e2e`` is the same metric through
the C ABI with host buffers (pinned host -> device copies of the step's inputs,
the GEMM, device -> host copy of D, every step).

Multi-GPU: one process per GPU (torchrun).  Strong scaling (the default): the
workload's global GEMM is cut into equal slabs, one per rank, with no
data-path collective -- M-row slabs (B replicated) for the dense projection,
long-K, tall-skinny and square shapes, N-column slabs of 32-column multiples (A
replicated) for the wide shape -- so each rank runs 1/N of the FLOPs and
``value`` is the global FLOPs over the max over ranks of the timed region.
``--scaling weak`` gives every rank a whole workload-sized slab instead (total
M = N x M); multi-GPU strong runs also report that figure under ``weak``.
torch.distributed carries only the barrier, the max over ranks and the optional
all-gather comparison (``gather``).

``--impl reference`` times the reference's own CPU implementation of the path
(gemm_reference_host + mxfp8_quantize_host from oracle/_ref, or the oracle's
restatement when the reference was not built) on the host cores, on a bounded
row sample of the same workload, extrapolated linearly in M (rows are
independent).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "MXFP8×BF16 GEMM TFLOPS/GPU & % of BF16 TC peak at 1/2/4/8 B200"
WORKLOADS = {
    # name: (M, N, K, seed, how the GEMM is cut across GPUs)
    "dense_projection": (4096, 12288, 4096, 43, "m"),
    "long_k": (4096, 4096, 11008, 44, "m"),
    "tall_skinny": (131072, 2048, 2048, 45, "m"),
    "wide": (2048, 28672, 8192, 46, "n"),
    "square": (16384, 16384, 16384, 46, "m"),
}
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    e = d.get(kernel, {}).get(workload)
    return None if e is None else e.get("bytes_per_launch")


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------
def gpu_pci_id(cuda_index: int) -> str:
    """PCI bus id of a CUDA device, which names the same GPU for nvidia-smi and NVML
    whatever CUDA_VISIBLE_DEVICES or the CUDA device order is."""
    import torch

    pr = torch.cuda.get_device_properties(cuda_index)
    return f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"


class NvmlSampler:
    """SM clock, clock-event reasons and power read through NVML every 10 ms on a
    thread: finer than nvidia-smi's loop, so a short timed region still gets a
    record.  Reading only; nothing is set."""
    BITS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
            "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
            "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
            "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, pci_id: str, period_s: float = 0.01):
        self.pci, self.period = pci_id, period_s
        self.samples = []
        self.stop_flag = threading.Event()
        self.t = None

    def start(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByPciBusId(self.pci)
        except Exception:
            return
        self.nv, self.h = nv, h
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        nv, h = self.nv, self.h
        while not self.stop_flag.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h),
                                     nv.nvmlDeviceGetPowerUsage(h) / 1000.0, time.monotonic()))
            except Exception:
                return
            time.sleep(self.period)

    def energy_mj(self):
        """The GPU's cumulative energy counter in millijoules (None if unreadable)."""
        try:
            return self.nv.nvmlDeviceGetTotalEnergyConsumption(self.h)
        except Exception:
            return None

    def stop(self, window=None):
        """Statistics over the samples taken inside window = (t0, t1) (monotonic
        seconds), or over all samples if none fall inside it."""
        if self.t is None:
            return None
        self.stop_flag.set()
        self.t.join(timeout=2)
        if not self.samples:
            return None
        inside = [x for x in self.samples if window and window[0] <= x[3] <= window[1]]
        sel = inside or self.samples
        sm = [x[0] for x in sel]
        reasons = sorted(n for n, a in self.BITS.items() if any(x[1] & getattr(self.nv, a) for x in sel))
        return {"samples": len(sm), "in_timed_region": bool(inside), "sm_mhz_median": statistics.median(sm),
                "sm_mhz_min": min(sm), "reasons": reasons,
                "power_w_max": round(max(x[2] for x in sel), 1)}


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str, period_ms: int = 50):
        self.gpu = gpu_id
        self.period = period_ms
        self.proc = None
        self.lines = []
        self.nvml = NvmlSampler(gpu_id)
        self.window = [None, None]

    def begin(self):
        """Marks the start of the timed region (host time, just before its launches)."""
        self.window[0] = time.monotonic()
        self.energy = [self.nvml.energy_mj() if self.nvml.t is not None else None, None]

    def end(self):
        """Marks its end (host time, after the device synchronised)."""
        self.window[1] = time.monotonic()
        self.energy[1] = self.nvml.energy_mj() if self.nvml.t is not None else None

    def joules(self):
        """GPU energy over the timed region from NVML's counter, or None."""
        e = getattr(self, "energy", [None, None])
        return None if None in e else (e[1] - e[0]) / 1000.0

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", f"-lms={self.period}"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        self.nvml.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def stop(self):
        win = tuple(self.window) if None not in self.window else None
        nvml = self.nvml.stop(win)
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0, "nvml": nvml}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # nvidia-smi lines that arrived inside the timed region (plus one period of
        # slack), or all of them when the region was shorter than the loop period
        lines = [ln for t, ln in self.lines if win and win[0] <= t <= win[1] + self.period / 1000.0]
        in_region = bool(lines)
        lines = lines or [ln for _, ln in self.lines]
        for ln in lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if nvml:
            reasons |= set(nvml["reasons"])
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "in_timed_region": in_region,
                "nvml": nvml}


# ----------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def barrier_sync(dist):
    import torch

    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(dist, value: float) -> float:
    import torch

    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------
# CPU baseline: the reference's own host implementation on a bounded row sample
# ----------------------------------------------------------------------------
class CpuBaseline:
    """gemm_reference_host + mxfp8_quantize_host (the reference's CPU path for
    D = MXFP8(A*B + C)) timed on row samples, one row slab per host thread.  B is
    drawn once; each sample draws fresh A and C rows.  Rows are independent, so the
    throughput extrapolates linearly in M."""

    def __init__(self, M, N, K, seed, threads: int | None = None):
        import numpy as np

        import oracle as O

        self.O, self.np = O, np
        self.M, self.N, self.K = M, N, K
        self.threads = threads or O.default_threads()
        self.kind = "reference" if O.ref_available() else "port"
        rng = np.random.default_rng(seed)
        B = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        self.B = O.bf16_bits_to_float(O.to_bf16_bits(B))
        self.rows = 1

    def run_rows(self, nrows_per_thread: int, seed: int) -> float:
        np, O, N, K, B = self.np, self.O, self.N, self.K, self.B
        threads = self.threads
        rng = np.random.default_rng(seed)
        f32 = ctypes.POINTER(ctypes.c_float)
        u8 = ctypes.POINTER(ctypes.c_uint8)
        A = (rng.standard_normal((threads * nrows_per_thread, K)) * 0.02).astype(np.float32)
        C = (rng.standard_normal((threads * nrows_per_thread, N)) * 0.02).astype(np.float32)
        A = O.dequantize(*O.quantize(A))
        C = O.dequantize(*O.quantize(C))
        D = np.empty((A.shape[0], N), np.float32)
        Dd = np.empty((A.shape[0], N), np.uint8)
        Ds = np.empty((A.shape[0], (N + 31) // 32), np.uint8)
        kind = self.kind

        def work(t):
            r0, r1 = t * nrows_per_thread, (t + 1) * nrows_per_thread
            a, c, d = A[r0:r1], C[r0:r1], D[r0:r1]
            if kind == "reference":
                R = O.ref()
                R.ref_gemm_reference_host(a.ctypes.data_as(f32), B.ctypes.data_as(f32),
                                          c.ctypes.data_as(f32), d.ctypes.data_as(f32),
                                          r1 - r0, N, K)
                R.ref_mxfp8_quantize_host(d.ctypes.data_as(f32), Dd[r0:r1].ctypes.data_as(u8),
                                          Ds[r0:r1].ctypes.data_as(u8), r1 - r0, N)
            else:
                d[...] = O.gemm_gold(a, B, c, threads=1)
                Dd[r0:r1], Ds[r0:r1] = O.quantize(d, threads=1)

        ths = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
        t0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return time.perf_counter() - t0

    def calibrate(self, budget_s: float, seed: int) -> None:
        """Rows per thread so that one sample takes about budget_s."""
        t1 = self.run_rows(1, seed)
        self.rows = max(1, min(64, int(budget_s / max(t1, 1e-3))))

    def sample(self, seed: int):
        """One timed sample; returns (TFLOP/s extrapolated to M, description)."""
        t = self.run_rows(self.rows, seed)
        tflops = 2.0 * self.threads * self.rows * self.N * self.K / t / 1e12
        desc = {"value": tflops, "unit": "TFLOPS", "cores": self.threads, "kind": self.kind,
                "sample": f"{self.threads * self.rows} rows x N={self.N} x K={self.K} "
                          f"({self.threads} threads x {self.rows} rows, {t:.2f} s), extrapolated "
                          f"linearly in M to M={self.M}; gemm_reference_host + mxfp8_quantize_host"}
        return tflops, desc


def cpu_baseline(M, N, K, seed, budget_s: float, threads: int | None = None):
    """One calibrated sample of the reference's CPU path (see CpuBaseline)."""
    cb = CpuBaseline(M, N, K, seed, threads)
    cb.calibrate(budget_s, seed + 1)
    return cb.sample(seed + 2)


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def make_inputs(mpk, M, N, K, seed, rank):
    """N(0, 0.02^2) sources drawn on the device, A and C quantized by the
    library's codec along K and N, B cast to BF16 with RNE."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed * 1000 + rank)
    A = torch.randn((M, K), generator=g, device="cuda") * 0.02
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    C = torch.randn((M, N), generator=g, device="cuda") * 0.02
    Ad, As = mpk.quantize(A)
    Cd, Cs = mpk.quantize(C)
    del A, C
    D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    Ds = torch.empty((M, (N + 31) // 32), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    return Ad, As, B, Cd, Cs, D, Ds


def layout(args, world, rank):
    """This rank's slab of the workload: (rows, cols, K, M_total, N_total, shards,
    mode, description).  Strong scaling cuts the workload's global GEMM; weak
    scaling gives every rank a whole workload-sized M slab."""
    from mix_precision_kernel_b200 import sharding as S

    M, N, K, _, mode = WORKLOADS[args.workload]
    if args.scaling == "weak" or world == 1:
        shards = [S.Shard(r, r * M, (r + 1) * M, 0, N) for r in range(world)]
        desc = (f"M-slab x{world}, {M} rows per GPU (global M = {M * world}), no collective" if world > 1
                else "one GPU")
        return M, N, K, M * world, N, shards, "m", desc
    shards = S.plan(M, N, world, mode)
    sh = shards[rank]
    if mode == "m":
        desc = f"M-row slabs x{world}: {shards[0].rows} rows per GPU, B replicated, no collective"
    else:
        desc = (f"N-column slabs x{world}: {shards[0].cols} columns per GPU (multiples of 32), A replicated, "
                f"no collective")
    return sh.rows, sh.cols, K, M, N, shards, mode, desc


def workload_config(args, world):
    """The `config` object both arms print."""
    M, N, K, seed, _ = WORKLOADS[args.workload]
    rows, cols, _, M_total, N_total, _, _, desc = layout(args, world, 0)
    return {"workload": f"{args.workload} GEMM D=A*B+C", "M_total": M_total, "N": N_total, "K": K,
            "M_per_gpu": rows, "N_per_gpu": cols, "scaling": args.scaling if world > 1 else "single GPU",
            "A": "MXFP8 e4m3+e8m0/32 along K", "B": "bf16 [K][N]", "C": "MXFP8 along N", "D": "MXFP8 along N",
            "seed": seed, "parallelism": desc,
            "l2": f"inputs+outputs per GPU "
                  f"{((rows * K * 33) // 32 + 2 * K * cols + 2 * (rows * cols * 33) // 32) / 2**20:.0f} MiB; "
                  f"no flush between steps"}


def timed_steps(step, steps, stream, dist):
    """CUDA-event time of `steps` calls between barriers (ms, this rank)."""
    import torch

    barrier_sync(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    barrier_sync(dist)
    return e0.elapsed_time(e1)


def run_gemm_arm(args, world, rank, local, dist):
    import torch

    import mix_precision_kernel_b200 as mpk

    _, _, _, seed, _ = WORKLOADS[args.workload]
    M, N, K, M_total, N_total, shards, mode, desc = layout(args, world, rank)
    Ad, As, B, Cd, Cs, D, Ds = make_inputs(mpk, M, N, K, seed, rank)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    L = mpk.lib()
    a = [Ad.data_ptr(), As.data_ptr(), B.data_ptr(), Cd.data_ptr(), Cs.data_ptr(), D.data_ptr(),
         Ds.data_ptr()]

    def step():
        rc = L.mpk_gemm_mxfp8_bf16(*a, M, N, K, sptr)
        if rc:
            raise mpk.MpkError(rc, L.mpk_last_error_string().decode())

    for _ in range(args.warmup):
        step()
    barrier_sync(dist)
    sampler = ClockSampler(gpu_pci_id(local))
    sampler.start()
    time.sleep(0.3)  # let the sampler start before the timed region
    barrier_sync(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.begin()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier_sync(dist)
    sampler.end()
    joules = sampler.joules()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    assert mpk.device_status() == 0, "device wait expired"
    ms_max = max_over_ranks(dist, ms)
    flops = 2.0 * M * N * K              # this rank's slab
    flops_job = 2.0 * M_total * N_total * K
    ms_per_step = ms_max / args.steps
    value = flops_job * args.steps / (ms_max / 1e3) / 1e12
    tiles, sk_tiles, sk_pairs = mpk.gemm_plan(M, N, K)

    # Sustained: the same call back to back for at least a second, with its own
    # clock record (10 ms NVML samples), so the burst figure above can be set
    # against the clock the power cap allows.
    sus_steps = max(args.steps, int(1.05e3 / max(ms / args.steps, 1e-3)) + 1)
    sus_sampler = ClockSampler(gpu_pci_id(local))
    sus_sampler.start()
    time.sleep(0.2)
    barrier_sync(dist)
    sus_sampler.begin()
    sus_ms = timed_steps(step, sus_steps, stream, dist)
    sus_sampler.end()
    sus_clocks = sus_sampler.stop()
    sus_ms_max = max_over_ranks(dist, sus_ms)

    # On the pre-pass path a step is two launches on `stream`: the A pre-pass
    # (MXFP8 -> BF16 into the pooled workspace) and the tensor-core kernel.  The
    # pre-pass is timed alone over as many launches; the tensor-core kernel's time is
    # the difference.  On the on-chip path (tall products with few columns) a step is
    # the one kernel that converts A itself.
    onchip = mpk.gemm_path(Ad, B, M, N, K) == mpk.PATH_ONCHIP
    ws = torch.empty((M, K), dtype=torch.bfloat16, device="cuda")
    pre_args = (Ad.data_ptr(), As.data_ptr(), ws.data_ptr(), M, K, sptr)
    for _ in range(3):
        L.mpk_mxfp8_dequantize_bf16(*pre_args)
    pre_ms = timed_steps(lambda: L.mpk_mxfp8_dequantize_bf16(*pre_args), args.steps, stream, dist) / args.steps
    # Library bar: cuBLAS BF16 x BF16 -> BF16 (torch.matmul) on the same, already
    # dequantized A and B -- a plain GEMM without the C term or the MXFP8 epilogue.
    lib_steps = min(args.steps, 100)
    out16 = torch.matmul(ws, B)
    for _ in range(3):
        torch.matmul(ws, B, out=out16)
    lib_ms = timed_steps(lambda: torch.matmul(ws, B, out=out16), lib_steps, stream, dist) / lib_steps
    del ws, out16
    gemm_ms = ms / args.steps - (0.0 if onchip else pre_ms)
    kernel_tflops = flops / (gemm_ms / 1e3) / 1e12
    step_tflops = flops / (ms / args.steps / 1e3) / 1e12

    # End to end through the C ABI with host buffers.  Every step uploads all of its
    # inputs (this rank's A, A scales, B, C, C scales) from pinned host memory and
    # downloads its D and D scales.  Two device buffer sets and three streams
    # (upload, GEMM, download) let step i+1's upload and step i-1's download run
    # beside step i's kernels, as a serving loop would pipeline them.
    hA = torch.empty_like(Ad, device="cpu").pin_memory(); hA.copy_(Ad)
    hAs = torch.empty_like(As, device="cpu").pin_memory(); hAs.copy_(As)
    hB = torch.empty_like(B, device="cpu").pin_memory(); hB.copy_(B)
    hC = torch.empty_like(Cd, device="cpu").pin_memory(); hC.copy_(Cd)
    hCs = torch.empty_like(Cs, device="cpu").pin_memory(); hCs.copy_(Cs)
    hD = [torch.empty_like(D, device="cpu").pin_memory() for _ in range(2)]
    hDs = [torch.empty_like(Ds, device="cpu").pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in (hA, hAs, hB, hC, hCs))
    d2h = hD[0].numel() + hDs[0].numel()
    bufs = [(Ad, As, B, Cd, Cs, D, Ds),
            tuple(torch.empty_like(t) for t in (Ad, As, B, Cd, Cs, D, Ds))]
    s_up, s_down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]    # set k's inputs uploaded
    ev_used = [torch.cuda.Event() for _ in range(2)]  # set k's GEMM done (inputs free, D ready)
    ev_out = [torch.cuda.Event() for _ in range(2)]   # set k's D downloaded (D free)
    for k in range(2):
        ev_used[k].record(stream)
        ev_out[k].record(stream)

    def e2e_step(i):
        k = i % 2
        a_d, a_s, b_, c_d, c_s, d_d, d_s = bufs[k]
        s_up.wait_event(ev_used[k])
        with torch.cuda.stream(s_up):
            for dst, src in ((a_d, hA), (a_s, hAs), (b_, hB), (c_d, hC), (c_s, hCs)):
                dst.copy_(src, non_blocking=True)
        ev_in[k].record(s_up)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_out[k])
        rc = L.mpk_gemm_mxfp8_bf16(a_d.data_ptr(), a_s.data_ptr(), b_.data_ptr(), c_d.data_ptr(),
                                   c_s.data_ptr(), d_d.data_ptr(), d_s.data_ptr(), M, N, K, sptr)
        if rc:
            raise mpk.MpkError(rc, L.mpk_last_error_string().decode())
        ev_used[k].record(stream)
        s_down.wait_event(ev_used[k])
        with torch.cuda.stream(s_down):
            hD[k].copy_(d_d, non_blocking=True)
            hDs[k].copy_(d_s, non_blocking=True)
        ev_out[k].record(s_down)

    e2e_steps = max(3, min(args.steps, 20))
    for i in range(2):
        e2e_step(i)
    barrier_sync(dist)
    e0.record(stream)
    s_up.wait_event(e0)
    for i in range(2, 2 + e2e_steps):
        e2e_step(i)
    for k in range(2):
        stream.wait_event(ev_out[k])
    e1.record(stream)
    barrier_sync(dist)
    e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1))
    e2e_value = flops_job * e2e_steps / (e2e_ms / 1e3) / 1e12
    same = bool(torch.equal(hD[0], hD[1])) and bool(torch.equal(hDs[0].to(D.device), Ds))
    del bufs

    gather = gather_measurement(args, world, rank, dist, mpk, L, M, N, K, M_total, N_total, shards, mode, Ad, As,
                                B, Cd, Cs, D, Ds, stream) if world > 1 and not args.no_gather else None
    weak = weak_measurement(args, world, rank, dist, mpk, L, stream) \
        if world > 1 and args.scaling == "strong" else None

    # Denominator: the burst cuBLAS figure, unless the clock record shows the power
    # cap acting during the timed region -- the sw_power_cap reason set and the
    # median SM clock below 95 % of its maximum -- in which case the sustained figure
    # (the same GEMM measured back to back under the cap).  Both fractions are
    # reported.
    peaks, peak_src = load_peaks()
    burst = float(peaks["bf16_tflops"])
    sustained = float(peaks.get("bf16_tflops_sustained", burst))
    med_mhz = (clocks.get("nvml") or {}).get("sm_mhz_median") or clocks.get("sm_mhz")
    max_mhz = clocks.get("sm_max_mhz")
    capped = "sw_power_cap" in clocks["reasons"] and (
        med_mhz is None or not max_mhz or med_mhz < 0.95 * max_mhz)
    peak = sustained if capped else burst
    hbm = float(peaks["hbm_gbs"])
    pre_bytes = M * K + M * ((K + 31) // 32) + 2 * M * K
    kernel_name = "gemm_mxfp8_bf16_kernel" if onchip else "gemm_bf16a_mxfp8_kernel"
    roofline = {"bound": "tensor", "kernel": kernel_name,
                "path": "on-chip conversion (one launch)" if onchip else "pre-pass + BF16-A kernel (two launches)",
                "achieved": round(kernel_tflops, 2), "peak": peak,
                "unit": "TFLOP/s", "frac": round(kernel_tflops / peak, 4),
                "traffic": load_traffic(kernel_name, args.workload) if world == 1 else None,
                "peak_source": (f"{peak_src} bf16_tflops_sustained (sw_power_cap active in the timed "
                                f"region, SM clock median {med_mhz} of {max_mhz} MHz)" if capped
                                else f"{peak_src} bf16_tflops (burst; SM clock median {med_mhz} of "
                                     f"{max_mhz} MHz in the timed region)"),
                "frac_of_burst": round(kernel_tflops / burst, 4),
                "frac_of_sustained": round(kernel_tflops / sustained, 4),
                "algorithmic": f"2*M*N*K = {flops:.4e} FLOP per launch (this GPU's slab {M}x{N}x{K})",
                "kernel_ms": round(gemm_ms, 5),
                "timing": ("step time (CUDA events over the timed region): the step is this one kernel"
                           if onchip else "step time (CUDA events over the timed region) minus the A pre-pass "
                                          "timed alone over the same number of launches"),
                "schedule": {"tiles": tiles, "stream_k_tiles": sk_tiles, "stream_k_pairs": sk_pairs},
                "step_achieved": round(step_tflops, 2), "step_frac": round(step_tflops / peak, 4),
                "prepass": {"kernel": "mxfp8_dequantize_bf16_flat_kernel", "ms": round(pre_ms, 5),
                            "bytes": pre_bytes, "achieved_gbs": round(pre_bytes / pre_ms / 1e6, 1),
                            "frac_of_hbm": round(pre_bytes / pre_ms / 1e6 / hbm, 4),
                            "in_step": not onchip}}
    nv = clocks.get("nvml") or {}
    snv = sus_clocks.get("nvml") or {}
    sus_tflops = flops_job * sus_steps / (sus_ms_max / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (N(0,0.02^2) drawn on device, torch Philox seeded; A/C quantized to "
                "MXFP8 by the library, B rounded to BF16)",
        "config": workload_config(args, world),
        "tflops_per_gpu": round(value / world, 2),
        "gpu_launches": (1 if onchip else 2) * args.steps,
        "pct_of_bf16_peak": round(100.0 * value / world / burst, 2),
        "e2e": {"value": round(e2e_value, 3), "unit": "TFLOPS",
                "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                "h2d_bytes_per_step_per_gpu": h2d, "d2h_bytes_per_step_per_gpu": d2h,
                "steps": e2e_steps, "ms_per_step": round(e2e_ms / e2e_steps, 4),
                "pipelining": "two buffer sets; upload, GEMM and download streams overlap across steps",
                "downloads_match_device_result": same},
        "roofline": roofline,
        "library_bar": {"what": "cuBLAS BF16xBF16->BF16 GEMM (torch.matmul) on the pre-dequantized A; "
                                "no C term, no MXFP8 epilogue",
                        "tflops": round(flops / (lib_ms / 1e3) / 1e12, 2), "ms": round(lib_ms, 5),
                        "gemm_kernel_over_library": round(lib_ms / gemm_ms, 4),
                        "step_over_library": round(lib_ms / (ms / args.steps), 4)},
        "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        "sustained": {"what": "the same call back to back for >= 1 s with a 10 ms NVML clock record",
                      "steps": sus_steps, "ms_per_step": round(sus_ms_max / sus_steps, 5),
                      "value": round(sus_tflops, 2),
                      "frac_of_sustained_peak": round(sus_tflops / world / sustained, 4),
                      "frac_of_burst_peak": round(sus_tflops / world / burst, 4),
                      "sm_mhz_median": snv.get("sm_mhz_median"), "samples": snv.get("samples"),
                      "in_timed_region": snv.get("in_timed_region"), "reasons": sus_clocks["reasons"],
                      "ms_x_ghz": (round(sus_ms_max / sus_steps * snv["sm_mhz_median"] / 1e3, 5)
                                   if snv.get("sm_mhz_median") else None)},
        "burst_ms_x_ghz": (round(ms_per_step * nv["sm_mhz_median"] / 1e3, 5)
                           if nv.get("sm_mhz_median") else None),
    }
    line["clocks"]["samples"] = clocks["samples"]
    line["clocks"]["in_timed_region"] = clocks.get("in_timed_region")
    # The counter moves in steps of tens of milliseconds: shorter regions gave
    # average powers above the board limit, so energy is reported from 1 s up.
    if joules and ms >= 1000.0:
        line["energy"] = {"joules_per_step": round(joules / args.steps, 4),
                          "avg_power_w": round(joules / (ms / 1e3), 1),
                          "tflop_per_joule": round(flops / 1e12 / (joules / args.steps), 3),
                          "source": "NVML total energy counter read at the timed region's ends (this "
                                    "GPU); reported for timed regions of 1 s or more"}
    line["clocks"]["nvml_10ms"] = clocks.get("nvml")
    if gather is not None:
        line["gather"] = gather
    if weak is not None:
        line["weak"] = weak
    if world == 1 and rank == 0 and not args.no_reference_gpu:
        line["reference_gpu_bar"] = reference_gpu_bar(Ad, As, B, Cd, Cs, M, N, K, ms / args.steps)
    return line


def weak_measurement(args, world, rank, dist, mpk, L, stream):
    """Weak scaling beside a strong run: every rank runs a whole workload-sized
    GEMM of its own (an independent M slab); whole-job TFLOP/s, max over ranks."""
    import torch

    M, N, K, seed, _ = WORKLOADS[args.workload]
    Ad, As, B, Cd, Cs, D, Ds = make_inputs(mpk, M, N, K, seed + 7, rank)
    a = [Ad.data_ptr(), As.data_ptr(), B.data_ptr(), Cd.data_ptr(), Cs.data_ptr(), D.data_ptr(), Ds.data_ptr()]
    sptr = stream.cuda_stream

    def step():
        rc = L.mpk_gemm_mxfp8_bf16(*a, M, N, K, sptr)
        if rc:
            raise mpk.MpkError(rc, L.mpk_last_error_string().decode())

    steps = max(5, min(args.steps, 50))
    for _ in range(3):
        step()
    ms = max_over_ranks(dist, timed_steps(step, steps, stream, dist))
    del Ad, As, B, Cd, Cs, D, Ds
    torch.cuda.empty_cache()
    value = world * 2.0 * M * N * K * steps / (ms / 1e3) / 1e12
    return {"what": f"weak scaling: {M}x{N}x{K} on every GPU (global M = {M * world})",
            "value": round(value, 2), "tflops_per_gpu": round(value / world, 2),
            "ms_per_step": round(ms / steps, 5), "steps": steps}


def reference_gpu_bar(Ad, As, B, Cd, Cs, M, N, K, our_step_ms):
    """The reference's own GPU launcher (gemm_fp8_tensorcore: WMMA fp16 into an FP32
    temporary, then its quantize kernel; src/kernels/gemm_fp8_tensorcore.cu:231-249),
    rebuilt for sm_100a in oracle/_ref, on the same device inputs: a baseline
    measurement beside ours, like the CPU baseline."""
    import torch

    import oracle as O

    if not O.ref_available():
        return {"unavailable": "oracle/_ref (the reference compiled here) is not built"}
    R = O.ref()
    D7 = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    S7 = torch.empty((M, (N + 31) // 32), dtype=torch.uint8, device="cuda")
    args = (Ad.data_ptr(), As.data_ptr(), B.data_ptr(), Cd.data_ptr(), Cs.data_ptr(), D7.data_ptr(),
            S7.data_ptr(), M, N, K, None)
    assert R.ref_gemm_fp8_tensorcore(*args) == 0
    torch.cuda.synchronize()
    n = 3
    t0 = time.perf_counter()
    for _ in range(n):
        assert R.ref_gemm_fp8_tensorcore(*args) == 0
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) / n * 1e3
    tflops = 2.0 * M * N * K / (ms / 1e3) / 1e12
    del D7, S7
    return {"what": "the reference's gemm_fp8_tensorcore (WMMA fp16 + FP32 temporary + quantize kernel, "
                    "per-call cudaMalloc/cudaFree) rebuilt for sm_100a, same inputs, same GPU",
            "ms": round(ms, 4), "tflops": round(tflops, 3), "calls": n,
            "timing": "host wall clock around synchronous calls (the launcher synchronizes on its "
                      "cudaMalloc/cudaFree)",
            "our_step_over_reference": round(ms / our_step_ms, 2)}


def gather_measurement(args, world, rank, dist, mpk, L, M, N, K, M_total, N_total, shards, mode, Ad, As, B, Cd,
                       Cs, D, Ds, stream):
    """GEMM + all-gather of D onto every GPU, two ways, over this run's slabs: the
    fused kernel (each D tile stored into every GPU's full-D buffer by the epilogue,
    then a cross-GPU barrier) and the GEMM followed by NCCL all-gathers of D and
    its scales.  Both run whole tiles (the fused kernel has no stream-K schedule),
    so their results must be identical.  Times are max over ranks."""
    import torch

    from mix_precision_kernel_b200 import sharding as S

    prev = mpk.set_gemm_schedule(mpk.SCHEDULE_TILES)
    try:
        gg = S.GatherGemm(M_total, N_total, K, shards, None)
        steps = max(5, min(args.steps, 50))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gathered = {}

        def fused():
            gg(Ad, As, B, Cd, Cs)

        def separate():
            rc = L.mpk_gemm_mxfp8_bf16(Ad.data_ptr(), As.data_ptr(), B.data_ptr(), Cd.data_ptr(), Cs.data_ptr(),
                                       D.data_ptr(), Ds.data_ptr(), M, N, K, stream.cuda_stream)
            if rc:
                raise mpk.MpkError(rc, L.mpk_last_error_string().decode())
            gathered["d"], gathered["s"] = S.gather_d(D, Ds, shards, mode)

        out = {}
        for name, fn in (("separate", separate), ("fused", fused)):
            for _ in range(3):
                fn()
            barrier_sync(dist)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            barrier_sync(dist)
            out[name] = max_over_ranks(dist, e0.elapsed_time(e1) / steps)
        same = bool(torch.equal(gg.D, gathered["d"])) and bool(torch.equal(gg.Ds, gathered["s"]))
        ok = torch.tensor([1 if same else 0], device="cuda")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        gg.close()
    finally:
        mpk.set_gemm_schedule(prev)
    d_bytes = M * N + M * ((N + 31) // 32)
    return {"what": f"D = A*B + C on {'M-row' if mode == 'm' else 'N-column'} slabs, then D and its scales "
                    f"on every GPU",
            "fused_ms": round(out["fused"], 5), "separate_ms": round(out["separate"], 5),
            "speedup": round(out["separate"] / out["fused"], 3),
            "separate": "mpk GEMM + NCCL all-gather of D and scales (all_gather_into_tensor for equal row "
                        "slabs, all_gather + reassembly for column slabs)",
            "fused": "GEMM epilogue stores every tile into all GPUs' full-D buffers (peer stores), "
                     "cross-GPU barrier before and after",
            "bytes_sent_per_gpu": d_bytes * (world - 1),
            "nvlink_gbs_per_gpu_fused": round(d_bytes * (world - 1) / out["fused"] / 1e6, 1),
            "results_identical": bool(ok.item()), "steps": steps}


def run_codec_arm(args, world, rank, local, dist):
    """Standalone MXFP8 quantize + dequantize of a 131072 x 2048 FP32 tensor
    (HBM bandwidth kernels); value is GB/s of algorithmic traffic."""
    import torch

    import mix_precision_kernel_b200 as mpk

    M, K = 131072, 2048
    g = torch.Generator(device="cuda").manual_seed(45 + rank)
    x = torch.randn((M, K), generator=g, device="cuda") * 0.02
    d = torch.empty((M, K), dtype=torch.uint8, device="cuda")
    s = torch.empty((M, K // 32), dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    L = mpk.lib()
    sptr = torch.cuda.current_stream().cuda_stream
    stream = torch.cuda.current_stream()
    bytes_one = M * K * 4 + M * K + M * K // 32

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        barrier_sync(dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        barrier_sync(dist)
        return e0.elapsed_time(e1) / args.steps

    q_ms = timed(lambda: L.mpk_mxfp8_quantize(x.data_ptr(), d.data_ptr(), s.data_ptr(), M, K, sptr))
    dq_ms = timed(lambda: L.mpk_mxfp8_dequantize(d.data_ptr(), s.data_ptr(), y.data_ptr(), M, K, sptr))
    # Companion kernels, reported beside the headline pair: BF16 -> MXFP8 and MXFP8 -> BF16.
    x16 = x.to(torch.bfloat16)
    del y
    qb_ms = timed(lambda: L.mpk_mxfp8_quantize_bf16(x16.data_ptr(), d.data_ptr(), s.data_ptr(), M, K, sptr))
    db_ms = timed(lambda: L.mpk_mxfp8_dequantize_bf16(d.data_ptr(), s.data_ptr(), x16.data_ptr(), M, K, sptr))
    bytes16 = M * K * 2 + M * K + M * K // 32
    # Quantize with the blocks along the rows (32 rows per column): same traffic.
    sc = torch.empty(((M + 31) // 32, K), dtype=torch.uint8, device="cuda")
    qc_ms = timed(lambda: L.mpk_mxfp8_quantize_cols(x.data_ptr(), d.data_ptr(), sc.data_ptr(), M, K, sptr))
    qcb_ms = timed(lambda: L.mpk_mxfp8_quantize_bf16_cols(x16.data_ptr(), d.data_ptr(), sc.data_ptr(), M, K, sptr))
    del sc
    peaks, src = load_peaks()
    hbm = float(peaks["hbm_gbs"])
    qg, dg = bytes_one / q_ms / 1e6, bytes_one / dq_ms / 1e6
    q_ms_max, dq_ms_max = max_over_ranks(dist, q_ms), max_over_ranks(dist, dq_ms)
    value = world * bytes_one * 2 / ((q_ms_max + dq_ms_max) / 1e3) / 1e9

    # End to end: every step uploads the FP32 tensor from pinned host memory,
    # quantizes and dequantizes it through the C ABI, and downloads the result.
    del x16
    hx = torch.empty((M, K), dtype=torch.float32).pin_memory()
    hx.copy_(x)
    y = torch.empty_like(x)
    hy = torch.empty_like(hx).pin_memory()

    def e2e_step():
        x.copy_(hx, non_blocking=True)
        L.mpk_mxfp8_quantize(x.data_ptr(), d.data_ptr(), s.data_ptr(), M, K, sptr)
        L.mpk_mxfp8_dequantize(d.data_ptr(), s.data_ptr(), y.data_ptr(), M, K, sptr)
        hy.copy_(y, non_blocking=True)

    e2e_steps = 3
    e2e_step()
    barrier_sync(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier_sync(dist)
    e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1) / e2e_steps)
    e2e_value = world * bytes_one * 2 / (e2e_ms / 1e3) / 1e9
    return {
        "metric": "MXFP8 quantize+dequantize HBM GB/s (131072x2048 FP32)", "value": round(value, 1),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(q_ms_max + dq_ms_max, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32/u8", "data": "synthetic N(0,0.02^2)",
        "config": {"workload": "codec quantize+dequantize", "M": M, "K": K,
                   "l2": "1 GiB FP32 tensor > L2"},
        "gpu_launches": 2 * args.steps,
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": M * K * 4,
                "d2h_bytes_per_step": M * K * 4, "steps": e2e_steps,
                "what": "pinned FP32 upload, quantize, dequantize, pinned FP32 download, every step"},
        "bf16_companions": {"quantize_bf16_gbs": round(bytes16 / qb_ms / 1e6, 1),
                            "quantize_bf16_frac": round(bytes16 / qb_ms / 1e6 / hbm, 4),
                            "dequantize_bf16_gbs": round(bytes16 / db_ms / 1e6, 1),
                            "dequantize_bf16_frac": round(bytes16 / db_ms / 1e6 / hbm, 4),
                            "bytes_per_launch": bytes16},
        "row_blocks": {"what": "quantize with blocks of 32 rows per column (mpk_mxfp8_quantize_cols, _bf16_cols)",
                       "quantize_cols_gbs": round(bytes_one / qc_ms / 1e6, 1),
                       "quantize_cols_frac": round(bytes_one / qc_ms / 1e6 / hbm, 4),
                       "quantize_bf16_cols_gbs": round(bytes16 / qcb_ms / 1e6, 1),
                       "quantize_bf16_cols_frac": round(bytes16 / qcb_ms / 1e6 / hbm, 4)},
        "roofline": {"bound": "hbm", "achieved": round(qg, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(qg / hbm, 4), "traffic": load_traffic("mxfp8_quantize_flat_kernel", "codec"),
                     "peak_source": f"{src} hbm_gbs", "dequantize_gbs": round(dg, 1),
                     "dequantize_frac": round(dg / hbm, 4),
                     "algorithmic": f"{bytes_one} B per launch (4 B in + 1 B + 1/32 B out per element)"},
    }


def run_reference_codec_arm(args, world):
    """The reference's host quantize + dequantize (mxfp8_quantize_host,
    mxfp8_dequantize_host) of 131072 x 2048 FP32, timed on row slabs, one per host
    thread, and reported in the codec line's unit (GB/s of algorithmic traffic)."""
    import numpy as np

    import oracle as O

    M, K = 131072, 2048
    threads = O.default_threads()
    kind = "reference" if O.ref_available() else "port"
    rows = int(os.environ.get("MPK_REF_CODEC_ROWS", "128"))
    rng = np.random.default_rng(45)
    f32 = ctypes.POINTER(ctypes.c_float)
    u8 = ctypes.POINTER(ctypes.c_uint8)
    x = (rng.standard_normal((threads * rows, K)) * 0.02).astype(np.float32)
    d = np.empty((threads * rows, K), np.uint8)
    s_ = np.empty((threads * rows, K // 32), np.uint8)
    y = np.empty_like(x)

    def step():
        def work(t):
            r0 = t * rows
            if kind == "reference":
                R = O.ref()
                R.ref_mxfp8_quantize_host(x[r0:r0 + rows].ctypes.data_as(f32), d[r0:r0 + rows].ctypes.data_as(u8),
                                          s_[r0:r0 + rows].ctypes.data_as(u8), rows, K)
                R.ref_mxfp8_dequantize_host(d[r0:r0 + rows].ctypes.data_as(u8), s_[r0:r0 + rows].ctypes.data_as(u8),
                                            y[r0:r0 + rows].ctypes.data_as(f32), rows, K)
            else:
                d[r0:r0 + rows], s_[r0:r0 + rows] = O.quantize(x[r0:r0 + rows], threads=1)
                y[r0:r0 + rows] = O.dequantize(d[r0:r0 + rows], s_[r0:r0 + rows], threads=1)

        ths = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
        t0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return time.perf_counter() - t0

    vals = []
    sample_bytes = 2 * threads * rows * K * (4 + 1 + 1 / 32)
    for i in range(args.warmup + args.steps):
        t = step()
        if i >= args.warmup:
            vals.append(sample_bytes / t / 1e9)
    value = statistics.mean(vals)
    desc = {"value": value, "unit": "GB/s", "cores": threads, "kind": kind, "cpu_model": cpu_model(),
            "sample": f"{threads * rows} rows x K={K} quantized and dequantized ({threads} threads x "
                      f"{rows} rows) per step; mxfp8_quantize_host + mxfp8_dequantize_host"}
    return {
        "metric": "MXFP8 quantize+dequantize HBM GB/s (131072x2048 FP32)", "value": value, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 2 * M * K * (4 + 1 + 1 / 32) / (value * 1e9) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32/u8", "data": "synthetic N(0,0.02^2)",
        "impl": "reference", "config": {"workload": "codec quantize+dequantize", "M": M, "K": K,
                                        "parallelism": "host threads, row slabs"},
        "cpu_baseline": desc,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def run_reference_arm(args, world, rank):
    if rank != 0:
        return None
    if args.workload == "codec":
        return run_reference_codec_arm(args, world)
    M, N, K, seed, _ = WORKLOADS[args.workload]
    # Each step is one timed row sample of the whole workload (rows are independent,
    # so the sample's throughput is the workload's); the per-step budget shrinks with
    # the step count so that the whole run stays within about two minutes of host
    # work.  The metric is a rate, so the sample gives it without extrapolation;
    # the time a whole workload-sized step would take is reported beside it.
    budget = float(os.environ.get("MPK_REF_STEP_BUDGET_S", "2.0"))
    budget = max(0.05, min(budget, 120.0 / (args.steps + args.warmup)))
    cb = CpuBaseline(M, N, K, seed)
    cb.calibrate(budget, seed + 1)
    vals, secs = [], []
    desc = None
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        v, desc = cb.sample(seed + 2 + i)
        if i >= args.warmup:
            vals.append(v)
            secs.append(time.perf_counter() - t0)
    value = statistics.mean(vals)
    desc = dict(desc, value=value)
    desc["cpu_model"] = cpu_model()
    sample_rows = cb.threads * cb.rows
    full_ms = 2.0 * M * N * K / (value * 1e12) * 1e3
    # The whole job at N GPUs is the same global workload (strong scaling) or N of
    # them (weak); the host cores run it once either way.
    return {
        "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(secs) * 1e3, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32", "data": "synthetic N(0,0.02^2)", "impl": "reference",
        "config": workload_config(args, world),
        "step": f"one timed sample of {sample_rows} rows of the {M}x{N}x{K} workload on {cb.threads} host threads",
        "extrapolated": True, "sample_rows": sample_rows, "sample_s": round(statistics.mean(secs), 4),
        "full_step_ms_extrapolated": round(full_ms, 1),
        "cpu_baseline": desc,
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(WORKLOADS) + ["codec"], default="dense_projection")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0,
                    help="seconds of host work for the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true",
                    help="with --gpus > 1: skip timing the fused GEMM + all-gather of D against the GEMM "
                         "followed by NCCL all-gathers (reported as `gather`)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the workload's global GEMM is split over the GPUs (default); weak: every "
                         "GPU runs a whole workload-sized M slab")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU launcher beside ours (reference_gpu_bar)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_env()

    if args.impl == "reference":
        line = run_reference_arm(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    dist = init_dist(world, local)
    try:
        if args.workload == "codec":
            line = run_codec_arm(args, world, rank, local, dist)
        else:
            line = run_gemm_arm(args, world, rank, local, dist)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            if args.workload == "codec":
                sub = argparse.Namespace(steps=3, warmup=1)
                line["cpu_baseline"] = run_reference_codec_arm(sub, 1)["cpu_baseline"]
            else:
                M, N, K, seed, _ = WORKLOADS[args.workload]
                _, desc = cpu_baseline(M, N, K, seed, args.cpu_budget_s)
                desc["cpu_model"] = cpu_model()
                line["cpu_baseline"] = desc
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
