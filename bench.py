"""Benchmark of the trnblas_b200 hot path (one JSON line on rank 0).

Default workload (benchmark case 5, the headline "1/2/4/8 B200" setting):
the 2-D output-block sharded GEMM C = A @ B, M = N = K = 32768, bf16
(`trnblas_b200.parallel.gemm_2d`), one step = the whole GEMM over all ranks;
value = whole-job TFLOP/s. The same line carries the DF-MP2 pair-energy step
of config 5 (nocc 96, nvir 2208, naux 6912, pairs sharded over ranks) in ms.
Other workloads (--workload): gemm_fp32 (config 5a fp32), gemm8192_bf16 /
gemm8192_fp32 (single-GPU 8192^3), gemm1024 (config 1: fp32 1024^3, transA,
beta 0.5), batched / batched_bf16 (config 2a), syrk / syrk_bf16 (config 2b),
gemm_fp64 (config 4), pair3 (config 3), pair5 (config 5b alone), pair5x4
(config 5b per-pair shape at nocc 4, a small case for profiling), dfmp2 (the
whole DF-MP2 energy, `parallel.df_mp2_energy`, at the reference's largest
benchmark shape nbasis/nocc/naux = 768/96/2304).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)

Inputs are seeded synthetic tensors with the benchmark cases' shapes and
distributions, generated on the device. Workloads whose operands are larger
than L2 run back to back; those that fit in L2 (gemm1024, batched_bf16, syrk,
syrk_bf16) overwrite a 256 MB buffer before every timed step, outside that
step's events. Timing: CUDA events on the launching stream, barrier +
synchronize around the K timed steps, max over ranks.

`--impl reference` times the reference's CPU path (its torch/CPU route,
restated in `oracle/`) on the host cores, rank 0 only, on a bounded sample of
the same workload; the other ranks exit without work.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
REASON_BITS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


def peaks():
    if PEAKS_FILE.exists():
        d = json.loads(PEAKS_FILE.read_text())
        return d, "measured"
    return FALLBACK, "fallback"


# ── distributed plumbing ─────────────────────────────────────────────────────


def setup_dist(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch with torchrun --nproc-per-node {n}")
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group(
            "nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
            device_id=torch.device("cuda", local),
        )
    return rank, world, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ── clocks during the timed region ───────────────────────────────────────────


class ClockSampler:
    """nvidia-smi samples of this GPU's SM clock and throttle reasons. The
    sampler is started, and its first sample awaited, before the warm-up steps
    (so its start-up does not fall inside the timed region); the summary keeps
    the samples taken between start() and stop() (all of them when the region
    is shorter than the 200 ms sampling period)."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu),
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,power.draw",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def ready(self, timeout: float = 5.0):
        end = time.monotonic() + timeout
        while self.proc is not None and not self.lines and time.monotonic() < end:
            time.sleep(0.01)

    def start(self):
        self.t0 = time.monotonic()

    def stop(self):
        self.t1 = time.monotonic()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        lines = self.lines
        if self.t0 is not None and self.t1 is not None:
            inside = [x for x in lines if self.t0 <= x[0] <= self.t1 + 0.25]
            lines = inside or lines
        for _, ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 3:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
                bits = int(parts[2], 16)
            except ValueError:
                continue
            for b, name in REASON_BITS.items():
                if bits & b:
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx,
            "reasons": sorted(reasons - {"gpu_idle"}),
            "samples": len(sm),
        }


# ── timing helpers ───────────────────────────────────────────────────────────


def timed_steps(step, steps, warmup, world, gpu):
    with ClockSampler(gpu) as cs:
        cs.ready()
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        cs.start()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            step()
        e.record()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        cs.stop()
    ms = s.elapsed_time(e) / steps
    return max_over_ranks(ms, world), cs.summary()


L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


def timed_steps_flushed(step, steps, warmup, world, gpu):
    """timed_steps for workloads whose operands fit in L2: before every step
    a 256 MB buffer is overwritten (outside the timed events), and each step
    is bracketed by its own CUDA events on the launching stream; the mean
    step time, max over ranks."""
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with ClockSampler(gpu) as cs:
        cs.ready()
        for _ in range(warmup):
            flush.fill_(1)
            step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        cs.start()
        for a, b in ev:
            flush.fill_(1)
            a.record()
            step()
            b.record()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        cs.stop()
    ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    del flush
    return max_over_ranks(ms, world), cs.summary()


# single-GPU workloads whose operands fit in L2 (timed with a flush between steps)
FLUSHED = ("syrk", "syrk_bf16", "batched_bf16", "gemm1024")

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum, one
# ncu capture of the workload's dominant kernel on the same shape; the
# summaries with their commands are under profiles/, named in the comments).
# None where no capture of the timed shape exists.
TRAFFIC = {
    "spmd_bf16_1x1": 70950000000,  # profiles/gemm_bf16_32768.md
    "spmd_fp32_1x1": 281190000000, # profiles/gemm_fp32_32768.md
    "gemm8192_bf16": 1199138448,   # profiles/gemm_bf16_8192.md
    "gemm8192_fp32": 4821362688,   # profiles/gemm_fp32_8192.md
    "batched": 313154560,          # profiles/gemm_batched_64x512.md
    "batched_bf16": 70896640,      # profiles/gemm_batched_bf16.md
    "syrk": 257120256,             # profiles/gemm_syrk_4096.md
    "syrk_bf16": 34854912,         # profiles/gemm_syrk_bf16_4096.md
    "gemm_fp64": 2161969960,       # profiles/ozaki_fp64_4096.md (the int8 GEMM kernel)
    "pair3": 350738688,            # profiles/pair_energy_pair3.md
    "pair5x4": 2716847520,         # profiles/pair_energy_pair5x4.md
    "pair5": 1643160000000,        # profiles/pair_energy_pair5_dram.md
}


def pair_int8_ops(npairs: int, nvir: int, naux: int) -> float:
    """int8 ops (2 per multiply-add) the fused pair-energy kernel issues for
    `npairs` pairs: units (128 rows of a x 64 columns of b, C >= 2R) x 2
    passes x the summed MMA N of one K step (10 base-254 products of 64
    columns) x 128 rows x naux padded to the 64-wide stage (any naux: longer
    ones run as K chunks of the same products)."""
    nR, nC = math.ceil(nvir / 128), math.ceil(nvir / 64)
    upp = sum(max(0, nC - 2 * r) for r in range(nR))
    naux_p = math.ceil(naux / 64) * 64
    return npairs * upp * 2 * 10 * 64 * 128 * naux_p * 2.0


def kernel_avg_ms(events):
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in events) / max(len(events), 1)


# ── metric names (one string per metric, shared by both arms) ───────────────


def gemm_metric(n: int, dtype: torch.dtype) -> str:
    return f"GEMM TFLOP/s (M=N=K={n}, {str(dtype).split('.')[-1]})"


def pair_metric(nocc: int, nvir: int, naux: int) -> str:
    return f"DF-MP2 pair-energy step ms ({nocc}/{nvir}/{naux})"


# The pair-energy block of the default line (config 5b): its own step counts,
# reported in the block (a config-5b step takes seconds on one GPU).
PAIR5_STEPS, PAIR5_WARMUP = 5, 3
# The fp32 GEMM block of the default line (config 5a in fp32, ~0.3 s a step
# on one GPU).
FP32_STEPS, FP32_WARMUP = 5, 3


# ── CPU baseline (the reference's CPU route, restated) ──────────────────────


def cpu_gemm_sample(n: int, dtype: torch.dtype, budget_s: float = 12.0):
    """TFLOP/s of torch CPU matmul (the reference's host route for gemm) on a
    row sample of an n x n x n product, sized to ~budget_s seconds."""
    threads = torch.get_num_threads()
    g = torch.Generator().manual_seed(5)
    B = (2 * torch.rand(n, n, generator=g) - 1).to(dtype)
    rows = 64
    A = (2 * torch.rand(rows, n, generator=g) - 1).to(dtype)
    t0 = time.perf_counter()
    torch.matmul(A, B)
    t1 = time.perf_counter()
    per_row = max((t1 - t0) / rows, 1e-6)
    rows = int(max(64, min(n, budget_s / 2 / per_row)))
    A = (2 * torch.rand(rows, n, generator=g) - 1).to(dtype)
    torch.matmul(A[:64], B)  # warm
    t0 = time.perf_counter()
    torch.matmul(A, B)
    dt = time.perf_counter() - t0
    return 2.0 * rows * n * n / dt / 1e12, threads, f"{rows} x {n} rows of the {n}^3 product, {dtype}"


def cpu_single_sample(wl: str, budget_s: float = 10.0):
    """TFLOP/s of the reference's host route (torch on the CPU, all threads)
    for a single-GPU workload, on a bounded sample: config 2a batched fp32 /
    bf16 (a subset of the 64 batch entries), config 2b syrk fp32 / bf16
    (A @ A^T on a row sample, lower-triangle flops), config 1 (whole 1024^3
    products, repeated), config 4 gemm_fp64 (fp64 matmul on a row sample: the
    reference's CPU gemm_fp64 is host BLAS), 8192^3 bf16/fp32."""
    threads = torch.get_num_threads()
    g = torch.Generator().manual_seed(7)
    ldt = torch.bfloat16 if wl.endswith("bf16") else torch.float32
    lname = str(ldt).split(".")[-1]
    if wl in ("batched", "batched_bf16"):
        A = torch.randn(64, 512, 512, generator=g).to(ldt)
        B = torch.randn(64, 512, 512, generator=g).to(ldt)
        torch.matmul(A[:2], B[:2])
        t0, nb = time.perf_counter(), 0
        while time.perf_counter() - t0 < budget_s / 2 and nb < 64:
            torch.matmul(A[nb:nb + 8], B[nb:nb + 8])
            nb += 8
        dt = time.perf_counter() - t0
        return {"value": round(nb * 2.0 * 512 ** 3 / dt / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
                "kind": "port", "sample": f"{nb} of 64 batch entries, torch CPU bmm {lname} (the reference's host route)"}
    if wl in ("syrk", "syrk_bf16"):
        n = 4096
        A = (torch.randn(n, n, generator=g) / 64).to(ldt)
        rows = 64
        torch.matmul(A[:16], A.T)
        t0 = time.perf_counter()
        torch.matmul(A[:rows], A.T)
        per_row = max((time.perf_counter() - t0) / rows, 1e-7)
        rows = int(max(64, min(n, budget_s / 2 / per_row)))
        t0 = time.perf_counter()
        torch.matmul(A[:rows], A.T)
        dt = time.perf_counter() - t0
        # the reference computes the full square then symmetrises: time per full product
        full_s = dt * n / rows
        return {"value": round(n * (n + 1) * n / full_s / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
                "kind": "port", "sample": f"{rows} of {n} rows of A @ A^T (torch CPU {lname}, the reference's full-square route), lower-triangle flops"}
    if wl == "gemm1024":
        n = 1024
        A = 2 * torch.rand(n, n, generator=g) - 1
        B = 2 * torch.rand(n, n, generator=g) - 1
        C = 2 * torch.rand(n, n, generator=g) - 1
        step = lambda: torch.addmm(C, A.T, B, beta=0.5, alpha=1.0)  # noqa: E731
        step()
        t0, reps = time.perf_counter(), 0
        while time.perf_counter() - t0 < budget_s / 4 and reps < 2000:
            step()
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        return {"value": round(2.0 * n ** 3 / dt / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"{reps} whole config-1 products (fp32 1024^3, transA, beta 0.5), torch CPU addmm (the reference's host route)"}
    dt_, n = (torch.float64, 4096) if wl == "gemm_fp64" else ((torch.bfloat16 if wl.endswith("bf16") else torch.float32), 8192)
    v, th, sample = cpu_gemm_sample(n, dt_, budget_s=budget_s)
    return {"value": round(v, 4), "unit": "TFLOP/s", "cores": th, "kind": "port",
            "sample": sample + (" (host fp64 BLAS: the reference's CPU gemm_fp64 route)" if wl == "gemm_fp64" else " (torch CPU matmul)")}


def cpu_pair_sample(nocc, nvir, naux, budget_s: float = 12.0):
    """Energy-step ms of the reference's chunked CPU energy (oracle restatement,
    fp32 torch on the host), extrapolated from a pair-count sample."""
    from oracle import pair_energy as PE

    threads = torch.get_num_threads()
    g = torch.Generator().manual_seed(6)
    npairs = PE.n_pairs(nocc)
    # sample: rows i (all j) of the reference's aten_rows route, on a subset of B
    B = (0.05 * torch.randn(nocc, nvir, naux, generator=g))
    eo = torch.sort(-20 + 19.7 * torch.rand(nocc, generator=g)).values
    ev = torch.sort(0.1 + 4.9 * torch.rand(nvir, generator=g)).values
    Bf = B.reshape(nocc * nvir, naux)
    t0 = time.perf_counter()
    done = 0
    i = 0
    while time.perf_counter() - t0 < budget_s and i < nocc:
        T = (Bf[i * nvir:(i + 1) * nvir] @ Bf.T).reshape(nvir, nocc, nvir).permute(1, 0, 2)
        den = (eo[i] + eo).reshape(nocc, 1, 1) - ev.reshape(1, nvir, 1) - ev.reshape(1, 1, nvir)
        float((T * (2 * T - T.transpose(-2, -1)) / den).sum())
        done += nocc  # ordered pairs (i, j) for all j
        i += 1
    dt = time.perf_counter() - t0
    full_ms = dt / done * (nocc * nocc) * 1e3
    return full_ms, threads, f"{i} occupied rows ({done} ordered pairs of {nocc * nocc}) of the chunked fp32 energy, extrapolated by pair count"


# ── workloads ────────────────────────────────────────────────────────────────


def run_gemm_spmd(args, rank, world, gpu, dtype, n=32768):
    import trnblas_b200 as tb
    from trnblas_b200 import _native as N
    from trnblas_b200 import parallel as tp

    grid = tp.Grid2D() if world > 1 else _SingleGrid()
    w = world
    mw, nw = n // w, n // w
    g = torch.Generator(device="cuda").manual_seed(5 + 1000 * rank)
    A_sh = (2 * torch.rand(mw, n, device="cuda", generator=g) - 1).to(dtype)
    B_sh = (2 * torch.rand(n, nw, device="cuda", generator=g) - 1).to(dtype)
    k_chunks = 1  # gather, then one GEMM: NCCL kernels running beside the persistent GEMM slow both
    events = []

    def step():
        tp.gemm_2d(A_sh, B_sh, grid, k_chunks=k_chunks, kernel_events=events)

    N.launch_count = 0
    ms, clocks = timed_steps(step, args.steps, args.warmup, world, gpu)
    launches_timed = N.launch_count  # includes warmup; normalised below
    per_step_launches = launches_timed // (args.steps + args.warmup)
    kern_ms = kernel_avg_ms(events[args.warmup * k_chunks:])
    flops = 2.0 * n ** 3
    value = flops / (ms / 1e3) / 1e12
    # dominant kernel: one local GEMM launch (M/pr x N/pc x K/k_chunks)
    pr, pc = grid.pr, grid.pc
    launch_flops = 2.0 * (n // pr) * (n // pc) * (n // k_chunks)
    achieved = launch_flops / (kern_ms / 1e3) / 1e12
    pk, src = peaks()
    peak = pk["bf16_tflops_sustained"] if dtype == torch.bfloat16 else pk["bf16_tflops_sustained"] / 6.0
    # e2e: host operands (pinned), H2D + 2-D GEMM + D2H of this rank's C block
    Ah = torch.empty(A_sh.shape, dtype=dtype, pin_memory=True).copy_(A_sh)
    Bh = torch.empty(B_sh.shape, dtype=dtype, pin_memory=True).copy_(B_sh)
    Ch = torch.empty((n // pr, n // pc), dtype=dtype, pin_memory=True)
    out_h = {}

    def e2e_step():
        if world == 1:
            # the public call on host operands: streamed through the GPU in
            # row blocks (uploads, GEMMs and downloads overlapped)
            out_h.pop("c", None)  # the previous result is read and released, as a caller's loop would
            out_h["c"] = tb.gemm(1.0, Ah, Bh)
            return
        a = Ah.to("cuda", non_blocking=True)
        b = Bh.to("cuda", non_blocking=True)
        c = tp.gemm_2d(a, b, grid, k_chunks=k_chunks)
        Ch.copy_(c, non_blocking=True)

    e2e_ms, _ = timed_steps(e2e_step, max(2, args.steps // 2), 3, world, gpu)
    out_h.clear()
    del Ah, Bh
    es = A_sh.element_size()
    line = {
        "metric": gemm_metric(n, dtype),
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16" if dtype == torch.bfloat16 else "f32 (3xTF32 on tensor cores)",
        "data": "synthetic (seeded uniform[-1,1] on device, benchmark case 5 shapes)",
        "config": {
            "workload": f"config5a spmd gemm {n}^3",
            "M": n, "N": n, "K": n, "grid": f"{pr}x{pc}", "k_chunks": k_chunks,
            "parallelism": f"2d-output-block {pr}x{pc}",
            "l2": "inputs larger than L2 (no flush needed)",
        },
        "roofline": {
            "bound": "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "peak_source": f"{src} {'bf16 sustained' if dtype == torch.bfloat16 else 'bf16 sustained / 6 (3 tf32 products at half the bf16 rate)'}",
            "kernel": "gemm_pair_kernel (CTA pairs, 256 x 256 tiles)" + ("" if dtype == torch.bfloat16 else " after the split pass"),
            "kernel_ms": round(kern_ms, 4),
            "traffic": TRAFFIC.get(f"spmd_{'bf16' if dtype == torch.bfloat16 else 'fp32'}_{pr}x{pc}"),
        },
        "e2e": {
            "value": round(flops / (e2e_ms / 1e3) / 1e12, 2),
            "unit": "TFLOP/s",
            "ms_per_step": round(e2e_ms, 3),
            "h2d_bytes_per_step": int((A_sh.numel() + B_sh.numel()) * es * world),
            "d2h_bytes_per_step": int((n // pr) * (n // pc) * es * world),
            "path": ("trnblas_b200.gemm on pinned host operands (streamed: row blocks up, GEMMs, rows down, overlapped)"
                     if world == 1 else "trnblas_b200.parallel.gemm_2d on pinned host operands (all ranks)"),
        },
        "clocks": clocks,
        "gpu_launches": per_step_launches * args.steps,
    }
    del A_sh, B_sh
    torch.cuda.empty_cache()
    return line


class _SingleGrid:
    """A 1x1 grid without process groups (N = 1)."""

    pr = pc = 1
    r = c = rank = 0
    world = 1
    row_group = col_group = None

    def block_rows(self, M):
        return 0, M

    def block_cols(self, N):
        return 0, N


def run_pair(args, rank, world, gpu, nocc, nvir, naux, steps=None, warmup=None):
    from trnblas_b200 import _native as N
    from trnblas_b200 import energy
    from trnblas_b200 import parallel as tp

    g = torch.Generator(device="cuda").manual_seed(6)  # same B on every rank
    B = (0.05 * torch.randn(nocc, nvir, naux, device="cuda", generator=g))
    eo = torch.sort(-20 + 19.7 * torch.rand(nocc, device="cuda", generator=g)).values
    ev = torch.sort(0.1 + 4.9 * torch.rand(nvir, device="cuda", generator=g)).values
    steps = steps or args.steps
    warmup = warmup if warmup is not None else args.warmup
    p0, p1 = energy.pair_ranges(nocc, world)[rank]
    out = {}

    def step():
        e = energy.pair_range_energy(B, eo, ev, p0, p1).reshape(1)
        if world > 1:
            dist.all_reduce(e)
        out["e"] = e

    N.launch_count = 0
    ms, clocks = timed_steps(step, steps, warmup, world, gpu)
    launches = N.launch_count // (steps + warmup) * steps
    E = float(out["e"].item())
    npairs = p1 - p0
    sym_flops = nocc * (nocc + 1) / 2 * 2.0 * nvir * nvir * naux
    # kernel-level: the fused kernel on this rank's range, timed alone
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    energy.pair_range_energy(B, eo, ev, p0, p1)
    e_ev.record()
    torch.cuda.synchronize()
    kern_ms = s_ev.elapsed_time(e_ev)
    int8_ops = pair_int8_ops(npairs, nvir, naux)
    # int8 dense rate = 2 x the bf16 dense rate (4.5 POPS vs 2.25 PFLOP/s nominal), both
    # counted as 2 ops per multiply-add; the burst bf16 figure for a launch under a second
    # (full clocks), the sustained one for longer launches (power-capped clocks)
    pk, src = peaks()
    which = "bf16_tflops_sustained" if kern_ms >= 1000.0 else "bf16_tflops"
    int8_peak = 2.0 * pk[which]
    # e2e: the public call on pinned host inputs (each rank uploads B)
    Bh = B.cpu().pin_memory()
    eoh, evh = eo.cpu(), ev.cpu()
    del B
    torch.cuda.empty_cache()

    def e2e_step():
        if world == 1:
            out["e2e"] = float(energy.batched_pair_energy(Bh, eoh, evh))
        else:
            out["e2e"] = tp.pair_energy(Bh, eoh, evh)

    e2e_ms, _ = timed_steps(e2e_step, max(1, min(steps, 2)), 1, world, gpu)
    # at N > 1 each rank uploads a 1/N slice of B and an all-gather shares them
    e2e_info = {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": int(Bh.numel() * 4),
                "d2h_bytes_per_step": 8 * world,
                "path": "trnblas_b200.batched_pair_energy / parallel.pair_energy on pinned host B"}
    del Bh
    return {
        "e2e": e2e_info,
        "ms_per_step": round(ms, 3),
        "energy": E,
        "tflops_sym_count": round(sym_flops / (ms / 1e3) / 1e12, 2),
        "clocks": clocks,
        "gpu_launches": launches,
        "kernel_ms_alone": round(kern_ms, 3),
        "int8_tops_achieved": round(int8_ops / (kern_ms / 1e3) / 1e12, 1),
        "int8_peak_tops": int8_peak,
        "int8_frac": round(int8_ops / (kern_ms / 1e3) / 1e12 / int8_peak, 4),
        "peak_source": f"{src}: 2 x {which} (int8 dense rate = 2 x bf16), int8 ops",
        "pairs_per_rank": npairs,
        "config": {"nocc": nocc, "nvir": nvir, "naux": naux, "sharding": "i<=j pair ranges by count"},
    }


# ── main ─────────────────────────────────────────────────────────────────────


# nocc, nvir, naux: config 3, config 5b, and config 5b's per-pair shape at
# nocc = 4 (a small case with the same units per pair, for profiling)
PAIR_DIMS = {"pair3": (48, 432, 1152), "pair5": (96, 2208, 6912), "pair5x4": (4, 2208, 6912)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="spmd",
                    choices=["spmd", "gemm_fp32", "gemm8192_bf16", "gemm8192_fp32", "pair3", "pair5",
                             "pair5x4", "dfmp2", "gemm_fp64", "batched", "syrk", "batched_bf16",
                             "syrk_bf16", "gemm1024"])
    ap.add_argument("--no-pair", action="store_true", help="skip the pair-energy block of the default line")
    ap.add_argument("--no-fp32", action="store_true", help="skip the fp32 GEMM block of the default line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        # the host cores of rank 0 alone; the other ranks exit without work
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(reference_arm(args, world)), flush=True)
        return
    rank, world, local = setup_dist(args.gpus)
    try:
        line = run_ours(args, rank, world, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


def run_ours(args, rank, world, gpu):
    torch.backends.cuda.matmul.allow_tf32 = False
    if args.workload in ("spmd", "gemm_fp32"):
        dt = torch.bfloat16 if args.workload == "spmd" else torch.float32
        line = run_gemm_spmd(args, rank, world, gpu, dt)
        if args.workload == "spmd" and not args.no_pair:
            pe = run_pair(args, rank, world, gpu, 96, 2208, 6912,
                          steps=min(args.steps, PAIR5_STEPS), warmup=PAIR5_WARMUP)
            line["pair_energy"] = {"metric": pair_metric(96, 2208, 6912), "value": pe["ms_per_step"],
                                   "unit": "ms", "higher_is_better": False,
                                   "steps": min(args.steps, PAIR5_STEPS), "warmup": PAIR5_WARMUP,
                                   "roofline": {"bound": "tensor", "achieved": pe["int8_tops_achieved"],
                                                "peak": pe["int8_peak_tops"], "unit": "TOP/s (int8)",
                                                "frac": pe["int8_frac"],
                                                "traffic": TRAFFIC["pair5"] if world == 1 else None},
                                   **pe}
        if args.workload == "spmd" and not args.no_fp32:
            # config 5a in fp32 (3xTF32), the reference's working precision:
            # its own block, step counts and metric
            sub = argparse.Namespace(**{**vars(args), "steps": min(args.steps, FP32_STEPS),
                                        "warmup": FP32_WARMUP})
            blk = run_gemm_spmd(sub, rank, world, gpu, torch.float32)
            blk.pop("vs_baseline", None)
            line["gemm_fp32"] = blk
        if rank == 0:
            line["cpu_baseline"] = cpu_baseline_gemm(dt) if world == 1 else None
            if "gemm_fp32" in line and world == 1:
                line["gemm_fp32"]["cpu_baseline"] = cpu_baseline_gemm(torch.float32)
        return line
    if args.workload == "dfmp2":
        return run_dfmp2(args, rank, world, gpu)
    if args.workload in PAIR_DIMS:
        dims = PAIR_DIMS[args.workload]
        r = run_pair(args, rank, world, gpu, *dims)
        line = {
            "metric": pair_metric(*dims),
            "value": r["ms_per_step"], "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 (base-254 digit slices, exact int32) + fp64 epilogue",
            "data": "synthetic (benchmark recipe, device generator)",
            "config": {"workload": args.workload, **r["config"]},
            "roofline": {"bound": "tensor", "achieved": r["int8_tops_achieved"], "peak": r["int8_peak_tops"],
                         "unit": "TOP/s (int8)", "frac": r["int8_frac"], "traffic": TRAFFIC.get(args.workload)},
            "clocks": r["clocks"], "gpu_launches": r["gpu_launches"], "e2e": r["e2e"], "detail": r,
        }
        if rank == 0 and world == 1:
            ms, th, sample = cpu_pair_sample(*dims)
            line["cpu_baseline"] = {"value": round(ms, 1), "unit": "ms", "cores": th, "kind": "port", "sample": sample}
        return line
    return run_single(args, rank, world, gpu)


# nbasis, nocc, naux: the reference's largest DF-MP2 benchmark shape
# ("large" in examples/df_mp2.py, docs/benchmarks.md "DF-MP2 end to end")
DFMP2_DIMS = (768, 96, 2304)


def run_dfmp2(args, rank, world, gpu):
    """The whole DF-MP2 energy through `trnblas_b200.parallel.df_mp2_energy`
    (metric factor, half transforms, metric contraction, pair energy; the
    integral rows split over the ranks, strong scaling). value: ms per energy
    with the inputs resident on every rank's GPU; e2e: the same call on
    host inputs (each rank uploads its rows of the integrals)."""
    from trnblas_b200 import _native as N
    from trnblas_b200 import parallel as tp

    nbasis, nocc, naux = DFMP2_DIMS
    nvir = nbasis - nocc
    g = torch.Generator(device="cuda").manual_seed(42)  # same inputs on every rank
    C_occ = 0.1 * torch.randn(nbasis, nocc, device="cuda", generator=g)
    C_vir = 0.1 * torch.randn(nbasis, nvir, device="cuda", generator=g)
    eri = 0.01 * torch.randn(nbasis, nbasis, naux, device="cuda", generator=g)
    R = 0.01 * torch.randn(naux, naux, device="cuda", generator=g)
    J = R @ R.T + naux * torch.eye(naux, device="cuda")  # input construction, untimed
    eo = -torch.sort(torch.rand(nocc, device="cuda", generator=g)).values - 0.5
    ev = torch.sort(torch.rand(nvir, device="cuda", generator=g)).values + 0.1
    ins = (C_occ, C_vir, eri, J, eo, ev)
    out = {}

    def step():
        out["e"] = tp.df_mp2_energy(*ins)

    N.launch_count = 0
    steps, warmup = min(args.steps, 5), args.warmup
    ms, clocks = timed_steps(step, steps, warmup, world, gpu)
    launches = N.launch_count // (steps + warmup) * steps
    t = {}
    tp.df_mp2_energy(*ins, timings=t)
    # e2e: host inputs, each rank uploads its rows of the integrals (pinned)
    rows = tp._eri_rows(nbasis, world, False)[rank]
    eri_h = torch.empty(eri.shape, dtype=eri.dtype, pin_memory=True)  # only this rank's rows are read
    eri_h[rows[0]:rows[1]] = eri[rows[0]:rows[1]].cpu()
    host = [x.cpu() for x in (C_occ, C_vir)] + [eri_h] + [x.cpu() for x in (J, eo, ev)]
    del eri
    torch.cuda.empty_cache()

    def e2e_step():
        out["e2e"] = tp.df_mp2_energy(*host)

    e2e_ms, _ = timed_steps(e2e_step, max(2, steps // 2), 1, world, gpu)
    h2d = (rows[1] - rows[0]) * nbasis * naux * 4 + sum(x.numel() * 4 for x in (C_occ, C_vir, J, eo, ev))
    flops = (2.0 * nbasis * nbasis * nocc * naux + 2.0 * nocc * nvir * nbasis * naux
             + 2.0 * nocc * nvir * naux * naux + nocc * (nocc + 1) / 2 * 2.0 * nvir * nvir * naux)
    # dominant stage: the fused pair energy (int8 pipe), timed by the stage clock
    npairs_rank = (lambda pr: pr[1] - pr[0])(__import__("trnblas_b200").energy.pair_ranges(nocc, world)[rank])
    int8_ops = pair_int8_ops(npairs_rank, nvir, naux)
    pk, src = peaks()
    e_ms = t.get("energy", float("nan")) * 1e3
    ach = int8_ops / (e_ms / 1e3) / 1e12
    line = {
        "metric": f"DF-MP2 energy ms ({nbasis}/{nocc}/{naux}, end to end)",
        "value": round(ms, 3), "unit": "ms", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 (3xTF32) GEMMs + int8 (base-254 digit slices) pair energy",
        "data": "synthetic (examples/df_mp2 distributions, device generator)",
        "config": {"workload": "dfmp2", "nbasis": nbasis, "nocc": nocc, "naux": naux,
                   "sharding": "integral rows by bytes, pairs by count"},
        "energy": out["e"], "stage_seconds": {k: round(v, 5) for k, v in t.items()},
        "tflops_fp32_equiv": round(flops / (ms / 1e3) / 1e12, 2),
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": 2.0 * pk["bf16_tflops"],
                     "unit": "TOP/s (int8)", "frac": round(ach / (2.0 * pk["bf16_tflops"]), 4),
                     "kernel": "pair_energy254_kernel (energy stage)", "stage_ms": round(e_ms, 3),
                     "traffic": None, "peak_source": f"{src}: 2 x bf16 burst (int8 dense rate)"},
        "e2e": {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": int(h2d * world),
                "d2h_bytes_per_step": 8 * world, "path": "parallel.df_mp2_energy on host inputs"},
        "clocks": clocks, "gpu_launches": launches,
    }
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_dfmp2_sample(nbasis, nocc, naux)
    return line


def cpu_dfmp2_sample(nbasis, nocc, naux, budget_s: float = 10.0):
    """The reference's CPU route for the whole DF-MP2 energy (torch fp32 on
    the host): the energy stage from a pair sample (`cpu_pair_sample`), the
    three GEMM stages from one timed sample GEMM scaled by flops."""
    nvir = nbasis - nocc
    e_ms, th, e_sample = cpu_pair_sample(nocc, nvir, naux, budget_s=budget_s)
    g = torch.Generator().manual_seed(7)
    cols = max(1, nbasis * naux // 16)
    Ct = torch.randn(nocc, nbasis, generator=g)
    E = torch.randn(nbasis, cols, generator=g)
    Ct @ E
    t0 = time.perf_counter()
    Ct @ E
    dt = time.perf_counter() - t0
    rate = 2.0 * nocc * nbasis * cols / dt
    gemm_flops = 2.0 * nbasis * nbasis * nocc * naux + 2.0 * nocc * nvir * nbasis * naux + 2.0 * nocc * nvir * naux * naux
    total = e_ms + gemm_flops / rate * 1e3
    return {"value": round(total, 1), "unit": "ms", "cores": th, "kind": "port",
            "sample": f"{e_sample}; GEMM stages from a 1/16 half-transform sample at {rate / 1e12:.2f} TFLOP/s scaled by flops"}


def cpu_baseline_gemm(dt):
    v, th, sample = cpu_gemm_sample(32768, dt)
    return {"value": round(v, 4), "unit": "TFLOP/s", "cores": th, "kind": "port",
            "sample": sample + " (torch CPU matmul: the reference's host route)"}


def run_single(args, rank, world, gpu):
    """Single-GPU workloads (each rank runs its own replica)."""
    import trnblas_b200 as tb
    from trnblas_b200 import _native as N

    g = torch.Generator(device="cuda").manual_seed(rank)
    wl = args.workload
    if wl.startswith("gemm8192"):
        dt = torch.bfloat16 if wl.endswith("bf16") else torch.float32
        n = 8192
        A = torch.randn(n, n, device="cuda", generator=g).to(dt)
        B = torch.randn(n, n, device="cuda", generator=g).to(dt)
        fn = lambda: tb.gemm(1.0, A, B)  # noqa: E731
        flops = 2.0 * n ** 3
    elif wl in ("batched", "batched_bf16"):
        dt = torch.bfloat16 if wl.endswith("bf16") else torch.float32
        A = torch.randn(64, 512, 512, device="cuda", generator=g).to(dt)
        B = torch.randn(64, 512, 512, device="cuda", generator=g).to(dt)
        fn = lambda: tb.batched_gemm(1.0, A, B)  # noqa: E731
        flops = 64 * 2.0 * 512 ** 3
    elif wl in ("syrk", "syrk_bf16"):
        dt = torch.bfloat16 if wl.endswith("bf16") else torch.float32
        A = (torch.randn(4096, 4096, device="cuda", generator=g) / 64).to(dt)
        B = None
        fn = lambda: tb.syrk(1.0, A, uplo="lower")  # noqa: E731
        flops = 4096 * 4097 * 4096.0
    elif wl == "gemm1024":  # config 1: A stored K x M, transA, beta 0.5
        n = 1024
        A = 2 * torch.rand(n, n, device="cuda", generator=g) - 1
        B = 2 * torch.rand(n, n, device="cuda", generator=g) - 1
        C = 2 * torch.rand(n, n, device="cuda", generator=g) - 1
        fn = lambda: tb.gemm(1.0, A, B, 0.5, C, transA=True)  # noqa: E731
        flops = 2.0 * n ** 3
    else:  # gemm_fp64, config 4
        n = 4096
        A = torch.randn(n, n, device="cuda", dtype=torch.float64, generator=g) * torch.exp2(
            torch.randint(-10, 11, (n, n), device="cuda", generator=g).double())
        B = torch.randn(n, n, device="cuda", dtype=torch.float64, generator=g) * torch.exp2(
            torch.randint(-10, 11, (n, n), device="cuda", generator=g).double())
        fn = lambda: tb.gemm_fp64(A, B)  # noqa: E731
        flops = 2.0 * n ** 3
    N.launch_count = 0
    timer = timed_steps_flushed if wl in FLUSHED else timed_steps
    ms, clocks = timer(fn, args.steps, args.warmup, world, gpu)
    launches = N.launch_count // (args.steps + args.warmup) * args.steps
    value = flops / (ms / 1e3) / 1e12 * world
    line = {"metric": f"{wl} TFLOP/s", "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": str(A.dtype).split(".")[-1],
            "data": "synthetic (seeded, device generator)",
            "config": {"workload": wl, "replicas": world,
                       "l2": "256 MB flush before each timed step" if wl in FLUSHED else "operands larger than L2"},
            "clocks": clocks, "gpu_launches": launches}
    line["roofline"] = single_roofline(wl, A, B, flops, C if wl == "gemm1024" else None)
    # e2e: the same public call on pinned host operands, result back on the host
    Ah = A.cpu().pin_memory()
    Bh = B.cpu().pin_memory() if B is not None else None
    Ch = C.cpu().pin_memory() if wl == "gemm1024" else None
    host_fn = {
        "gemm_fp64": lambda: tb.gemm_fp64(Ah, Bh),
        "batched": lambda: tb.batched_gemm(1.0, Ah, Bh),
        "batched_bf16": lambda: tb.batched_gemm(1.0, Ah, Bh),
        "syrk": lambda: tb.syrk(1.0, Ah, uplo="lower"),
        "syrk_bf16": lambda: tb.syrk(1.0, Ah, uplo="lower"),
        "gemm1024": lambda: tb.gemm(1.0, Ah, Bh, 0.5, Ch, transA=True),
    }.get(wl, lambda: tb.gemm(1.0, Ah, Bh))
    res = {}

    def e2e_step():
        res.pop("r", None)
        res["r"] = host_fn()

    e2e_ms, _ = timed_steps(e2e_step, max(2, min(args.steps, 5)), 3, world, gpu)
    out_bytes = res["r"].numel() * res["r"].element_size()
    line["e2e"] = {"value": round(flops / (e2e_ms / 1e3) / 1e12 * world, 2), "unit": "TFLOP/s",
                   "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": int((Ah.numel() + (Bh.numel() if Bh is not None else 0)
                                              + (Ch.numel() if Ch is not None else 0)) * Ah.element_size() * world),
                   "d2h_bytes_per_step": int(out_bytes * world),
                   "path": "the same public call on pinned host operands"}
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_single_sample(wl)
    return line


def single_roofline(wl, A, B, flops, C=None):
    """Roofline of the library call alone (device time between CUDA events on
    the launching stream, no host checks; an L2 flush before each call for the
    workloads whose operands fit in L2): gemm_fp64 against the int8 tensor
    pipe (k (k + 1) / 2 int8 slice products, the split included in the time),
    bf16 batched against HBM (its operands and result: 100.7 MB a call; the
    MMA work needs 7.6 us at the bf16 peak), the others against the bf16 /
    3xTF32 tensor rate."""
    import trnblas_b200 as tb
    from trnblas_b200 import level3

    pk, src = peaks()
    if wl == "gemm_fp64":
        k = level3.DEFAULT_SLICES
        call = lambda: level3._gemm_fp64_device(A, B, k)  # noqa: E731
    elif wl.startswith("gemm8192"):
        call = lambda: tb.gemm(1.0, A, B)  # noqa: E731
    elif wl == "gemm1024":
        call = lambda: tb.gemm(1.0, A, B, 0.5, C, transA=True)  # noqa: E731
    elif wl.startswith("batched"):
        call = lambda: tb.batched_gemm(1.0, A, B)  # noqa: E731
    else:
        call = lambda: tb.syrk(1.0, A, uplo="lower")  # noqa: E731
    for _ in range(2):
        call()
    reps = 5
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if wl in FLUSHED:
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for a, b in ev:
            flush.fill_(1)
            a.record()
            call()
            b.record()
        torch.cuda.synchronize()
        kms = sum(a.elapsed_time(b) for a, b in ev) / reps
        del flush
    else:
        s.record()
        for _ in range(reps):
            call()
        e.record()
        torch.cuda.synchronize()
        kms = s.elapsed_time(e) / reps
    if wl == "gemm_fp64":
        M, K = A.shape
        ops = k * (k + 1) / 2 * 2.0 * M * B.shape[1] * K
        achieved = ops / (kms / 1e3) / 1e12
        peak = 2.0 * pk["bf16_tflops"]
        # context: cuBLAS DGEMM (torch.matmul fp64) on the same operands
        torch.matmul(A, B)
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            torch.matmul(A, B)
        e.record()
        torch.cuda.synchronize()
        dgemm = flops / (s.elapsed_time(e) / reps / 1e3) / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TOP/s (int8)",
                "frac": round(achieved / peak, 4), "traffic": TRAFFIC["gemm_fp64"],
                "kernel": "ozk split + ozaki_gemm_kernel (one trnblas_gemm_fp64 call)",
                "kernel_ms": round(kms, 4), "fp64_tflops_of_call": round(flops / (kms / 1e3) / 1e12, 2),
                "cublas_dgemm_tflops": round(dgemm, 2),
                "peak_source": f"{src}: 2 x bf16 burst (int8 dense rate = 2 x bf16), int8 ops"}
    bf16 = A.dtype == torch.bfloat16
    if wl == "batched_bf16":
        nbytes = 3.0 * A.numel() * A.element_size()  # A, B read; C written
        gbs = nbytes / (kms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": TRAFFIC["batched_bf16"],
                "kernel_ms": round(kms, 4), "algorithmic_bytes": int(nbytes),
                "peak_source": f"{src} HBM copy bandwidth"}
    peak = pk["bf16_tflops"] if bf16 else pk["bf16_tflops"] / 6.0
    achieved = flops / (kms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "traffic": TRAFFIC.get(wl),
            "kernel_ms": round(kms, 4),
            "peak_source": f"{src} bf16 burst" + ("" if bf16 else " / 6 (3 tf32 products at half the bf16 rate)")}


def _ref_line(args, world, metric, unit, hib, value, ms_per_step, cb, extra=None, steps=None, warmup=None):
    """The reference arm's JSON line: the same metric, unit and direction as
    this repo's line for the workload, the step counts it ran (the driver's
    for the default workload) with the wall time of one timed step, and the
    sample it timed."""
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit, "higher_is_better": hib,
            "n_gpus": world, "steps": args.steps if steps is None else steps,
            "warmup": args.warmup if warmup is None else warmup, "ms_per_step": round(ms_per_step, 3),
            "config": {"workload": args.workload, "timed": "each step is a bounded sample of the workload on the host cores"},
            "cpu_baseline": {**cb, "value": value},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if extra:
        line.update(extra)
    return line


def _ref_steps(args, step):
    """Run `step` (one bounded sample; returns (work units, seconds)) W times
    untimed and K times timed; (units per second, mean seconds per step)."""
    for _ in range(args.warmup):
        step()
    units = secs = 0.0
    for _ in range(args.steps):
        u, t = step()
        units += u
        secs += t
    return units / secs, secs / args.steps


def reference_arm(args, world):
    """The reference's CPU route for the workload (its torch host path,
    restated in oracle/ and torch CPU) on the host cores with all threads,
    rank 0 only: --warmup untimed and --steps timed steps, each a bounded
    sample of the workload; value in this repo's metric and unit."""
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    wl = args.workload
    per_step = max(0.3, min(2.0, 60.0 / max(args.steps + args.warmup, 1)))  # seconds per sample
    # other workloads: one bounded sample (one step), timed on the wall clock
    t0 = time.perf_counter()
    if wl == "dfmp2":
        cb = cpu_dfmp2_sample(*DFMP2_DIMS, budget_s=8.0)
        nb, no, na = DFMP2_DIMS
        return _ref_line(args, world, f"DF-MP2 energy ms ({nb}/{no}/{na}, end to end)", "ms", False,
                         cb["value"], (time.perf_counter() - t0) * 1e3, cb, steps=1, warmup=0)
    if wl in PAIR_DIMS:
        dims = PAIR_DIMS[wl]
        ms, th, sample = cpu_pair_sample(*dims, budget_s=8.0)
        cb = {"unit": "ms", "cores": th, "kind": "port", "sample": sample}
        return _ref_line(args, world, pair_metric(*dims), "ms", False, round(ms, 1),
                         (time.perf_counter() - t0) * 1e3, cb, steps=1, warmup=0)
    if wl in ("batched", "syrk", "gemm_fp64", "batched_bf16", "syrk_bf16", "gemm1024"):
        cb = cpu_single_sample(wl, budget_s=8.0)
        return _ref_line(args, world, f"{wl} TFLOP/s", "TFLOP/s", True, cb["value"],
                         (time.perf_counter() - t0) * 1e3, cb, steps=1, warmup=0)
    dt = torch.float32 if wl in ("gemm_fp32", "gemm8192_fp32") else torch.bfloat16
    n = 32768 if wl in ("spmd", "gemm_fp32") else 8192
    g = torch.Generator().manual_seed(5)
    B = (2 * torch.rand(n, n, generator=g) - 1).to(dt)
    A = (2 * torch.rand(64, n, generator=g) - 1).to(dt)
    torch.matmul(A, B)  # thread-pool warm-up
    t0 = time.perf_counter()
    torch.matmul(A, B)
    per_row = max((time.perf_counter() - t0) / 64, 1e-6)
    rows = int(max(64, min(n, per_step / per_row)))
    A = (2 * torch.rand(rows, n, generator=g) - 1).to(dt)

    def step():
        t = time.perf_counter()
        torch.matmul(A, B)
        return 2.0 * rows * n * n, time.perf_counter() - t

    rate, sec = _ref_steps(args, step)
    v = round(rate / 1e12, 4)
    cb = {"unit": "TFLOP/s", "cores": threads, "kind": "port",
          "sample": f"{rows} x {n} rows of the {n}^3 product per step, {dt} (torch CPU matmul: the reference's host route)"}
    extra = {}
    if wl == "spmd" and not args.no_pair:
        ms, th, sample = cpu_pair_sample(96, 2208, 6912, budget_s=8.0)
        extra["pair_energy"] = {"metric": pair_metric(96, 2208, 6912), "value": round(ms, 1), "unit": "ms",
                                "higher_is_better": False, "steps": 1, "warmup": 0,
                                "cpu_baseline": {"value": round(ms, 1), "unit": "ms", "cores": th, "kind": "port",
                                                 "sample": sample}}
    if wl == "spmd" and not args.no_fp32:
        del A, B
        v32, th, sample = cpu_gemm_sample(n, torch.float32, budget_s=8.0)
        extra["gemm_fp32"] = {"metric": gemm_metric(n, torch.float32), "value": round(v32, 4), "unit": "TFLOP/s",
                              "higher_is_better": True, "steps": 1, "warmup": 1,
                              "cpu_baseline": {"value": round(v32, 4), "unit": "TFLOP/s", "cores": th, "kind": "port",
                                               "sample": sample + " (torch CPU matmul: the reference's host route)"}}
    return _ref_line(args, world, gemm_metric(n, dt), "TFLOP/s", True, v, sec * 1e3, cb, extra)


if __name__ == "__main__":
    main()
