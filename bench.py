"""Benchmark of the B200 hot path behind the VC runtime API.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--only gemm,fa_causal,fa_bf16,stream,fa_f32,gemm_f32]

One JSON line on rank 0. The headline workload is the dense GEMM
C = A*B, M = N = K = 4096, fp16 inputs drawn U[-1, 1), fp32 accumulate and
output (weak scaling: every rank runs its own 4096-row block). A step is a
batch of GEMMS_PER_STEP such products; inputs rotate over 4 buffer sets
(512 MiB, larger than the 126 MB L2), so every product reads cold operands.
The other benchmark configurations ride along in "also":
  fa_causal  flash-attention fwd fp16, B=8, H=16, N=4096, d=128, causal
  fa_bf16    flash-attention fwd bf16, B=32, H=32, N=8192, d=128, sharded
             over ranks by batch x heads (strong scaling)
  stream     vadd c = a + b then sum(c), n = 2^30 fp32, sharded contiguously
             over ranks, the ranks' fp64 sums combined inside the kernel over
             NVLink (an NCCL all-reduce after the kernel is timed beside it)
  fa_f32     flash-attention fwd fp32, B=1, H=1, N=256, d=64 (the demo's
             precision; latency bound: timed as CUDA-graph replays of 16
             launches each)
  gemm_f32   fp32 GEMM 4096^3 (the fp32 demo kernel's contract) on the tensor
             cores from a hi/lo split (hi*hi in tf32, corrections in bf16);
             the CUDA-core path of the same call timed beside it
Under torchrun (N > 1) ranks time on the device with CUDA events between
barriers; rank 0 prints the max over ranks.

`--impl reference` times the reference's own CPU algorithm for the headline
workload (the oracle's restatement of the demos' host loops, all host
threads) on a bounded sample, on rank 0 only.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "attn-fwd & GEMM TFLOP/s (% of B200 dense peak), reduce GB/s, at 1/2/4/8 GPU"
GEMM_N = 4096
GEMMS_PER_STEP = 400
ROTATE = 4
E2E_LANES = 3  # streams the end-to-end GEMM rotates over
E2E_STEPS = 32
FA_F32_GRAPH = 16  # demo-precision attention launches per CUDA-graph replay
LOG2E = 1.4426950408889634


# ---------------------------------------------------------------- helpers
def set_gemms_per_step(n: int) -> None:
    global GEMMS_PER_STEP
    GEMMS_PER_STEP = max(1, int(n))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm": p["hbm_gbs"], "bf16": p["bf16_tflops"],
                "bf16_sustained": p["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def traffic_table():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        return json.load(open(path))
    return {}


def flash_traffic(name, bh):
    """DRAM bytes of one launch over `bh` slices: a whole-launch capture of
    this workload when there is one, else a per-slice figure (a capture of
    fewer slices of the same shape, whose traffic grows with the slice
    count) times `bh`."""
    tt = traffic_table()
    if name in tt:
        return tt[name]
    per_slice = tt.get(name + "_per_slice")
    return None if per_slice is None else int(per_slice * bh)


def stream_traffic(n):
    """DRAM bytes of one fused vadd+sum launch over `n` elements: a capture
    of the same kernel on fewer elements (inputs still larger than L2), per
    element, times `n`."""
    per_elem = traffic_table().get("stream_fused_per_elem")
    return None if per_elem is None else int(per_elem * n)


class ClockSampler:
    """nvidia-smi samples (every 50 ms), each stamped on arrival; started before
    the idle period and the warm-up (nvidia-smi takes a moment to produce its
    first line), summarised over the samples that arrived inside the timed
    window `window` = (t0, t1) of time.monotonic()."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str):
        self.uuid = device_uuid
        self.proc = None
        self.lines = []
        self.window = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.uuid, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = list(self.lines)
        if self.window is not None:
            t0, t1 = self.window
            # a sample arriving up to one period after the window describes it
            lines = [(t, l) for t, l in lines if t0 <= t <= t1 + 0.05]
        for _, line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:7]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend="nccl"):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group(backend, timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def shard(total: int, world: int, rank: int):
    """Contiguous [begin, end) share of `total` units for `rank`."""
    base, rem = divmod(total, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def check(err, what):
    if int(err) != 0:
        raise RuntimeError(f"{what} failed with VCError {int(err)}")


IDLE_BEFORE_S = 1.0  # every workload starts from an idle GPU (as the peaks were measured)
# A timed region of at least this many ms of back-to-back launches is judged
# against the sustained (power-capped) peak, a shorter one against burst.
SUSTAINED_REGION_MS = 1000.0


def timed(dist, stream, fn, steps, warmup, sampler=None, stats=None):
    """After IDLE_BEFORE_S seconds idle, run fn() warmup times, then time
    `steps` calls with CUDA events on `stream` between barriers; returns the
    max over ranks, in ms. With `stats` (a dict), an event between steps also
    gives this rank's median and best step time (`median_ms`, `best_ms`)."""
    import torch
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        torch.cuda.synchronize()
        time.sleep(IDLE_BEFORE_S)
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        events = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        t0 = time.monotonic()
        events[0].record(stream)
        for i in range(steps):
            fn()
            events[i + 1].record(stream)
        torch.cuda.synchronize()
        t1 = time.monotonic()
    if sampler is not None:
        sampler.window = (t0, t1)
    dist.barrier()
    if stats is not None:
        per = [events[i].elapsed_time(events[i + 1]) for i in range(steps)]
        stats["median_ms"] = round(statistics.median(per), 4)
        stats["best_ms"] = round(min(per), 4)
    return dist.max(events[0].elapsed_time(events[-1]))


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ---------------------------------------------------------------- workloads
def colsum_parity(dist, A, B, C):
    """Cross-rank check of a product split over the ranks by M-blocks (rank r
    holds rows of A and C, B replicated): the column sums of the assembled C
    (summed over the ranks) against (column sums of the assembled A) * B, in
    fp64. Returns the largest |difference| over the columns in units of the
    bar sqrt(M_total) * 1e-3 * sqrt(K) (each element within 1e-3 sqrt(K),
    errors of independent rows adding as a random walk); <= 1 passes."""
    import torch
    K = A.shape[1]
    cs = C.double().sum(0)
    asum = A.double().sum(0)
    rows = torch.tensor([float(A.shape[0])], dtype=torch.float64, device="cuda")
    if dist.pg:
        for t in (cs, asum, rows):
            dist.pg.all_reduce(t)
    ref = asum @ B.double()
    bar = math.sqrt(rows.item()) * 1e-3 * math.sqrt(K)
    return float((cs - ref).abs().max().item() / bar)


def gemm_workload(vc, dist, steps, warmup, pk, device_uuid, want_e2e=True):
    """Rank r computes rows [4096 r, 4096 (r + 1)) of one (4096 N_ranks) x
    4096 x 4096 product: its own M-block of A, B the same on every rank
    (generated from one seed), no communication."""
    import torch
    N = GEMM_N
    ga = torch.Generator(device="cuda").manual_seed(1 + dist.rank)
    gb = torch.Generator(device="cuda").manual_seed(1000)
    sets = []
    for _ in range(ROTATE):
        A = (torch.rand(N, N, device="cuda", generator=ga) * 2 - 1).half()
        B = (torch.rand(N, N, device="cuda", generator=gb) * 2 - 1).half()
        C = torch.empty(N, N, device="cuda", dtype=torch.float32)
        sets.append((A, B, C))
    stream = torch.cuda.current_stream()
    state = {"i": 0}

    def one():
        A, B, C = sets[state["i"] % ROTATE]
        state["i"] += 1
        check(vc.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), None, N, N, N, N, N, N, 0,
                      vc.Dtype.F16, True, stream.cuda_stream), "vc_gemm")

    def step():
        for _ in range(GEMMS_PER_STEP):
            one()

    # Quick parity guard on the first set (row sample vs torch fp32 matmul).
    one()
    torch.cuda.synchronize()
    A, B, C = sets[0]
    ref = A[:64].float() @ B.float()
    err = dist.max((C[:64] - ref).abs().max().item())
    if not err <= 1e-3 * math.sqrt(N):
        raise RuntimeError(f"GEMM parity guard failed: max err {err}")
    colsum = dist.max(colsum_parity(dist, A, B, C))
    if not colsum <= 1.0:
        raise RuntimeError(f"GEMM cross-rank column-sum check failed: {colsum}")

    sampler = ClockSampler(device_uuid)
    step_stats = {}
    ms = timed(dist, stream, step, steps, warmup, sampler, stats=step_stats)
    flop_step = 2.0 * N ** 3 * GEMMS_PER_STEP
    per_launch_ms = ms / (steps * GEMMS_PER_STEP)
    value = flop_step * steps * dist.world / (ms * 1e-3) / 1e12
    achieved = 2.0 * N ** 3 / (per_launch_ms * 1e-3) / 1e12
    # The timed region runs the kernel back to back; a region of a second or
    # more is the power-capped regime the sustained peak was measured in
    # (seconds of back-to-back GEMMs); a shorter one is judged against burst.
    sustained = ms >= SUSTAINED_REGION_MS
    peak = pk["bf16_sustained"] if sustained else pk["bf16"]
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s",
        "ms_per_step": round(ms / steps, 4),
        "ms_per_step_median": step_stats["median_ms"], "ms_per_step_best": step_stats["best_ms"],
        "per_launch_ms": round(per_launch_ms, 5),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_kind": ("bf16 dense sustained" if sustained else "bf16 dense burst")
                     + f" ({pk['source']}); timed region {ms / 1e3:.2f} s back to back",
                     "frac_vs_burst": round(achieved / pk["bf16"], 4),
                     "traffic": traffic_table().get("gemm_f16_4096")},
        "clocks": sampler.summary(),
        "gpu_launches": steps * GEMMS_PER_STEP,
        "parity": {"row_sample_max_err_all_ranks": err, "bar": 1e-3 * math.sqrt(N),
                   "colsum_all_ranks_over_bar": round(colsum, 5), "ranks": dist.world},
    }
    if want_e2e:
        # 32 steps (~50 ms): the first upload and the last download, which
        # nothing overlaps, stay a small part of the timed region.
        out["e2e"] = gemm_e2e(vc, dist, steps=E2E_STEPS, warmup=E2E_LANES)
    del sets
    torch.cuda.empty_cache()
    return out


def gemm_e2e(vc, dist, steps, warmup):
    """The same GEMM through the reference-facing API: pinned host A, B ->
    vcMemcpyAsyncS H2D -> vcLaunchKernel('vc.gemm') -> vcMemcpyAsyncS D2H of
    C, every step moving its inputs in and its result out. Three streams, one
    per stage (uploads, GEMMs, downloads), ordered by vcEvents, over
    E2E_LANES buffer sets: each direction of the PCIe link works through its
    copies in order without waiting on the other, and a buffer set is reused
    only after the step that last used it has finished with it. Timed with
    vcEvents from the first upload to the last download."""
    import ctypes
    N = GEMM_N
    nb16, nb32 = N * N * 2, N * N * 4
    rng = np.random.default_rng(100 + dist.rank)
    a = (rng.random(N * N, dtype=np.float32) * 2 - 1).astype(np.float16)
    b = (rng.random(N * N, dtype=np.float32) * 2 - 1).astype(np.float16)

    def event():
        err, e = vc.vcEventCreate()
        check(err, "vcEventCreate")
        return e

    lanes = []
    for _ in range(E2E_LANES):
        lane = {}
        for key, nb in (("hA", nb16), ("hB", nb16), ("hC", nb32)):
            err, lane[key] = vc.vcMallocHost(nb)
            check(err, "vcMallocHost")
        for key, nb in (("dA", nb16), ("dB", nb16), ("dC", nb32)):
            err, lane[key] = vc.vcMalloc(nb)
            check(err, "vcMalloc")
        ctypes.memmove(lane["hA"], a.ctypes.data, nb16)
        ctypes.memmove(lane["hB"], b.ctypes.data, nb16)
        lane["up"], lane["gemm"], lane["down"] = event(), event(), event()
        lane["args"] = [vc.ptr(lane["dA"]), vc.ptr(lane["dB"]), vc.ptr(lane["dC"]), vc.ptr(0),
                        vc.i32(N), vc.i32(N), vc.i32(N), vc.i64(N), vc.i64(N), vc.i64(N),
                        vc.i64(0), vc.i32(int(vc.Dtype.F16)), vc.i32(1)]
        lanes.append(lane)
    streams = {}
    for name in ("up", "gemm", "down"):
        err, streams[name] = vc.vcStreamCreate()
        check(err, "vcStreamCreate")
    s_up, s_gemm, s_down = streams["up"], streams["gemm"], streams["down"]
    err, k = vc.vcGetKernel("vc.gemm")
    check(err, "vcGetKernel")
    H2D, D2H = vc.VCMemcpyKind.HostToDevice, vc.VCMemcpyKind.DeviceToHost
    used = set()

    def step(i):
        L = lanes[i % E2E_LANES]
        reuse = id(L) in used
        used.add(id(L))
        if reuse:  # the previous GEMM on this set has read dA, dB
            vc.vcStreamWaitEvent(s_up, L["gemm"])
        check(vc.vcMemcpyAsyncS(L["dA"], L["hA"], nb16, H2D, s_up), "H2D A")
        check(vc.vcMemcpyAsyncS(L["dB"], L["hB"], nb16, H2D, s_up), "H2D B")
        vc.vcEventRecord(L["up"], s_up)
        vc.vcStreamWaitEvent(s_gemm, L["up"])
        if reuse:  # the previous download of this set has read dC
            vc.vcStreamWaitEvent(s_gemm, L["down"])
        check(vc.vcLaunchKernel(k, 1, 1, L["args"], s_gemm), "launch vc.gemm")
        vc.vcEventRecord(L["gemm"], s_gemm)
        vc.vcStreamWaitEvent(s_down, L["gemm"])
        check(vc.vcMemcpyAsyncS(L["hC"], L["dC"], nb32, D2H, s_down), "D2H C")
        vc.vcEventRecord(L["down"], s_down)

    for i in range(warmup):
        step(i)
    for st_ in (s_up, s_gemm, s_down):
        check(vc.vcStreamSynchronize(st_), "sync")
    dist.barrier()
    e0, e1, e_end = event(), event(), event()
    vc.vcEventRecord(e0, s_up)
    for i in range(steps):
        step(warmup + i)
    vc.vcEventRecord(e_end, s_down)
    vc.vcStreamWaitEvent(s_up, e_end)
    vc.vcEventRecord(e1, s_up)
    check(vc.vcEventSynchronize(e1), "event sync")
    err, ms = vc.vcEventElapsedTime(e0, e1)
    check(err, "elapsed")
    ms = dist.max(ms)
    ref = a.reshape(N, N)[0].astype(np.float64) @ b.reshape(N, N).astype(np.float64)
    for L in lanes:
        c_row = np.frombuffer((ctypes.c_float * N).from_address(L["hC"]), np.float32)
        if not np.abs(c_row - ref).max() <= 1e-3 * math.sqrt(N):
            raise RuntimeError("e2e GEMM result check failed")
    for L in lanes:
        for key in ("dA", "dB", "dC", "hA", "hB", "hC"):
            vc.vcFree(L[key])
        for key in ("up", "gemm", "down"):
            vc.vcEventDestroy(L[key])
    for st_ in (s_up, s_gemm, s_down):
        vc.vcStreamDestroy(st_)
    for e in (e0, e1, e_end):
        vc.vcEventDestroy(e)
    vc.vcReleaseKernel(k)
    value = 2.0 * N ** 3 * steps * dist.world / (ms * 1e-3) / 1e12
    return {"value": round(value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": 2 * nb16,
            "d2h_bytes_per_step": nb32, "ms_per_step": round(ms / steps, 4),
            "path": "vcMallocHost + vcMemcpyAsyncS + vcLaunchKernel(vc.gemm) + vcMemcpyAsyncS; "
                    f"upload, GEMM and download streams ordered by vcEvents over {E2E_LANES} "
                    "buffer sets; bound: PCIe Gen5 x16, 44-48 GB/s each way with both "
                    "directions busy (64 MiB each way per step)"}


MBLOCK_M = 8 * GEMM_N  # rows of the one product the M-block GEMM splits over the ranks
MBLOCK_PER_STEP = 20


def gemm_mblock_workload(vc, dist, steps, warmup, pk):
    """One product C = A * B of MBLOCK_M x 4096 x 4096 (fp16 in, fp32 out)
    split over the ranks by M-blocks: rank r owns a contiguous share of the
    rows of A and C, B (32 MiB) is the same on every rank, no communication
    (strong scaling: the total work is fixed, at 8 ranks each computes a
    4096^3 block). A step is MBLOCK_PER_STEP products, alternating over two
    sets of A and C. Whole-job TFLOP/s = the product's FLOP / the slowest
    rank's time; the assembled result is checked across the ranks by column
    sums."""
    import torch
    N = GEMM_N
    r0, r1 = shard(MBLOCK_M, dist.world, dist.rank)
    m = r1 - r0
    gb = torch.Generator(device="cuda").manual_seed(2000)
    B = (torch.rand(N, N, device="cuda", generator=gb) * 2 - 1).half()
    sets = []
    for si in range(2):
        ga = torch.Generator(device="cuda").manual_seed(3000 + 100 * si + dist.rank)
        A = (torch.rand(m, N, device="cuda", generator=ga) * 2 - 1).half()
        sets.append((A, torch.empty(m, N, device="cuda", dtype=torch.float32)))
    stream = torch.cuda.current_stream()
    state = {"i": 0}

    def one():
        A, C = sets[state["i"] % 2]
        state["i"] += 1
        check(vc.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), None, m, N, N, N, N, N, 0,
                      vc.Dtype.F16, True, stream.cuda_stream), "vc_gemm")

    def step():
        for _ in range(MBLOCK_PER_STEP):
            one()

    one()
    torch.cuda.synchronize()
    A, C = sets[0]
    ref = A[-64:].float() @ B.float()
    err = dist.max((C[-64:] - ref).abs().max().item())
    colsum = dist.max(colsum_parity(dist, A, B, C))
    if not (err <= 1e-3 * math.sqrt(N) and colsum <= 1.0):
        raise RuntimeError(f"M-block GEMM parity failed: {err}, {colsum}")
    step_stats = {}
    ms = timed(dist, stream, step, steps, warmup, stats=step_stats)
    per_launch = ms / (steps * MBLOCK_PER_STEP)
    value = 2.0 * MBLOCK_M * N * N / (per_launch * 1e-3) / 1e12
    achieved = 2.0 * m * N * N / (per_launch * 1e-3) / 1e12
    sustained = ms >= SUSTAINED_REGION_MS
    peak = pk["bf16_sustained"] if sustained else pk["bf16"]
    res = {"workload": "gemm_mblock", "value": round(value, 2), "unit": "TFLOP/s",
           "ms_per_step": round(ms / steps, 4), "per_launch_ms": round(per_launch, 5),
           "ms_per_step_median": step_stats["median_ms"], "ms_per_step_best": step_stats["best_ms"],
           "scaling": "strong",
           "config": {"M": MBLOCK_M, "N": N, "K": N, "dtype": "f16 in, f32 out",
                      "rows_per_rank": m, "gemms_per_step": MBLOCK_PER_STEP,
                      "split": "M-blocks of one product, B replicated, no collective"},
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                        "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                        "peak_kind": ("bf16 dense sustained" if sustained else "bf16 dense burst")
                        + f" ({pk['source']}); timed region {ms / 1e3:.2f} s",
                        "frac_vs_burst": round(achieved / pk["bf16"], 4), "traffic": None},
           "gpu_launches": steps * MBLOCK_PER_STEP,
           "parity": {"row_sample_max_err_all_ranks": err,
                      "colsum_all_ranks_over_bar": round(colsum, 5), "ranks": dist.world}}
    del sets, B
    torch.cuda.empty_cache()
    return res


def measured_tf32_tflops(n=8192, reps=10):
    """Dense TF32 tensor-core rate of this GPU, measured the way the bf16 peak
    of MEASURED_PEAKS.json is: a library (cuBLAS) TF32 GEMM of n^3, best of
    `reps` launches, CUDA events. A denominator only, never on the hot path."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.rand(n, n, device="cuda")
        b = torch.rand(n, n, device="cuda")
        for _ in range(3):
            torch.mm(a, b)
        torch.cuda.synchronize()
        best = None
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            torch.mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        del a, b
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def gemm_f32_workload(vc, dist, steps, warmup, pk):
    """fp32 C = A * B at 4096^3 (the reference's fp32 GEMM, matmulTiled in
    examples/matmul_bench.vc, at the headline size): tensor-core path, hi*hi
    as one tf32 MMA and lo*hi + hi*lo as one bf16 MMA per 8-deep K step.
    Reported as fp32 TFLOP/s delivered; the roofline counts the tensor pipe's
    work as 4 N^3 tf32-equivalent FLOP (2 N^3 tf32 + 4 N^3 bf16 at twice the
    rate) against the dense tf32 rate measured on this GPU (a cuBLAS tf32
    GEMM, best of 10). The CUDA-core path of the same API (taken for strides TMA cannot serve:
    lda = N + 1) is timed beside it."""
    import torch
    N, per_step = 4096, 16
    g = torch.Generator(device="cuda").manual_seed(11 + dist.rank)
    sets = []
    for _ in range(2):  # 192 MiB per set > 126 MB L2
        A = torch.rand(N, N, device="cuda", generator=g) * 2 - 1
        B = torch.rand(N, N, device="cuda", generator=g) * 2 - 1
        sets.append((A, B, torch.empty(N, N, device="cuda")))
    stream = torch.cuda.current_stream()
    state = {"i": 0}

    def one():
        A, B, C = sets[state["i"] % 2]
        state["i"] += 1
        check(vc.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), None, N, N, N, N, N, N, 0,
                      vc.Dtype.F32, True, stream.cuda_stream), "vc_gemm f32")

    def step():
        for _ in range(per_step):
            one()

    one()
    torch.cuda.synchronize()
    A, B, C = sets[0]
    ref = A[:64].double() @ B.double()
    mag = A[:64].abs().double() @ B.abs().double()
    perr = ((C[:64].double() - ref).abs() / mag).max().item()
    if not perr <= 2e-5:
        raise RuntimeError(f"fp32 GEMM parity guard failed: {perr}")
    step_stats = {}
    ms = timed(dist, stream, step, steps, warmup, stats=step_stats)
    per_launch = ms / (steps * per_step)
    value = 2.0 * N ** 3 * dist.world / (per_launch * 1e-3) / 1e12
    achieved = 4.0 * N ** 3 / (per_launch * 1e-3) / 1e12
    tf32_peak = measured_tf32_tflops()
    peak = round(tf32_peak, 1)
    # CUDA-core path of the same call: A with a row stride of N + 1 floats.
    Ap = torch.zeros(N, N + 1, device="cuda")
    Ap[:, :N] = A

    def simt():
        check(vc.gemm(Ap.data_ptr(), B.data_ptr(), C.data_ptr(), None, N, N, N, N + 1, N, N, 0,
                      vc.Dtype.F32, True, stream.cuda_stream), "vc_gemm f32 simt")

    simt()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(3):
        simt()
    e1.record()
    torch.cuda.synchronize()
    simt_ms = e0.elapsed_time(e1) / 3
    res = {"workload": "gemm_f32", "value": round(value, 2), "unit": "TFLOP/s",
           "ms_per_step": round(ms / steps, 4), "per_launch_ms": round(per_launch, 4),
           "ms_per_step_median": step_stats["median_ms"], "ms_per_step_best": step_stats["best_ms"],
           "scaling": "weak",
           "config": {"M": N, "N": N, "K": N, "dtype": "f32", "layout": "row-major, B [K][N]",
                      "gemms_per_step": per_step, "method": "hi/lo split: hi*hi tf32, "
                      "lo*hi + hi*lo bf16; 512-deep K chunks added with round-to-nearest"},
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                        "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                        "peak_kind": "tf32-equivalent work 4 N^3 (2 N^3 tf32 + 4 N^3 bf16 at twice "
                        "the tf32 rate) against the dense tf32 rate measured on this GPU in this run "
                        "(cuBLAS tf32 8192^3, best of 10)",
                        "frac_vs_half_bf16_burst": round(achieved / (pk["bf16"] / 2), 4),
                        "traffic": traffic_table().get("gemm_f32_4096")},
           "simt_path_tflops": round(2.0 * N ** 3 / (simt_ms * 1e-3) / 1e12, 2),
           "gpu_launches": steps * per_step, "parity_guard_max_rel_err": perr}
    del sets, Ap
    torch.cuda.empty_cache()
    return res


def flash_workload(vc, dist, name, B, H, N, d, causal, dtype, steps, warmup, pk, shard_bh):
    import torch
    BH = B * H
    b0, b1 = shard(BH, dist.world, dist.rank) if shard_bh else (0, BH)
    bh = b1 - b0
    tdt = {vc.Dtype.F16: torch.float16, vc.Dtype.BF16: torch.bfloat16, vc.Dtype.F32: torch.float32}[dtype]
    g = torch.Generator(device="cuda").manual_seed(3 + dist.rank)
    amp = 0.5 if dtype == vc.Dtype.BF16 else 1.0
    Q, K, V = ((torch.randn(bh, N, d, device="cuda", generator=g) * amp).to(tdt) for _ in range(3))
    O = torch.empty_like(Q)
    scale = LOG2E / math.sqrt(d)
    stream = torch.cuda.current_stream()

    def launch(stream_handle):
        check(vc.flash_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), bh, N, d, scale,
                           causal, dtype, stream_handle), "vc_flash_fwd")

    def step():
        launch(stream.cuda_stream)

    step()
    torch.cuda.synchronize()
    per_step = 1
    if dtype == vc.Dtype.F32:
        # The demo-precision launch runs ~10 us on the GPU, less than a host
        # call through the C ABI takes: a CUDA graph of FA_F32_GRAPH launches
        # is replayed per step, so the timing is the GPU's, every launch
        # still doing its full work.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(FA_F32_GRAPH):
                launch(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        per_step = FA_F32_GRAPH
        step = graph.replay  # noqa: F811
        step()
        torch.cuda.synchronize()
    # parity guard: 32 rows of the last slice against torch fp32 SDPA
    q = Q[-1:].float()
    ref = torch.nn.functional.scaled_dot_product_attention(
        q[:, -32:], K[-1:].float(), V[-1:].float(), is_causal=False,
        attn_mask=(torch.arange(N, device="cuda")[None, :] <= torch.arange(N - 32, N, device="cuda")[:, None])
        if causal else None)
    # Every rank checks the last slice of its own shard; the line carries the
    # largest error over the ranks.
    perr = dist.max((O[-1:, -32:].float() - ref).abs().max().item())
    tol = {vc.Dtype.F16: 2e-3, vc.Dtype.BF16: 1e-2, vc.Dtype.F32: 1e-4}[dtype]
    if not perr <= tol:
        raise RuntimeError(f"{name} parity guard failed: {perr}")
    step_stats = {}
    ms = timed(dist, stream, step, steps, warmup, stats=step_stats)
    flop = (2.0 if causal else 4.0) * BH * N * N * d  # whole job
    per_launch = ms / (steps * per_step)
    value = flop / (per_launch * 1e-3) / 1e12 if shard_bh else flop * dist.world / (per_launch * 1e-3) / 1e12
    local_flop = (2.0 if causal else 4.0) * bh * N * N * d
    achieved = local_flop / (per_launch * 1e-3) / 1e12
    long_kernel = ms >= SUSTAINED_REGION_MS
    peak = pk["bf16_sustained"] if long_kernel else pk["bf16"]
    res = {"workload": name, "value": round(value, 2), "unit": "TFLOP/s",
           "ms_per_step": round(per_launch, 4), "ms_per_step_median": step_stats["median_ms"],
           "ms_per_step_best": step_stats["best_ms"],
           "scaling": "strong" if shard_bh else "weak",
           "config": {"B": B, "H": H, "N": N, "d": d, "causal": causal,
                      "dtype": {1: "f16", 2: "bf16", 0: "f32"}[int(dtype)],
                      "bh_per_rank": bh},
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                        "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                        "peak_kind": ("bf16 dense sustained" if long_kernel else "bf16 dense burst")
                        + f" ({pk['source']}); timed region {ms / 1e3:.2f} s",
                        "frac_vs_burst": round(achieved / pk["bf16"], 4),
                        "traffic": flash_traffic(name, bh)},
           "gpu_launches": steps * per_step, "parity_guard_max_err": perr,
           "parity": {"check": "last 32 query rows of the last slice of every rank's shard vs "
                               "torch fp32 SDPA", "max_err_all_ranks": perr, "bar": tol,
                      "ranks": dist.world}}
    if dtype == vc.Dtype.F32:
        res["roofline"]["note"] = "fp32 CUDA-core path; latency bound at this size"
        res["launches_per_step"] = per_step
        res["timing"] = f"CUDA graph of {per_step} launches replayed per step; ms_per_step is per launch"
        for key in ("ms_per_step_median", "ms_per_step_best"):
            res[key] = round(res[key] / per_step, 5)
    del Q, K, V, O
    torch.cuda.empty_cache()
    return res


def stream_workload(vc, dist, steps, warmup, pk, log2n=30):
    import torch
    n_total = 1 << log2n
    b0, b1 = shard(n_total, dist.world, dist.rank)
    n = b1 - b0
    g = torch.Generator(device="cuda").manual_seed(5 + dist.rank)
    a = torch.rand(n, device="cuda", generator=g)
    b = torch.rand(n, device="cuda", generator=g)
    c = torch.empty_like(a)
    part = torch.zeros(1, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream()
    cs = stream.cuda_stream
    # N > 1: the per-GPU sums are combined inside the kernel through the
    # ranks' mailboxes (NVLink peer stores); the handles travel once over the
    # process group.
    from vkcuda_b200 import peer
    boxes = peer.open_mailboxes(dist.pg, dist.rank, dist.world) if dist.pg else None
    epoch = [0]

    def fused():
        if boxes is None:
            check(vc.vadd_sum_f32(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, part.data_ptr(),
                                  cs), "vc_vadd_sum_f32")
            return
        epoch[0] += 1
        check(vc.vadd_sum_f32_allreduce(a.data_ptr(), b.data_ptr(), c.data_ptr(), n,
                                        part.data_ptr(), boxes, dist.rank, epoch[0], cs),
              "vc_vadd_sum_f32_allreduce")

    def fused_then_nccl():
        check(vc.vadd_sum_f32(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, part.data_ptr(), cs),
              "vc_vadd_sum_f32")
        dist.pg.all_reduce(part)

    def vadd_only():
        check(vc.vadd_f32(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, cs), "vc_vadd_f32")

    def sum_only():
        check(vc.sum_f32(c.data_ptr(), n, part.data_ptr(), cs), "vc_sum_f32")

    fused()
    torch.cuda.synchronize()
    total = part.item()
    # parity guard: fp64 sum of c on the device (torch) vs ours
    ref = c.double().sum()
    if dist.pg:
        dist.pg.all_reduce(ref)
    rel = dist.max(abs(total - ref.item()) / abs(ref.item()))
    if not rel <= 1e-6:
        raise RuntimeError(f"stream parity guard failed: {total} vs {ref.item()}")
    ms_fused = timed(dist, stream, fused, steps, warmup)
    ms_vadd = timed(dist, stream, vadd_only, steps, warmup)
    ms_sum = timed(dist, stream, sum_only, steps, warmup)
    # For comparison (ranks > 1): the kernel followed by an NCCL all-reduce of
    # the partial, and that all-reduce on its own.
    ms_nccl = timed(dist, stream, fused_then_nccl, steps, warmup) if dist.pg else None
    ms_ar = timed(dist, stream, lambda: dist.pg.all_reduce(part), steps, warmup) if dist.pg else None
    if boxes is not None:
        torch.cuda.synchronize()
        peer.close_mailboxes(dist.pg, dist.rank, boxes)
    per = ms_fused / steps
    gbs = 12.0 * n_total / (per * 1e-3) / 1e9
    local_gbs = 12.0 * n / (per * 1e-3) / 1e9
    vadd_gbs = 12.0 * n / (ms_vadd / steps * 1e-3) / 1e9
    sum_gbs = 4.0 * n / (ms_sum / steps * 1e-3) / 1e9
    pair_gbs = 16.0 * n / ((ms_vadd + ms_sum) / steps * 1e-3) / 1e9
    res = {"workload": "stream", "value": round(gbs, 1), "unit": "GB/s",
           "ms_per_step": round(per, 4), "scaling": "strong",
           "config": {"n": n_total, "n_per_rank": n, "dtype": "f32",
                      "step": "fused vadd+sum kernel; with N > 1 the per-GPU fp64 sums are "
                              "combined inside the kernel through NVLink peer stores"},
           "roofline": {"bound": "hbm", "achieved": round(local_gbs, 1), "peak": pk["hbm"],
                        "unit": "GB/s", "frac": round(local_gbs / pk["hbm"], 4),
                        "bytes_per_elem": 12, "traffic": stream_traffic(n)},
           "separate_kernels": {"vadd_gbs": round(vadd_gbs, 1), "sum_gbs": round(sum_gbs, 1),
                                "pair_gbs_16B": round(pair_gbs, 1),
                                "vadd_frac": round(vadd_gbs / pk["hbm"], 4),
                                "sum_frac": round(sum_gbs / pk["hbm"], 4)},
           "allreduce_us": round(ms_ar / steps * 1e3, 2) if ms_ar is not None else None,
           "nccl_step_ms": round(ms_nccl / steps, 4) if ms_nccl is not None else None,
           "gpu_launches": steps, "sum_check_rel_err": rel,
           "parity": {"check": "every rank's combined sum vs the fp64 sum of c all-reduced "
                               "over the ranks", "max_rel_err_all_ranks": rel, "bar": 1e-6,
                      "ranks": dist.world}}
    del a, b, c
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------- CPU baseline
# The reference's CPU path for each configuration is the demos' host loops,
# restated in the oracle (oracle/oracle.c): fp64 GEMM rows
# (matmul_coopmat_bench.vc:171-176), referenceAttn rows (flash_attn.vc:129-165),
# vadd and the sum (test/vadd.vc:40-43, test/reduce.vc:64-75). Each is timed on
# this box's host cores at 1 thread (the demos' form) and at all threads
# (OpenMP over rows / elements), on a bounded sample of the configuration's
# own work, and extrapolated by the work the sample covers (stated per entry).
def cpu_info():
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    avail = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    return {"cpu_model": model, "nproc": os.cpu_count(), "threads_available": avail}


def _cpu_threads():
    # All host cores this process may run on (torchrun sets OMP_NUM_THREADS=1
    # for its workers; the oracle takes the thread count explicitly).
    return cpu_info()["threads_available"]


def _timed_sample(run, units_min, units_max, target_s):
    """run(units) -> None. Calibrates on units_min, then times calls on as
    many units as target_s allows (at most units_max); a call shorter than
    0.1 s is repeated and averaged. Returns (units, seconds per call)."""
    t0 = time.perf_counter()
    run(units_min)
    dt = time.perf_counter() - t0
    units = int(min(units_max, max(units_min, units_min * target_s / max(dt, 1e-4))))
    est = dt * units / units_min
    reps = 1 if est >= 0.1 else int(min(1000, math.ceil(0.1 / max(est, 1e-5))))
    t0 = time.perf_counter()
    for _ in range(reps):
        run(units)
    return units, (time.perf_counter() - t0) / reps


def _baseline(unit, kind_desc, measure, target_s):
    """measure(threads, target_s) -> (value, sample text, seconds)."""
    threads = _cpu_threads()
    v_all, sample_all, s_all = measure(threads, target_s)
    v_one, sample_one, s_one = measure(1, target_s / 2)
    out = {"value": round(v_all, 6), "unit": unit, "cores": threads, "kind": "port",
           "sample": f"{sample_all}, {s_all:.4g} s per call at {threads} threads; {kind_desc}",
           "threads_1": round(v_one, 6), "threads_1_sample": f"{sample_one}, {s_one:.4g} s per call",
           "seconds": round(s_all + s_one, 2)}
    out.update(cpu_info())
    return out


def cpu_gemm_baseline(target_s=4.0, N=GEMM_N, fp32_inputs=False):
    """fp64 GEMM loop over C's rows (A, B: fp16-rounded U[-1,1), or fp32 for
    the fp32 config); TFLOP/s = 2 * rows * N^2 / seconds."""
    from oracle import oracle
    rng = np.random.default_rng(7)
    a = rng.random((N, N), dtype=np.float32) * 2 - 1
    b = rng.random((N, N), dtype=np.float32) * 2 - 1
    if not fp32_inputs:
        a = a.astype(np.float16).astype(np.float32)
        b = b.astype(np.float16).astype(np.float32)

    def measure(threads, budget):
        rows, dt = _timed_sample(
            lambda r: oracle.gemm(a, b, N, N, N, N, N, True, rows=(0, r), threads=threads),
            max(2, threads), N, budget)
        return 2.0 * rows * N * N / dt / 1e12, f"{rows} of {N} rows of C", dt

    return _baseline("TFLOP/s", f"fp64 loop over {'fp32' if fp32_inputs else 'fp16'} inputs "
                     f"(matmul_coopmat_bench.vc:171-176 form), {N}^3, extrapolated per row",
                     measure, target_s)


def cpu_attention_baseline(BH, N, d, causal, target_s=4.0):
    """referenceAttn (fp64, two passes per row) over a sample of query rows of
    one slice, taken from the end of the slice (the heaviest rows when
    causal), extrapolated to all BH * N rows by the keys each row visits
    (N per row; i + 1 for causal row i). FLOP counted as the configuration
    counts them (4 BH N^2 d; half of it causal)."""
    from oracle import oracle
    rng = np.random.default_rng(9)
    q, k, v = (rng.standard_normal(N * d).astype(np.float32) for _ in range(3))
    out = np.zeros(N * d, np.float32)
    scale = LOG2E / math.sqrt(d)
    job_flop = (2.0 if causal else 4.0) * BH * N * N * d
    keys_all = BH * (N * (N + 1) / 2 if causal else float(N) * N)

    def keys(r0, r1):
        return (r1 * (r1 + 1) - r0 * (r0 + 1)) / 2 if causal else float(r1 - r0) * N

    def measure(threads, budget):
        rows, dt = _timed_sample(
            lambda r: oracle.attention(q, k, v, 1, N, d, scale, causal, row_range=(N - r, N),
                                       threads=threads, out=out),
            min(N, max(4, threads)), N, budget)
        t_full = dt * keys_all / keys(N - rows, N)
        return job_flop / t_full / 1e12, f"the last {rows} of {N} rows of 1 of {BH} slices", dt

    return _baseline("TFLOP/s", f"referenceAttn fp64 rows (flash_attn.vc:129-165), "
                     f"BH={BH} N={N} d={d} causal={int(causal)}, extrapolated by keys visited",
                     measure, target_s)


def cpu_stream_baseline(log2n=30, reps=2):
    """vadd (c = a + b, fp32) then the fp64 sum of c over the whole 2^log2n
    arrays; GB/s at 12 bytes per element (the fused pair's accounting)."""
    from oracle import oracle
    n = 1 << log2n
    a = np.full(n, 0.25, np.float32)
    b = np.full(n, 0.5, np.float32)
    c = np.empty_like(a)
    L = oracle.lib()
    L.oracle_vadd(a.ctypes.data, b.ctypes.data, c.ctypes.data, n, 0)  # first touch, untimed

    def measure(threads, _budget):
        best = None
        for _ in range(reps):
            t0 = time.perf_counter()
            L.oracle_vadd(a.ctypes.data, b.ctypes.data, c.ctypes.data, n, threads)
            L.oracle_sum_f64(c.ctypes.data, n, threads)
            dt = time.perf_counter() - t0
            best = dt if best is None else min(best, dt)
        return 12.0 * n / best / 1e9, f"all {n} elements, best of {reps}", best

    res = _baseline("GB/s", "vadd fp32 + fp64 sum loops (test/vadd.vc:40-43, "
                    "test/reduce.vc:64-75), whole arrays, no extrapolation", measure, 0.0)
    del a, b, c
    return res


def cpu_baselines(workloads):
    """CPU baselines for the configurations the bench ran (rank 0, one GPU)."""
    table = {
        "gemm": lambda: cpu_gemm_baseline(),
        "fa_causal": lambda: cpu_attention_baseline(128, 4096, 128, True),
        "fa_bf16": lambda: cpu_attention_baseline(1024, 8192, 128, False),
        "stream": lambda: cpu_stream_baseline(),
        "fa_f32": lambda: cpu_attention_baseline(1, 256, 64, False, target_s=0.5),
        "gemm_f32": lambda: cpu_gemm_baseline(fp32_inputs=True),
    }
    out = {}
    for name in workloads:
        if name == "gemm_mblock" and "gemm" in out:
            out[name] = out["gemm"]  # the same fp64 GEMM loop, per row
            continue
        if name == "gemm_mblock":
            name_fn = table["gemm"]
            try:
                out[name] = name_fn()
            except Exception as e:
                out[name] = {"error": f"{type(e).__name__}: {e}"}
            continue
        if name in table:
            try:
                out[name] = table[name]()
            except Exception as e:  # report, keep the GPU numbers
                out[name] = {"error": f"{type(e).__name__}: {e}"}
    return out


def reference_arm(args, config):
    """`--impl reference`: the reference's CPU path for the headline (the fp64
    GEMM loop of matmul_coopmat_bench.vc:171-176, restated in the oracle), all
    host threads, on this arm's metric and config. Each step is one bounded
    sample: `rows` rows of C of one 4096^3 product (about 0.4 s of CPU work);
    W samples warm up, K are timed, and the value is the K samples' FLOP over
    their measured time."""
    from oracle import oracle
    N = GEMM_N
    rng = np.random.default_rng(7)
    a = (rng.random((N, N), dtype=np.float32) * 2 - 1).astype(np.float16).astype(np.float32)
    b = (rng.random((N, N), dtype=np.float32) * 2 - 1).astype(np.float16).astype(np.float32)
    threads = _cpu_threads()
    rows, _ = _timed_sample(
        lambda r: oracle.gemm(a, b, N, N, N, N, N, True, rows=(0, r), threads=threads),
        max(2, threads), N, 0.4)
    r0 = [0]

    def sample():
        lo = r0[0] % (N - rows + 1)
        oracle.gemm(a, b, N, N, N, N, N, True, rows=(lo, lo + rows), threads=threads)
        r0[0] += rows

    for _ in range(args.warmup):
        sample()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sample()
    dt = time.perf_counter() - t0
    value = 2.0 * rows * N * N * args.steps / dt / 1e12
    ms = dt / args.steps * 1e3
    base = {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"each step {rows} of {N} rows of C = A*B (4096^3, fp16 inputs), fp64 loop "
                      f"(matmul_coopmat_bench.vc:171-176 form); {args.steps} steps timed in "
                      f"{dt:.2f} s", "seconds": round(dt, 2)}
    base.update(cpu_info())
    cfg = {k: v for k, v in config.items() if k not in ("gemms_per_step", "l2")}
    cfg["step"] = f"one sample: {rows} rows of C of one {N}^3 product"
    return {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic", "config": cfg,
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--only", default="gemm,fa_causal,fa_bf16,stream,fa_f32,gemm_f32,gemm_mblock")
    ap.add_argument("--fa-bf16-heads", type=int, default=32,
                    help="heads of the bf16 attention config (32); a smaller count gives a "
                         "launch small enough for an ncu capture, whose DRAM traffic scales "
                         "with batch x heads")
    ap.add_argument("--stream-log2n", type=int, default=30,
                    help="log2 of the streaming pair's element count (30); a smaller size "
                         "gives a launch small enough for an ncu capture, whose DRAM traffic "
                         "scales with the element count")
    ap.add_argument("--gemms-per-step", type=int, default=GEMMS_PER_STEP,
                    help="GEMM products per step (small values for profiler captures)")
    args = ap.parse_args()
    set_gemms_per_step(args.gemms_per_step)
    dist = Dist()
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 warm-up steps

    config = {"workload": "gemm_f16_4096x4096x4096_fp32out", "M": GEMM_N, "N": GEMM_N,
              "K": GEMM_N, "layout": "row-major A[M][K], B[K][N], C[M][N]",
              "gemms_per_step": GEMMS_PER_STEP,
              "l2": f"inputs rotate over {ROTATE} buffer sets (512 MiB > 126 MB L2)",
              "parallelism": f"weak: {dist.world} rank(s), each the next 4096-row M-block of one "
                             f"({GEMM_N}*{dist.world}) x {GEMM_N} x {GEMM_N} product, B replicated"}

    if args.impl == "reference":
        if dist.rank != 0:
            return
        print(json.dumps(reference_arm(args, config)), flush=True)
        return

    import torch
    torch.cuda.set_device(dist.local)
    dist.init()
    from vkcuda_b200 import vc
    check(vc.vcInit(), "vcInit")
    check(vc.vcSetDevice(dist.local), "vcSetDevice")
    pk = peaks()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dist.local).uuid)
    only = set(args.only.split(","))

    head = gemm_workload(vc, dist, args.steps, args.warmup, pk, uuid) if "gemm" in only else None
    also = []
    jobs = [("fa_causal", lambda: flash_workload(vc, dist, "fa_causal", 8, 16, 4096, 128, True,
                                                 vc.Dtype.F16, max(args.steps, 20), args.warmup, pk,
                                                 shard_bh=False)),
            ("fa_bf16", lambda: flash_workload(vc, dist, "fa_bf16", 32, args.fa_bf16_heads, 8192, 128,
                                               False,
                                               vc.Dtype.BF16, max(3, min(args.steps, 5)),
                                               args.warmup, pk, shard_bh=True)),
            ("stream", lambda: stream_workload(vc, dist, max(args.steps, 10), args.warmup, pk,
                                               args.stream_log2n)),
            ("fa_f32", lambda: flash_workload(vc, dist, "fa_f32", 1, 1, 256, 64, False,
                                              vc.Dtype.F32, max(args.steps, 20), args.warmup, pk,
                                              shard_bh=False)),
            ("gemm_f32", lambda: gemm_f32_workload(vc, dist, max(3, min(args.steps, 10)),
                                                   args.warmup, pk)),
            ("gemm_mblock", lambda: gemm_mblock_workload(vc, dist, max(3, min(args.steps, 10)),
                                                         args.warmup, pk))]
    for name, fn in jobs:
        if name in only:
            try:
                also.append(fn())
            except Exception as e:  # report, keep the headline
                also.append({"workload": name, "error": f"{type(e).__name__}: {e}"})
    kerr = vc.kernel_error(True)

    if dist.rank == 0:
        # CPU baselines on one GPU only (rank 0 of a one-rank job).
        bases = cpu_baselines((["gemm"] if head else []) + [a.get("workload") for a in also]
                              ) if dist.world == 1 else {}
        base = bases.get("gemm")
        for a in also:
            if a.get("workload") in bases:
                a["cpu_baseline"] = bases[a["workload"]]
        line = {"metric": METRIC, "value": head["value"] if head else None, "unit": "TFLOP/s",
                "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": head["ms_per_step"] if head else None,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic (seeded U[-1,1) fp16 inputs)",
                "config": config}
        if head:
            for key in ("ms_per_step_median", "ms_per_step_best", "roofline", "clocks", "e2e",
                        "gpu_launches", "per_launch_ms", "parity"):
                line[key] = head[key]
            line["cpu_baseline"] = base
        line["also"] = also
        line["device_error_word"] = kerr
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.close()


if __name__ == "__main__":
    main()
