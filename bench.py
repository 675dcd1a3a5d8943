#!/usr/bin/env python3
"""Benchmark of the fused relu(A @ B + bias) ("mbr") hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode fp32|tf32|bf16|fp32_exact]
                    [--m M --n N --k K] [--impl ours|reference]

One step = one call of the library's fused operator (tforge_mbr, the C-ABI of
include/tforge.h) on one batch: A (M x K), B (K x N), bias (N) -> out (M x N), f32,
U[-1, 1] synthetic inputs drawn by the reference's generator (NumPy default_rng(0),
tforge_cpu.make_inputs; rank r > 0 draws its A rows from default_rng(r)).  Default
workload: BASELINE config 2, M = N = K = 2048 in the fp32-accurate (3xTF32) mode.  With
N GPUs (torchrun, one rank per GPU, NCCL) each rank owns a 2048-row shard of an
(N * 2048) x 2048 x 2048 problem: B and bias are broadcast once from rank 0 over NCCL
before timing, outputs stay sharded (weak scaling; no collective inside the timed region).

The same run also measures BASELINE config 4 at every N (`config4` in the JSON line,
`--no-config4` skips it): M = 131072 rows in total split over the N GPUs, N = K = 8192,
TF32, A, B ~ N(0, 1/sqrt(K)), bias ~ N(0, 0.1) (device generators), W and bias
NCCL-broadcast once (its first and a repeated broadcast are timed), a few steps timed with
CUDA events per rank (max over ranks), per-rank SM clocks, and an FP64 check of 16 rows
per rank.  NCCL prints its communicator set-up to stderr (NCCL_DEBUG=INFO, subsystem
INIT) unless the caller set NCCL_DEBUG.

Timing: W untimed warm-up steps; then K steps between a barrier + synchronize on both
sides; before every step a 256 MiB buffer is written to flush L2 (126 MB), outside the
step's CUDA-event pair on the launching stream; the step times are summed; the max over
ranks is reported.  `value` = total FLOP of all ranks / that time (2 M N K per call, the
reference's convention, python/tforge_cpu.py:154-157).

Also reported: `roofline` of the GEMM kernel against the measured bf16 peak scaled to the
mode (TF32 = bf16 / 2, 3xTF32 = TF32 / 3); `cpu_baseline` (the CPU restatement of the
reference kernel, pinned to the reference's published numerics, on every host core with
one thread pinned per core, plus the reference's own single-core harness on config 1 and
the host's CPU model); `e2e` through the C-ABI's host-buffer entry (tforge_gemm_host) on
pinned host buffers, with the chunked, overlapped copies in the timed region; `clocks`
sampled through NVML during the timed region.

`--impl reference` times the reference's own CPU implementation of the path (its MLIR
pipeline cannot be built on this image or on the GPU host, so the pinned C restatement
stands in) on all host cores, one pinned thread per core, on the same inputs, and prints
the same JSON keys with "impl": "reference".
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import pathlib
import re
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused MBR TFLOP/s (2048^3 fp32, device-timed), % tensor peak, 1/2/4/8 B200"
FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--mode", default="fp32", choices=["fp32", "tf32", "bf16", "fp32_exact"])
    ap.add_argument("--m", type=int, default=2048, help="rows per GPU (weak scaling)")
    ap.add_argument("--m-total", type=int, default=0,
                    help="total rows split over the GPUs (strong scaling, e.g. 131072 for config 4)")
    ap.add_argument("--dist", default="uniform", choices=["uniform", "normal"],
                    help="uniform: U[-1,1]; normal: A, B ~ N(0, std 1/sqrt(K)), bias ~ N(0, 0.1) (config 4)")
    ap.add_argument("--n", type=int, default=2048)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--shape", default="",
                    help="MxNxK, same as --m/--n/--k (use this form under torchrun, whose own flags "
                         "make --m/--n ambiguous abbreviations)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the BASELINE config-4 measurement (131072x8192x8192 TF32, M-sharded)")
    ap.add_argument("--nccl-debug", default="INFO",
                    help="NCCL_DEBUG level for the communicator set-up lines on stderr (N > 1); off: leave the env")
    args = ap.parse_args()
    if args.shape:
        args.m, args.n, args.k = (int(x) for x in args.shape.lower().split("x"))
    return args


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------- CPU restatement timing
WORKLOAD_LABEL = "mbr relu(A@B+bias) {m}x{n}x{k} f32, A/B/bias U[-1,1] from NumPy default_rng(0) (BASELINE config 2)"


def host_cpu_info() -> dict:
    """CPU model, sockets, cores and SMT of this host (lscpu), and the CPUs this process may use."""
    import subprocess

    info = {"cpus_allowed": host_threads()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=20).stdout
    except (OSError, subprocess.TimeoutExpired):
        return info
    keys = {"Model name": "model", "Socket(s)": "sockets", "Core(s) per socket": "cores_per_socket",
            "Thread(s) per core": "threads_per_core", "CPU(s)": "cpus", "Hypervisor vendor": "hypervisor",
            "L2 cache": "l2", "L3 cache": "l3"}
    for line in out.splitlines():
        key, _, val = line.partition(":")
        if key.strip() in keys:
            info[keys[key.strip()]] = val.strip()
    return info


def pinned_cpus() -> list[int]:
    """One CPU per physical core among those this process may use (the first SMT sibling of each)."""
    allowed = sorted(os.sched_getaffinity(0))
    seen, cpus = set(), []
    for c in allowed:
        sib = pathlib.Path(f"/sys/devices/system/cpu/cpu{c}/topology/thread_siblings_list")
        core = sib.read_text().strip() if sib.exists() else str(c)
        if core not in seen:
            seen.add(core)
            cpus.append(c)
    return cpus


def restatement_runner(ins):
    """(run, rows, out, cpus): one call of the CPU restatement of the reference kernel
    (oracle/, pinned to the reference's published numerics) over all physical cores: one
    worker thread per core, each pinned to its core, each making one single-threaded call on
    its slice of rows -- the way the single-threaded reference kernel would use every core."""
    import concurrent.futures as cf
    import itertools

    import numpy as np

    from tests import oracle_lib

    subprocess_build_oracle()
    a, b, bias = ins["a"], ins["b"], ins["bias"]
    m, k = a.shape
    n = b.shape[1]
    cpus = pinned_cpus()
    out = np.empty((m, n), dtype=np.float32)
    rows = [(i * m // len(cpus), (i + 1) * m // len(cpus)) for i in range(len(cpus))]
    rows = [r for r in rows if r[1] > r[0]]
    slot = itertools.count()

    def pin():  # Linux: sched_setaffinity(0, ...) binds the calling thread only
        os.sched_setaffinity(0, {cpus[next(slot) % len(cpus)]})

    ex = cf.ThreadPoolExecutor(max_workers=len(rows), initializer=pin)

    def part(r):
        r0, r1 = r
        oracle_lib._lib.oracle_gemm(1, a[r0:].ctypes.data, b.ctypes.data, bias.ctypes.data,
                                    out[r0:].ctypes.data, r1 - r0, n, k, 1)

    def run():
        list(ex.map(part, rows))

    return run, rows, out, cpus[:len(rows)]


def cpu_restatement_tflops(ins, seconds=10.0, max_reps=50):
    """Median TFLOP/s of the restatement on all cores over a bounded sample (about `seconds` of CPU time)."""
    m, k = ins["a"].shape
    n = ins["b"].shape[1]
    run, rows, _, cpus = restatement_runner(ins)
    run()  # warm-up (also starts and pins the worker threads)
    times = []
    t_end = time.perf_counter() + seconds / max(1, len(rows))
    while len(times) < max_reps:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 3:
            break
    med = statistics.median(times)
    return 2.0 * m * n * k / med / 1e12, len(rows), len(times), med


def reference_harness_one_core(m, n, k, seed, warmup, reps):
    """The reference's own CPU harness (runners/cpu/tforge-cpu-bench.cpp, built into oracle/_ref/)
    driving the restatement kernel (oracle/build/k_mbr.so, the reference's `_mlir_ciface_entry` ABI)
    on NumPy default_rng(seed) inputs: pinned to one CPU by the harness itself
    (tforge-cpu-bench.cpp:174-186), steady_clock per call, median of `reps` after `warmup`
    (:255-289).  Returns a dict with GFLOP/s, or None where the harness was not built."""
    import subprocess
    import tempfile

    from tensorforge_b200 import tforge_cpu as tc

    harness = ROOT / "oracle" / "_ref" / "tforge-cpu-bench"
    kern = ROOT / "oracle" / "build" / "k_mbr.so"
    if not harness.exists():
        return None
    subprocess_build_oracle()
    ins = tc.make_inputs("mbr", m, n, k, seed)
    with tempfile.TemporaryDirectory() as d:
        for name in ("a", "b", "bias"):
            ins[name].tofile(pathlib.Path(d) / f"{name}.bin")
        cmd = [str(harness), "--lib", str(kern), "--workload", "mbr", "--m", str(m), "--n", str(n), "--k", str(k),
               "--warmup", str(warmup), "--reps", str(reps), "--in-dir", d]
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if r.returncode != 0:
        return {"error": r.stderr.strip()[-200:]}
    j = json.loads(r.stdout)
    return {"shape": f"{m}x{n}x{k}", "seed": seed, "gflops": 2.0 * m * n * k / j["median_ns"],
            "median_ns": j["median_ns"], "warmup": warmup, "reps": reps, "cpu": j["cpu"], "threads": j["threads"]}


def cpu_baseline_leg(ins) -> dict:
    """`cpu_baseline` of the GPU arm (rank 0, N = 1): the all-core figure on the headline
    workload, the reference harness on one core, and the host it ran on."""
    m, k = ins["a"].shape
    n = ins["b"].shape[1]
    v, cores, reps, med = cpu_restatement_tflops(ins)
    one = {f"config1_seed{s}": reference_harness_one_core(256, 256, 128, s, 10, 100) for s in (0, 1234)}
    # Why the per-core figure at 2048^3 is far below config 1's: each 6-row register tile walks a
    # 16-column strip of B down all K rows (one 64-byte line per k, N floats apart), and the next
    # tile walks the next strip, so all of B is re-read for every 6 rows of A.  With B in the
    # core's L2 (config 1: 128 KB; 2048x128x2048: 1 MB) that is cheap; at 2048^3 B is 16 MB and
    # every strip comes from L3.  Same K and M, one core, B of 1 MB versus 16 MB:
    one["config2_2048x2048x2048"] = reference_harness_one_core(2048, 2048, 2048, 0, 1, 3)
    one["b_in_l2_2048x128x2048"] = reference_harness_one_core(2048, 128, 2048, 0, 2, 5)
    return {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"full {m}x{n}x{k} mbr, {reps} timed reps (median {med:.3f} s), {cores} row slices, one "
                      "worker thread pinned per physical core, each one single-threaded call of the C restatement "
                      "of the reference kernel",
            "host": host_cpu_info(),
            "one_core_reference_harness": one,
            "published_one_core": "98.08 GFLOP/s at 256x256x128, seed 1234, one EPYC 9554 core (README.md:90)"}


def reference_arm(args):
    """--impl reference: the reference's CPU implementation of the path on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    from tensorforge_b200 import tforge_cpu as tc

    m = args.m_total if args.m_total else args.m
    n, k = args.n, args.k
    ins = tc.make_inputs("mbr", m, n, k, 0)
    run, rows, out, cpus = restatement_runner(ins)
    for _ in range(args.warmup):
        run()
    step_t = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        step_t.append(time.perf_counter() - t0)
    total = sum(step_t)
    value = 2.0 * m * n * k * args.steps / total / 1e12
    res = tc.check_output("mbr", ins, out, "fp32_exact", rows=np.arange(0, m, max(1, m // 64)))
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": WORKLOAD_LABEL.format(m=m, n=n, k=k),
                       "implementation": "C restatement of the reference's tforge-cpu-pipeline kernel "
                                         "(6x16 register tiles, sequential-k FMA); the MLIR pipeline that "
                                         "generates the real kernel is absent here and on the GPU host",
                       "err_over_bound": res["err_over_bound"], "host": host_cpu_info()},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": len(rows), "kind": "port",
                             "sample": f"the full {m}x{n}x{k} problem per step, {len(rows)} row slices, one "
                                       f"worker thread pinned per physical core (CPUs {cpus}), one "
                                       "single-threaded call each"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def subprocess_build_oracle():
    import subprocess

    if not (ROOT / "oracle" / "build" / "liboracle.so").exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)


# ---------------------------------------------------------------- clocks (NVML)
class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML in a thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.01):
        self.samples, self.period, self.stop_ev = [], period_s, threading.Event()
        self.ok = False
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv, self.h = nv, nv.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: clocks reported as unavailable
            self.err = str(e)
        self.th = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((sm, pw, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.th.start()
        return self

    def __exit__(self, *exc):
        self.stop_ev.set()
        if self.ok:
            self.th.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable: " + self.err}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "power_w_median": statistics.median(s[1] for s in self.samples),
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- roofline inputs
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else {}


def profiled_traffic(kernel: str, mode: str, m: int, n: int, k: int):
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary, or None."""
    path = ROOT / "profiles" / f"gemm_tcgen05_{mode}_mbr_{m}x{n}x{k}.md"
    if not path.exists():
        return None
    mt = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", path.read_text())
    return float(mt.group(1)) if mt else None


# ---------------------------------------------------------------- our arm
def ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from tensorforge_b200 import _lib, tforge_cpu as tc, tforge_gpu as tg

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    L = _lib.lib()
    _lib.check(L.tforge_set_device(local))
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        # NCCL reports its communicator set-up (ranks, devices, NVLink/NVLS, channels) on stderr
        # (`--nccl-debug off` leaves the environment's NCCL_DEBUG settings as they are).
        if args.nccl_debug != "off":
            os.environ.update({"NCCL_DEBUG": args.nccl_debug, "NCCL_DEBUG_SUBSYS": "INIT",
                               "NCCL_DEBUG_FILE": "/dev/stderr"})
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    from tensorforge_b200.shard import broadcast_weights, row_partition

    n, k, mode = args.n, args.k, args.mode
    strong = args.m_total > 0
    if strong:
        r0, r1 = row_partition(args.m_total, world, rank)
        m = r1 - r0
        m_total = args.m_total
    else:
        m, m_total = args.m, args.m * world
    # Inputs: the reference's generator (NumPy default_rng, tforge_cpu.make_inputs), seed 0 on
    # rank 0 -- the reference arm's inputs exactly; rank r > 0 draws its A rows with seed r.
    # B and bias come from rank 0.
    gen = tc.make_inputs_normal if args.dist == "normal" else (lambda mm, nn, kk, seed: tc.make_inputs("mbr", mm, nn, kk, seed))
    host = gen(m, n, k, rank)
    A = torch.from_numpy(host["a"]).to(dev)
    B = torch.from_numpy(host["b"]).to(dev)
    bias = torch.from_numpy(host["bias"]).to(dev)
    del host
    bcast_ms = None
    if world > 1:
        # Communicator and broadcast-channel set-up are not part of the broadcast time: one
        # small broadcast first (NCCL connects a collective's channels on its first use).
        dist.barrier()
        warm = torch.zeros(1 << 18, device=dev)
        dist.broadcast(warm, 0)
        del warm
    torch.cuda.synchronize()
    # Once per weight set, outside the timed region; timed with CUDA events on this rank's
    # stream (the collective's completion is ordered before the second event), max over ranks.
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(torch.cuda.current_stream(dev))
    broadcast_weights(B, bias, src=0)
    b1.record(torch.cuda.current_stream(dev))
    torch.cuda.synchronize()
    if world > 1:
        bt = torch.tensor([b0.elapsed_time(b1)], device=dev, dtype=torch.float64)
        dist.all_reduce(bt, op=dist.ReduceOp.MAX)
        bcast_ms = float(bt.item())
    out = torch.empty((m, n), device=dev, dtype=torch.float32)
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step():
        rc = L.tforge_mbr(A.data_ptr(), B.data_ptr(), bias.data_ptr(), out.data_ptr(), m, n, k,
                          _lib.MODES[mode], sp)
        if rc:
            raise _lib.TforgeError(rc, "tforge_mbr")

    launch = _lib.describe("mbr", m, n, k, mode)
    launches_per_step = 1 + (1 if mode == "bf16" else 0)  # bf16 mode converts A and B first (one launch)

    for _ in range(args.warmup):
        flush.fill_(1.0)
        step()
    torch.cuda.synchronize()
    assert _lib.device_status(sp) == 0

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.fill_(float(i))
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    status = _lib.device_status(sp)
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    flops_rank = 2.0 * m * n * k
    value = 2.0 * m_total * n * k * args.steps / (total_ms * 1e-3) / 1e12

    # Correctness of the timed output (row subset vs FP64, the reference's bound); B and bias
    # as broadcast.
    rows = np.arange(0, m, max(1, m // 64))
    ins = {"a": A.cpu().numpy(), "b": B.cpu().numpy(), "bias": bias.cpu().numpy()}
    res = tc.check_output("mbr", ins, out.cpu().numpy(), mode, rows=rows)

    result = None
    if rank == 0:
        peaks = measured_peaks()
        peak, basis = tg.tensor_roofline_tflops(mode, peaks)
        achieved = flops_rank / (statistics.mean(step_ms) * 1e-3) / 1e12
        traffic = profiled_traffic(launch["kernel"], mode, m, n, k)
        roof = None
        if peak:
            roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic,
                    "kernel": launch["kernel"],
                    "peak_basis": (f"{basis} bf16 GEMM peak {peaks.get('bf16_tflops', 1590.0)} TFLOP/s (burst, "
                                   "MEASURED_PEAKS.json) scaled to the mode: TF32 = bf16/2, 3xTF32 = TF32/3"),
                    "algorithmic_flop_per_launch": flops_rank}
        comparators = cublas_comparator(m, n, k, A, B, bias, flush, stream) if mode in ("fp32", "fp32_exact") else {}
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_baseline_leg(ins)
        e2e = None if args.no_e2e else e2e_measure(L, _lib, m, n, k, mode, A, B, bias, world, dev)
        result = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                  "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
                  "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32",
                  "data": "synthetic",
                  "config": {"workload": workload_label(args, world, m, m_total, n, k),
                             "precision": f"mode {mode}" + (" (3xTF32 split products, f32 accumulate)"
                                                            if mode == "fp32" else ""),
                             "M_total": m_total, "M_rank0": m, "N": n, "K": k, "mode": mode,
                             "l2": "flushed before every step (256 MiB write outside the step's events)",
                             "parallelism": f"M-sharded rows over {world} GPU(s); B and bias NCCL-broadcast once "
                                            "before timing; outputs stay sharded",
                             "kernel": launch["kernel"], "tile": launch["tile"], "stages": launch["stages"],
                             "broadcast_ms": bcast_ms,
                             # the same K steps with the one-time B + bias broadcast counted once
                             "value_including_broadcast_once": (
                                 2.0 * m_total * n * k * args.steps / ((total_ms + bcast_ms) * 1e-3) / 1e12
                                 if bcast_ms is not None else value),
                             "err_over_bound": res["err_over_bound"], "check_pass": bool(res["pass"]),
                             "device_status": status},
                  "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
                  "gpu_launches": launches_per_step * args.steps,
                  "comparators": comparators}
    del A, B, bias, out, flush
    torch.cuda.empty_cache()
    c4 = None if args.no_config4 else config4_leg(L, _lib, tc, world, rank, local, dev)
    if result is not None:
        result["config4"] = c4
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def workload_label(args, world, m, m_total, n, k) -> str:
    if args.m_total:
        return (f"mbr relu(A@B+bias) {m_total}x{n}x{k} f32 split over {world} GPU(s), "
                + ("A,B ~ N(0,1/sqrt(K)), bias ~ N(0,0.1) from NumPy default_rng" if args.dist == "normal"
                   else "A/B/bias U[-1,1] from NumPy default_rng"))
    if world == 1 and args.dist == "uniform":
        return WORKLOAD_LABEL.format(m=m, n=n, k=k)  # the reference arm's label, same inputs
    return (f"mbr relu(A@B+bias) {m}x{n}x{k} f32 per GPU, "
            + ("A,B ~ N(0,1/sqrt(K)), bias ~ N(0,0.1)" if args.dist == "normal" else "A/B/bias U[-1,1]")
            + " from NumPy default_rng(rank) (B and bias from rank 0, broadcast)")


# ---------------------------------------------------------------- BASELINE config 4
C4_M, C4_N, C4_K, C4_MODE = 131072, 8192, 8192, "tf32"


def config4_leg(L, _lib, tc, world, rank, local, dev, target_ms=200.0) -> dict | None:
    """BASELINE config 4 on this run's N GPUs: relu(A @ W + bias), M = 131072 rows in total
    split over the ranks (row_partition), N = K = 8192, TF32; A, W ~ N(0, 1/sqrt(K)), bias ~
    N(0, 0.1) drawn on the device (A per rank with seed 4000 + rank, W and bias on rank 0 with
    seed 4); W and bias NCCL-broadcast from rank 0 -- the first broadcast (the once-per-weight-set
    cost) and a repeated one are both timed.  Steps: enough for about `target_ms` of timed work
    (5 to 50), each timed with CUDA events on the launching stream; value = all rows' FLOP /
    the slowest rank's summed time.  Every rank samples its SM clock during its steps and checks
    16 of its rows against FP64 with the TF32 bound.  Collectives run in the same order on every
    rank; rank 0 returns the object, the others None."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from tensorforge_b200.shard import broadcast_weights, row_partition

    r0, r1 = row_partition(C4_M, world, rank)
    m, n, k = r1 - r0, C4_N, C4_K
    g = torch.Generator(device=dev)
    g.manual_seed(4000 + rank)
    A = torch.empty((m, k), device=dev).normal_(0.0, 1.0 / k ** 0.5, generator=g)
    W = torch.empty((k, n), device=dev)
    bias = torch.empty((n,), device=dev)
    if rank == 0:
        g0 = torch.Generator(device=dev)
        g0.manual_seed(4)
        W.normal_(0.0, 1.0 / k ** 0.5, generator=g0)
        bias.normal_(0.0, 0.1, generator=g0)
    out = torch.empty((m, n), device=dev)
    stream = torch.cuda.current_stream(dev)
    bcast = []
    for _ in range(2):  # the first broadcast of the weight set, then the same again (steady state)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        broadcast_weights(W, bias, src=0)
        b1.record(stream)
        torch.cuda.synchronize()
        bcast.append(b0.elapsed_time(b1))

    def step():
        _lib.check(L.tforge_mbr(A.data_ptr(), W.data_ptr(), bias.data_ptr(), out.data_ptr(), m, n, k,
                                _lib.MODES[C4_MODE], stream.cuda_stream), "tforge_mbr (config 4)")

    est_ms = 2.0 * m * n * k / 650e12 * 1e3
    steps = int(min(50, max(5, round(target_ms / est_ms))))
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with ClockSampler(local, period_s=0.005) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for e0, e1 in evs:  # A (>= 512 MiB per rank) exceeds L2: no flush needed
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
    status = _lib.device_status(stream.cuda_stream)
    ms = sum(a.elapsed_time(b) for a, b in evs)
    sel = np.sort(np.random.default_rng(rank).choice(m, 16, replace=False))
    idx = torch.from_numpy(sel).to(dev)
    res = tc.check_output("mbr", {"a": A[idx].cpu().numpy(), "b": W.cpu().numpy(), "bias": bias.cpu().numpy()},
                          out[idx].cpu().numpy(), C4_MODE)
    launch = _lib.describe("mbr", m, n, k, C4_MODE)
    props = torch.cuda.get_device_properties(dev)
    gpu = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}"
    mine = {"rank": rank, "rows": m, "ms": ms, "broadcast_ms": bcast, "clocks": clk.summary(),
            "err_over_bound": res["err_over_bound"], "pass": bool(res["pass"]), "device_status": status,
            "kernel": launch["kernel"], "gpu_pci": gpu}
    ranks = [None] * world
    if world > 1:
        dist.all_gather_object(ranks, mine)
    else:
        ranks = [mine]
    del A, W, bias, out
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    t_max = max(r["ms"] for r in ranks)
    b_first = max(r["broadcast_ms"][0] for r in ranks) if world > 1 else None
    b_steady = max(r["broadcast_ms"][1] for r in ranks) if world > 1 else None
    flop = 2.0 * C4_M * n * k * steps
    wbytes = (k * n + n) * 4
    return {"workload": f"mbr relu(A@W+bias) {C4_M}x{n}x{k} f32 split over {world} GPU(s), A,W ~ N(0,1/sqrt(K)), "
                        "bias ~ N(0,0.1) (device generators), BASELINE config 4",
            "mode": C4_MODE, "steps": steps, "warmup": 3, "scaling": "strong",
            "value": flop / (t_max * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step_max_rank": t_max / steps,
            "broadcast_ms": b_first, "broadcast_ms_repeat": b_steady,
            "broadcast_gbs": wbytes / (b_first * 1e-3) / 1e9 if b_first else None,
            "broadcast_gbs_repeat": wbytes / (b_steady * 1e-3) / 1e9 if b_steady else None,
            "value_including_broadcast_once": flop / ((t_max + (b_first or 0.0)) * 1e-3) / 1e12,
            "check": "16 rows per rank vs FP64, TF32 bound", "pass": all(r["pass"] and r["device_status"] == 0
                                                                          for r in ranks),
            "max_err_over_bound": max(r["err_over_bound"] for r in ranks),
            "nccl": ".".join(map(str, torch.cuda.nccl.version())) if world > 1 else None,
            "distinct_gpus": len({r["gpu_pci"] for r in ranks}),
            "per_rank": [{"rank": r["rank"], "gpu_pci": r["gpu_pci"], "rows": r["rows"], "ms_per_step": r["ms"] / steps,
                          "sm_mhz": r["clocks"].get("sm_mhz"), "reasons": r["clocks"].get("reasons"),
                          "kernel": r["kernel"]} for r in ranks]}


def cublas_comparator(m, n, k, A, B, bias, flush, stream):
    """The reference's comparator on the same GPU: cuBLAS SGEMM (FP32, no TF32) followed by
    a separate bias + ReLU pass (runners/gpu/tforge-gpu-bench.cu:303-318)."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        C_ = torch.empty((m, n), device=A.device, dtype=torch.float32)

        def run():
            torch.matmul(A, B, out=C_)
            C_.add_(bias).clamp_(min=0.0)

        for _ in range(5):
            run()
        ts = []
        for i in range(20):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        med = statistics.median(ts)
        out = {"cublas_sgemm_plus_bias_relu": {"tflops": 2.0 * m * n * k / (med * 1e-3) / 1e12, "ms": med}}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    out.update(runner_comparators(m, n, k))
    return out


def runner_comparators(m, n, k):
    """More cuBLAS paths through the runner (same GPU, L2 flushed, median of 20): FP32
    emulated on bf16 tensor cores (CUBLAS_COMPUTE_32F_EMULATED_16BFX9), the fp32-accurate
    comparator closest to this mode, and cuBLASLt TF32 with the bias + relu fused into its
    epilogue (TF32 precision, for context)."""
    import subprocess

    runner = pathlib.Path(__file__).resolve().parent / "tensorforge_b200" / "tforge-gpu-bench"
    res = {}
    for key, math in (("cublas_fp32_emulated_bf16x9_plus_bias_relu", "bf16x9"),
                      ("cublaslt_tf32_relu_bias_epilogue", "lt_tf32")):
        cmd = [str(runner), "--mode", "cublas", "--math", math, "--workload", "mbr", "--m", str(m), "--n", str(n),
               "--k", str(k), "--warmup", "5", "--reps", "20", "--flush"]
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
            d = json.loads(r.stdout) if r.returncode == 0 else None
        except (OSError, ValueError, subprocess.TimeoutExpired):
            d = None
        if d:
            res[key] = {"tflops": d["tflops"], "ms": d["median_ms"], "kernel": d["kernel"]}
    return res


def e2e_measure(L, _lib, m, n, k, mode, A, B, bias, world, dev, steps=20, warmup=3):
    """The same operator through the C-ABI on HOST buffers (tforge_gemm_host): A, B and bias
    in page-locked host memory are copied in, the fused kernel runs per row chunk as the
    chunk lands, and out is copied back per chunk, all inside the timed region (CUDA events
    on the caller's stream, which the call joins)."""
    import torch

    hA, hB, hb = A.cpu().pin_memory(), B.cpu().pin_memory(), bias.cpu().pin_memory()
    hO = torch.empty((m, n), dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    h2d = hA.numel() * 4 + hB.numel() * 4 + hb.numel() * 4
    d2h = hO.numel() * 4

    def one():
        _lib.gemm_host("mbr", hA.data_ptr(), hB.data_ptr(), hO.data_ptr(), m, n, k, mode,
                       bias=hb.data_ptr(), stream=sp)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"value": 2.0 * m * n * k / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "steps": steps,
            "h2d_plus_d2h_gbs": (h2d + d2h) / (ms * 1e-3) / 1e9,
            "path": "tforge_gemm_host (pinned host A, B, bias, out; B first, A in row chunks, "
                    "per-chunk kernels and copy-back overlapped), rank 0"}


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    return ours(args)


if __name__ == "__main__":
    sys.exit(main())
