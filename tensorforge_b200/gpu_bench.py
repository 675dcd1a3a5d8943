#!/usr/bin/env python3
"""Check, then time, the library's GPU operators over workloads x shapes x variants.

The reference's GPU driver (bench/gpu_bench.py:33-103) on this library: every
(variant, workload, shape) is first checked against FP64 with the reference's bound and
compared with cuBLAS on the same inputs, then timed by the runner (CUDA events, NVML
clock), and written as one CSV row with the provenance columns.  A variant is
`NAME=OPTIONS`, the options being the library's (`precision=fp32|tf32|bf16|fp32_exact`,
`bn=`, `stages=`), in place of the reference's MLIR pipeline options.

    python -m tensorforge_b200.gpu_bench --csv results/gpu/b200.csv --tag r1 \\
        --variant fp32="precision=fp32" --variant tf32="precision=tf32" --cublas \\
        --workloads matmul,mbr,matmul_add --shapes 512x512x512,2048x2048x2048
"""

from __future__ import annotations

import argparse
import sys

import numpy as np

from . import provenance
from . import tforge_cpu as tc
from . import tforge_gpu as tg

SHAPES = [(256, 256, 256), (512, 512, 512), (1024, 1024, 1024), (2048, 2048, 2048),
          (4096, 4096, 4096), (1000, 1000, 1000), (777, 1111, 333)]
# squares plus the two skinny shapes.
SWEEP_SHAPES = [(512, 512, 512), (1024, 1024, 1024), (4096, 4096, 4096), (8192, 8192, 8192),
                (8192, 4096, 1024), (256, 16384, 4096)]


def parse_shapes(text: str):
    return [tuple(int(x) for x in s.split("x")) for s in text.split(",") if s]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--csv", default="")
    ap.add_argument("--tag", default="default")
    ap.add_argument("--variant", action="append", default=[], help="NAME=OPTIONS (repeatable)")
    ap.add_argument("--workloads", default="matmul,mbr")
    ap.add_argument("--shapes", default="", help="MxNxK,... (default: the reference's shape list)")
    ap.add_argument("--sweep", action="store_true", help="BASELINE config 3 shapes")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--reps", type=int, default=100)
    ap.add_argument("--flush", action="store_true")
    ap.add_argument("--cublas", action="store_true", help="also time cuBLAS (+ separate epilogue)")
    ap.add_argument("--check-only", action="store_true")
    args = ap.parse_args(argv)

    variants = [v.split("=", 1) if "=" in v else (v, "") for v in args.variant] or [("fp32", "precision=fp32")]
    shapes = parse_shapes(args.shapes) if args.shapes else (SWEEP_SHAPES if args.sweep else SHAPES)
    base = provenance.common()
    out = None if (args.check_only or not args.csv) else provenance.CsvWriter(args.csv)
    failures = 0
    for workload in args.workloads.split(","):
        for m, n, k in shapes:
            gemm = workload in ("matmul", "mbr", "matmul_add")
            flops = 2.0 * m * n * k if gemm else 0.0
            # Above 2^33 multiply-adds the FP64 reference is checked on 64 seeded rows.
            rows_sel = (np.sort(np.random.default_rng(0).choice(m, 64, replace=False))
                        if gemm and m * n * k > (1 << 33) else None)
            ins = tc.make_inputs(workload, m, n, k, 1234)
            ref_cublas = tg.check(workload, m, n, k, mode="cublas", ins=ins, rows=rows_sel)[1] if gemm else None
            rows = [(name, opts, "kernel") for name, opts in variants]
            if args.cublas and gemm:
                rows.append(("cublas", "", "cublas"))
            for name, opts, mode in rows:
                kdir = launch = None
                if mode == "kernel":
                    kdir, launch = tg.compile_kernel(workload, m, n, k, opts, tag=f"{args.tag}/{name}")
                chk, got = tg.check(workload, m, n, k, kdir, launch, mode, ins=ins, rows=rows_sel)
                diff = (float(np.nanmax(np.abs(got.astype(np.float64) - ref_cublas)))
                        if ref_cublas is not None and got.size else 0.0)
                status = "PASS" if chk["pass"] else "FAIL"
                print(f"[{status}] {name:>12} {workload:>10} {m}x{n}x{k:<6} err/bound={chk['err_over_bound']:.3g} "
                      f"max|x-cublas|={diff:.3g}", flush=True)
                if not chk["pass"]:
                    failures += 1
                    continue
                if args.check_only:
                    continue
                r = tg.bench(workload, m, n, k, kdir, launch, mode, args.warmup, args.reps, args.flush)
                if not gemm:  # elementwise: bytes moved, the reference's GB/s metric
                    metric, work = tc.flops_or_bytes(workload, m, n, k)
                    gbs = work / (r["median_ms"] * 1e-3) / 1e9
                    print(f"        median {r['median_ms']:.4f} ms  {gbs:.1f} {metric}", flush=True)
                    if out is not None:
                        out.row(**base, device=r["gpu"], workload=workload, shape=f"{m}x{n}", dtype="f32",
                                pipeline=r["kernel"], params=name, threads="", warmup=r["warmup"], reps=r["reps"],
                                median_ms=r["median_ms"], min_ms=r["min_ms"], std_ms=r["std_ms"], metric=metric,
                                metric_value=gbs, sm_clock_median_mhz=r["sm_clock_median_mhz"],
                                clock_adjusted_metric="", alloc_bytes_per_call=0,
                                correctness="bit-exact" if chk["pass"] else "mismatch",
                                notes=f"l2_flush={r['l2_flush']}")
                    continue
                gflops = flops / (r["median_ms"] * 1e-3) / 1e9
                clk = r["sm_clock_median_mhz"]
                prec = (launch or {}).get("precision", "fp32") if mode == "kernel" else "fp32"
                roof, basis = tg.tensor_roofline_tflops(prec) if mode == "kernel" else (None, "")
                adj = (f"{100.0 * gflops / 1e3 / roof:.1f}% of {prec} tensor roofline ({basis})" if roof
                       else f"{100.0 * gflops / tg.fp32_peak_gflops(clk):.1f}% of FP32 SIMT peak at median clock"
                       if clk > 0 else "")
                pipeline = (f"{r['kernel']} {opts}" if mode == "kernel" else
                            "cublasSgemm FP32 default math" + (" + bias_relu kernel" if workload == "mbr" else ""))
                params = (f"{name}; grid={r['grid']} block={r['block']} tile={r.get('tile', '')} "
                          f"stages={r.get('stages', '')}; regs={r['regs']} dyn_smem={r.get('dyn_smem', '')}")
                print(f"        median {r['median_ms']:.4f} ms  {gflops / 1e3:.2f} TFLOP/s  {adj}", flush=True)
                if out is not None:
                    out.row(**base, device=r["gpu"], workload=workload, shape=f"{m}x{n}x{k}", dtype="f32",
                            pipeline=pipeline, params=params, threads="", warmup=r["warmup"], reps=r["reps"],
                            median_ms=r["median_ms"], min_ms=r["min_ms"], std_ms=r["std_ms"], metric="GFLOP/s",
                            metric_value=gflops, sm_clock_median_mhz=clk, clock_adjusted_metric=adj,
                            alloc_bytes_per_call=0,
                            correctness=(f"err/bound={chk['err_over_bound']:.3g}; max|x-cublas|={diff:.3g}"
                                         + ("; FP64 check on 64 seeded rows" if rows_sel is not None else "")),
                            notes=(f"l2_flush={r['l2_flush']}; sm_clock {r['sm_clock_min_mhz']}-"
                                   f"{r['sm_clock_max_mhz']} MHz; power {r['power_median_w']} W; "
                                   f"driver {r['cuda_driver']}"))
    print(f"failures: {failures}")
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
