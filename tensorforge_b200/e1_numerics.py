#!/usr/bin/env python3
"""Numerics of the precision modes against FP64 (the reference's E1 study, on B200).

For relu(A @ B + bias) and matmul on the reference's E1 shapes (bench/e1_numerics.py:33)
and its inputs (seed 1234), every variant runs on the same inputs and reports
max |x - x64|, RMS, err/bound with the reference's bound gamma_{K+1}(|A||B|+|bias|)
(bench/e1_numerics.py:68-74), err/bound against the mode's stated bound, and the fraction
of outputs that differ bitwise from `fp32_exact` (sequential-k FFMA: the reference's
generated kernels, docs/numerics.md:3,53).

Variants: fp32_exact, fp32 (3xTF32), tf32, bf16 (this library), cuBLAS SGEMM (+ bias/relu),
NumPy float32 (1 thread).

    python -m tensorforge_b200.e1_numerics [--csv out.csv] [--shapes 256x256x256,...]
"""

from __future__ import annotations

import argparse
import csv
import os
import sys

os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")

import numpy as np  # noqa: E402

from . import provenance  # noqa: E402
from . import tforge_cpu as tc  # noqa: E402
from . import tforge_gpu as tg  # noqa: E402

SHAPES = [(256, 256, 256), (1000, 1000, 1000), (777, 1111, 333), (512, 512, 4096)]
MODES = ["fp32_exact", "fp32", "tf32", "bf16"]
COLUMNS = ["commit", "cuda_version", "date", "workload", "shape", "variant", "max_abs_err", "rms_err",
           "err_over_bound_fp32", "err_over_bound_mode", "bitwise_diff_vs_fp32_exact", "bitwise_diff_fraction"]


def run(shapes, workloads=("mbr", "matmul")):
    base = provenance.common()
    rows = []
    for workload in workloads:
        for m, n, k in shapes:
            ins = tc.make_inputs(workload, m, n, k, 1234)
            outs = []
            for mode in MODES:
                outs.append((mode, mode, tg.run_op(workload, ins, m, n, k, mode)))
            _, ob = tg.check(workload, m, n, k, mode="cublas", ins=ins)
            outs.append(("cublas", "fp32", ob))
            npo = ins["a"] @ ins["b"]
            if workload == "mbr":
                npo = np.maximum(npo + ins["bias"], np.float32(0))
            outs.append(("numpy", "fp32", npo.astype(np.float32)))
            exact = outs[0][2].view(np.uint32)
            for name, mode, o in outs:
                r32 = tc.check_output(workload, ins, o, "fp32")
                rmode = tc.check_output(workload, ins, o, mode)
                diff = int(np.count_nonzero(o.view(np.uint32) != exact))
                rows.append({**{c: base.get(c, "") for c in ("commit", "cuda_version", "date")},
                             "workload": workload, "shape": f"{m}x{n}x{k}", "variant": name,
                             "max_abs_err": f"{r32['max_abs_err']:.4g}", "rms_err": f"{r32['rms_err']:.4g}",
                             "err_over_bound_fp32": f"{r32['err_over_bound']:.4g}",
                             "err_over_bound_mode": f"{rmode['err_over_bound']:.4g}",
                             "bitwise_diff_vs_fp32_exact": diff,
                             "bitwise_diff_fraction": f"{diff / o.size:.4f}"})
                print(f"{workload} {m}x{n}x{k} {name:>10}: max_err={r32['max_abs_err']:.3g} "
                      f"err/bound(fp32)={r32['err_over_bound']:.3g} err/bound({mode})={rmode['err_over_bound']:.3g} "
                      f"bitwise-diff={diff / o.size:.3f}", flush=True)
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--csv", default="")
    ap.add_argument("--shapes", default="")
    args = ap.parse_args(argv)
    shapes = [tuple(int(x) for x in s.split("x")) for s in args.shapes.split(",") if s] or SHAPES
    rows = run(shapes)
    if args.csv:
        with open(args.csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=COLUMNS)
            w.writeheader()
            w.writerows(rows)
    return 0


if __name__ == "__main__":
    sys.exit(main())
