"""Regenerate tests/golden/golden.json from the reference tree (run where it exists).

    python tests/golden/make_golden.py --reference <reference tree>   (or TF_REFERENCE=<tree>)

What it records, and from where:

* ``e1_pins``: the reference's published numerics (results/numerics/e1.csv): per
  workload and shape, max |x - x64| and max err/bound of the sequential-k FMA variant
  (``cpu-vec-kr4``, bitwise identical to the reference's GPU kernels, docs/numerics.md:3)
  and of the unfused ``cpu-scalar`` variant.  Inputs: the reference generator, seed 1234.
* ``readme_pin``: README.md:90, mbr 256x256x128 seed 1234: err/bound 0.0237, max_abs 5.98e-06.
* ``inputs``: sha256 of the reference's own ``make_inputs`` (python/tforge_cpu.py:89-100),
  imported from the reference tree, for several workloads, shapes and seeds.
* ``reference_check``: the reference's own ``tforge_cpu.check`` (FP64 bound), driving the
  reference's own CPU harness (runners/cpu/tforge-cpu-bench.cpp, built by
  ``make -C oracle ref``) with the CPU restatement ``oracle/build/k_<workload>.so``.
* ``provenance_fields``: the reference's CSV schema (python/provenance.py:11-16).
* ``outputs``: sha256 of the harness's output bytes for small cases, plus the full
  output of a tiny case, so CPU tests can check the restatement without the reference.

Nothing at test time reads the reference tree: the tests read only this JSON.
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import json
import os
import pathlib
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent


def sha(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TF_REFERENCE"),
                    help="the reference source tree (default: $TF_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <reference tree> or set TF_REFERENCE")
    ref = pathlib.Path(args.reference)
    sys.path.insert(0, str(ref / "python"))
    import tforge_cpu as rtc  # the reference's host library (imports only numpy)

    subprocess.run(["make", "-C", str(REPO / "oracle"), "all", "ref", f"REF={ref}"], check=True,
                   capture_output=True)
    rtc.BENCH = REPO / "oracle" / "_ref" / "tforge-cpu-bench"

    def kdir(workload):
        d = pathlib.Path(tempfile.mkdtemp())
        shutil.copy(REPO / "oracle" / "build" / f"k_{workload}.so", d / "k.so")
        return d

    golden: dict = {"source": "the reference tree (NirakChoun/TensorForge sources; values below are copied from it)"}

    # Published E1 numerics.
    pins = []
    with open(ref / "results" / "numerics" / "e1.csv") as f:
        for r in csv.DictReader(f):
            if r["variant"] in ("cpu-vec-kr4", "cpu-scalar"):
                pins.append({"workload": r["workload"], "shape": [int(x) for x in r["shape"].split("x")],
                             "variant": "fma" if r["variant"] == "cpu-vec-kr4" else "scalar",
                             "max_abs_err": r["max_abs_err"], "rms_err": r["rms_err"],
                             "err_over_bound": r["max_err_over_bound"],
                             "cite": "results/numerics/e1.csv"})
    golden["e1_pins"] = pins
    golden["readme_pin"] = {"workload": "mbr", "shape": [256, 256, 128], "seed": 1234,
                            "err_over_bound": "0.0237", "max_abs_err": "5.98e-06", "cite": "README.md:90"}

    # The reference generator's inputs.
    cases = [("mbr", 256, 256, 128, 1234), ("mbr", 256, 256, 128, 0), ("matmul", 33, 17, 9, 1234),
             ("mbr", 777, 1111, 333, 1234), ("add", 33, 17, None, 1234), ("relu", 33, 17, None, 1234),
             ("bias_add", 33, 17, None, 1234), ("mbr", 2048, 2048, 2048, 0)]
    golden["inputs"] = []
    for w, m, n, k, s in cases:
        ins = rtc.make_inputs(w, m, n, k, s)
        golden["inputs"].append({"workload": w, "m": m, "n": n, "k": k, "seed": s,
                                 "sha256": {name: sha(a) for name, a in ins.items()}})

    # The reference's own check through the reference's own harness.
    golden["reference_check"] = []
    for w, m, n, k, s in [("mbr", 256, 256, 128, 1234), ("mbr", 256, 256, 128, 0),
                          ("matmul", 256, 256, 256, 1234), ("mbr", 777, 1111, 333, 1234)]:
        res = rtc.check(w, m, n, k, kdir(w), seed=s)
        golden["reference_check"].append({"workload": w, "m": m, "n": n, "k": k, "seed": s,
                                          "err_over_bound": res["err_over_bound"],
                                          "max_abs_err": res["max_abs_err"], "pass": res["pass"]})

    # Harness outputs (restatement driven by the reference harness).
    golden["outputs"] = []
    for w, m, n, k, s in [("mbr", 256, 256, 128, 1234), ("mbr", 256, 256, 128, 0),
                          ("matmul", 33, 17, 9, 1234), ("mbr", 7, 19, 5, 1234), ("add", 33, 17, None, 1234),
                          ("relu", 33, 17, None, 1234)]:
        ins = rtc.make_inputs(w, m, n, k, s)
        with tempfile.TemporaryDirectory() as td:
            for name, arr in ins.items():
                arr.tofile(f"{td}/{name}.bin")
            subprocess.run([str(rtc.BENCH), "--lib", str(kdir(w) / "k.so"), "--workload", w, "--m", str(m),
                            "--n", str(n), "--k", str(k or 0), "--warmup", "0", "--reps", "1", "--in-dir", td,
                            "--out", f"{td}/o.bin"], check=True, capture_output=True)
            out = np.fromfile(f"{td}/o.bin", dtype=np.float32).reshape(m, n)
        entry = {"workload": w, "m": m, "n": n, "k": k, "seed": s, "sha256": sha(out)}
        if m * n <= 200:
            entry["values_hex"] = [format(int(v), "08x") for v in out.view(np.uint32).ravel()]
        golden["outputs"].append(entry)

    import provenance as rprov  # the reference's CSV schema (python/provenance.py:11-16)

    golden["provenance_fields"] = list(rprov.FIELDS)

    (HERE / "golden.json").write_text(json.dumps(golden, indent=1) + "\n")
    print("wrote", HERE / "golden.json")
    return 0


if __name__ == "__main__":
    sys.exit(main())
