"""Provenance columns shared by every results CSV row.

The column set is the reference's (python/provenance.py:11-16) so that its summary tools
read these CSVs unchanged; `mlir_llvm_version` records "none" (no MLIR toolchain is
involved on this path).
"""

from __future__ import annotations

import csv
import datetime
import os
import pathlib
import subprocess

ROOT = pathlib.Path(__file__).resolve().parent.parent

FIELDS = [
    "commit", "mlir_llvm_version", "cuda_version", "device", "job_id", "date",
    "workload", "shape", "dtype", "pipeline", "params", "threads", "warmup", "reps",
    "median_ms", "min_ms", "std_ms", "metric", "metric_value", "sm_clock_median_mhz",
    "clock_adjusted_metric", "alloc_bytes_per_call", "correctness", "notes",
]


def _run(args: list[str]) -> str:
    try:
        return subprocess.run(args, capture_output=True, text=True, timeout=30).stdout.strip()
    except (OSError, subprocess.SubprocessError):
        return ""


def git_commit() -> str:
    sha = _run(["git", "-C", str(ROOT), "rev-parse", "--short", "HEAD"])
    dirty = _run(["git", "-C", str(ROOT), "status", "--porcelain", "--untracked-files=no"])
    return sha + ("-dirty" if sha and dirty else "")


def cuda_version() -> str:
    out = _run(["nvcc", "--version"])
    for tok in out.replace(",", " ").split():
        if tok[:1].isdigit() and "." in tok and tok.count(".") == 1:
            return tok
    return ""


def common() -> dict:
    """The per-run provenance columns."""
    return {
        "commit": git_commit(),
        "mlir_llvm_version": "none",
        "cuda_version": cuda_version(),
        "job_id": os.environ.get("SLURM_JOB_ID", "none"),
        "date": datetime.datetime.now().astimezone().isoformat(timespec="seconds"),
    }


def cpu_model() -> str:
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return ""


class CsvWriter:
    """Appends rows with exactly FIELDS; the header is written only for a new file."""

    def __init__(self, path):
        self.path = pathlib.Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        new = not self.path.exists() or self.path.stat().st_size == 0
        self._f = open(self.path, "a", newline="")
        self._w = csv.DictWriter(self._f, fieldnames=FIELDS)
        if new:
            self._w.writeheader()

    def row(self, **kw) -> None:
        unknown = set(kw) - set(FIELDS)
        if unknown:
            raise KeyError(sorted(unknown))
        self._w.writerow(kw)
        self._f.flush()

    def close(self) -> None:
        self._f.close()
