"""bench.py's reference arm and its contract with the GPU arm, on the CPU.

The reference arm times the CPU restatement of the reference kernel on the host cores (one
pinned thread per core) and prints one JSON line with the GPU arm's keys; at one GPU both arms
describe the same workload with the same label (same NumPy default_rng(0) inputs), so a
driver comparing the two lines sees the same configuration.
"""

import argparse
import json
import pathlib
import subprocess
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, str(REPO))
    import bench as b

    return b


def test_reference_arm_prints_the_contract_line(oracle):
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "1",
                        "--shape", "256x256x128"], capture_output=True, text=True, timeout=300, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])
    for key in ("metric", "impl", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["steps"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["config"]["err_over_bound"] <= 1.0
    assert "256x256x128" in line["config"]["workload"]


def test_both_arms_share_the_workload_label(bench):
    args = argparse.Namespace(m_total=0, dist="uniform")
    gpu_label = bench.workload_label(args, 1, 2048, 2048, 2048, 2048)
    assert gpu_label == bench.WORKLOAD_LABEL.format(m=2048, n=2048, k=2048)
    assert "default_rng(0)" in gpu_label


def test_pinned_cpus_are_distinct_and_allowed(bench):
    import os

    cpus = bench.pinned_cpus()
    assert cpus and len(set(cpus)) == len(cpus)
    assert set(cpus) <= set(os.sched_getaffinity(0))
    info = bench.host_cpu_info()
    assert info["cpus_allowed"] >= len(cpus)
