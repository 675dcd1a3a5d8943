"""The CPU restatement (oracle/) pinned against the reference's published numbers.

Every pin comes from tests/golden/golden.json, generated from the reference tree by
tests/golden/make_golden.py: README.md:90 (mbr 256x256x128), results/numerics/e1.csv
(mbr and matmul at 256^3, 1000^3, 777x1111x333, 512x512x4096 for the sequential-k FMA
and the unfused scalar variants), the reference generator's input hashes and the
reference harness's output bytes.
"""

import hashlib
import json
import pathlib

import numpy as np
import pytest

from tensorforge_b200 import tforge_cpu as tc

GOLDEN = json.loads((pathlib.Path(__file__).parent / "golden" / "golden.json").read_text())


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_readme_pin(oracle):
    p = GOLDEN["readme_pin"]
    m, n, k = p["shape"]
    ins = tc.make_inputs("mbr", m, n, k, p["seed"])
    res = tc.check_output("mbr", ins, oracle.gemm("mbr", ins))
    assert f"{res['err_over_bound']:.3g}" == p["err_over_bound"]
    assert f"{res['max_abs_err']:.3g}" == p["max_abs_err"]
    assert res["pass"]


@pytest.mark.parametrize("pin", GOLDEN["e1_pins"],
                         ids=lambda p: f"{p['workload']}-{'x'.join(map(str, p['shape']))}-{p['variant']}")
def test_e1_pins(oracle, pin):
    m, n, k = pin["shape"]
    ins = tc.make_inputs(pin["workload"], m, n, k, 1234)
    out = oracle.gemm(pin["workload"], ins, fma=pin["variant"] == "fma")
    res = tc.check_output(pin["workload"], ins, out)
    assert f"{res['max_abs_err']:.4g}" == pin["max_abs_err"]
    assert f"{res['err_over_bound']:.4g}" == pin["err_over_bound"]
    assert f"{res['rms_err']:.4g}" == pin["rms_err"]


@pytest.mark.parametrize("case", GOLDEN["reference_check"], ids=lambda c: f"{c['workload']}-{c['m']}x{c['n']}x{c['k']}-s{c['seed']}")
def test_reference_check_values(oracle, case):
    """The reference's own check() on its own harness gave these; the restatement agrees."""
    ins = tc.make_inputs(case["workload"], case["m"], case["n"], case["k"], case["seed"])
    res = tc.check_output(case["workload"], ins, oracle.gemm(case["workload"], ins))
    assert res["err_over_bound"] == pytest.approx(case["err_over_bound"], rel=1e-12)
    assert res["max_abs_err"] == pytest.approx(case["max_abs_err"], rel=1e-12)


@pytest.mark.parametrize("case", GOLDEN["inputs"], ids=lambda c: f"{c['workload']}-{c['m']}x{c['n']}-s{c['seed']}")
def test_make_inputs_matches_reference_generator(case):
    ins = tc.make_inputs(case["workload"], case["m"], case["n"], case["k"], case["seed"])
    assert {k: sha(v) for k, v in ins.items()} == case["sha256"]


@pytest.mark.parametrize("case", GOLDEN["outputs"], ids=lambda c: f"{c['workload']}-{c['m']}x{c['n']}-s{c['seed']}")
def test_outputs_match_reference_harness(oracle, case):
    w = case["workload"]
    ins = tc.make_inputs(w, case["m"], case["n"], case["k"], case["seed"])
    out = oracle.gemm(w, ins) if w in tc.GEMM_WORKLOADS else oracle.elementwise(w, ins)
    assert sha(out) == case["sha256"]
    if "values_hex" in case:
        assert [format(int(v), "08x") for v in out.view(np.uint32).ravel()] == case["values_hex"]


@pytest.mark.parametrize("shape", [(1, 1, 1), (7, 19, 5), (13, 35, 9), (6, 16, 4), (12, 32, 8), (5, 3, 0),
                                   (0, 4, 4), (37, 50, 131)])
@pytest.mark.parametrize("workload", ["matmul", "mbr", "matmul_add"])
def test_tiled_equals_scalar_fma_loop(oracle, workload, shape):
    """docs/numerics.md:3,53: tiling does not change bits; sequential-k FMA is the target."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 7)
    a = oracle.gemm(workload, ins)
    b = oracle.gemm(workload, ins, naive=True)
    assert a.view(np.uint32).tobytes() == b.view(np.uint32).tobytes()


def test_relu_known_answers(oracle):
    """test/Transforms/canonicalize.mlir:90-100: relu of [-1, -0, NaN, 2.5, 0]."""
    a = np.array([[-1.0, -0.0, np.nan, 2.5, 0.0]], dtype=np.float32)
    out = oracle.elementwise("relu", {"a": a})
    assert out.view(np.uint32).tolist() == [[0, 0, 0x7FC00000, np.float32(2.5).view(np.uint32), 0]]
    # tforge_cpu's bit-exact check uses the same semantics.
    assert tc.check_elementwise("relu", {"a": a}, out)["pass"]


def test_bias_add_relu_known_answer(oracle):
    """test/Transforms/canonicalize.mlir:104-116: relu([[1,2],[3,4]] + [10,-20])."""
    a = np.array([[1.0, 2.0], [3.0, 4.0]], dtype=np.float32)
    b = np.array([10.0, -20.0], dtype=np.float32)
    y = oracle.elementwise("bias_add", {"a": a, "bias": b})
    z = oracle.elementwise("relu", {"a": y})
    assert z.tolist() == [[11.0, 0.0], [13.0, 0.0]]
    # The fused path: identity weights make A @ B = A.
    fused = oracle.gemm("mbr", {"a": a, "b": np.eye(2, dtype=np.float32), "bias": b})
    assert fused.tolist() == [[11.0, 0.0], [13.0, 0.0]]


def test_planted_error_is_caught(oracle):
    """The check rejects an output with one element off by far more than the bound."""
    ins = tc.make_inputs("mbr", 64, 48, 32, 3)
    out = oracle.gemm("mbr", ins)
    assert tc.check_output("mbr", ins, out)["pass"]
    bad = out.copy()
    bad[5, 7] += 1e-3
    assert not tc.check_output("mbr", ins, bad)["pass"]
    nan = out.copy()
    nan[0, 0] = np.nan
    assert not tc.check_output("mbr", ins, nan)["pass"]
