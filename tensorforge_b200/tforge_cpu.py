"""Workload inputs, the FP64 error-bound check and the work metric (host side, NumPy).

Mirrors python/tforge_cpu.py of the reference:

* ``make_inputs`` draws exactly the reference's inputs: NumPy ``default_rng(seed)``,
  U[-1, 1] in float32, in the order a, b, bias (python/tforge_cpu.py:89-100).  The new
  ``matmul_add`` workload draws its residual ``c`` after ``b``.
* ``check_output`` is the reference's FP64 check (python/tforge_cpu.py:103-145,
  python/tforge_gpu.py:134-144, bench/e1_numerics.py:68-74):
  ``|out - ref64| <= gamma_{K+1} (|A||B| + |bias|)``, ``gamma_j = j u / (1 - j u)``,
  ``u = 2^-24``, plus float32 ``tiny``; pass = err/bound <= 1 and no NaN.  For the
  tensor-core input roundings (TF32, BF16) the stated looser bound adds the input
  rounding term ``(2 u_in + u_in^2) |A||B|`` with u_in the unit roundoff of the input
  conversion.
* ``flops_or_bytes`` is the reference's work metric (python/tforge_cpu.py:154-159):
  2 M N K FLOP for GEMM workloads (the epilogue is not counted).
"""

from __future__ import annotations

import numpy as np

F32_EPS = 2.0 ** -24  # unit roundoff of f32, round to nearest
F32_TINY = float(np.finfo(np.float32).tiny)

# Unit roundoff of the operand rounding each precision mode applies before the products.
#   tf32: the tensor core reads f32 operands as TF32 (10 explicit mantissa bits); the
#         hardware discards the low 13 bits, so the stated bound uses the truncation
#         figure u_in = 2^-10 (2^-11 would hold for round-to-nearest).
#   bf16: operands are rounded to nearest bf16 (7 explicit bits), u_in = 2^-8.
INPUT_UNIT = {"fp32": 0.0, "fp32_exact": 0.0, "tf32": 2.0 ** -10, "bf16": 2.0 ** -8}

GEMM_WORKLOADS = ("matmul", "mbr", "matmul_add")


def make_inputs(workload: str, m: int, n: int, k: int | None, seed: int = 1234) -> dict:
    """Inputs of one workload, bit-identical to the reference generator for its workloads."""
    rng = np.random.default_rng(seed)

    def u(*s):
        return rng.uniform(-1.0, 1.0, size=s).astype(np.float32)

    if workload == "add":
        return {"a": u(m, n), "b": u(m, n)}
    if workload == "relu":
        return {"a": u(m, n)}
    if workload == "bias_add":
        return {"a": u(m, n), "bias": u(n)}
    if workload == "matmul":
        return {"a": u(m, k), "b": u(k, n)}
    if workload == "matmul_add":
        return {"a": u(m, k), "b": u(k, n), "c": u(m, n)}
    if workload == "mbr":
        return {"a": u(m, k), "b": u(k, n), "bias": u(n)}
    raise ValueError(workload)


def make_inputs_normal(m: int, n: int, k: int, seed: int = 0) -> dict:
    """Large M-sharded MBR inputs: A, B ~ N(0, std 1/sqrt(K)), bias ~ N(0, std 0.1), f32."""
    rng = np.random.default_rng(seed)
    s = 1.0 / np.sqrt(k)
    return {"a": rng.normal(0.0, s, size=(m, k)).astype(np.float32),
            "b": rng.normal(0.0, s, size=(k, n)).astype(np.float32),
            "bias": rng.normal(0.0, 0.1, size=n).astype(np.float32)}


def make_mlp_inputs(m: int, d: int, h: int, seed: int = 0) -> dict:
    """Two-layer MLP: X U[-1,1] (m x d); Xavier-uniform W1 (d x h), W2 (h x d),
    U(+-sqrt(6 / (fan_in + fan_out))); biases N(0, std 0.02)."""
    rng = np.random.default_rng(seed)
    lim = np.sqrt(6.0 / (d + h))
    return {"x": rng.uniform(-1.0, 1.0, size=(m, d)).astype(np.float32),
            "w1": rng.uniform(-lim, lim, size=(d, h)).astype(np.float32),
            "b1": rng.normal(0.0, 0.02, size=h).astype(np.float32),
            "w2": rng.uniform(-lim, lim, size=(h, d)).astype(np.float32),
            "b2": rng.normal(0.0, 0.02, size=d).astype(np.float32)}


def reference64(workload: str, ins: dict, rows=None):
    """FP64 result and |A||B| (+|bias| or +|C_res|) magnitude, optionally on a row subset."""
    a = ins["a"] if rows is None else ins["a"][rows]
    a64, b64 = a.astype(np.float64), ins["b"].astype(np.float64)
    ref, mag = a64 @ b64, np.abs(a64) @ np.abs(b64)
    if workload == "mbr":
        bias64 = ins["bias"].astype(np.float64)
        ref, mag = np.maximum(ref + bias64, 0.0), mag + np.abs(bias64)
    elif workload == "matmul_add":
        c64 = (ins["c"] if rows is None else ins["c"][rows]).astype(np.float64)
        ref, mag = ref + c64, mag + np.abs(c64)
    return ref, mag


def error_bound(mag, k: int, workload: str, mode: str = "fp32", ab_mag=None):
    """Deterministic error bound of the reference check, widened for input rounding."""
    steps = k + 1 if workload in ("mbr", "matmul_add") else k
    gamma = steps * F32_EPS / (1 - steps * F32_EPS)
    bound = gamma * mag + F32_TINY
    u_in = INPUT_UNIT[mode]
    if u_in:
        bound = bound + (2 * u_in + u_in * u_in) * (mag if ab_mag is None else ab_mag)
    return bound


def check_output(workload: str, ins: dict, out: np.ndarray, mode: str = "fp32", rows=None,
                 out_unit: float = 0.0) -> dict:
    """Reference FP64 check of a GEMM output (optionally on a row subset).  `out_unit` is the
    unit roundoff of an output stored below f32 precision (2^-8 for a bf16 output rounded to
    nearest): the bound grows by out_unit * |ref|."""
    k = ins["a"].shape[1]
    o = out if rows is None else out[rows]
    ref, mag = reference64(workload, ins, rows)
    ab_mag = None
    if INPUT_UNIT[mode]:
        a = ins["a"] if rows is None else ins["a"][rows]
        ab_mag = np.abs(a.astype(np.float64)) @ np.abs(ins["b"].astype(np.float64))
    bound = error_bound(mag, k, workload, mode, ab_mag)
    if out_unit:
        bound = bound + out_unit * np.abs(ref)
    err = np.abs(o.astype(np.float64) - ref)
    res = {"nan_count": int(np.isnan(o).sum()),
           "max_abs_err": float(np.nanmax(err)) if err.size else 0.0,
           "err_over_bound": float(np.nanmax(err / bound)) if err.size else 0.0,
           "rms_err": float(np.sqrt(np.nanmean(err ** 2))) if err.size else 0.0,
           "tolerance": (f"gamma_{k + (workload != 'matmul')}*(|A||B|+|aux|)" +
                         (f" + (2u+u^2)|A||B|, u={INPUT_UNIT[mode]:.3g}" if INPUT_UNIT[mode] else "") +
                         (f" + {out_unit:.3g}|ref|" if out_unit else ""))}
    res["pass"] = res["nan_count"] == int(np.isnan(ref).sum()) and res["err_over_bound"] <= 1.0
    return res


def check_elementwise(workload: str, ins: dict, out: np.ndarray) -> dict:
    """Elementwise ops must be bit-exact against NumPy float32 (python/tforge_gpu.py:116-126).

    Compared bit for bit; relu's reference is IEEE-2019 maximum(x, +0.0) (NaN kept,
    -0.0 -> +0.0, docs/dialect.md:27-30), stricter than the reference's value compare."""
    if workload == "bias_add":
        ref = ins["a"] + ins["bias"]
    elif workload == "relu":
        a = ins["a"]
        ref = np.where(np.isnan(a), a, np.where(a > 0, a, np.float32(0))).astype(np.float32)
    elif workload == "add":
        ref = ins["a"] + ins["b"]
    else:
        raise ValueError(workload)
    exact = bool(np.array_equal(out.view(np.uint32), ref.view(np.uint32)))
    return {"pass": exact, "nan_count": int(np.isnan(out).sum()),
            "err_over_bound": 0.0 if exact else float("inf"),
            "max_abs_err": float(np.max(np.abs(out.astype(np.float64) - ref))) if out.size else 0.0}


def flops_or_bytes(workload: str, m: int, n: int, k: int | None):
    """(metric name, amount of work) for the derived metric."""
    if workload in GEMM_WORKLOADS:
        return "GFLOP/s", 2.0 * m * n * k
    arrays = 3 if workload == "add" else 2
    return "GB/s", arrays * m * n * 4.0
