"""ctypes access to the CPU restatement in oracle/ (the checker; test infrastructure only)."""

from __future__ import annotations

import ctypes as C
import pathlib

import numpy as np

REPO = pathlib.Path(__file__).resolve().parent.parent
_lib = C.CDLL(str(REPO / "oracle" / "build" / "liboracle.so"))
_P, _I64 = C.c_void_p, C.c_int64
_lib.oracle_gemm.argtypes = [C.c_int, _P, _P, _P, _P, _I64, _I64, _I64, C.c_int]
_lib.oracle_gemm_fma_naive.argtypes = [C.c_int, _P, _P, _P, _P, _I64, _I64, _I64]
_lib.oracle_elementwise.argtypes = [C.c_int, _P, _P, _P, _I64, _I64]

WORKLOAD = {"matmul": 0, "mbr": 1, "matmul_add": 2}
ELEMENTWISE = {"add": 0, "relu": 1, "bias_add": 2}


def _ptr(a):
    return None if a is None else a.ctypes.data


def gemm(workload: str, ins: dict, fma: bool = True, naive: bool = False) -> np.ndarray:
    """Reference CPU kernel result: sequential-k FMA (fma=True) or the unfused scalar order."""
    a = np.ascontiguousarray(ins["a"], dtype=np.float32)
    b = np.ascontiguousarray(ins["b"], dtype=np.float32)
    aux = ins.get("bias") if workload == "mbr" else ins.get("c")
    aux = None if aux is None else np.ascontiguousarray(aux, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.float32)
    if naive:
        rc = _lib.oracle_gemm_fma_naive(WORKLOAD[workload], _ptr(a), _ptr(b), _ptr(aux), _ptr(out), m, n, k)
    else:
        rc = _lib.oracle_gemm(WORKLOAD[workload], _ptr(a), _ptr(b), _ptr(aux), _ptr(out), m, n, k, int(fma))
    assert rc == 0
    return out


def elementwise(workload: str, ins: dict) -> np.ndarray:
    a = np.ascontiguousarray(ins["a"], dtype=np.float32)
    y = ins.get("b") if workload == "add" else ins.get("bias")
    y = None if y is None else np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty_like(a)
    assert _lib.oracle_elementwise(ELEMENTWISE[workload], _ptr(a), _ptr(y), _ptr(out), a.shape[0], a.shape[1]) == 0
    return out
