"""tforge_gemm_host: the operators on HOST buffers with chunked, overlapped copies.

Same numerics bar as the device entry (tests/test_gpu_parity.py): fp32_exact bit-exact
against the CPU restatement, tensor-core modes within the FP64 bound.  Covers page-locked
and pageable host memory, pitched host arrays, ragged chunking, K = 0 and the BF16 mode's
one-time conversion of B.
"""

import ctypes as C

import numpy as np
import pytest

from tensorforge_b200 import _lib, tforge_cpu as tc

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def pinned(arr):
    import torch

    t = torch.empty(arr.shape, dtype=torch.float32, pin_memory=True)
    t.numpy()[...] = arr
    return t


def run_host(workload, ins, m, n, k, mode, chunk_rows=0, pin=True, pitch=0):
    """Call tforge_gemm_host on host copies of `ins` (optionally pitched by `pitch` extra
    elements per row) and return the M x N result."""
    keep = []

    def host(arr):
        if pitch and arr.ndim == 2:
            wide = np.full((arr.shape[0], arr.shape[1] + pitch), np.nan, np.float32)
            wide[:, : arr.shape[1]] = arr
            arr = wide
        if pin:
            t = pinned(arr)
            keep.append(t)
            return t.data_ptr()
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        keep.append(arr)
        return arr.ctypes.data

    A, B = host(ins["a"]), host(ins["b"])
    bias = host(ins["bias"]) if "bias" in ins else None
    c_res = host(ins["c"]) if "c" in ins else None
    out = host(np.full((m, n), np.nan, np.float32))  # padded to n + pitch columns by host()
    _lib.gemm_host(workload, A, B, out, m, n, k, mode, bias=bias, c_res=c_res, chunk_rows=chunk_rows,
                   lda=(k + pitch) if pitch else 0, ldb=(n + pitch) if pitch else 0,
                   ldc=(n + pitch) if pitch else 0)
    _lib.check(_lib.lib().tforge_stream_sync(None), "sync")
    _lib.check(_lib.device_status(None), "device status")
    res = keep[-1]
    res = res.numpy() if hasattr(res, "numpy") else res
    full = np.array(res).reshape(m, n + pitch)
    if pitch:  # the pad columns of out are never written
        assert np.isnan(full[:, n:]).all()
    return np.ascontiguousarray(full[:, :n])


@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("shape", [(777, 1111, 333), (1000, 520, 300), (5, 7, 3)], ids=lambda s: "x".join(map(str, s)))
def test_host_fp32_exact_bitwise(gpu, oracle, workload, shape):
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 1234)
    out = run_host(workload, ins, m, n, k, "fp32_exact", chunk_rows=128)
    assert np.array_equal(bits(out), bits(oracle.gemm(workload, ins)))


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul_add"])
def test_host_tensor_core_modes_within_bound(gpu, workload, mode):
    m, n, k = 1000, 520, 304
    ins = tc.make_inputs(workload, m, n, k, 7)
    out = run_host(workload, ins, m, n, k, mode)
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


def test_host_2048_fp32_pinned(gpu):
    """BASELINE config 2's shape through the host entry (8 chunks of 256 rows)."""
    ins = tc.make_inputs("mbr", 2048, 2048, 2048, 0)
    out = run_host("mbr", ins, 2048, 2048, 2048, "fp32")
    res = tc.check_output("mbr", ins, out, "fp32")
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("chunk_rows", [1, 100, 256, 4096])
def test_host_chunking_pitched_pageable(gpu, oracle, chunk_rows):
    """Ragged chunks (1 row rounds up to M/64), pitched host rows, pageable memory."""
    m, n, k = 777, 264, 96
    ins = tc.make_inputs("matmul_add", m, n, k, 3)
    ref = oracle.gemm("matmul_add", ins)
    out = run_host("matmul_add", ins, m, n, k, "fp32_exact", chunk_rows=chunk_rows, pin=False, pitch=4)
    assert np.array_equal(bits(out), bits(ref))
    out = run_host("matmul_add", ins, m, n, k, "fp32", chunk_rows=chunk_rows, pin=True, pitch=4)
    res = tc.check_output("matmul_add", ins, out, "fp32")
    assert res["err_over_bound"] <= 1.0, res


def test_host_k0_and_empty(gpu, oracle):
    ins = tc.make_inputs("mbr", 300, 64, 0, 5)
    out = run_host("mbr", ins, 300, 64, 0, "tf32")
    assert np.array_equal(bits(out), bits(oracle.gemm("mbr", ins)))
    L = _lib.lib()
    args = _lib.GemmArgs(_lib.WORKLOADS["mbr"], 0, _lib.F32, _lib.F32, None, None, None, None, None,
                         0, 16, 16, 0, 0, 0)
    assert L.tforge_gemm_host(C.byref(args), 0, None) == 0


def test_host_bf16_matches_device_entry(gpu):
    """BF16 mode converts B once for all chunks; each chunk's result equals the device
    entry's on the same rows (same kernel family and rounding)."""
    m, n, k = 2048, 512, 1024
    ins = tc.make_inputs("mbr", m, n, k, 11)
    host = run_host("mbr", ins, m, n, k, "bf16", chunk_rows=256)
    from tensorforge_b200 import tforge_gpu as tg

    dev = np.concatenate([tg.run_op("mbr", {"a": ins["a"][r:r + 256], "b": ins["b"], "bias": ins["bias"]},
                                    256, n, k, "bf16") for r in range(0, m, 256)])
    assert np.array_equal(bits(host), bits(dev))
    res = tc.check_output("mbr", ins, host, "bf16")
    assert res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul_add"])
def test_host_wide_ragged_pitched_within_bound(gpu, workload, mode):
    """A wide, ragged problem through the host entry: several row chunks, N not a multiple
    of the tile width, pitched host rows, every tensor-core mode."""
    m, n, k = 1500, 1304, 256
    ins = tc.make_inputs(workload, m, n, k, 19)
    out = run_host(workload, ins, m, n, k, mode, pitch=4)
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res
