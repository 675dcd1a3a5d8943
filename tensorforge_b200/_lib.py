"""ctypes binding of ``libtforge_gpu.so`` (the C-ABI declared in ``include/tforge.h``).

The library is the product path: there is no Python or CPU fallback.  ``lib()`` raises
``RuntimeError`` when the shared object is missing or fails to load.
"""

from __future__ import annotations

import ctypes as C
import pathlib
import threading

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG / "libtforge_gpu.so"

# enum tforge_status
OK, ERR_SHAPE, ERR_ALIGN, ERR_ALIAS, ERR_MODE, ERR_CUDA, ERR_TIMEOUT, ERR_NULL, ERR_UNSUPPORTED, ERR_NOMEM = range(10)
# enum tforge_mode
MODES = {"fp32": 0, "tf32": 1, "bf16": 2, "fp32_exact": 3}
# enum tforge_workload
WORKLOADS = {"matmul": 0, "mbr": 1, "matmul_add": 2, "bias_add": 3, "relu": 4, "add": 5}
F32, BF16 = 0, 1


class GemmArgs(C.Structure):
    _fields_ = [("workload", C.c_int32), ("mode", C.c_int32), ("a_dtype", C.c_int32),
                ("b_dtype", C.c_int32), ("A", C.c_void_p), ("B", C.c_void_p), ("bias", C.c_void_p),
                ("C_res", C.c_void_p), ("out", C.c_void_p), ("M", C.c_int64), ("N", C.c_int64),
                ("K", C.c_int64), ("lda", C.c_int64), ("ldb", C.c_int64), ("ldc", C.c_int64),
                ("out_dtype", C.c_int32)]


class Launch(C.Structure):
    _fields_ = [("kernel", C.c_char * 64), ("grid", C.c_int32 * 3), ("block", C.c_int32 * 3),
                ("cluster", C.c_int32 * 3), ("smem_bytes", C.c_int32), ("tile", C.c_int32 * 3),
                ("stages", C.c_int32), ("tmem_cols", C.c_int32), ("mode", C.c_int32),
                ("persistent", C.c_int32), ("split_k", C.c_int32), ("regs", C.c_int32),
                ("static_smem", C.c_int32), ("blocks_per_sm", C.c_int32)]

    def as_dict(self) -> dict:
        return {"kernel": self.kernel.decode(), "grid": list(self.grid), "block": list(self.block),
                "cluster": list(self.cluster), "smem_bytes": self.smem_bytes, "tile": list(self.tile),
                "stages": self.stages, "tmem_cols": self.tmem_cols, "mode": self.mode,
                "persistent": self.persistent, "split_k": self.split_k, "regs": self.regs,
                "static_smem": self.static_smem, "blocks_per_sm": self.blocks_per_sm}


class Config(C.Structure):
    _fields_ = [("kernel", C.c_int32), ("bn", C.c_int32), ("stages", C.c_int32),
                ("persistent", C.c_int32), ("split_k", C.c_int32), ("b_layout", C.c_int32)]


# Every symbol include/tforge.h declares, with its ctypes signature.
_P, _I, _I64, _U64 = C.c_void_p, C.c_int, C.c_int64, C.c_uint64
SIGNATURES = {
    "tforge_gemm": (_I, [C.POINTER(GemmArgs), _P]),
    "tforge_gemm_host": (_I, [C.POINTER(GemmArgs), _I64, _P]),
    "tforge_matmul": (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "tforge_mbr": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "tforge_matmul_add": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "tforge_bias_add": (_I, [_P, _P, _P, _I64, _I64, _P]),
    "tforge_relu": (_I, [_P, _P, _I64, _I64, _P]),
    "tforge_add": (_I, [_P, _P, _P, _I64, _I64, _P]),
    "tforge_convert_bf16": (_I, [_P, _P, _I64, _P]),
    "tforge_mbr_bf16_noalloc": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "tforge_describe": (_I, [_I, _I64, _I64, _I64, _I, C.POINTER(Launch)]),
    "tforge_set_config": (_I, [C.POINTER(Config)]),
    "tforge_device_status": (_I, [_P]),
    "tforge_set_wait_limit_ns": (_I, [_U64]),
    "tforge_debug_skip_load": (_I, [_I]),
    "tforge_debug_pool_usage": (_I, [C.POINTER(_U64), C.POINTER(_U64), _I]),
    "tforge_status_string": (C.c_char_p, [_I]),
    "tforge_last_error": (C.c_char_p, []),
    "tforge_version": (C.c_char_p, []),
    "tforge_malloc": (_I, [C.POINTER(_P), _U64]),
    "tforge_free": (_I, [_P]),
    "tforge_memcpy_h2d": (_I, [_P, _P, _U64, _P]),
    "tforge_memcpy_d2h": (_I, [_P, _P, _U64, _P]),
    "tforge_memset": (_I, [_P, _I, _U64, _P]),
    "tforge_stream_sync": (_I, [_P]),
    "tforge_device_count": (_I, [C.POINTER(C.c_int)]),
    "tforge_set_device": (_I, [_I]),
}

_lock = threading.Lock()
_lib = None


def lib() -> C.CDLL:
    """Load the library once; raise if it is absent (no fallback exists)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: run tensorforge_b200.build.build() first")
            lib_ = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib_, name)
                fn.restype, fn.argtypes = res, args
            _lib = lib_
    return _lib


class TforgeError(RuntimeError):
    def __init__(self, code: int, what: str):
        L = lib()
        msg = L.tforge_status_string(code).decode()
        if code == ERR_CUDA:
            msg += f" ({L.tforge_last_error().decode()})"
        super().__init__(f"{what}: {msg} [status {code}]")
        self.code = code


def check(code: int, what: str = "tforge") -> None:
    if code != OK:
        raise TforgeError(code, what)


def describe(workload: str, m: int, n: int, k: int, mode: str = "fp32") -> dict:
    out = Launch()
    check(lib().tforge_describe(WORKLOADS[workload], m, n, k, MODES[mode], C.byref(out)), "tforge_describe")
    return out.as_dict()


def set_config(kernel: int = 0, bn: int = 0, stages: int = 0, persistent: int = 0, split_k: int = 0,
               b_layout: int = 0) -> None:
    """Force a kernel configuration (kernel 1 = one-CTA tcgen05, 2 = SIMT, 3 = CTA pair;
    split_k: pairs per tile for the pair kernel, 1 = none; b_layout (TF32 pair kernels):
    1 = B as given, 2 = a transposed K-major copy, 3 = B as given in 128-byte column blocks
    instead of k-group-major tiles); all zeros = table."""
    if kernel == 0 and bn == 0 and stages == 0 and persistent == 0 and split_k == 0 and b_layout == 0:
        check(lib().tforge_set_config(None), "tforge_set_config")
        return
    cfg = Config(kernel, bn, stages, persistent, split_k, b_layout)
    check(lib().tforge_set_config(C.byref(cfg)), "tforge_set_config")


def gemm(workload: str, A: int, B: int, out: int, M: int, N: int, K: int, mode: str = "fp32",
         bias: int | None = None, c_res: int | None = None, stream: int | None = None,
         a_dtype: int = F32, b_dtype: int = F32, lda: int = 0, ldb: int = 0, ldc: int = 0,
         out_dtype: int = F32) -> None:
    """tforge_gemm on device pointers (ints), asynchronous on `stream`."""
    args = GemmArgs(WORKLOADS[workload], MODES[mode], a_dtype, b_dtype, A, B, bias, c_res, out,
                    M, N, K, lda, ldb, ldc, out_dtype)
    check(lib().tforge_gemm(C.byref(args), stream), f"tforge_gemm({workload}, {M}x{N}x{K}, {mode})")


def gemm_host(workload: str, A: int, B: int, out: int, M: int, N: int, K: int, mode: str = "fp32",
              bias: int | None = None, c_res: int | None = None, stream: int | None = None,
              chunk_rows: int = 0, a_dtype: int = F32, b_dtype: int = F32, lda: int = 0, ldb: int = 0,
              ldc: int = 0) -> None:
    """tforge_gemm_host on HOST pointers (ints): overlapped chunked copies and kernels,
    asynchronous on `stream` (out is complete once the stream synchronizes)."""
    args = GemmArgs(WORKLOADS[workload], MODES[mode], a_dtype, b_dtype, A, B, bias, c_res, out,
                    M, N, K, lda, ldb, ldc)
    check(lib().tforge_gemm_host(C.byref(args), chunk_rows, stream),
          f"tforge_gemm_host({workload}, {M}x{N}x{K}, {mode})")


def device_status(stream: int | None = None) -> int:
    return lib().tforge_device_status(stream)


def pool_usage(reset_high: bool = False) -> tuple[int, int]:
    """(bytes in use now, high-water mark) of the library's scratch pool on the current device."""
    now, high = C.c_uint64(), C.c_uint64()
    check(lib().tforge_debug_pool_usage(C.byref(now), C.byref(high), int(reset_high)), "tforge_debug_pool_usage")
    return now.value, high.value
