"""Select, check and time TensorForge GPU operators on B200 (sm_100a).

Same functions and return shapes as the reference's python/tforge_gpu.py:66-160, over
the CUDA library's C-ABI instead of an MLIR/LLVM backend chain:

* ``compile_kernel(workload, m, n, k, options, tag)`` no longer generates code: it asks
  the library which kernel its dispatch table picks (``tforge_describe``) and writes the
  same ``launch.json`` keys (kernel, grid, block, args, padded) plus the new ones
  (cluster, smem_bytes, tile, stages, tmem_cols, precision).  ``options`` is a
  space-separated ``key=value`` list: ``precision=fp32|tf32|bf16|fp32_exact`` and the
  table overrides ``bn=`` and ``stages=``.
* ``check`` runs the operator once in this process through ctypes (NaN-prefilled
  output, as the runner does, tforge-gpu-bench.cu:323-325) and applies the FP64 bound;
  ``mode="cublas"`` runs the runner's cuBLAS comparator instead.
* ``bench`` and ``info`` run the ``tforge-gpu-bench`` runner (CUDA-event timing, NVML
  clocks) and return its JSON object.
* ``padded_shape`` returns the shape unchanged: TMA zero-fill and predicated stores
  replace the reference's padding copies.

No PyTorch and no CPU fallback: the library must load, or these functions raise.
"""

from __future__ import annotations

import ctypes as C
import json
import os
import pathlib
import re
import subprocess
import tempfile

import numpy as np

from . import _lib
from . import tforge_cpu as tc

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
GPU_BENCH = PKG / "tforge-gpu-bench"
ART = ROOT / "build" / "artifacts" / "gpu"
SM = os.environ.get("TF_GPU_ARCH", "sm_100a")
SMS = int(os.environ.get("TF_GPU_SMS", "148"))
FP32_LANES_PER_SM = 128  # B200: 128 FP32 lanes per SM (SIMT FFMA peak, the reference's convention)
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"


def fp32_peak_gflops(sm_mhz):
    """SIMT FP32 FFMA peak at a clock (the reference's % of FP32 peak, tforge_gpu.py:34-35)."""
    return SMS * FP32_LANES_PER_SM * 2 * sm_mhz * 1e6 / 1e9


def tensor_roofline_tflops(precision: str, peaks: dict | None = None) -> tuple[float, str]:
    """Dense tensor roofline of a precision mode, from the measured bf16 GEMM peak.

    TF32 runs at half the bf16 rate on B200 (1.1 vs 2.25 PFLOP/s dense nominal), and the
    fp32-accurate 3xTF32 mode issues three TF32 products per K step: P_tf32 / 3."""
    if peaks is None:
        peaks = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else {}
    bf16 = peaks.get("bf16_tflops")
    src = "of measured"
    if not bf16:
        bf16, src = 1590.0, "of fallback"
    tf32 = bf16 / 2.0
    table = {"bf16": bf16, "tf32": tf32, "fp32": tf32 / 3.0, "fp32_exact": None}
    return table[precision], src


def run(cmd, **kw):
    cmd = [str(c) for c in cmd]
    kw.setdefault("timeout", 600)
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stderr}")
    return r.stdout


def parse_options(options: str) -> dict:
    opts = dict(o.split("=", 1) for o in options.split() if "=" in o)
    return {"precision": opts.get("precision", "fp32"), "bn": int(opts.get("bn", 0)),
            "stages": int(opts.get("stages", 0)), "kernel": opts.get("kernel", ""),
            "split": int(opts.get("split", 0)), "persistent": int(opts.get("persistent", 0)),
            "b_layout": int(opts.get("b_layout", 0))}


def _forced_kind(o: dict) -> int:
    """tforge_config.kernel for parsed options: 0 table, 1 one-CTA, 2 SIMT, 3 CTA pair."""
    k = o.get("kernel", "")
    if k == "pair" or ((o.get("split") or o.get("persistent")) and not k):
        return 3
    if k == "simt":
        return 2
    return 1 if (k == "cta" or o["bn"] or o["stages"]) else 0


def padded_shape(m, n, k, options=""):
    """The shape the kernel runs on: unchanged (no padding copies on this path)."""
    return m, n, k


def parse_launch(path) -> dict:
    return json.loads(pathlib.Path(path).read_text())


def compile_kernel(workload, m, n, k, options="", tag="default"):
    """Pick the kernel for one problem and record its launch; returns (dir, launch)."""
    o = parse_options(options)
    d = ART / tag / f"{workload}_{m}x{n}x{k}"
    d.mkdir(parents=True, exist_ok=True)
    kind = _forced_kind(o)
    if kind or o.get("b_layout"):
        _lib.set_config(kind, o["bn"], o["stages"], o.get("persistent", 0), o.get("split", 0), o.get("b_layout", 0))
    try:
        desc = _lib.describe(workload, m, n, k or 0, o["precision"])
    finally:
        if kind or o.get("b_layout"):
            _lib.set_config()
    args = {"matmul": ["arg0", "arg1", "arg2"], "mbr": ["arg0", "arg1", "arg2", "arg3"],
            "matmul_add": ["arg0", "arg1", "arg2", "arg3"], "bias_add": ["arg0", "arg1", "arg2"],
            "relu": ["arg0", "arg1"], "add": ["arg0", "arg1", "arg2"]}[workload]
    launch = {"kernel": desc["kernel"], "grid": desc["grid"], "block": desc["block"], "args": args,
              "padded": [m, n, k], "cluster": desc["cluster"], "smem_bytes": desc["smem_bytes"],
              "tile": desc["tile"], "stages": desc["stages"], "tmem_cols": desc["tmem_cols"],
              "precision": o["precision"], "options": options}
    (d / "launch.json").write_text(json.dumps(launch))
    return d, launch


def _bench_cmd(workload, m, n, k, kdir=None, launch=None, mode="kernel"):
    cmd = [GPU_BENCH, "--mode", "cublas" if mode == "cublas" else "lib", "--workload", workload,
           "--m", m, "--n", n, "--k", k or 1]
    if mode != "cublas" and launch:
        o = parse_options(launch.get("options", ""))
        cmd += ["--precision", o["precision"]]
        if o["bn"]:
            cmd += ["--bn", o["bn"]]
        if o["stages"]:
            cmd += ["--stages", o["stages"]]
        if o["kernel"]:
            cmd += ["--kernel", o["kernel"]]
        if o.get("split"):
            cmd += ["--split", o["split"]]
        if o.get("persistent"):
            cmd += ["--persistent"]
        if o.get("b_layout"):
            cmd += ["--b-layout", o["b_layout"]]
    return cmd


def info(workload, m, n, k, kdir=None, launch=None):
    """Registers, shared memory and occupancy of the selected kernel (CUDA occupancy API)."""
    return json.loads(run(_bench_cmd(workload, m, n, k, kdir, launch) + ["--info-only"]))


class DeviceBuffer:
    """Device allocation through the library (the shim has no other CUDA binding)."""

    def __init__(self, nbytes: int):
        self.ptr = C.c_void_p()
        _lib.check(_lib.lib().tforge_malloc(C.byref(self.ptr), nbytes), "tforge_malloc")
        self.nbytes = nbytes

    @classmethod
    def upload(cls, arr: np.ndarray) -> "DeviceBuffer":
        arr = np.ascontiguousarray(arr)
        b = cls(arr.nbytes)
        _lib.check(_lib.lib().tforge_memcpy_h2d(b.ptr, arr.ctypes.data, arr.nbytes, None), "H2D")
        return b

    def download(self, shape, dtype=np.float32) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        _lib.check(_lib.lib().tforge_memcpy_d2h(out.ctypes.data, self.ptr, out.nbytes, None), "D2H")
        _lib.check(_lib.lib().tforge_stream_sync(None), "sync")
        return out

    @property
    def addr(self) -> int:
        return self.ptr.value

    def free(self):
        if self.ptr:
            _lib.lib().tforge_free(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def run_op(workload: str, ins: dict, m: int, n: int, k: int | None, precision: str = "fp32",
           options: str = "") -> np.ndarray:
    """One call of an operator on host arrays through the C-ABI; returns the output."""
    L = _lib.lib()
    bufs = {name: DeviceBuffer.upload(arr) for name, arr in ins.items()}
    out = DeviceBuffer(m * n * 4)
    _lib.check(L.tforge_memset(out.ptr, 0xFF, m * n * 4, None), "memset")  # NaN prefill
    o = parse_options(options)
    kind = _forced_kind(o)
    if kind or o.get("b_layout"):
        _lib.set_config(kind, o["bn"], o["stages"], o.get("persistent", 0), o.get("split", 0), o.get("b_layout", 0))
    try:
        if workload in tc.GEMM_WORKLOADS:
            _lib.gemm(workload, bufs["a"].addr, bufs["b"].addr, out.addr, m, n, k, precision,
                      bias=bufs["bias"].addr if "bias" in bufs else None,
                      c_res=bufs["c"].addr if "c" in bufs else None)
        elif workload == "bias_add":
            _lib.check(L.tforge_bias_add(bufs["a"].ptr, bufs["bias"].ptr, out.ptr, m, n, None), "bias_add")
        elif workload == "relu":
            _lib.check(L.tforge_relu(bufs["a"].ptr, out.ptr, m, n, None), "relu")
        elif workload == "add":
            _lib.check(L.tforge_add(bufs["a"].ptr, bufs["b"].ptr, out.ptr, m, n, None), "add")
        else:
            raise ValueError(workload)
        _lib.check(_lib.device_status(None), "device status")
        return out.download((m, n))
    finally:
        if kind or o.get("b_layout"):
            _lib.set_config()
        for b in bufs.values():
            b.free()
        out.free()


def check(workload, m, n, k, kdir=None, launch=None, mode="kernel", seed=1234, ins=None, rows=None):
    """Run once on the reference's inputs and apply the FP64 bound; returns (res, out).

    Elementwise workloads must match NumPy float32 bit for bit."""
    if ins is None:
        ins = tc.make_inputs(workload, m, n, k, seed)
    precision = parse_options(launch.get("options", ""))["precision"] if launch else "fp32"
    if mode == "cublas":
        with tempfile.TemporaryDirectory() as td:
            for name, arr in ins.items():
                arr.tofile(f"{td}/{name}.bin")
            run(_bench_cmd(workload, m, n, k, mode="cublas") +
                ["--warmup", 0, "--reps", 1, "--in-dir", td, "--out", f"{td}/out.bin"])
            out = np.fromfile(f"{td}/out.bin", dtype=np.float32).reshape(m, n)
    else:
        out = run_op(workload, ins, m, n, k, precision, launch.get("options", "") if launch else "")
    if workload not in tc.GEMM_WORKLOADS:
        return tc.check_elementwise(workload, ins, out), out
    return tc.check_output(workload, ins, out, "fp32" if mode == "cublas" else precision, rows=rows), out


def bench(workload, m, n, k, kdir=None, launch=None, mode="kernel", warmup=10, reps=100, flush=False):
    cmd = _bench_cmd(workload, m, n, k, kdir, launch, mode) + ["--warmup", warmup, "--reps", reps]
    if flush:
        cmd.append("--flush")
    return json.loads(run(cmd))


def ptxas_resources(kdir=None, launch=None):
    """Registers, spill stores/loads and shared memory from the build's ptxas -v report.

    Reports the largest figures over the instantiations of the selected kernel family."""
    t = (PKG / "_build" / "ptxas.txt").read_text() if (PKG / "_build" / "ptxas.txt").exists() else ""
    fam = {"tf_gemm_tcgen05_tf32": "gemm_tc_kernelILi0E", "tf_gemm_tcgen05_3xtf32": "gemm_tc_kernelILi1E",
           "tf_gemm_tcgen05_bf16": "gemm_tc_kernelILi2E", "tf_gemm_simt_ffma": "gemm_simt_kernel"}
    key = fam.get((launch or {}).get("kernel", ""), "gemm_tc_kernel")
    res = {"regs": 0, "spill_stores": 0, "spill_loads": 0, "smem": 0}
    blocks = t.split("Compiling entry function")
    for b in blocks:
        if key not in b.split("\n", 1)[0]:
            continue
        g = lambda pat: int(m.group(1)) if (m := re.search(pat, b)) else 0
        res["regs"] = max(res["regs"], g(r"Used (\d+) registers"))
        res["spill_stores"] = max(res["spill_stores"], g(r"(\d+) bytes spill stores"))
        res["spill_loads"] = max(res["spill_loads"], g(r"(\d+) bytes spill loads"))
        res["smem"] = max(res["smem"], g(r"(\d+) bytes smem"))
    return res
