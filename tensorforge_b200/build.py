"""Build recipe for the native parts of tensorforge_b200.

Compiles the CUDA sources in ``csrc/`` for sm_100a into ``libtforge_gpu.so`` (the C-ABI
of ``include/tforge.h``) and the ``tforge-gpu-bench`` runner, in-tree, so the built
files travel with the source tree.  The ptxas resource report (registers, spills,
shared memory per kernel) is kept in ``_build/ptxas.txt``.

    python -m tensorforge_b200.build          # or tensorforge_b200.build.build()
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libtforge_gpu.so"
RUNNER = PKG / "tforge-gpu-bench"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB_SOURCES = ["tf_api.cu", "tf_gemm_tc.cu", "tf_gemm_2sm.cu", "tf_simt.cu", "tf_noalloc.cu", "tf_host.cu",
               "tf_gemm_2sm_persist.cu"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not pathlib.Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def _flags() -> list[str]:
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                   "-I", str(ROOT / "include")]


def _newer(target: pathlib.Path, deps: list[pathlib.Path]) -> bool:
    return target.exists() and all(target.stat().st_mtime >= d.stat().st_mtime for d in deps)


def _compile(src: pathlib.Path) -> tuple[pathlib.Path, str]:
    obj = BUILD / (src.stem + ".o")
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *CSRC.glob("*.inc"), ROOT / "include" / "tforge.h"]
    log = BUILD / (src.stem + ".ptxas.txt")
    if _newer(obj, deps) and log.exists():
        return obj, log.read_text()
    cmd = [nvcc(), *_flags(), "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    log.write_text(r.stderr)
    return obj, r.stderr


def build(force: bool = False) -> pathlib.Path:
    """Compile every CUDA source for sm_100a; returns the library path."""
    BUILD.mkdir(exist_ok=True)
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    srcs = [CSRC / s for s in LIB_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 1)) as ex:
        results = list(ex.map(_compile, srcs))
    objs = [o for o, _ in results]
    (BUILD / "ptxas.txt").write_text("".join(log for _, log in results))
    if not _newer(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    runner_src = CSRC / "runner" / "tforge_gpu_bench.cu"
    if runner_src.exists() and not _newer(RUNNER, [runner_src, LIB, ROOT / "include" / "tforge.h"]):
        cmd = [nvcc(), *_flags(), str(runner_src), "-o", str(RUNNER), "-L", str(PKG), "-ltforge_gpu",
               f"-Xlinker=-rpath,$ORIGIN", "-lcublasLt", "-lcublas", "-lcuda", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("runner build failed:\n" + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force=os.environ.get("TF_FORCE_BUILD") == "1"))
