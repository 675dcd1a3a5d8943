"""tensorforge_b200: B200-native (sm_100a) TensorForge operators behind a C-ABI.

The product is ``libtforge_gpu.so`` (include/tforge.h): tcgen05/TMA GEMM kernels with the
bias-add, ReLU and residual-add epilogue fused, a bit-exact SIMT kernel, and elementwise
ops.  ``tforge_gpu`` and ``tforge_cpu`` keep the reference's host-library API;
``gpu_bench`` keeps its driver; ``shard`` row-shards large problems over GPUs.
"""

__all__ = ["tforge_gpu", "tforge_cpu"]
__version__ = "0.1.0"
