"""Row-sharded fused dense layers over several GPUs of one node.

The reference runs on one device (runners/gpu/tforge-gpu-bench.cu:180) and has no
collective.  For large M the fused layer out = relu(A @ W + bias) shards naturally over
output rows: rank r of n owns rows [floor(r M / n), floor((r + 1) M / n)) of A and of
out; W (K x N) and bias (N) are broadcast once per weight set from one rank over NCCL;
outputs stay sharded, so there is no collective after the GEMM and none in the hot loop.

One process per GPU with torch.distributed for the plumbing (NCCL on GPUs; gloo runs
the host-side logic in CPU tests).  The GEMM itself is the library's C-ABI call on each
rank's own rows (include/tforge.h); PyTorch only holds the device memory and streams.
"""

from __future__ import annotations

from dataclasses import dataclass

from . import _lib


def row_partition(m: int, n_ranks: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of rank `rank` when M rows are split over `n_ranks` ranks."""
    if n_ranks <= 0 or not 0 <= rank < n_ranks or m < 0:
        raise ValueError(f"bad partition request m={m} n_ranks={n_ranks} rank={rank}")
    return (rank * m) // n_ranks, ((rank + 1) * m) // n_ranks


def all_partitions(m: int, n_ranks: int) -> list[tuple[int, int]]:
    return [row_partition(m, n_ranks, r) for r in range(n_ranks)]


@dataclass
class WeightSet:
    """A broadcast weight set: W (K x N) and bias (N) resident on this rank's device."""

    weight: "object"
    bias: "object"
    version: int = 0


def broadcast_weights(weight, bias, src: int = 0, group=None, version: int = 0) -> WeightSet:
    """Broadcast W and bias from rank `src` to every rank (in place), once per weight set.

    Every rank passes tensors of the final shape; non-source ranks' contents are
    overwritten.  Returns the rank's WeightSet."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.broadcast(weight, src=src, group=group)
        dist.broadcast(bias, src=src, group=group)
    return WeightSet(weight, bias, version)


def mbr_rows(a_rows, ws: WeightSet, out_rows, mode: str = "fp32", stream=None) -> None:
    """out_rows = relu(a_rows @ W + bias) on this rank's rows through the C-ABI.

    a_rows (rows x K) and out_rows (rows x N) are this rank's row blocks (contiguous
    tensors on this rank's GPU); the call is asynchronous on `stream` (torch's current
    stream of the device when None)."""
    import torch

    rows, k = a_rows.shape
    n = ws.weight.shape[1]
    if ws.weight.shape[0] != k or out_rows.shape != (rows, n) or ws.bias.shape != (n,):
        raise ValueError("shape mismatch between A rows, W, bias and out rows")
    if stream is None:
        stream = torch.cuda.current_stream(a_rows.device).cuda_stream
    L = _lib.lib()
    _lib.check(L.tforge_mbr(a_rows.data_ptr(), ws.weight.data_ptr(), ws.bias.data_ptr(),
                            out_rows.data_ptr(), rows, n, k, _lib.MODES[mode], stream), "tforge_mbr")


class ShardedMBR:
    """relu(A @ W + bias) with A's and out's rows sharded over the ranks of `group`.

    Construct on every rank with W and bias tensors of full shape on the rank's device
    (rank `src` holds the values); they are broadcast once.  Call with this rank's rows
    of A; returns this rank's rows of the output."""

    def __init__(self, weight, bias, mode: str = "fp32", src: int = 0, group=None):
        self.ws = broadcast_weights(weight, bias, src=src, group=group)
        self.mode = mode
        self.group = group

    def rows(self, m_total: int) -> tuple[int, int]:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            return row_partition(m_total, dist.get_world_size(self.group), dist.get_rank(self.group))
        return 0, m_total

    def __call__(self, a_rows, out_rows=None, stream=None):
        import torch

        if out_rows is None:
            out_rows = torch.empty((a_rows.shape[0], self.ws.weight.shape[1]), device=a_rows.device,
                                   dtype=torch.float32)
        mbr_rows(a_rows, self.ws, out_rows, self.mode, stream)
        return out_rows
