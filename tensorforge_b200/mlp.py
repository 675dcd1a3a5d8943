"""Two-layer MLP chain out = relu(relu(X @ W1 + b1) @ W2 + b2), each layer one fused call.

The direct consumer of the fused dense layer: layer 1 writes H into a caller-owned buffer,
layer 2 reads it; nothing else is materialised.  In BF16 mode the weights are rounded to
bf16 once (tforge_convert_bf16) and passed as bf16 operands, and H is kept in bf16 by
default: layer 1's epilogue rounds its output to bf16 (out_dtype = TFORGE_BF16), which is
exactly what layer 2 would do to an f32 H before its MMAs, so the result is the same bits
with half the H traffic and no conversion pass (`--h-dtype f32` keeps an f32 H).  Rows of X shard over GPUs like tensorforge_b200.shard: weights are
broadcast once, H and the output stay on the rank that owns the rows.

    python -m tensorforge_b200.mlp --shape 65536x4096x16384 --mode fp32        # one GPU
    torchrun --nproc-per-node 8 -m tensorforge_b200.mlp --shape 65536x4096x16384  # M-sharded
"""

from __future__ import annotations

import argparse
import json
import os
import sys

from . import _lib
from .shard import broadcast_weights, row_partition


class MLP2:
    """relu(relu(X @ W1 + b1) @ W2 + b2) on torch tensors of one GPU, through the C-ABI."""

    def __init__(self, w1, b1, w2, b2, mode: str = "fp32", h_bf16: bool | None = None):
        import torch

        self.mode = mode
        # BF16 mode: H in bf16 unless asked otherwise; other modes keep an f32 H.
        self.h_bf16 = (mode == "bf16") if h_bf16 is None else bool(h_bf16)
        if self.h_bf16 and mode != "bf16":
            raise ValueError("a bf16 H needs mode='bf16'")
        self.b1, self.b2 = b1, b2
        self.d, self.h = w1.shape
        if w2.shape != (self.h, self.d) or b1.shape != (self.h,) or b2.shape != (self.d,):
            raise ValueError("MLP2 expects W1 d x h, b1 h, W2 h x d, b2 d")
        if mode == "bf16":
            # Weights converted once; activations are converted inside each call.
            L = _lib.lib()
            self.w1 = torch.empty(w1.shape, device=w1.device, dtype=torch.bfloat16)
            self.w2 = torch.empty(w2.shape, device=w2.device, dtype=torch.bfloat16)
            stream = torch.cuda.current_stream(w1.device).cuda_stream
            _lib.check(L.tforge_convert_bf16(w1.data_ptr(), self.w1.data_ptr(), w1.numel(), stream), "convert W1")
            _lib.check(L.tforge_convert_bf16(w2.data_ptr(), self.w2.data_ptr(), w2.numel(), stream), "convert W2")
            self.b_dtype = _lib.BF16
        else:
            self.w1, self.w2 = w1, w2
            self.b_dtype = _lib.F32

    @property
    def h_dtype(self):
        import torch

        return torch.bfloat16 if self.h_bf16 else torch.float32

    def layer(self, x, w, b, out, stream) -> None:
        import torch

        m, k = x.shape
        n = w.shape[1]
        dt = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}
        _lib.gemm("mbr", x.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, self.mode, bias=b.data_ptr(),
                  stream=stream, a_dtype=dt[x.dtype], b_dtype=self.b_dtype, out_dtype=dt[out.dtype])

    def __call__(self, x, h=None, out=None, stream=None):
        import torch

        m = x.shape[0]
        if h is None:
            h = torch.empty((m, self.h), device=x.device, dtype=self.h_dtype)
        if out is None:
            out = torch.empty((m, self.d), device=x.device, dtype=torch.float32)
        if stream is None:
            stream = torch.cuda.current_stream(x.device).cuda_stream
        self.layer(x, self.w1, self.b1, h, stream)
        self.layer(h, self.w2, self.b2, out, stream)
        return h, out


def flops(m: int, d: int, h: int) -> float:
    """2 M N K per layer (the reference's convention), two layers."""
    return 2.0 * m * d * h * 2


def main(argv=None) -> int:
    import numpy as np
    import torch
    import torch.distributed as dist

    from . import tforge_cpu as tc

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--shape", default="65536x4096x16384",
                    help="MxDxH: rows of X in total (sharded over ranks), model width, hidden width")
    ap.add_argument("--mode", default="fp32", choices=["fp32", "tf32", "bf16"])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--check-rows", type=int, default=16, help="rows checked against FP64 per layer")
    ap.add_argument("--h-dtype", default="auto", choices=["auto", "f32", "bf16"],
                    help="hidden activation storage (auto: bf16 in BF16 mode, else f32)")
    args = ap.parse_args(argv)
    args.m, args.d, args.h = (int(x) for x in args.shape.lower().split("x"))

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    r0, r1 = row_partition(args.m, world, rank)
    rows = r1 - r0
    # Xavier-uniform weights, N(0, 0.02) biases, X U[-1, 1]; X rows generated per rank.
    g = torch.Generator(device=dev)
    g.manual_seed(100 + rank)
    x = torch.empty((rows, args.d), device=dev).uniform_(-1, 1, generator=g)
    lim = float(np.sqrt(6.0 / (args.d + args.h)))
    w1 = torch.empty((args.d, args.h), device=dev)
    w2 = torch.empty((args.h, args.d), device=dev)
    b1 = torch.empty((args.h,), device=dev)
    b2 = torch.empty((args.d,), device=dev)
    if rank == 0:
        g0 = torch.Generator(device=dev)
        g0.manual_seed(5)
        w1.uniform_(-lim, lim, generator=g0)
        w2.uniform_(-lim, lim, generator=g0)
        b1.normal_(0.0, 0.02, generator=g0)
        b2.normal_(0.0, 0.02, generator=g0)
    broadcast_weights(w1, b1)
    broadcast_weights(w2, b2)
    model = MLP2(w1, b1, w2, b2, args.mode, None if args.h_dtype == "auto" else args.h_dtype == "bf16")
    h = torch.empty((rows, args.h), device=dev, dtype=model.h_dtype)
    out = torch.empty((rows, args.d), device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        model(x, h, out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(args.steps):
        model(x, h, out)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    status = _lib.device_status(stream.cuda_stream)

    # Per-layer FP64 check on a seeded subset of this rank's rows (layer 2 on our own H).
    sel = np.sort(np.random.default_rng(rank).choice(rows, min(args.check_rows, rows), replace=False))
    xs, hs, os_ = x[sel].cpu().numpy(), h[sel].float().cpu().numpy(), out[sel].cpu().numpy()
    r_1 = tc.check_output("mbr", {"a": xs, "b": w1.cpu().numpy(), "bias": b1.cpu().numpy()}, hs, args.mode,
                          out_unit=2.0 ** -8 if model.h_bf16 else 0.0)
    r_2 = tc.check_output("mbr", {"a": hs, "b": w2.cpu().numpy(), "bias": b2.cpu().numpy()}, os_, args.mode)
    ok = torch.tensor([int(r_1["pass"] and r_2["pass"] and status == 0)], device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0:
        t = float(ms.item())
        print(json.dumps({"workload": f"mlp2 X {args.m}x{args.d}, W1 {args.d}x{args.h}, W2 {args.h}x{args.d}",
                          "mode": args.mode, "h_dtype": "bf16" if model.h_bf16 else "f32",
                          "n_gpus": world, "ms_per_step": t,
                          "tflops": flops(args.m, args.d, args.h) / (t * 1e-3) / 1e12,
                          "err_over_bound_layer1": r_1["err_over_bound"], "err_over_bound_layer2": r_2["err_over_bound"],
                          "checked_rows_per_rank": int(len(sel)), "pass": bool(ok.item())}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if ok.item() else 1


if __name__ == "__main__":
    sys.exit(main())
