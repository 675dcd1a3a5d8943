"""BF16 mode with f32 operands against the same call on bf16 operands.

tforge_gemm in TFORGE_MODE_BF16 with f32 A and B rounds both to bf16 (round to nearest
even) into pooled scratch and runs the tensor-core kernel on the copies.  The result must be
the same bits as rounding the operands first (tforge_convert_bf16) and calling tforge_gemm
with bf16 operands, and meet the BF16 bound.  Shapes: one round of 256 x 256 pair tiles
(2048^3), several rounds with ragged edges and a K tail, many rounds with few panels; every
epilogue; A and B in row pitches that are not multiples of 8 elements (read in place, still
on the tensor cores); calls in flight on two streams; a wait that expires (the skip-load
hook) must be reported and the next call right.
"""

import numpy as np
import pytest

from tensorforge_b200 import _lib, tforge_cpu as tc

pytestmark = pytest.mark.gpu

SHAPES = [(2048, 2048, 2048), (3000, 2600, 520), (4096, 1024, 1024), (300, 264, 136), (2560, 512, 4096)]


def _bf16_operand_reference(t, wl, m, n, k, lda, ldb):
    """Convert A and B with tforge_convert_bf16, then tforge_gemm on the bf16 copies."""
    import torch

    L = _lib.lib()
    a16 = torch.empty((m, k), device=t["a"].device, dtype=torch.bfloat16)
    b16 = torch.empty((k, n), device=t["a"].device, dtype=torch.bfloat16)
    a32 = t["a"][:, :k].contiguous() if lda != k else t["a"]
    b32 = t["b"][:, :n].contiguous() if ldb != n else t["b"]
    _lib.check(L.tforge_convert_bf16(a32.data_ptr(), a16.data_ptr(), m * k, None), "convert A")
    _lib.check(L.tforge_convert_bf16(b32.data_ptr(), b16.data_ptr(), k * n, None), "convert B")
    out = torch.full((m, n), float("nan"), device=t["a"].device)
    _lib.gemm(wl, a16.data_ptr(), b16.data_ptr(), out.data_ptr(), m, n, k, "bf16",
              bias=t["bias"].data_ptr() if "bias" in t else None, c_res=t["c"].data_ptr() if "c" in t else None,
              a_dtype=_lib.BF16, b_dtype=_lib.BF16)
    return out


@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_f32_operands_match_converted_operands_bitwise(gpu, workload, shape):
    import torch

    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 61)
    ins["a"][3, 5] = np.nan  # a NaN row stays NaN through the conversion
    dev = torch.device("cuda", 0)
    t = {name: torch.from_numpy(arr).to(dev) for name, arr in ins.items()}
    out = torch.full((m, n), float("nan"), device=dev)
    _lib.gemm(workload, t["a"].data_ptr(), t["b"].data_ptr(), out.data_ptr(), m, n, k, "bf16",
              bias=t["bias"].data_ptr() if "bias" in t else None, c_res=t["c"].data_ptr() if "c" in t else None)
    ref = _bf16_operand_reference(t, workload, m, n, k, k, n)
    torch.cuda.synchronize()
    assert _lib.device_status(None) == _lib.OK
    assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
    o = out.cpu().numpy()
    assert np.isnan(o[3]).all()
    rows = np.array([r for r in range(0, m, max(1, m // 48)) if r != 3])
    res = tc.check_output(workload, ins, o, "bf16", rows=rows)
    assert res["pass"], res


@pytest.mark.parametrize("shape", [(2300, 2064, 776), (700, 520, 264)], ids=lambda s: "x".join(map(str, s)))
def test_f32_operands_pitched(gpu, shape):
    """A and B in wider row pitches (lda = K + 12, ldb = N + 4, not multiples of 8 elements):
    read in place into the packed bf16 copies, same bits as converting first, on the tensor
    cores (not the exact SIMT kernel)."""
    import torch

    m, n, k = shape
    ins = tc.make_inputs("mbr", m, n, k, 62)
    dev = torch.device("cuda", 0)
    abig = torch.zeros((m, k + 12), device=dev)
    bbig = torch.zeros((k, n + 4), device=dev)
    abig[:, :k] = torch.from_numpy(ins["a"]).to(dev)
    bbig[:, :n] = torch.from_numpy(ins["b"]).to(dev)
    bias = torch.from_numpy(ins["bias"]).to(dev)
    out = torch.full((m, n), float("nan"), device=dev)
    _lib.gemm("mbr", abig.data_ptr(), bbig.data_ptr(), out.data_ptr(), m, n, k, "bf16", bias=bias.data_ptr(),
              lda=k + 12, ldb=n + 4)
    t = {"a": abig, "b": bbig, "bias": bias}
    ref = _bf16_operand_reference(t, "mbr", m, n, k, k + 12, n + 4)
    torch.cuda.synchronize()
    assert _lib.device_status(None) == _lib.OK
    assert torch.equal(out.view(torch.int32), ref.view(torch.int32))


def test_f32_operands_two_streams(gpu):
    """Calls in flight on two streams each take their own scratch from the pool."""
    import torch

    dev = torch.device("cuda", 0)
    cases = [(2048, 2048, 1024, 63), (1536, 3072, 512, 64)]
    data = []
    for m, n, k, seed in cases:
        ins = tc.make_inputs("mbr", m, n, k, seed)
        data.append((m, n, k, {name: torch.from_numpy(arr).to(dev) for name, arr in ins.items()}))
    refs = [_bf16_operand_reference(t, "mbr", m, n, k, k, n) for m, n, k, t in data]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    # Outputs are filled on the default stream and finished before the side streams start.
    outs = [(i, torch.full((m, n), float("nan"), device=dev)) for _ in range(3) for i, (m, n, _, _) in enumerate(data)]
    torch.cuda.synchronize()
    for j, (i, o) in enumerate(outs):
        m, n, k, t = data[i]
        _lib.gemm("mbr", t["a"].data_ptr(), t["b"].data_ptr(), o.data_ptr(), m, n, k, "bf16",
                  bias=t["bias"].data_ptr(), stream=streams[(j // len(data) + i) % 2].cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_status(None) == _lib.OK
    for i, o in outs:
        assert torch.equal(o.view(torch.int32), refs[i].view(torch.int32))


def test_f32_operands_timeout_reported_and_recovers(gpu):
    import torch

    L = _lib.lib()
    m, n, k = 2048, 2048, 512
    ins = tc.make_inputs("mbr", m, n, k, 65)
    dev = torch.device("cuda", 0)
    t = {name: torch.from_numpy(arr).to(dev) for name, arr in ins.items()}
    out = torch.empty((m, n), device=dev)

    def call():
        _lib.gemm("mbr", t["a"].data_ptr(), t["b"].data_ptr(), out.data_ptr(), m, n, k, "bf16",
                  bias=t["bias"].data_ptr())

    try:
        assert L.tforge_set_wait_limit_ns(50_000_000) == 0
        assert L.tforge_debug_skip_load(1) == 0
        call()
        assert _lib.device_status(None) == _lib.ERR_TIMEOUT
    finally:
        L.tforge_debug_skip_load(0)
        L.tforge_set_wait_limit_ns(0)
    call()
    ref = _bf16_operand_reference(t, "mbr", m, n, k, k, n)
    torch.cuda.synchronize()
    assert _lib.device_status(None) == _lib.OK
    assert torch.equal(out.view(torch.int32), ref.view(torch.int32))


def test_runner_bf16_operands_match_f32_operands(gpu, tmp_path):
    """The runner's --operands bf16 (A and B rounded once before timing, the GEMM timed on the
    bf16 copies) writes the same output bits as the BF16-mode call on f32 operands."""
    import json
    import subprocess

    from tensorforge_b200 import tforge_gpu as tg

    outs = {}
    for ops in ("f32", "bf16"):
        path = tmp_path / f"{ops}.bin"
        r = subprocess.run([str(tg.GPU_BENCH), "--mode", "lib", "--workload", "mbr", "--m", "700", "--n", "520",
                            "--k", "264", "--precision", "bf16", "--operands", ops, "--warmup", "1", "--reps", "2",
                            "--seed", "71", "--out", str(path)], capture_output=True, text=True, check=True)
        assert json.loads(r.stdout)["median_ms"] > 0
        outs[ops] = np.fromfile(path, dtype=np.uint32)
    assert outs["f32"].size == 700 * 520
    assert np.array_equal(outs["f32"], outs["bf16"])
