"""GPU parity at the shapes and input distributions of the benchmark configurations.

Each case goes through the C-ABI with the kernel the dispatch picks (nothing forced unless
a comparison needs it) and is checked against FP64 on a seeded subset of 64 rows with the
reference's bound, gamma_{K+1}(|A||B| + |aux|) (python/tforge_cpu.py:103-145), widened by
the stated input-rounding term (2u + u^2)|A||B| for TF32 (u = 2^-10) and BF16 (u = 2^-8):

* config 3: 4096^3, 8192x4096x1024 and 256x16384x4096, U[-1, 1], matmul / mbr /
  matmul_add in the fp32-accurate (3xTF32) mode; 256x16384x4096 takes 256x240 pair tiles.
* config 4: the per-GPU shard of the M-sharded problem at 8 GPUs, 16384x8192x8192, with
  A, B ~ N(0, 1/sqrt(K)) and bias ~ N(0, 0.1), in TF32 and BF16.  TF32 reads B as given, in
  k-group-major tiles; that result must equal reading a transposed (K-major) copy of B
  bit for bit.
* config 5: the two-layer MLP at its full widths, D = 4096 and H = 16384, with 2048 rows,
  Xavier-uniform weights and N(0, 0.02) biases, each layer checked against its own FP64
  reference (layer 2 on the kernel's own H), fp32 and BF16 with a bf16 H.
"""

import numpy as np
import pytest

from tensorforge_b200 import _lib, tforge_cpu as tc, tforge_gpu as tg

pytestmark = pytest.mark.gpu

CHECK_ROWS = 64


def _rows(m, seed):
    return np.sort(np.random.default_rng(seed).choice(m, min(CHECK_ROWS, m), replace=False))


@pytest.mark.parametrize("workload", ["matmul", "mbr", "matmul_add"])
@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (8192, 4096, 1024), (256, 16384, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_config3_shapes_fp32_row_subset(gpu, workload, shape):
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 3)
    d = _lib.describe(workload, m, n, k, "fp32")
    assert d["kernel"] == "tf_gemm_tcgen05_3xtf32_pair"
    if shape == (256, 16384, 4096):
        assert d["tile"][:2] == [256, 240] and d["split_k"] == 1
    out = tg.run_op(workload, ins, m, n, k, "fp32")
    assert not np.isnan(out).any()
    res = tc.check_output(workload, ins, out, "fp32", rows=_rows(m, 31))
    assert res["pass"], res


@pytest.fixture(scope="module")
def config4_shard():
    """16384 x 8192 x 8192 with config 4's distributions, resident on the device."""
    import torch

    m, n, k = 16384, 8192, 8192
    ins = tc.make_inputs_normal(m, n, k, seed=4)
    dev = torch.device("cuda", 0)
    t = {name: torch.from_numpy(arr).to(dev) for name, arr in ins.items()}
    yield (m, n, k), ins, t
    del t
    torch.cuda.empty_cache()


def _mbr_device(t, m, n, k, mode):
    import torch

    out = torch.full((m, n), float("nan"), device=t["a"].device)
    _lib.gemm("mbr", t["a"].data_ptr(), t["b"].data_ptr(), out.data_ptr(), m, n, k, mode, bias=t["bias"].data_ptr())
    torch.cuda.synchronize()
    assert _lib.device_status(None) == 0
    return out


def test_config4_shard_tf32_transposed_b_bitwise_and_bound(gpu, config4_shard):
    (m, n, k), ins, t = config4_shard
    d = _lib.describe("mbr", m, n, k, "tf32")
    assert d["kernel"].startswith("tf_gemm_tcgen05_tf32_pair")
    auto = _mbr_device(t, m, n, k, "tf32")        # dispatch: B as given, k-group-major tiles
    _lib.set_config(b_layout=2)                    # the same kernel on a transposed copy of B
    try:
        tcopy = _mbr_device(t, m, n, k, "tf32")
    finally:
        _lib.set_config()
    import torch

    assert torch.equal(auto.view(torch.int32), tcopy.view(torch.int32))
    rows = _rows(m, 41)
    o = auto[torch.from_numpy(rows).to(auto.device)].cpu().numpy()
    res = tc.check_output("mbr", {"a": ins["a"][rows], "b": ins["b"], "bias": ins["bias"]}, o, "tf32")
    assert res["pass"], res


def test_config4_shard_bf16_bound(gpu, config4_shard):
    import torch

    (m, n, k), ins, t = config4_shard
    out = _mbr_device(t, m, n, k, "bf16")
    rows = _rows(m, 43)
    o = out[torch.from_numpy(rows).to(out.device)].cpu().numpy()
    res = tc.check_output("mbr", {"a": ins["a"][rows], "b": ins["b"], "bias": ins["bias"]}, o, "bf16")
    assert res["pass"], res


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_config5_mlp_full_widths_per_layer_bound(gpu, mode):
    import torch

    from tensorforge_b200.mlp import MLP2

    m, d, h = 2048, 4096, 16384
    ins = tc.make_mlp_inputs(m, d, h, seed=5)
    dev = torch.device("cuda", 0)
    t = {name: torch.from_numpy(v).to(dev) for name, v in ins.items()}
    model = MLP2(t["w1"], t["b1"], t["w2"], t["b2"], mode)
    assert model.h_bf16 == (mode == "bf16")
    hid, out = model(t["x"])
    torch.cuda.synchronize()
    assert _lib.device_status(None) == 0
    rows = _rows(m, 51)
    sel = torch.from_numpy(rows).to(dev)
    hn, on = hid[sel].float().cpu().numpy(), out[sel].cpu().numpy()
    r1 = tc.check_output("mbr", {"a": ins["x"][rows], "b": ins["w1"], "bias": ins["b1"]}, hn, mode,
                         out_unit=2.0 ** -8 if model.h_bf16 else 0.0)
    r2 = tc.check_output("mbr", {"a": hn, "b": ins["w2"], "bias": ins["b2"]}, on, mode)
    assert r1["pass"] and r2["pass"], (r1, r2)
    assert not torch.isnan(out).any()
