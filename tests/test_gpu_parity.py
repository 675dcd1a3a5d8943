"""GPU parity: every kernel through the C-ABI against the CPU restatement and the
reference's FP64 check.

* fp32_exact (SIMT FFMA, sequential k): bit-exact against the restatement, i.e. the
  reference's generated kernels (docs/numerics.md:3,53).
* fp32 (3xTF32 on tcgen05): err/bound <= 1 with the reference's bound
  gamma_{K+1}(|A||B| + |bias|) (python/tforge_cpu.py:128-145).
* tf32 / bf16: err/bound <= 1 against the stated looser bound that adds the input
  rounding term (2u + u^2)|A||B|, u = 2^-10 (TF32 truncation) or 2^-8 (bf16).
* elementwise ops: bit-exact.
"""

import ctypes as C
import json
import subprocess

import numpy as np
import pytest

from tensorforge_b200 import _lib, tforge_cpu as tc, tforge_gpu as tg

pytestmark = pytest.mark.gpu

# 1664x1536x96 has 156 tiles of 128x128 (the large-tile SIMT kernel); the others use 64x64.
EXACT_SHAPES = [(256, 256, 128), (777, 1111, 333), (1000, 1000, 1000), (7, 19, 5), (1, 1, 1),
                (130, 260, 36), (256, 256, 0), (1664, 1536, 96), (1665, 1537, 97)]
TC_SHAPES = [(256, 256, 128), (2048, 2048, 2048), (1000, 1000, 1000), (512, 512, 4096), (129, 264, 36),
             (300, 8, 64), (4, 2048, 128), (1, 4, 16), (513, 1000, 520), (128, 256, 2048)]


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("shape", EXACT_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("workload", ["matmul", "mbr", "matmul_add"])
def test_fp32_exact_is_bitwise_reference(gpu, oracle, workload, shape):
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 1234)
    out = tg.run_op(workload, ins, m, n, k, "fp32_exact")
    ref = oracle.gemm(workload, ins)
    assert np.array_equal(bits(out), bits(ref))


@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
def test_tensor_core_modes_within_bound(gpu, workload, mode, shape):
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 1234)
    out = tg.run_op(workload, ins, m, n, k, mode)
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0
    assert res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("seed", [0, 1234])
def test_config1_fp32_mode(gpu, seed):
    """relu(x @ w + b), x 256x128, w 128x256, seeds 0 and 1234."""
    ins = tc.make_inputs("mbr", 256, 256, 128, seed)
    d = _lib.describe("mbr", 256, 256, 128, "fp32")
    assert d["kernel"].startswith("tf_gemm_tcgen05_3xtf32")  # whichever 3xTF32 kernel the sweep measured fastest
    out = tg.run_op("mbr", ins, 256, 256, 128, "fp32")
    res = tc.check_output("mbr", ins, out)
    assert res["pass"] and res["err_over_bound"] < 0.25, res


@pytest.mark.parametrize("bn,stages", [(256, 2), (128, 3), (64, 4)])
@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_every_instantiated_config(gpu, mode, bn, stages):
    st = {"fp32": stages, "tf32": {256: 4, 128: 6, 64: 8}[bn], "bf16": {256: 4, 128: 6, 64: 8}[bn]}[mode]
    m, n, k = 384, 520, 200
    ins = tc.make_inputs("mbr", m, n, k, 5)
    out = tg.run_op("mbr", ins, m, n, k, mode, options=f"bn={bn} stages={st}")
    res = tc.check_output("mbr", ins, out, mode)
    assert res["pass"], res


@pytest.mark.parametrize("shape", [(33, 17), (256, 1024), (1000, 999), (1, 1), (4096, 4096)])
@pytest.mark.parametrize("workload", ["relu", "bias_add", "add"])
def test_elementwise_bitwise(gpu, oracle, workload, shape):
    m, n = shape
    ins = tc.make_inputs(workload, m, n, None, 99)
    if workload == "relu":
        ins["a"].ravel()[:5] = np.array([-1.0, -0.0, np.nan, 2.5, 0.0], dtype=np.float32)[: ins["a"].size]
    out = tg.run_op(workload, ins, m, n, None)
    assert np.array_equal(bits(out), bits(oracle.elementwise(workload, ins)))
    assert tc.check_elementwise(workload, ins, out)["pass"]


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16", "fp32_exact"])
def test_epilogue_nan_and_signed_zero(gpu, mode):
    """relu = IEEE maximum: NaN propagates, no -0.0 ever leaves the kernel."""
    m, n, k = 256, 256, 64
    ins = tc.make_inputs("mbr", m, n, k, 11)
    ins["a"][3, 5] = np.nan
    ins["bias"][:8] = -0.0
    out = tg.run_op("mbr", ins, m, n, k, mode)
    assert np.isnan(out[3]).all()
    rest = np.delete(out, 3, axis=0)
    assert not np.isnan(rest).any()
    assert not (bits(rest) == 0x80000000).any()
    assert (rest >= 0).all()


def test_pitched_views(gpu):
    """Sub-matrix views through lda/ldb/ldc (row shards and column blocks)."""
    M, N, K, lda, ldb, ldc = 300, 200, 96, 128, 256, 256
    rng = np.random.default_rng(3)
    Abig = rng.uniform(-1, 1, (M, lda)).astype(np.float32)
    Bbig = rng.uniform(-1, 1, (K, ldb)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    a, b, bb = (tg.DeviceBuffer.upload(x) for x in (Abig, Bbig, bias))
    out = tg.DeviceBuffer(M * ldc * 4)
    try:
        for mode in ("fp32", "tf32", "fp32_exact"):
            _lib.check(_lib.lib().tforge_memset(out.ptr, 0, M * ldc * 4, None))
            _lib.gemm("mbr", a.addr, b.addr, out.addr, M, N, K, mode, bias=bb.addr, lda=lda, ldb=ldb, ldc=ldc)
            got = out.download((M, ldc))
            ins = {"a": Abig[:, :K].copy(), "b": Bbig[:, :N].copy(), "bias": bias}
            assert tc.check_output("mbr", ins, got[:, :N], mode)["pass"]
            assert (got[:, N:] == 0).all()  # nothing written outside the view
    finally:
        for x in (a, b, bb, out):
            x.free()


def test_bf16_operands_match_f32_input_bf16_mode(gpu):
    m, n, k = 512, 384, 256
    ins = tc.make_inputs("mbr", m, n, k, 8)
    ref = tg.run_op("mbr", ins, m, n, k, "bf16")
    L = _lib.lib()
    a, b, bias = (tg.DeviceBuffer.upload(ins[x]) for x in ("a", "b", "bias"))
    a16, b16, out = tg.DeviceBuffer(m * k * 2), tg.DeviceBuffer(k * n * 2), tg.DeviceBuffer(m * n * 4)
    try:
        _lib.check(L.tforge_convert_bf16(a.ptr, a16.ptr, m * k, None))
        _lib.check(L.tforge_convert_bf16(b.ptr, b16.ptr, k * n, None))
        _lib.gemm("mbr", a16.addr, b16.addr, out.addr, m, n, k, "bf16", bias=bias.addr,
                  a_dtype=_lib.BF16, b_dtype=_lib.BF16)
        got = out.download((m, n))
        assert np.array_equal(bits(got), bits(ref))
    finally:
        for x in (a, b, bias, a16, b16, out):
            x.free()


def test_large_square_row_subset(gpu):
    """cfg3 8192^3 in fp32 mode: FP64 check on a seeded subset of 64 rows."""
    m = n = k = 8192
    ins = tc.make_inputs("mbr", m, n, k, 1234)
    out = tg.run_op("mbr", ins, m, n, k, "fp32")
    rows = np.sort(np.random.default_rng(0).choice(m, 64, replace=False))
    res = tc.check_output("mbr", ins, out, "fp32", rows=rows)
    assert res["pass"], res
    assert not np.isnan(out).any()


def test_bounded_wait_reports_timeout_and_context_survives(gpu):
    """A stage that never fills: the consumer's bounded wait expires, the kernel drains
    and returns, the status word says TIMEOUT, and the next call is correct."""
    L = _lib.lib()
    m, n, k = 256, 256, 256
    ins = tc.make_inputs("mbr", m, n, k, 2)
    a, b, bias = (tg.DeviceBuffer.upload(ins[x]) for x in ("a", "b", "bias"))
    out = tg.DeviceBuffer(m * n * 4)
    try:
        assert L.tforge_set_wait_limit_ns(50_000_000) == 0
        assert L.tforge_debug_skip_load(1) == 0
        _lib.gemm("mbr", a.addr, b.addr, out.addr, m, n, k, "tf32", bias=bias.addr)
        assert _lib.device_status(None) == _lib.ERR_TIMEOUT
    finally:
        L.tforge_debug_skip_load(0)
        L.tforge_set_wait_limit_ns(0)
    _lib.gemm("mbr", a.addr, b.addr, out.addr, m, n, k, "tf32", bias=bias.addr)
    assert _lib.device_status(None) == 0
    assert tc.check_output("mbr", ins, out.download((m, n)), "tf32")["pass"]
    for x in (a, b, bias, out):
        x.free()


def test_describe_reports_device_resources(gpu):
    d = _lib.describe("mbr", 2048, 2048, 2048, "fp32")
    assert d["regs"] > 0 and d["blocks_per_sm"] >= 1


def test_runner_lib_and_cublas_modes(gpu, tmp_path):
    for mode in ("lib", "cublas"):
        r = json.loads(subprocess.run([str(tg.GPU_BENCH), "--mode", mode, "--workload", "mbr", "--m", "512",
                                       "--n", "512", "--k", "512", "--warmup", "1", "--reps", "3"],
                                      capture_output=True, text=True, check=True).stdout)
        for key in ("gpu", "median_ms", "grid", "block", "sm_clock_median_mhz", "cuda_driver"):
            assert key in r
        assert r["median_ms"] > 0


@pytest.mark.parametrize("splits", [2, 3, 8])
@pytest.mark.parametrize("mode", ["fp32", "tf32"])
@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("shape", [(300, 264, 1024), (512, 512, 2048)], ids=lambda s: "x".join(map(str, s)))
def test_pair_split_k_within_bound_and_deterministic(gpu, workload, mode, splits, shape):
    """Split-K on the pair kernel: S pairs per tile over K / S each, partial sums summed in a
    fixed order; ragged M and N, every epilogue; two runs agree bit for bit."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 21)
    _lib.set_config(3, split_k=splits)
    try:
        assert _lib.describe(workload, m, n, k, mode)["split_k"] == splits
        out = tg.run_op(workload, ins, m, n, k, mode)
        again = tg.run_op(workload, ins, m, n, k, mode)
    finally:
        _lib.set_config()
    assert np.array_equal(bits(out), bits(again))
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("shape", [(300, 2152, 200), (520, 1936, 96), (256, 240, 64)],
                         ids=lambda s: "x".join(map(str, s)))
def test_pair_240_wide_tiles_within_bound(gpu, workload, mode, shape):
    """256 x 240 pair tiles: each CTA's MMA half is the first 120 of the 128 B columns it
    loads and the last 16 columns of a tile are stored without TMA.  N = 2152 ends inside a
    tile's last 16 columns, N = 1936 leaves the last tile's second CTA wholly out of range,
    256 x 240 is one tile; ragged M."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 23)
    _lib.set_config(3, 240)
    try:
        d = _lib.describe(workload, m, n, k, mode)
        assert d["tile"][1] == 240 and d["grid"][0] == 2 * -(-n // 240)
        out = tg.run_op(workload, ins, m, n, k, mode)
    finally:
        _lib.set_config()
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_pair_240_matches_256_bitwise(gpu, mode):
    """Each output element sees the same k-block order and the same per-k-step MMA sequence
    whichever tile width covers it, so 256 x 240 and 256 x 256 tiles agree bit for bit (both
    without split-K, which the 256-wide tiles would take here by default)."""
    m, n, k = 512, 1024, 512
    ins = tc.make_inputs("mbr", m, n, k, 29)
    outs = []
    for bn in (256, 240):
        _lib.set_config(3, bn, split_k=1)
        try:
            outs.append(tg.run_op("mbr", ins, m, n, k, mode))
        finally:
            _lib.set_config()
    assert np.array_equal(bits(outs[0]), bits(outs[1]))


def test_automatic_split_k_small_square(gpu):
    """1024^3 has 16 pair tiles for 74 SM pairs: the dispatch splits K and stays in bound."""
    d = _lib.describe("mbr", 1024, 1024, 1024, "fp32")
    assert d["kernel"].endswith("_pair") and d["split_k"] >= 2 and d["grid"][2] == d["split_k"]
    ins = tc.make_inputs("mbr", 1024, 1024, 1024, 5)
    out = tg.run_op("mbr", ins, 1024, 1024, 1024, "fp32")
    res = tc.check_output("mbr", ins, out, "fp32")
    assert res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("math,precision", [("default", "fp32"), ("bf16x9", "fp32"), ("lt", "fp32"),
                                            ("lt_tf32", "tf32"), ("tf32", "tf32"), ("bf16", "bf16"),
                                            ("lt_bf16", "bf16")])
def test_runner_cublas_comparators_within_bound(gpu, tmp_path, math, precision):
    """Every cuBLAS comparator path of the runner computes relu(A@B+bias) on the reference's
    inputs within the bound of its precision (bf16x9 emulation and FP32 paths: the fp32
    bound; TF32 and bf16 paths: their looser bounds)."""
    m, n, k = 384, 512, 256
    ins = tc.make_inputs("mbr", m, n, k, 1234)
    for name, arr in ins.items():
        arr.tofile(tmp_path / f"{name}.bin")
    subprocess.run([str(tg.GPU_BENCH), "--mode", "cublas", "--math", math, "--workload", "mbr", "--m", str(m),
                    "--n", str(n), "--k", str(k), "--warmup", "0", "--reps", "1", "--in-dir", str(tmp_path),
                    "--out", str(tmp_path / "out.bin")], capture_output=True, text=True, check=True)
    out = np.fromfile(tmp_path / "out.bin", dtype=np.float32).reshape(m, n)
    res = tc.check_output("mbr", ins, out, precision)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


def test_shim_check_matches_reference_api(gpu):
    """tg.check returns (res, out) like python/tforge_gpu.py:112-145, for lib and cuBLAS."""
    for mode in ("kernel", "cublas"):
        res, out = tg.check("mbr", 256, 256, 256, mode=mode)
        assert res["pass"] and out.shape == (256, 256)
    res, out = tg.check("relu", 64, 48, 1)
    assert res["pass"]


PAIR_SHAPES = [(256, 256, 32), (300, 520, 200), (1000, 1000, 1000), (512, 256, 2048), (257, 260, 36),
               (2048, 2048, 2048)]


@pytest.mark.parametrize("shape", PAIR_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul_add"])
def test_pair_kernel_within_bound(gpu, workload, mode, shape):
    """The CTA-pair (cta_group::2) kernel, forced, on ragged and full tiles."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 77)
    _lib.set_config(3)
    try:
        # bf16 rows must be 16-byte multiples for TMA (N, K multiples of 8); otherwise the
        # table routes the call to the exact SIMT kernel.
        tma_ok = mode != "bf16" or (n % 8 == 0 and k % 8 == 0)
        assert _lib.describe(workload, m, n, k, mode)["kernel"].endswith("_pair") == tma_ok
        out = tg.run_op(workload, ins, m, n, k, mode)
    finally:
        _lib.set_config()
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


def test_pair_kernel_bounded_wait(gpu):
    """Timeout path of the pair kernel: both CTAs drain, status is TIMEOUT, next call is right."""
    L = _lib.lib()
    m, n, k = 512, 512, 256
    ins = tc.make_inputs("mbr", m, n, k, 4)
    a, b, bias = (tg.DeviceBuffer.upload(ins[x]) for x in ("a", "b", "bias"))
    out = tg.DeviceBuffer(m * n * 4)
    _lib.set_config(3)
    try:
        for mode in ("fp32", "tf32"):
            assert L.tforge_set_wait_limit_ns(50_000_000) == 0
            assert L.tforge_debug_skip_load(1) == 0
            try:
                _lib.gemm("mbr", a.addr, b.addr, out.addr, m, n, k, mode, bias=bias.addr)
                assert _lib.device_status(None) == _lib.ERR_TIMEOUT
            finally:
                L.tforge_debug_skip_load(0)
                L.tforge_set_wait_limit_ns(0)
            _lib.gemm("mbr", a.addr, b.addr, out.addr, m, n, k, mode, bias=bias.addr)
            assert _lib.device_status(None) == 0
            assert tc.check_output("mbr", ins, out.download((m, n)), mode)["pass"]
    finally:
        _lib.set_config()
        for x in (a, b, bias, out):
            x.free()


@pytest.mark.parametrize("mode", ["tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("shape", [(2600, 2400, 96), (4100, 4000, 64), (300, 264, 520)],
                         ids=lambda s: "x".join(map(str, s)))
def test_persistent_pair_within_bound(gpu, workload, mode, shape):
    """Persistent CTA-pair kernel: clusters loop over tiles with two TMEM accumulators
    (110 and 272 tiles: every cluster reuses both accumulators; ragged M and N; one cluster
    with a single ragged tile and a K tail)."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 31)
    _lib.set_config(3, 0, 0, 1)
    try:
        d = _lib.describe(workload, m, n, k, mode)
        assert d["kernel"].endswith("_pair_persistent") and d["persistent"] == 1 and d["tmem_cols"] == 512
        tiles = -(-m // 256) * -(-n // 256)
        assert d["grid"][0] == 2 * min(tiles, d["grid"][0] // 2) and d["grid"][1] == 1
        out = tg.run_op(workload, ins, m, n, k, mode)
    finally:
        _lib.set_config()
    res = tc.check_output(workload, ins, out, mode)
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("mode", ["tf32", "bf16"])
@pytest.mark.parametrize("workload", ["mbr", "matmul_add"])
def test_persistent_pair_matches_pair_bitwise(gpu, workload, mode):
    """Per tile the persistent kernel runs the pair kernel's k-block order and MMA sequence,
    so the two agree bit for bit (160 tiles: two to three per cluster)."""
    m, n, k = 4096, 2560, 256
    ins = tc.make_inputs(workload, m, n, k, 37)
    outs = []
    for persistent in (0, 1):
        _lib.set_config(3, 0, 0, persistent, 1)
        try:
            outs.append(tg.run_op(workload, ins, m, n, k, mode))
        finally:
            _lib.set_config()
    assert np.array_equal(bits(outs[0]), bits(outs[1]))


def test_persistent_pair_bounded_wait(gpu):
    """Timeout path of the persistent kernel: the MMA issuer, the producers and both CTAs'
    epilogues give up, drain and meet; status is TIMEOUT; the next call is right."""
    L = _lib.lib()
    m, n, k = 1024, 1024, 256
    ins = tc.make_inputs("mbr", m, n, k, 41)
    a, b, bias = (tg.DeviceBuffer.upload(ins[x]) for x in ("a", "b", "bias"))
    out = tg.DeviceBuffer(m * n * 4)
    _lib.set_config(3, 0, 0, 1)
    try:
        for mode in ("tf32", "bf16"):
            assert L.tforge_set_wait_limit_ns(50_000_000) == 0
            assert L.tforge_debug_skip_load(1) == 0
            try:
                _lib.gemm("mbr", a.addr, b.addr, out.addr, m, n, k, mode, bias=bias.addr)
                assert _lib.device_status(None) == _lib.ERR_TIMEOUT
            finally:
                L.tforge_debug_skip_load(0)
                L.tforge_set_wait_limit_ns(0)
            _lib.gemm("mbr", a.addr, b.addr, out.addr, m, n, k, mode, bias=bias.addr)
            assert _lib.device_status(None) == 0
            assert tc.check_output("mbr", ins, out.download((m, n)), mode)["pass"]
    finally:
        _lib.set_config()
        for x in (a, b, bias, out):
            x.free()


def test_tf32_operands_are_read_truncated(gpu):
    """The truncation split of the 3xTF32 pair kernel relies on the tensor core reading an
    f32 operand as TF32 by discarding its low 13 mantissa bits (not rounding): pin it.

    One nonzero product per output: A[m, 0] = 1 + (m + 1) 2^-16 (m < 63: only discarded
    bits set), B[0, n] = 1, so a truncating read gives exactly 1.0 and a rounding read
    gives 1 + 2^-10 for m >= 31.  Then the same with the roles of A and B swapped."""
    m, n, k = 128, 64, 32
    a = np.zeros((m, k), np.float32)
    b = np.zeros((k, n), np.float32)
    a[:63, 0] = 1 + (np.arange(63) + 1) * 2.0 ** -16
    b[0, :] = 1
    _lib.set_config(1, 64, 8)
    try:
        out = tg.run_op("matmul", {"a": a, "b": b}, m, n, k, "tf32")
        assert (out[:63] == 1.0).all(), out[:63, 0]
        a2 = np.zeros((m, k), np.float32)
        b2 = np.zeros((k, n), np.float32)
        a2[:, 0] = 1
        b2[0, :63] = 1 + (np.arange(63) + 1) * 2.0 ** -16
        out2 = tg.run_op("matmul", {"a": a2, "b": b2}, m, n, k, "tf32")
        assert (out2[:, :63] == 1.0).all(), out2[0]
    finally:
        _lib.set_config()


def test_row_sharded_calls_cover_the_full_problem(gpu):
    """Rank-style row blocks (uneven split of M) through shard.mbr_rows equal the bound-checked
    full problem; every row is written exactly once."""
    import torch
    from tensorforge_b200.shard import WeightSet, all_partitions, mbr_rows

    m, n, k = 1000, 512, 384
    ins = tc.make_inputs("mbr", m, n, k, 21)
    dev = torch.device("cuda", 0)
    A = torch.from_numpy(ins["a"]).to(dev)
    ws = WeightSet(torch.from_numpy(ins["b"]).to(dev), torch.from_numpy(ins["bias"]).to(dev))
    out = torch.full((m, n), float("nan"), device=dev)
    for r0, r1 in all_partitions(m, 3):
        mbr_rows(A[r0:r1], ws, out[r0:r1], "fp32")
    torch.cuda.synchronize()
    res = tc.check_output("mbr", ins, out.cpu().numpy(), "fp32")
    assert res["pass"] and res["nan_count"] == 0, res


@pytest.mark.parametrize("mode", ["fp32", "bf16", "tf32"])
def test_mlp_chain_per_layer_bound(gpu, mode):
    """relu(relu(X W1 + b1) W2 + b2), Xavier weights, N(0, 0.02) biases; each layer checked
    against FP64 with its own bound (layer 2 on the kernel's own H)."""
    import torch
    from tensorforge_b200.mlp import MLP2

    ins = tc.make_mlp_inputs(640, 256, 1024, seed=3)
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in ins.items()}
    model = MLP2(t["w1"], t["b1"], t["w2"], t["b2"], mode)
    h, out = model(t["x"])
    torch.cuda.synchronize()
    assert _lib.device_status(None) == 0
    assert model.h_bf16 == (mode == "bf16")  # BF16 mode keeps H in bf16 by default
    hn, on = h.float().cpu().numpy(), out.cpu().numpy()
    r1 = tc.check_output("mbr", {"a": ins["x"], "b": ins["w1"], "bias": ins["b1"]}, hn, mode,
                         out_unit=2.0 ** -8 if model.h_bf16 else 0.0)
    r2 = tc.check_output("mbr", {"a": hn, "b": ins["w2"], "bias": ins["b2"]}, on, mode)
    assert r1["pass"] and r2["pass"], (r1, r2)


def test_mlp_bf16_h_matches_f32_h_bitwise(gpu):
    """A bf16 H (layer 1 rounds in its epilogue) gives the same H values as rounding an f32
    H, and the same final output bits (layer 2 rounds an f32 H to bf16 before its MMAs)."""
    import torch
    from tensorforge_b200.mlp import MLP2

    ins = tc.make_mlp_inputs(1100, 512, 2048, seed=8)
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in ins.items()}
    h16, out16 = MLP2(t["w1"], t["b1"], t["w2"], t["b2"], "bf16", h_bf16=True)(t["x"])
    h32, out32 = MLP2(t["w1"], t["b1"], t["w2"], t["b2"], "bf16", h_bf16=False)(t["x"])
    torch.cuda.synchronize()
    assert h16.dtype == torch.bfloat16 and h32.dtype == torch.float32
    ref16 = torch.empty_like(h16)
    _lib.check(_lib.lib().tforge_convert_bf16(h32.data_ptr(), ref16.data_ptr(), h32.numel(), None), "convert")
    torch.cuda.synchronize()
    assert torch.equal(h16.view(torch.int16), ref16.view(torch.int16))
    assert torch.equal(out16.view(torch.int32), out32.view(torch.int32))


@pytest.mark.parametrize("case", [
    ("mbr", 2048, 2048, 512, 0, None),          # pair kernel, bf16 epilogue
    ("mbr", 1000, 2048, 512, 8, None),          # ragged M, pitched out
    ("mbr", 2600, 2400, 96, 0, (3, 0, 0, 1)),   # persistent pair kernel, 110 tiles
    ("mbr", 300, 264, 520, 0, (3, 0, 0, 1)),    # persistent, one ragged tile, K tail
    ("mbr", 256, 256, 128, 0, None),            # one-CTA kernel: f32 scratch then rounded
    ("mbr", 300, 1004, 64, 0, None),            # N % 8 != 0: f32 scratch path
    ("matmul", 1024, 1024, 256, 0, None),       # matmul: f32 scratch path
    ("matmul_add", 512, 768, 128, 0, None),
    ("mbr", 512, 512, 2048, 0, (3, 0, 0, 0, 2)),  # forced split-K: f32 reduction, then rounded
], ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}x{c[3]}-ld{c[4]}-{'forced' if c[5] else 'table'}")
def test_bf16_output_matches_f32_then_convert(gpu, case):
    """out_dtype = TFORGE_BF16: the bf16 output equals tforge_convert_bf16 of the f32 output
    bit for bit, on the direct epilogue paths and the f32-scratch ones; a NaN row too."""
    import torch

    wl, m, n, k, pad, cfg = case
    ins = tc.make_inputs(wl, m, n, k, 43)
    ins["a"][0, 0] = np.nan
    dev = torch.device("cuda", 0)
    t = {name: torch.from_numpy(arr).to(dev) for name, arr in ins.items()}
    ldc = n + pad
    out32 = torch.empty((m, n), device=dev)
    out16 = torch.full((m, ldc), 7.0, device=dev, dtype=torch.bfloat16)
    if cfg:
        _lib.set_config(*cfg)
    try:
        for out, od, ld in ((out32, _lib.F32, 0), (out16, _lib.BF16, ldc)):
            _lib.gemm(wl, t["a"].data_ptr(), t["b"].data_ptr(), out.data_ptr(), m, n, k, "bf16",
                      bias=t["bias"].data_ptr() if "bias" in t else None,
                      c_res=t["c"].data_ptr() if "c" in t else None, ldc=ld, out_dtype=od)
    finally:
        _lib.set_config()
    ref = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
    _lib.check(_lib.lib().tforge_convert_bf16(out32.data_ptr(), ref.data_ptr(), m * n, None), "convert")
    torch.cuda.synchronize()
    assert _lib.device_status(None) == 0
    assert torch.equal(out16[:, :n].contiguous().view(torch.int16), ref.view(torch.int16))
    if pad:
        assert bool((out16[:, n:] == 7.0).all())  # the pitch's padding is untouched
    assert bool(torch.isnan(out16[0, :n].float()).all())


@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("cfg", [(3, 0, 0, 0, 1), (3, 0, 0, 1, 0), (3, 0, 0, 0, 3)],
                         ids=["pair", "persistent", "pair-split3"])
@pytest.mark.parametrize("shape", [(700, 900, 300), (2600, 2400, 96)], ids=lambda s: "x".join(map(str, s)))
def test_tf32_transposed_b_within_bound_and_bitwise(gpu, workload, cfg, shape):
    """TF32 with B read from a transposed, K-major copy (b_layout = 2): within the TF32
    bound, and bit for bit the result of reading B as given (b_layout = 1) -- the same
    products in the same order; ragged M and N, a K tail, every epilogue, split-K."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 47)
    outs = []
    for layout in (1, 2):
        _lib.set_config(*cfg, b_layout=layout)
        try:
            outs.append(tg.run_op(workload, ins, m, n, k, "tf32"))
        finally:
            _lib.set_config()
    res = tc.check_output(workload, ins, outs[1], "tf32")
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res
    assert np.array_equal(bits(outs[0]), bits(outs[1]))


@pytest.mark.parametrize("workload", ["mbr", "matmul", "matmul_add"])
@pytest.mark.parametrize("cfg", [(3, 256, 0, 0, 1), (3, 0, 0, 1, 0), (3, 256, 0, 0, 3)],
                         ids=["pair", "persistent", "pair-split3"])
@pytest.mark.parametrize("shape", [(700, 2080, 520), (2600, 1024, 264), (300, 4096, 1028), (384, 96, 200)],
                         ids=lambda s: "x".join(map(str, s)))
def test_tf32_b_tile_layouts_bitwise(gpu, workload, cfg, shape):
    """TF32, B as given, loaded as k-group-major tiles (the default where N and K allow it, one
    4-D box per tile) or in 128-byte column blocks (b_layout = 3): the tensor core reads the
    same values in the same order, so the results are the same bits, and within the TF32
    bound; ragged M, N a multiple of 32 but not of the tile width (down to fewer column blocks
    than one tile's box holds), K tails, every epilogue, split-K."""
    m, n, k = shape
    ins = tc.make_inputs(workload, m, n, k, 53)
    outs = []
    for layout in (1, 3):
        _lib.set_config(*cfg, b_layout=layout)
        try:
            outs.append(tg.run_op(workload, ins, m, n, k, "tf32"))
        finally:
            _lib.set_config()
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    res = tc.check_output(workload, ins, outs[0], "tf32")
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


@pytest.mark.parametrize("persistent", [0, 1], ids=["pair", "persistent"])
def test_tf32_b_tile_layouts_pitched_b(gpu, persistent):
    """The k-group-major B map takes B's row pitch in two of its strides: B in a wider buffer
    (ldb = N + 4) gives the same bits through both tilings and stays within the TF32 bound."""
    import torch

    m, n, k = 1000, 1024, 776
    ins = tc.make_inputs("mbr", m, n, k, 57)
    dev = torch.device("cuda", 0)
    a = torch.from_numpy(ins["a"]).to(dev)
    bbig = torch.full((k, n + 4), float("nan"), device=dev)  # the pitch padding is never read
    bbig[:, :n] = torch.from_numpy(ins["b"]).to(dev)
    bias = torch.from_numpy(ins["bias"]).to(dev)
    outs = []
    for layout in (1, 3):
        out = torch.full((m, n), float("nan"), device=dev)
        _lib.set_config(3, 256 if not persistent else 0, 0, persistent, 1 if not persistent else 0, layout)
        try:
            _lib.gemm("mbr", a.data_ptr(), bbig.data_ptr(), out.data_ptr(), m, n, k, "tf32", bias=bias.data_ptr(),
                      ldb=n + 4)
            torch.cuda.synchronize()
        finally:
            _lib.set_config()
        assert _lib.device_status(None) == _lib.OK
        outs.append(out.cpu().numpy())
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    res = tc.check_output("mbr", ins, outs[0], "tf32")
    assert res["nan_count"] == 0 and res["err_over_bound"] <= 1.0, res


def _bf16_rne_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (NaNs left to the caller)."""
    u = x.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("n,xoff,yoff", [(1, 0, 0), (7, 0, 0), (8, 0, 0), (1000003, 0, 0), (4099, 1, 0),
                                         (4099, 0, 3), (65536, 4, 8)])
def test_convert_bf16_rounds_to_nearest_even(gpu, n, xoff, yoff):
    """tforge_convert_bf16: 8-element vector steps when both ends are 16-byte aligned, the
    scalar kernel for the n % 8 tail and for misaligned buffers; every element rounded to
    nearest even (ties, subnormals, infinities; NaN stays NaN)."""
    import torch

    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * np.float32(2.0) ** rng.integers(-130, 120, n)).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, 1e-45,
                        -3.4e38, 1.17e-38], np.float32)
    x[: min(n, special.size)] = special[: min(n, special.size)]
    dev = torch.device("cuda", 0)
    xb = torch.zeros(n + 8, device=dev)
    xb[xoff:xoff + n] = torch.from_numpy(x).to(dev)
    yb = torch.zeros(n + 8, device=dev, dtype=torch.int16)
    _lib.check(_lib.lib().tforge_convert_bf16(xb.data_ptr() + 4 * xoff, yb.data_ptr() + 2 * yoff, n, None), "convert")
    torch.cuda.synchronize()
    got = yb[yoff:yoff + n].cpu().numpy().view(np.uint16)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], _bf16_rne_bits(x)[~nan])
    assert bool(np.all((got[nan] & 0x7F80) == 0x7F80) and np.all(got[nan] & 0x7F))
    assert bool((yb[:yoff] == 0).all()) and bool((yb[yoff + n:] == 0).all())  # nothing outside


def test_concurrent_streams_match_single_stream(gpu):
    """Calls interleaved on two streams (split-K workspace and bf16 scratch come from the
    stream-ordered pool) give the same bits as the same calls on one stream."""
    import torch

    cases = [("mbr", (1024, 1024, 1024), "fp32"),   # split-K: pooled workspace
             ("mbr", (512, 384, 256), "bf16"),      # bf16 operand scratch from the pool
             ("matmul_add", (2048, 1024, 512), "tf32")]
    dev = torch.device("cuda", 0)
    data = []
    for wl, (m, n, k), mode in cases:
        ins = tc.make_inputs(wl, m, n, k, 77)
        t = {name: torch.from_numpy(arr).to(dev) for name, arr in ins.items()}
        data.append((wl, m, n, k, mode, t))

    def launch(i, stream, out):
        wl, m, n, k, mode, t = data[i]
        _lib.gemm(wl, t["a"].data_ptr(), t["b"].data_ptr(), out.data_ptr(), m, n, k, mode,
                  bias=t["bias"].data_ptr() if "bias" in t else None,
                  c_res=t["c"].data_ptr() if "c" in t else None, stream=stream.cuda_stream)

    torch.cuda.synchronize()  # inputs uploaded on the default stream before the side streams read them
    ref = []
    s0 = torch.cuda.Stream()
    for i, (wl, m, n, k, mode, t) in enumerate(data):
        out = torch.empty((m, n), device=dev)
        launch(i, s0, out)
        ref.append(out)
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [[torch.full((m, n), float("nan"), device=dev) for (_, m, n, _, _, _) in data] for _ in range(4)]
    torch.cuda.synchronize()  # the fills (default stream) finish before the side streams write
    for r in range(4):
        for i in range(len(data)):
            launch(i, streams[(r + i) % 2], outs[r][i])
    torch.cuda.synchronize()
    assert _lib.device_status(None) == _lib.OK
    for r in range(4):
        for i in range(len(data)):
            assert torch.equal(outs[r][i].view(torch.int32), ref[i].view(torch.int32)), (r, data[i][:5])
