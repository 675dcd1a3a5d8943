"""The C-ABI library loads, exports every declared symbol, and validates arguments
without a GPU (no compute calls here)."""

import ctypes as C
import pathlib
import re

import pytest

from tensorforge_b200 import _lib, tforge_gpu as tg

REPO = pathlib.Path(__file__).resolve().parent.parent


def declared_symbols():
    text = "\n".join(p.read_text() for p in (REPO / "include").glob("*.h"))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tforge_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s
    # and the ctypes signature table covers them all
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)


def test_version_and_status_strings():
    L = _lib.lib()
    assert b"sm_100a" in L.tforge_version()
    for code in range(10):
        assert L.tforge_status_string(code)
    assert L.tforge_status_string(_lib.ERR_TIMEOUT) == b"device-side wait timed out"


P = 1 << 20  # fake, 16-byte aligned "device" addresses: validation happens before any CUDA call


@pytest.mark.parametrize("call,code", [
    (lambda L: L.tforge_mbr(None, None, None, None, 4, 4, 4, 0, None), _lib.ERR_NULL),
    (lambda L: L.tforge_mbr(P, 2 * P, 3 * P, 4 * P, -1, 4, 4, 0, None), _lib.ERR_SHAPE),
    (lambda L: L.tforge_mbr(P, 2 * P, 3 * P, 4 * P, 4, 4, 4, 9, None), _lib.ERR_MODE),
    (lambda L: L.tforge_mbr(P + 2, 2 * P, 3 * P, 4 * P, 4, 4, 4, 0, None), _lib.ERR_ALIGN),
    (lambda L: L.tforge_mbr(P, 2 * P, 3 * P, P + 16, 8, 8, 8, 0, None), _lib.ERR_ALIAS),
    (lambda L: L.tforge_matmul_add(P, 2 * P, 4 * P + 8, 4 * P, 8, 8, 8, 0, None), _lib.ERR_ALIAS),
    (lambda L: L.tforge_matmul(P, None, 4 * P, 8, 8, 8, 0, None), _lib.ERR_NULL),
    (lambda L: L.tforge_relu(P, P, 4, 4, None), _lib.ERR_ALIAS),
    (lambda L: L.tforge_add(P, 2 * P, 3 * P, -2, 4, None), _lib.ERR_SHAPE),
    (lambda L: L.tforge_bias_add(P, None, 3 * P, 2, 4, None), _lib.ERR_NULL),
    (lambda L: L.tforge_convert_bf16(P, P + 2, 16, None), _lib.ERR_ALIAS),
])
def test_argument_validation(call, code):
    assert call(_lib.lib()) == code


def test_empty_problems_are_noops():
    L = _lib.lib()
    assert L.tforge_mbr(None, None, None, None, 0, 16, 16, 0, None) == 0
    assert L.tforge_matmul(None, None, None, 16, 0, 16, 0, None) == 0
    assert L.tforge_relu(None, None, 0, 0, None) == 0


def test_bf16_operands_need_bf16_mode():
    args = _lib.GemmArgs(0, 0, _lib.BF16, _lib.F32, P, 2 * P, None, None, 4 * P, 8, 8, 8, 0, 0, 0)
    assert _lib.lib().tforge_gemm(C.byref(args), None) == _lib.ERR_MODE


def test_bf16_output_needs_bf16_mode_and_device_buffers():
    """out_dtype = TFORGE_BF16 is a BF16-mode option of tforge_gemm; other modes, unknown
    dtypes and the host-buffer entry reject it before any CUDA call."""
    L = _lib.lib()
    for mode, out_dtype in ((0, _lib.BF16), (1, _lib.BF16), (2, 7)):  # fp32, tf32, bad dtype
        args = _lib.GemmArgs(0, mode, _lib.F32, _lib.F32, P, 2 * P, None, None, 4 * P, 8, 8, 8, 0, 0, 0, out_dtype)
        assert L.tforge_gemm(C.byref(args), None) == _lib.ERR_MODE
    args = _lib.GemmArgs(0, 2, _lib.F32, _lib.F32, P, 2 * P, None, None, 4 * P, 8, 8, 8, 0, 0, 0, _lib.BF16)
    assert L.tforge_gemm_host(C.byref(args), 0, None) == _lib.ERR_MODE
    # An odd out address is misaligned for bf16 as well as f32.
    args = _lib.GemmArgs(0, 2, _lib.F32, _lib.F32, P, 2 * P, None, None, 4 * P + 1, 8, 8, 8, 0, 0, 0, _lib.BF16)
    assert L.tforge_gemm(C.byref(args), None) == _lib.ERR_ALIGN


def test_pitch_smaller_than_row_is_rejected():
    args = _lib.GemmArgs(0, 0, _lib.F32, _lib.F32, P, 2 * P, None, None, 4 * P, 8, 8, 8, 4, 0, 0)
    assert _lib.lib().tforge_gemm(C.byref(args), None) == _lib.ERR_SHAPE


def test_host_entry_validates_before_any_cuda_call():
    """tforge_gemm_host applies tforge_gemm's checks to its host pointers first."""
    L = _lib.lib()
    assert L.tforge_gemm_host(None, 0, None) == _lib.ERR_NULL
    args = _lib.GemmArgs(0, 0, _lib.F32, _lib.F32, P, 2 * P, None, None, 4 * P, 8, 8, 8, 4, 0, 0)
    assert L.tforge_gemm_host(C.byref(args), 0, None) == _lib.ERR_SHAPE
    args = _lib.GemmArgs(1, 0, _lib.F32, _lib.F32, P, 2 * P, None, None, 4 * P, 8, 8, 8, 0, 0, 0)
    assert L.tforge_gemm_host(C.byref(args), 0, None) == _lib.ERR_NULL  # mbr without bias
    args = _lib.GemmArgs(0, 0, _lib.F32, _lib.F32, P, 2 * P, None, None, P, 8, 8, 8, 0, 0, 0)
    assert L.tforge_gemm_host(C.byref(args), 0, None) == _lib.ERR_ALIAS  # out overlaps A
    args = _lib.GemmArgs(0, 0, _lib.F32, _lib.F32, None, None, None, None, None, 0, 8, 8, 0, 0, 0)
    assert L.tforge_gemm_host(C.byref(args), 0, None) == _lib.OK


@pytest.mark.parametrize("shape,mode,kernel", [
    ((2048, 2048, 2048), "fp32", "tf_gemm_tcgen05_3xtf32_pair"),
    ((2048, 2048, 2048), "tf32", "tf_gemm_tcgen05_tf32_pair"),
    ((2048, 2048, 2048), "bf16", "tf_gemm_tcgen05_bf16_pair_persistent"),  # measured: even with the pair kernel
    ((256, 256, 128), "fp32", "tf_gemm_tcgen05_3xtf32"),       # measured: 128x64 tiles by a hair
    ((1000, 1000, 1000), "bf16", "tf_gemm_tcgen05_bf16"),       # measured: 128x64 tiles
    ((300, 8, 64), "tf32", "tf_gemm_tcgen05_tf32"),             # outside the table: the model
    ((2048, 2048, 2048), "fp32_exact", "tf_gemm_simt_ffma"),
    ((777, 1111, 333), "fp32", "tf_gemm_simt_ffma"),   # pitches not 16-byte multiples
    ((256, 256, 8), "fp32", "tf_gemm_simt_ffma"),      # K < 16: exact kernel keeps the fp32 bound
    ((256, 256, 0), "tf32", "tf_gemm_simt_ffma"),      # K = 0: out = epilogue(+0)
])
def test_dispatch_table(shape, mode, kernel):
    d = _lib.describe("mbr", *shape, mode)
    assert d["kernel"] == kernel
    assert d["block"] == [384 if kernel == "tf_gemm_tcgen05_3xtf32_pair" else 256, 1, 1]
    if kernel.endswith("_persistent"):  # one cluster of two CTAs per tile, up to the SM pairs
        m, n, _ = shape
        assert d["grid"] == [2 * min(-(-m // 256) * -(-n // 256), 74), 1, 1]
    elif kernel.startswith("tf_gemm_tcgen05"):
        m, n, _ = shape
        pair = kernel.endswith("_pair")
        assert d["grid"] == [-(-n // d["tile"][1]) * (2 if pair else 1), -(-m // d["tile"][0]), 1]
        assert d["cluster"] == [2 if pair else 1, 1, 1]
        assert d["smem_bytes"] <= 232448
        assert d["tmem_cols"] <= 512
        if not pair:
            assert d["tmem_cols"] == d["tile"][1]


def _tune_table():
    text = (pathlib.Path(tg.PKG) / "csrc" / "tf_tune_table.inc").read_text()
    rows = re.findall(r"\{(\d+), (\d+), (\d+), (\d+), (\d+), (\d+), (\d+), ([0-9.]+)\}", text)
    return [tuple(int(x) for x in r[:7]) + (float(r[7]),) for r in rows]


def test_tuned_table_entries_are_what_dispatch_picks():
    """Every measured entry is a supported configuration and the dispatch returns it for
    its own shape; shapes within a factor of two take the nearest entry."""
    entries = _tune_table()
    assert len(entries) >= 60
    modes = {0: "tf32", 1: "fp32", 2: "bf16"}
    for prec, m, n, k, pair, bn, stages, tflops in entries:
        assert tflops > 0
        d = _lib.describe("mbr", m, n, k, modes[prec])
        assert ("_pair" in d["kernel"]) == bool(pair), (prec, m, n, k)
        assert d["kernel"].endswith("_pair_persistent") == (pair == 2), (prec, m, n, k)
        assert d["tile"][1] == bn, (prec, m, n, k)
        if not pair:  # the pair kernel has one instantiated depth per precision
            assert d["stages"] == stages
    # (1100, 1000, 904) is nearest to the measured (1000, 1000, 1000) bf16 entry.
    assert _lib.describe("mbr", 1100, 1000, 904, "bf16")["tile"][1] == 64


def test_forced_config_and_reset():
    _lib.set_config(1, 128, 6)
    try:
        d = _lib.describe("mbr", 2048, 2048, 2048, "tf32")
        assert d["tile"] == [128, 128, 32] and d["stages"] == 6
        _lib.set_config(3)  # CTA-pair kernel
        d = _lib.describe("mbr", 256, 256, 128, "fp32")
        assert d["kernel"] == "tf_gemm_tcgen05_3xtf32_pair" and d["tmem_cols"] == 512
        _lib.set_config(1, 96, 6)  # not instantiated
        with pytest.raises(_lib.TforgeError):
            _lib.describe("mbr", 2048, 2048, 2048, "tf32")
        _lib.set_config(3, 240)  # 256 x 240 pair tiles
        d = _lib.describe("mbr", 2048, 2048, 2048, "fp32")
        assert d["tile"][:2] == [256, 240] and d["grid"][:2] == [18, 8] and d["split_k"] == 1
        _lib.set_config(3, 240, split_k=2)  # the 240-wide tile takes no split-K
        with pytest.raises(_lib.TforgeError):
            _lib.describe("mbr", 2048, 2048, 2048, "fp32")
        _lib.set_config(3, 0, 0, 1)  # persistent pair kernel: TF32 / BF16 only
        d = _lib.describe("mbr", 8192, 8192, 8192, "tf32")
        assert d["kernel"] == "tf_gemm_tcgen05_tf32_pair_persistent" and d["persistent"] == 1
        assert d["tmem_cols"] == 512 and d["grid"][1] == 1 and d["split_k"] == 1
        assert d["grid"][0] == 148  # without a device: 74 SM pairs
        d = _lib.describe("mbr", 300, 264, 64, "bf16")
        assert d["kernel"] == "tf_gemm_tcgen05_bf16_pair_persistent" and d["grid"][0] == 8  # 2 x 2 tiles
        with pytest.raises(_lib.TforgeError):
            _lib.describe("mbr", 8192, 8192, 8192, "fp32")
        _lib.set_config(3, 0, 0, 1, 2)  # no split-K either
        with pytest.raises(_lib.TforgeError):
            _lib.describe("mbr", 8192, 8192, 8192, "tf32")
        _lib.set_config(3, 0, 0, 0, 0, 3)  # b_layout is 0 .. 3
        with pytest.raises(_lib.TforgeError):
            _lib.set_config(3, 0, 0, 0, 0, 4)
    finally:
        _lib.set_config()
    assert _lib.describe("mbr", 2048, 2048, 2048, "tf32")["kernel"] == "tf_gemm_tcgen05_tf32_pair"


def test_model_picks_240_wide_pair_tiles_when_waves_allow():
    """Outside the measured table the pair kernel takes 256 x 240 tiles when that needs no
    more waves of SM pairs: 2048 x 2048 is 72 such tiles on 74 pairs instead of 64 of 256 x 256;
    8192 x 8192 would need more waves and keeps 256."""
    assert _lib.describe("mbr", 2048, 2048, 64, "fp32")["tile"][:2] == [256, 240]
    assert _lib.describe("mbr", 65536, 65536, 64, "fp32")["tile"][:2] == [256, 256]


def test_model_picks_persistent_pair_for_multi_wave_tf32_bf16():
    """Outside the measured table, TF32 and BF16 shapes with more 256x256 tiles than SM
    pairs, up to 32 tiles per pair, take the persistent pair kernel; one wave or fewer, and
    very long calls (config 4's 131072 x 8192 x 8192 on one GPU: 16384 tiles), keep the
    one-launch-per-tile pair kernel."""
    for mode in ("tf32", "bf16"):
        assert _lib.describe("mbr", 16384, 8192, 64, mode)["kernel"].endswith("_pair_persistent")  # 2048 tiles
        assert _lib.describe("mbr", 131072, 8192, 8192, mode)["kernel"].endswith("_pair")
        assert _lib.describe("mbr", 65536, 16384, 4096, mode)["kernel"].endswith("_pair")
    assert _lib.describe("mbr", 2048, 2048, 64, "tf32")["kernel"] == "tf_gemm_tcgen05_tf32_pair"
    assert _lib.describe("mbr", 131072, 8192, 8192, "fp32")["kernel"] == "tf_gemm_tcgen05_3xtf32_pair"


def test_compile_kernel_writes_launch_json(tmp_path, monkeypatch):
    monkeypatch.setattr(tg, "ART", tmp_path)
    d, launch = tg.compile_kernel("mbr", 512, 512, 512, "precision=tf32 bn=128 stages=6", tag="t")
    assert tg.parse_launch(d / "launch.json") == launch
    for key in ("kernel", "grid", "block", "args", "padded"):  # the reference's launch.json keys
        assert key in launch
    assert launch["args"] == ["arg0", "arg1", "arg2", "arg3"]
    assert launch["padded"] == [512, 512, 512]
    assert launch["tile"] == [128, 128, 32]
    assert tg.padded_shape(777, 1111, 333, "") == (777, 1111, 333)


def test_ptxas_resources_reports_no_spills():
    res = tg.ptxas_resources(launch={"kernel": "tf_gemm_tcgen05_3xtf32"})
    assert res["regs"] > 0
    assert res["spill_stores"] == 0 and res["spill_loads"] == 0


def test_tensor_roofline_from_measured_peaks():
    peaks = {"bf16_tflops": 1600.0}
    assert tg.tensor_roofline_tflops("bf16", peaks) == (1600.0, "of measured")
    assert tg.tensor_roofline_tflops("tf32", peaks)[0] == 800.0
    assert tg.tensor_roofline_tflops("fp32", peaks)[0] == pytest.approx(800.0 / 3)
    assert tg.tensor_roofline_tflops("fp32", {})[1] == "of fallback"


def test_csv_schema_is_the_references(tmp_path):
    import csv
    import json

    from tensorforge_b200 import provenance

    golden = json.loads((REPO / "tests" / "golden" / "golden.json").read_text())
    assert provenance.FIELDS == golden["provenance_fields"]
    w = provenance.CsvWriter(tmp_path / "r.csv")
    w.row(**provenance.common(), workload="mbr", shape="2x2x2")
    with pytest.raises(KeyError):
        w.row(bogus=1)
    w.close()
    rows = list(csv.DictReader(open(tmp_path / "r.csv")))
    assert rows[0]["workload"] == "mbr" and list(rows[0]) == provenance.FIELDS


def test_autotune_table_round_trip(tmp_path):
    """The sweep's table writer and reader agree (the reader backs `--merge`, which keeps the
    entries of modes not swept)."""
    from tensorforge_b200 import autotune
    entries = autotune.read_table(autotune.TABLE)
    assert len(entries) == len(_tune_table())
    out = tmp_path / "t.inc"
    autotune.write_table(entries, out)
    assert autotune.read_table(out) == entries


def test_option_strings_carry_pair_kernel_knobs():
    """compile_kernel / check / bench option strings reach tforge_config: persistent, split
    and b_layout imply the pair kernel except b_layout alone, which keeps the table's."""
    o = tg.parse_options("precision=tf32 kernel=pair persistent=1 split=0 b_layout=2")
    assert (o["persistent"], o["b_layout"], tg._forced_kind(o)) == (1, 2, 3)
    assert tg._forced_kind(tg.parse_options("b_layout=1")) == 0
    assert tg._forced_kind(tg.parse_options("split=4")) == 3
