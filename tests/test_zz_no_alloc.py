"""The allocation-free BF16 entry point, tforge_mbr_bf16_noalloc, against tforge_mbr.

tforge_mbr in BF16 mode takes scratch for the bf16 copies of its f32 operands from a
memory pool; callers that must not allocate device memory during a call (a serving loop
that reserved all of its memory up front, a framework that owns every device byte) use
tforge_mbr_bf16_noalloc, which keeps that scratch in a 16 MiB static device array.

Two calls of the new entry point in a row, on different inputs, so the second call has to
overwrite what the first left in the shared array: each output must equal the regular
entry point's output bit for bit (same conversion, same kernel) and meet the bf16 error
bound the other tests use.  Around those two calls neither the device's free memory nor
the library's scratch pool may change.  A call whose bounded wait expires must be
reported by tforge_device_status, and the next call must be correct.  This file is
collected last; it passes alone in a fresh process and after the rest of the suite.
"""

import ctypes as C

import numpy as np
import pytest

from tensorforge_b200 import _lib, tforge_cpu as tc, tforge_gpu as tg

pytestmark = pytest.mark.gpu

CASES = [(11, (512, 384, 256)), (12, (2048, 2048, 2048))]


def _upload_case(L, seed, m, n, k):
    x = tc.make_inputs("mbr", m, n, k, seed)
    b = {name: tg.DeviceBuffer.upload(x[name]) for name in ("a", "b", "bias")}
    b["ref"] = tg.DeviceBuffer(m * n * 4)
    b["out"] = tg.DeviceBuffer(m * n * 4)
    _lib.check(L.tforge_mbr(b["a"].ptr, b["b"].ptr, b["bias"].ptr, b["ref"].ptr, m, n, k,
                            _lib.MODES["bf16"], None), "tforge_mbr")
    return x, b


def _noalloc(L, b, m, n, k):
    _lib.check(L.tforge_mbr_bf16_noalloc(b["a"].ptr, b["b"].ptr, b["bias"].ptr, b["out"].ptr,
                                         m, n, k, None), "tforge_mbr_bf16_noalloc")


def test_noalloc_entry_matches_tforge_mbr_bf16(gpu):
    import torch

    L = _lib.lib()
    ins, bufs = [], []
    try:
        for seed, (m, n, k) in CASES:
            x, b = _upload_case(L, seed, m, n, k)
            ins.append(x)
            bufs.append(b)
        _lib.check(_lib.device_status(None), "status")
        # Set-up call (resolves the array's address on this device), then the measurements.
        _noalloc(L, bufs[0], *CASES[0][1])
        _lib.check(L.tforge_stream_sync(None), "sync")
        free_before = torch.cuda.mem_get_info(0)[0]
        pool_now, _ = _lib.pool_usage(reset_high=True)
        # The two calls in a row under test.
        for (seed, (m, n, k)), b in zip(CASES, bufs):
            _noalloc(L, b, m, n, k)
        _lib.check(L.tforge_stream_sync(None), "sync")
        assert _lib.device_status(None) == _lib.OK
        assert torch.cuda.mem_get_info(0)[0] == free_before  # no cudaMalloc
        assert _lib.pool_usage()[1] == pool_now               # nothing taken from the pool
        for (seed, (m, n, k)), x, b in zip(CASES, ins, bufs):
            ref = b["ref"].download((m, n))
            out = b["out"].download((m, n))
            assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), (m, n, k)
            res = tc.check_output("mbr", x, out, "bf16")
            assert res["pass"], res
    finally:
        for b in bufs:
            for d in b.values():
                d.free()


def test_noalloc_entry_reports_a_timeout_and_recovers(gpu):
    """A stage that never fills (the skip-load test hook, 50 ms wait limit): the kernel gives
    up, tforge_device_status reports TFORGE_ERR_TIMEOUT once, and the next call is right."""
    L = _lib.lib()
    m, n, k = 2048, 2048, 2048
    _, b = _upload_case(L, 13, m, n, k)
    try:
        _lib.check(_lib.device_status(None), "status")
        assert L.tforge_set_wait_limit_ns(50_000_000) == 0
        assert L.tforge_debug_skip_load(1) == 0
        try:
            _noalloc(L, b, m, n, k)
            assert _lib.device_status(None) == _lib.ERR_TIMEOUT
        finally:
            L.tforge_debug_skip_load(0)
            L.tforge_set_wait_limit_ns(0)
        assert _lib.device_status(None) == _lib.OK  # reading cleared it
        _noalloc(L, b, m, n, k)
        assert _lib.device_status(None) == _lib.OK
        assert np.array_equal(b["out"].download((m, n)).view(np.uint32), b["ref"].download((m, n)).view(np.uint32))
    finally:
        for d in b.values():
            d.free()


def test_noalloc_entry_rejects_problems_beyond_its_scratch(gpu):
    L = _lib.lib()
    dummy = tg.DeviceBuffer(256)
    try:
        p = dummy.ptr
        # bf16(A) + bf16(B) = 2 * 4096 * 4096 * 2 bytes = 64 MiB > 16 MiB: rejected up front,
        # before any pointer is touched (the pointers here only need to be aligned).
        assert L.tforge_mbr_bf16_noalloc(p, C.c_void_p(p.value + 4096), C.c_void_p(p.value + 8192),
                                         C.c_void_p(p.value + (1 << 30)), 4096, 4096, 4096, None) == _lib.ERR_SHAPE
        assert b"16 MiB" in L.tforge_last_error()
    finally:
        dummy.free()
