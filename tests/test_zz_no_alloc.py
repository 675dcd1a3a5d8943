"""The allocation-free BF16 entry point, tforge_mbr_bf16_noalloc, against tforge_mbr.

tforge_mbr in BF16 mode takes scratch for the bf16 copies of its f32 operands from a
memory pool; callers that must not allocate device memory during a call (a serving loop
that reserved all of its memory up front, a framework that owns every device byte) use
tforge_mbr_bf16_noalloc, which keeps that scratch in a 16 MiB static device array.

Two calls of the new entry point in a row, on different inputs, so the second call has to
overwrite what the first left in the shared array: each output must equal the regular
entry point's output bit for bit (same conversion, same kernel) and meet the bf16 error
bound the other tests use.  This file is collected last; it passes alone in a fresh
process and after the rest of the suite.
"""

import ctypes as C

import numpy as np
import pytest

from tensorforge_b200 import _lib, tforge_cpu as tc, tforge_gpu as tg

pytestmark = pytest.mark.gpu

CASES = [(11, (512, 384, 256)), (12, (2048, 2048, 2048))]


def test_noalloc_entry_matches_tforge_mbr_bf16(gpu):
    L = _lib.lib()
    ins = [tc.make_inputs("mbr", m, n, k, seed) for seed, (m, n, k) in CASES]
    bufs = []
    try:
        for (seed, (m, n, k)), x in zip(CASES, ins):
            b = {name: tg.DeviceBuffer.upload(x[name]) for name in ("a", "b", "bias")}
            b["ref"] = tg.DeviceBuffer(m * n * 4)
            b["out"] = tg.DeviceBuffer(m * n * 4)
            bufs.append(b)
            _lib.check(L.tforge_mbr(b["a"].ptr, b["b"].ptr, b["bias"].ptr, b["ref"].ptr, m, n, k,
                                    _lib.MODES["bf16"], None), "tforge_mbr")
        _lib.check(_lib.device_status(None), "status")
        # The two calls in a row under test.
        for (seed, (m, n, k)), b in zip(CASES, bufs):
            _lib.check(L.tforge_mbr_bf16_noalloc(b["a"].ptr, b["b"].ptr, b["bias"].ptr, b["out"].ptr,
                                                 m, n, k, None), "tforge_mbr_bf16_noalloc")
        _lib.check(L.tforge_stream_sync(None), "sync")
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
