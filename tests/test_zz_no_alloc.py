"""Cuda_Attention_VarLen_NoAlloc against Cuda_Attention_VarLen.

The no-allocation entry point serves callers that may not allocate device memory during a call
(memory fully reserved by admission control, or an allocator owned by the host framework): it
keeps its launch metadata in a fixed device array instead of a per-call allocation.  This test
calls both entry points through the C ABI on the same inputs and expects the same result, on
two calls in a row with different batches, so that contents left in the shared array by the
first call cannot leak into the second.  It lives in a file that pytest collects last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fl():
    import build
    build.build()
    import fletcher
    return fletcher


def _run(fl, be, entry, q, k, v, lengths, heads, scale, dtype):
    T, H = q.shape
    tq, tk, tv = (be.new_tensor(T, H, a, dtype) for a in (q, k, v))
    out = be.new_tensor(T, H, None, dtype)
    lens = np.ascontiguousarray(lengths, np.int32)
    be.check(getattr(fl.lib(), entry)(be.ctx, tq.buf, tk.buf, tv.buf, out.buf,
                                      lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), lens.size, H, heads,
                                      ctypes.c_float(scale)))
    return out.to_host()


@pytest.mark.parametrize("dtype,H,heads", [("bf16", 768, 12), ("f16", 768, 12), ("f32", 128, 2)])
def test_no_alloc_matches_allocating_entry_point(fl, dtype, H, heads):
    be = fl.Backend(0)
    dt = fl.DTYPES[dtype]
    rng = np.random.default_rng(42)
    for lengths in ([300, 1, 64, 65, 17], [5, 129, 2]):  # two calls in a row, different batches
        T = sum(lengths)
        q, k, v = (rng.standard_normal((T, H)).astype(np.float32) for _ in range(3))
        want = _run(fl, be, "Cuda_Attention_VarLen", q, k, v, lengths, heads, 0.125, dt)
        got = _run(fl, be, "Cuda_Attention_VarLen_NoAlloc", q, k, v, lengths, heads, 0.125, dt)
        np.testing.assert_allclose(got, want, rtol=0, atol=0)
        # The property the entry point exists for: the call itself allocates nothing (the
        # context's device-allocation counter is unchanged across it).
        T, H_ = q.shape
        tq, tk, tv = (be.new_tensor(T, H_, a, dt) for a in (q, k, v))
        out = be.new_tensor(T, H_, None, dt)
        lens = np.ascontiguousarray(lengths, np.int32)
        before = be.vram_usage()[0]
        be.check(fl.lib().Cuda_Attention_VarLen_NoAlloc(be.ctx, tq.buf, tk.buf, tv.buf, out.buf,
                                                        lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                        lens.size, H_, heads, ctypes.c_float(0.125)))
        be.synchronize()
        assert be.vram_usage()[0] == before
        np.testing.assert_allclose(out.to_host(), want, rtol=0, atol=0)
    be.close()


def test_no_alloc_rejects_oversized_batches(fl):
    be = fl.Backend(0)
    H, heads = 768, 12
    lens = np.ones(300000, np.int32)  # 300001 cu_seqlens entries > 262144
    t = be.new_tensor(int(lens.sum()), H, None, fl.BF16)
    rc = fl.lib().Cuda_Attention_VarLen_NoAlloc(be.ctx, t.buf, t.buf, t.buf, t.buf,
                                                lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), lens.size, H,
                                                heads, ctypes.c_float(0.125))
    assert rc == 1
    buf = ctypes.create_string_buffer(512)
    fl.lib().Cuda_GetLastError(be.ctx, buf, 512)
    assert b"FLETCHER_NOALLOC_SCRATCH_INTS" in buf.value
    be.close()
