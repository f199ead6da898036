"""Page-locked staging with asynchronous uploads (``rvc_cuda_host_alloc`` /
``rvc_cuda_h2d_async``, what the device pipeline uploads through) and
concurrent f0 segments (``CudaRmvpe.infer_many``, sibling models on their own
streams): each result equals the plain path's."""

import numpy as np
import pytest

from rvc_cuda import _lib
from rvc_cuda import synthetic as syn

pytestmark = pytest.mark.gpu


def test_pinned_buffer_async_upload_roundtrip():
    ctx = _lib.get_context(None)
    buf = _lib.PinnedBuffer(1 << 20)
    a = buf.view(np.float32, 1000, 0)
    a[:] = np.arange(1000, dtype=np.float32) * 0.5
    b = buf.view(np.int64, 100, 4096)
    b[:] = np.arange(100, dtype=np.int64) * 7
    d1, d2 = ctx.alloc(4000), ctx.alloc(800)
    try:
        ctx.h2d_async(d1, a)
        ctx.h2d_async(d2, b)
        out1, out2 = np.empty(1000, np.float32), np.empty(100, np.int64)
        ctx.d2h(out1, d1)  # waits for the stream, so both uploads have landed
        ctx.d2h(out2, d2)
        np.testing.assert_array_equal(out1, a)
        np.testing.assert_array_equal(out2, b)
    finally:
        ctx.free(d1)
        ctx.free(d2)
        buf.close()
    small = _lib.PinnedBuffer(64)
    with pytest.raises(ValueError):
        small.view(np.float32, 100)
    small.close()


def test_rmvpe_infer_many_equals_per_segment():
    from rvc_cuda.rmvpe import CudaRmvpe

    m = CudaRmvpe(syn.make_rmvpe_weights(0), own_stream=True)
    xs = [syn.make_rmvpe_input(T, s) for T, s in ((16000, 1), (9000, 2), (24000, 3))]
    many = m.infer_many(xs)
    assert len(many) == 3
    for x, f in zip(xs, many):
        np.testing.assert_array_equal(f, m.infer_from_audio(x))
    assert [f.shape[0] for f in m.infer_many(xs[:1])] == [101]


def test_rmvpe_infer_many_lane_cap(monkeypatch):
    """More segments than lanes: the lanes stay at the cap and every segment
    still equals its own ``infer_from_audio``."""
    from rvc_cuda.rmvpe import CudaRmvpe

    monkeypatch.setenv("RVC_CUDA_RMVPE_LANES", "2")
    m = CudaRmvpe(syn.make_rmvpe_weights(0), own_stream=True)
    xs = [syn.make_rmvpe_input(T, s) for T, s in ((8000, 1), (9000, 2), (7000, 3), (12000, 4), (6000, 5))]
    many = m.infer_many(xs)
    assert len(m._lanes) == 1
    for x, f in zip(xs, many):
        np.testing.assert_array_equal(f, m.infer_from_audio(x))
    m.close()
