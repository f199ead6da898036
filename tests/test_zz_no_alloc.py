"""rvc_cuda_rel_attention_noalloc: the attention operator for callers that
cannot allocate device memory (for example an audio callback that must not
stall on the allocator, or a host whose device memory belongs to its own
arena).  Its intermediates live in a fixed array in device global memory; the
test feeds it caller-owned device buffers and checks it against the allocating
entry point (rvc_cuda_rel_attention) on two calls in a row, at the tolerance
of the other attention tests.  This file is named to be collected last.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from rvc_cuda import ops  # noqa: E402  (a missing library fails the module, it does not skip it)


def _noalloc(ctx, q, k, v, ek, ev, heads, window):
    from rvc_cuda import _lib

    B, H, P = q.shape
    kc = H // heads
    bufs = [ctx.alloc(a.nbytes) for a in (q, k, v, ek, ev)]
    for p, a in zip(bufs, (q, k, v, ek, ev)):
        ctx.h2d(p, a)
    dy = ctx.alloc(q.nbytes)
    try:
        rc = _lib.lib.rvc_cuda_rel_attention_noalloc(ctx.handle, *[C.c_void_p(p) for p in bufs], B, heads, kc, P,
                                                      window, C.c_void_p(dy))
        _lib.check(rc)
        ctx.sync()
        y = np.empty_like(q)
        ctx.d2h(y, dy)
        return y
    finally:
        for p in bufs + [dy]:
            ctx.free(p)


def test_noalloc_matches_allocating_entry_point_twice():
    from rvc_cuda import _lib

    ctx = _lib.get_context()
    rs = np.random.RandomState(11)
    for call, (B, P) in enumerate([(2, 130), (1, 57)]):
        q, k, v = (rs.standard_normal((B, 192, P)).astype(np.float32) for _ in range(3))
        ek = (rs.standard_normal((1, 21, 96)) * 0.1).astype(np.float32)
        ev = (rs.standard_normal((1, 21, 96)) * 0.1).astype(np.float32)
        ref = ops.rel_attention(q, k, v, ek, ev, 2, 10)
        got = _noalloc(ctx, q, k, v, ek.reshape(21, 96), ev.reshape(21, 96), 2, 10)
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5, err_msg=f"call {call}")


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    from rvc_cuda import _lib

    ctx = _lib.get_context()
    # 4 * B * heads * kc * P = 4 * 8 * 192 * 400 > 2**21
    rc = _lib.lib.rvc_cuda_rel_attention_noalloc(ctx.handle, C.c_void_p(16), C.c_void_p(16), C.c_void_p(16),
                                                  C.c_void_p(16), C.c_void_p(16), 8, 2, 96, 400, 10,
                                                  C.c_void_p(16))
    assert rc == _lib.RVC_E_ARG
    assert "scratch" in _lib.last_error()


def test_noalloc_rejects_unsupported_head_dim_before_queueing_work():
    """A head dimension above 128 (or a window above 16) is refused with the
    same argument error before any kernel is queued on the shared array: the
    library's launch counter does not move.  The buffers are real and sized
    for the call, so nothing could read outside them either way."""
    from rvc_cuda import _lib

    ctx = _lib.get_context()
    B, heads, kc, P, window = 1, 1, 129, 8, 10
    n = B * heads * kc * P
    bufs = [ctx.alloc(4 * n) for _ in range(3)] + [ctx.alloc(4 * (2 * window + 1) * kc) for _ in range(2)]
    dy = ctx.alloc(4 * n)
    try:
        before = _lib.launch_count()
        rc = _lib.lib.rvc_cuda_rel_attention_noalloc(ctx.handle, *[C.c_void_p(p) for p in bufs], B, heads, kc, P,
                                                      window, C.c_void_p(dy))
        assert rc == _lib.RVC_E_ARG
        assert "head dim" in _lib.last_error()
        assert _lib.launch_count() == before
    finally:
        for p in bufs + [dy]:
            ctx.free(p)
