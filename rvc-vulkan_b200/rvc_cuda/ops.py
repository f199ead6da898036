"""Operator module for ``RVC_BACKEND=cuda``.

``runtime.backend`` (``runtime/backend.py:57-70``, ``:189-197``) looks ops up
by name in the registered module and calls them with numpy arrays; each
function here keeps the signature and numpy semantics of the corresponding
``runtime.backend`` wrapper (``runtime/backend.py:205-319``) and returns a new
float32 array.  The math runs in librvc_cuda on the GPU; shapes the library
does not take raise ``ValueError``, which the reference's ``nn`` callers catch
to pick their own path (``runtime/nn.py:286-289``, ``:382-387``, ``:590-593``).

``buf_*`` arguments (the Vulkan engine's resident-buffer handles) are accepted
and ignored.
"""

from __future__ import annotations

import numpy as np

from . import _lib
from ._lib import check, fptr, iptr, lib

__all__ = [
    "matmul", "add", "mul", "relu", "conv1d", "conv_transpose1d", "embedding",
    "add_inplace", "mul_inplace", "layer_norm", "softmax", "leaky_relu", "gelu",
    "gating", "rel_attention", "im2col_1d",
]


def _ctx():
    return _lib.get_context().handle


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _mm2(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError(f"matmul: shapes {a.shape} and {b.shape} not aligned")
    out = np.empty((M, N), np.float32)
    if M == 0 or N == 0:
        return out
    if K == 0:
        out[:] = 0
        return out
    check(lib.rvc_cuda_matmul(_ctx(), fptr(_f32(a)), fptr(_f32(b)), M, K, N, fptr(out)))
    return out


def matmul(a, b, buf_a=None, buf_b=None):
    """``np.asarray(a) @ np.asarray(b)`` (``runtime/backend.py:205-209``)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.ndim == 1 or b.ndim == 1:
        a2 = a[None, :] if a.ndim == 1 else a
        b2 = b[:, None] if b.ndim == 1 else b
        r = matmul(a2, b2)
        if a.ndim == 1:
            r = r[..., 0, :]
        if b.ndim == 1:
            r = r[..., 0]
        return r
    if b.ndim == 2:
        lead = a.shape[:-1]
        out = _mm2(a.reshape(-1, a.shape[-1]), b)
        return out.reshape(lead + (b.shape[1],))
    # batched right operand: broadcast the batch dims, one GEMM per matrix
    shape = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    ab = np.broadcast_to(a, shape + a.shape[-2:])
    bb = np.broadcast_to(b, shape + b.shape[-2:])
    out = np.empty(shape + (a.shape[-2], b.shape[-1]), np.float32)
    for idx in np.ndindex(*shape):
        out[idx] = _mm2(ab[idx], bb[idx])
    return out


def _binary(op: int, a, b) -> np.ndarray:
    a, b = np.broadcast_arrays(np.asarray(a, np.float32), np.asarray(b, np.float32))
    a, b = _f32(a), _f32(b)
    out = np.empty(a.shape, np.float32)
    if a.size:
        check(lib.rvc_cuda_elementwise(_ctx(), op, fptr(a), fptr(b), a.size, 0.0, fptr(out)))
    return out


def _unary(op: int, a, alpha: float = 0.0) -> np.ndarray:
    a = _f32(a)
    out = np.empty(a.shape, np.float32)
    if a.size:
        check(lib.rvc_cuda_elementwise(_ctx(), op, fptr(a), None, a.size, float(alpha), fptr(out)))
    return out


def add(a, b):
    """``a + b`` with numpy broadcasting (``runtime/backend.py:212-216``)."""
    return _binary(0, a, b)


def mul(a, b):
    """``a * b`` (``runtime/backend.py:219-223``)."""
    return _binary(1, a, b)


def add_inplace(a, b, buf_a=None, buf_b=None):
    """Same value as ``a + b`` (``runtime/backend.py:270-274``)."""
    return _binary(0, a, b)


def mul_inplace(a, b, buf_a=None, buf_b=None):
    """Same value as ``a * b`` (``runtime/backend.py:277-281``)."""
    return _binary(1, a, b)


def relu(a):
    """``maximum(a, 0)`` (``runtime/backend.py:226-230``)."""
    return _unary(2, a)


def leaky_relu(x, negative_slope=0.1):
    """``x if x >= 0 else slope*x`` (``runtime/nn.py:507-517``)."""
    return _unary(3, x, negative_slope)


def gelu(x):
    """Exact-erf GELU (``runtime/models/hubert.py:229-244``)."""
    return _unary(4, x)


def _pads(padding):
    if isinstance(padding, (tuple, list)):
        return int(padding[0]), int(padding[1])
    return int(padding), int(padding)


def conv1d(x, w, b=None, stride=1, padding=0, dilation=1, buf_w=None, buf_b=None):
    """torch-semantics conv1d on ``[B,C,T]`` (``runtime/backend.py:233-239``,
    numpy reference ``runtime/nn.py:90-135``)."""
    x = _f32(x)
    w = _f32(w)
    if x.ndim != 3 or w.ndim != 3 or x.shape[1] != w.shape[1]:
        raise ValueError(f"conv1d: x {x.shape} / w {w.shape} mismatch")
    pl, pr = _pads(padding)
    B, Cc, T = x.shape
    O, _, K = w.shape
    stride, dilation = int(stride), int(dilation)
    oL = (T + pl + pr - dilation * (K - 1) - 1) // stride + 1
    if oL <= 0:
        return np.zeros((B, O, 0), np.float32)
    out = np.empty((B, O, oL), np.float32)
    bb = _f32(b) if b is not None else None
    check(lib.rvc_cuda_conv1d(_ctx(), fptr(x), B, Cc, T, fptr(w), O, K, fptr(bb) if bb is not None else None,
                              stride, pl, pr, dilation, fptr(out), oL))
    return out


def conv_transpose1d(x, w, b=None, stride=1, padding=0, output_padding=0, dilation=1, buf_w=None, buf_b=None):
    """torch-semantics transposed conv1d, ``w [C_in, C_out, K]``
    (``runtime/backend.py:242-251``, numpy reference ``runtime/nn.py:294-346``)."""
    x = _f32(x)
    w = _f32(w)
    if x.ndim != 3 or w.ndim != 3 or x.shape[1] != w.shape[0]:
        raise ValueError(f"conv_transpose1d: x {x.shape} / w {w.shape} mismatch")
    B, Ci, T = x.shape
    _, Co, K = w.shape
    stride, padding = int(stride), int(padding)
    oL = (T - 1) * stride - 2 * padding + int(dilation) * (K - 1) + int(output_padding) + 1
    if oL <= 0:
        return np.zeros((B, Co, 0), np.float32)
    out = np.empty((B, Co, oL), np.float32)
    bb = _f32(b) if b is not None else None
    check(lib.rvc_cuda_conv_transpose1d(_ctx(), fptr(x), B, Ci, T, fptr(w), Co, K,
                                        fptr(bb) if bb is not None else None, stride, padding,
                                        int(output_padding), int(dilation), fptr(out), oL))
    return out


def embedding(ids, table, buf_table=None):
    """Row gather, negative ids count from the end (``runtime/nn.py:574-594``)."""
    ids = np.asarray(ids)
    table = np.asarray(table)
    if not np.issubdtype(ids.dtype, np.integer) or table.ndim != 2:
        raise TypeError("embedding: integer ids and a 2-D table are required")
    t = _f32(table)
    V, E = t.shape
    flat = np.ascontiguousarray(ids.reshape(-1), dtype=np.int64)
    if flat.size and (flat.min() < -V or flat.max() >= V):
        raise ValueError("embedding: id out of range")
    out = np.empty((flat.size, E), np.float32)
    if flat.size:
        check(lib.rvc_cuda_embedding(_ctx(), iptr(flat), flat.size, fptr(t), V, E, fptr(out)))
    return out.reshape(ids.shape + (E,))


def layer_norm(x, gamma, beta, eps=1e-5, buf_gamma=None, buf_beta=None):
    """LayerNorm over the last axis, biased variance (``runtime/backend.py:286-296``)."""
    x = _f32(x)
    C = x.shape[-1]
    out = np.empty(x.shape, np.float32)
    rows = x.size // C if C else 0
    if rows:
        check(lib.rvc_cuda_layer_norm(_ctx(), fptr(x), rows, C, fptr(_f32(gamma)), fptr(_f32(beta)),
                                      float(eps), fptr(out)))
    return out


def rmsnorm(x, gamma, eps=1e-5, buf_gamma=None):
    """RMSNorm over the last axis: ``x / sqrt(mean(x^2) + eps) * gamma``
    (``runtime/backend.py:309-316``)."""
    x = _f32(x)
    C = x.shape[-1]
    out = np.empty(x.shape, np.float32)
    rows = x.size // C if C else 0
    if rows:
        check(lib.rvc_cuda_rmsnorm(_ctx(), fptr(x), rows, C, fptr(_f32(gamma)), float(eps), fptr(out)))
    return out


def _pair(v, name):
    if isinstance(v, (tuple, list)):
        if len(v) != 2:
            raise ValueError(f"conv2d: {name} must be an int or a pair, got {v!r}")
        return int(v[0]), int(v[1])
    return int(v), int(v)


def conv2d(x, w, b=None, stride=1, padding=0, buf_w=None, buf_b=None):
    """2-D convolution with ``torch.nn.functional.conv2d`` semantics (symmetric
    zero padding), ``runtime/backend.py:254-260`` / ``runtime/nn.py:259-290``:
    ``x [B,C,H,W]``, ``w [O,C,KH,KW]``, ``b [O]`` or None -> ``[B,O,Ho,Wo]``.
    Shape errors raise ``ValueError`` (the caller then takes its numpy path)."""
    x, w = _f32(x), _f32(w)
    if x.ndim != 4 or w.ndim != 4 or x.shape[1] != w.shape[1]:
        raise ValueError(f"conv2d: x {x.shape} and w {w.shape} do not match [B,C,H,W] / [O,C,KH,KW]")
    sh, sw = _pair(stride, "stride")
    ph, pw = _pair(padding, "padding")
    B, C, H, W = x.shape
    O, _, KH, KW = w.shape
    if sh < 1 or sw < 1 or ph < 0 or pw < 0 or H + 2 * ph < KH or W + 2 * pw < KW:
        raise ValueError("conv2d: bad stride / padding for these shapes")
    Ho, Wo = (H + 2 * ph - KH) // sh + 1, (W + 2 * pw - KW) // sw + 1
    bb = None if b is None else _f32(b).reshape(-1)
    if bb is not None and bb.size != O:
        raise ValueError(f"conv2d: bias of {bb.size} values for {O} output channels")
    out = np.empty((B, O, Ho, Wo), np.float32)
    if B:
        check(lib.rvc_cuda_conv2d(_ctx(), fptr(x), B, C, H, W, fptr(w), O, KH, KW,
                                  fptr(bb) if bb is not None else None, sh, sw, ph, pw, fptr(out)))
    return out


def softmax(x):
    """Row softmax over the last axis (``runtime/backend.py:298-306``)."""
    x = _f32(x)
    C = x.shape[-1]
    out = np.empty(x.shape, np.float32)
    rows = x.size // C if C else 0
    if rows:
        check(lib.rvc_cuda_softmax(_ctx(), fptr(x), rows, C, fptr(out)))
    return out


def gating(x, g=None):
    """WaveNet gate ``tanh(x[:, :H] + g[:, :H]) * sigmoid(x[:, H:] + g[:, H:])``
    on ``x [B, 2H, T]``, ``g [B, 2H, 1]`` (``runtime/models/vits.py:1131-1132``)."""
    x = _f32(x)
    B, H2, T = x.shape
    H = H2 // 2
    out = np.empty((B, H, T), np.float32)
    gg = _f32(np.broadcast_to(np.asarray(g, np.float32), (B, H2, 1))) if g is not None else None
    check(lib.rvc_cuda_gating(_ctx(), fptr(x), fptr(gg) if gg is not None else None, B, H, T, fptr(out)))
    return out


def rel_attention(q, k, v, emb_rel_k, emb_rel_v, heads, window=10):
    """Text-encoder attention with T5 relative positions for one layer.

    ``q, k, v [B, heads*kc, P]`` (projected), ``emb_rel_k/v [1, 2*window+1, kc]``
    -> ``[B, heads*kc, P]``; ``runtime/models/vits.py:993-1014``.
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hc, P = q.shape
    kc = Hc // int(heads)
    ek = _f32(np.asarray(emb_rel_k).reshape(-1, kc))
    ev = _f32(np.asarray(emb_rel_v).reshape(-1, kc))
    out = np.empty((B, Hc, P), np.float32)
    check(lib.rvc_cuda_rel_attention(_ctx(), fptr(q), fptr(k), fptr(v), fptr(ek), fptr(ev), B, int(heads), kc, P,
                                     int(window), fptr(out)))
    return out


def im2col_1d(x, kernel_size, stride=1, padding=0, dilation=1):
    """``x [B,C,T]`` -> ``cols [B, oL, C*K]`` (column c*K+k), the layout of the
    reference engine's im2col_1d (``runtime/vulkan_ops.py:2727``)."""
    x = _f32(x)
    B, Cc, T = x.shape
    pl, pr = _pads(padding)
    K = int(kernel_size)
    oL = (T + pl + pr - int(dilation) * (K - 1) - 1) // int(stride) + 1
    out = np.empty((B, max(oL, 0), Cc * K), np.float32)
    if oL > 0:
        check(lib.rvc_cuda_im2col1d(_ctx(), fptr(x), B, Cc, T, K, int(stride), pl, int(dilation), oL, fptr(out)))
    return out
