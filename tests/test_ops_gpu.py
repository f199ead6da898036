"""Tier-1 operator parity: rvc_cuda.ops (GPU, through the C ABI) against the
oracle's restatement of the reference's numpy operators.

Tolerances: GEMM-shaped ops run BF16x3 split precision on the tensor cores
(or fp32 SIMT), relative error ~1e-5; the bar here is rtol/atol 2e-4 on
unit-scale data.  Elementwise/normalisation ops are fp32 and checked at 1e-5.
"""

import numpy as np
import pytest

from oracle import ops as O
from oracle import vits as OV

pytestmark = pytest.mark.gpu

from rvc_cuda import ops  # noqa: E402

RS = np.random.RandomState(7)


def rnd(*s, scale=1.0):
    return (RS.standard_normal(s) * scale).astype(np.float32)


CONV = [  # B, C, T, O, K, stride, pad, dil
    (1, 192, 50, 192, 1, 1, 0, 1), (2, 192, 37, 768, 3, 1, 1, 1), (1, 256, 300, 256, 11, 1, 25, 5),
    (1, 32, 1000, 32, 3, 1, 1, 1), (1, 64, 129, 64, 7, 1, 9, 3), (3, 128, 257, 128, 5, 1, 2, 1),
    (1, 48, 99, 48, 128, 1, 64, 1), (1, 96, 40, 192, 1, 1, 0, 1), (1, 5, 37, 7, 3, 1, 1, 1),
    (1, 1, 400, 16, 10, 5, 0, 1), (1, 512, 101, 512, 3, 2, 0, 1), (1, 16, 3, 16, 5, 1, (2, 1), 1),
    (1, 384, 130, 192, 1, 1, 0, 1),
]


@pytest.mark.parametrize("case", CONV)
def test_conv1d(case):
    B, C, T, Oc, K, s, p, d = case
    x, w, b = rnd(B, C, T), rnd(Oc, C, K, scale=1.0 / np.sqrt(C * K)), rnd(Oc)
    y = ops.conv1d(x, w, b, s, p, d)
    ref = O.conv1d(x.astype(np.float64), w.astype(np.float64), b, s, p, d)
    assert y.shape == ref.shape
    np.testing.assert_allclose(y, ref, rtol=2e-4, atol=2e-4)


# Long square convs: these take the time-rows-as-N kernel (tcn_conv.cu; at
# least one wave of 256-row tiles): C = 32 (tap pairs stacked with the split),
# 64 (stacked hi/lo weight rows), 128 and 256 (hi and lo planes, two channel
# tiles), odd and even tap counts, dilations, ragged last tiles.
CONV_TCN = [(1, 64, 40000, 3, 1, 1), (1, 64, 40001, 11, 25, 5), (1, 128, 40000, 7, 9, 3),
            (2, 256, 19000, 3, 1, 1), (1, 128, 38000, 11, 5, 1),
            (1, 32, 40000, 3, 1, 1), (1, 32, 40003, 11, 25, 5), (2, 32, 20000, 7, 9, 3), (1, 32, 39000, 11, 5, 1)]


@pytest.mark.parametrize("case", CONV_TCN)
def test_conv1d_time_as_n_kernel(case):
    import torch
    B, C, T, K, p, d = case
    x, w, b = rnd(B, C, T), rnd(C, C, K, scale=1.0 / np.sqrt(C * K)), rnd(C)
    y = ops.conv1d(x, w, b, 1, p, d)
    ref = torch.nn.functional.conv1d(torch.from_numpy(x).double(), torch.from_numpy(w).double(),
                                     torch.from_numpy(b).double(), padding=p, dilation=d).numpy()
    assert y.shape == ref.shape
    np.testing.assert_allclose(y, ref, rtol=2e-4, atol=2e-4)


CONVT = [(1, 512, 20, 256, 16, 10, 3), (2, 64, 33, 32, 4, 2, 1), (1, 256, 17, 128, 20, 10, 5),
         (1, 512, 9, 256, 24, 12, 6), (1, 6, 11, 4, 16, 10, 3)]


@pytest.mark.parametrize("case", CONVT)
def test_conv_transpose1d(case):
    B, Ci, T, Co, K, s, p = case
    x, w, b = rnd(B, Ci, T), rnd(Ci, Co, K, scale=1.0 / np.sqrt(Ci)), rnd(Co)
    y = ops.conv_transpose1d(x, w, b, s, p)
    ref = O.conv_transpose1d(x.astype(np.float64), w.astype(np.float64), b, s, p)
    np.testing.assert_allclose(y, ref, rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("mkn", [(499, 768, 2304), (1, 768, 192), (1000, 192, 576), (33, 17, 5), (3, 4, 2, 5)])
def test_matmul(mkn):
    if len(mkn) == 4:  # batched right operand
        a, b = rnd(mkn[0], mkn[1], mkn[2]), rnd(mkn[0], mkn[2], mkn[3])
    else:
        M, K, N = mkn
        a, b = rnd(M, K), rnd(K, N, scale=1.0 / np.sqrt(K))
    y = ops.matmul(a, b)
    np.testing.assert_allclose(y, a.astype(np.float64) @ b.astype(np.float64), rtol=2e-4, atol=2e-4)


def test_layer_norm_softmax_elementwise():
    x = rnd(7, 33, 192, scale=3.0) + 1.0
    g, bt = rnd(192), rnd(192)
    np.testing.assert_allclose(ops.layer_norm(x, g, bt, 1e-5), O.layer_norm(x, g, bt, 1e-5), rtol=1e-5, atol=2e-5)
    s = rnd(5, 1000, scale=10.0)
    s[0] += 1000.0
    np.testing.assert_allclose(ops.softmax(s), O.softmax(s), rtol=1e-5, atol=1e-7)
    a, b = rnd(4, 5, 6), rnd(5, 1)
    np.testing.assert_allclose(ops.add(a, b), a + b, rtol=0, atol=0)
    np.testing.assert_allclose(ops.mul(a, b), a * b, rtol=0, atol=0)
    np.testing.assert_array_equal(ops.relu(a), O.relu(a))
    np.testing.assert_array_equal(ops.leaky_relu(a, 0.1), O.leaky_relu(a, 0.1))
    np.testing.assert_allclose(ops.gelu(a), O.gelu_erf(a), rtol=1e-5, atol=1e-6)


def test_embedding_and_errors():
    t = rnd(256, 192)
    ids = np.array([[0, 5, 255, -1]], np.int64)
    np.testing.assert_array_equal(ops.embedding(ids, t), O.embedding(ids, t))
    with pytest.raises(ValueError):
        ops.embedding(np.array([256]), t)
    with pytest.raises(ValueError):
        ops.conv1d(rnd(1, 3, 10), rnd(4, 5, 3))


def test_gating_and_rel_attention():
    x, g = rnd(2, 384, 50), rnd(2, 384, 1)
    ref = np.tanh(x[:, :192] + g[:, :192]) * O.sigmoid(x[:, 192:] + g[:, 192:])
    np.testing.assert_allclose(ops.gating(x, g), ref, rtol=1e-5, atol=1e-6)
    for P in (7, 50, 130):
        q, k, v = rnd(1, 192, P), rnd(1, 192, P), rnd(1, 192, P)
        ek, ev = rnd(1, 21, 96, scale=0.1), rnd(1, 21, 96, scale=0.1)
        qh = q.reshape(1, 2, 96, P).transpose(0, 1, 3, 2) / np.sqrt(96)
        kh = k.reshape(1, 2, 96, P).transpose(0, 1, 3, 2)
        vh = v.reshape(1, 2, 96, P).transpose(0, 1, 3, 2)
        sc = qh @ kh.swapaxes(-1, -2) + OV.rel_to_abs(qh @ OV.rel_embeddings(ek, P)[0].T)
        pa = O.softmax(sc)
        out = pa @ vh + OV.abs_to_rel(pa) @ OV.rel_embeddings(ev, P)[0]
        ref = out.transpose(0, 1, 3, 2).reshape(1, 192, P)
        np.testing.assert_allclose(ops.rel_attention(q, k, v, ek, ev, 2, 10), ref, rtol=1e-4, atol=1e-5)


def test_im2col():
    x = rnd(2, 3, 20)
    cols = ops.im2col_1d(x, 5, stride=2, padding=2, dilation=1)
    xp = np.pad(x, ((0, 0), (0, 0), (2, 2)))
    oL = (20 + 4 - 5) // 2 + 1
    ref = np.stack([xp[:, :, t * 2:t * 2 + 5].reshape(2, -1) for t in range(oL)], axis=1)
    np.testing.assert_array_equal(cols, ref)


CONV2D = [  # B, C, H, W, O, KH, KW, stride, padding
    (1, 16, 64, 32, 16, 3, 3, 1, 1), (2, 3, 17, 9, 5, 3, 3, (2, 1), (1, 0)), (1, 64, 16, 8, 32, 1, 1, 1, 0),
    (1, 4, 11, 13, 6, 5, 3, 2, 2),
]


@pytest.mark.parametrize("case", CONV2D)
def test_conv2d(case):
    """Tier-1 conv2d (``runtime/backend.py:254``) against torch conv2d in float64."""
    import torch
    B, C, H, W, Oc, KH, KW, st, pd = case
    x, w, b = rnd(B, C, H, W), rnd(Oc, C, KH, KW, scale=1.0 / np.sqrt(C * KH * KW)), rnd(Oc)
    y = ops.conv2d(x, w, b, st, pd)
    ref = torch.nn.functional.conv2d(torch.from_numpy(x).double(), torch.from_numpy(w).double(),
                                     torch.from_numpy(b).double(), stride=st, padding=pd).numpy()
    assert y.shape == ref.shape
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError):
        ops.conv2d(x, w[:, :1], b, st, pd)


def test_rmsnorm():
    """Tier-1 rmsnorm (``runtime/backend.py:309-316``) against the reference formula."""
    x = rnd(7, 33, 192, scale=3.0)
    g = rnd(192)
    y = ops.rmsnorm(x, g, 1e-5)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 * x64).mean(-1, keepdims=True) + 1e-5) * g
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)
