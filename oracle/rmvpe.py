"""Oracle for the RMVPE F0 estimator CPU path.

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``).  A numpy restatement of the
reference's numpy ``RMVPE.infer_from_audio`` (``runtime/models/rmvpe.py:927-952``):
log-mel front end (``:632-641`` with ``runtime/dsp/fft.py:59-113`` and the HTK
filter bank of ``runtime/dsp/mel.py:66-122``), the deep U-Net (``:643-760``),
cnn + BiGRU + linear + sigmoid (``:878-897``) and the local-average decode
(``:899-925``).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
SR, N_FFT, HOP, N_MELS, FMIN, FMAX = 16000, 1024, 160, 128, 30.0, 8000.0


def mel_basis() -> np.ndarray:
    """HTK triangular filters, each row normalised to sum 1 (``runtime/dsp/mel.py:97-122``)."""
    n_bins = N_FFT // 2 + 1
    fft_f = np.linspace(0.0, SR / 2.0, n_bins)
    m_lo, m_hi = 1127.0 * np.log1p(FMIN / 700.0), 1127.0 * np.log1p(FMAX / 700.0)
    f_pts = 700.0 * np.expm1(np.linspace(m_lo, m_hi, N_MELS + 2) / 1127.0)
    w = np.zeros((N_MELS, n_bins))
    for i in range(N_MELS):
        lo, c, hi = f_pts[i], f_pts[i + 1], f_pts[i + 2]
        up = (fft_f - lo) / (c - lo) if c - lo > 0 else np.zeros(n_bins)
        down = (hi - fft_f) / (hi - c) if hi - c > 0 else np.zeros(n_bins)
        tri = np.maximum(0.0, np.minimum(up, down))
        s = tri.sum()
        w[i] = tri / s if s > 0 else tri
    return w.astype(F32)


def log_mel(x: np.ndarray) -> np.ndarray:
    """``[T]`` -> ``[128, F]``: hann (symmetric) STFT, centre reflect pad,
    |X| in float64 -> f32, filter bank, log(clip(., 1e-5)) (``runtime/models/rmvpe.py:632-641``)."""
    x = np.asarray(x, dtype=np.float64)
    w = np.hanning(N_FFT)
    xp = np.pad(x, (N_FFT // 2, N_FFT // 2), mode="reflect")
    nf = 1 + (len(xp) - N_FFT) // HOP
    idx = np.arange(N_FFT)[None, :] + HOP * np.arange(nf)[:, None]
    mag = np.abs(np.fft.rfft(xp[idx] * w[None, :], axis=1).T).astype(F32)
    return np.log(np.clip(mel_basis() @ mag, 1e-5, None)).astype(F32)


def conv2d(x, w, b=None, pad=1):
    """Stride-1 conv2d by im2col + matmul (``runtime/models/rmvpe.py:165-196``)."""
    _, C, H, W = x.shape
    O, _, KH, KW = w.shape
    xp = np.pad(x[0], ((0, 0), (pad, pad), (pad, pad)))
    OH, OW = H + 2 * pad - KH + 1, W + 2 * pad - KW + 1
    cols = np.empty((C, KH, KW, OH, OW), dtype=F32)
    for i in range(KH):
        for j in range(KW):
            cols[:, i, j] = xp[:, i:i + OH, j:j + OW]
    out = (w.reshape(O, -1) @ cols.reshape(C * KH * KW, OH * OW)).reshape(1, O, OH, OW)
    if b is not None:
        out = out + b.reshape(1, -1, 1, 1)
    return out


def bn_scale_shift(sd, p):
    """``scale = gamma / sqrt(var + eps)``, ``shift = beta - mean * scale`` (``:507-515``)."""
    g, b = sd[p + ".weight"].astype(F32), sd[p + ".bias"].astype(F32)
    rm, rv = sd[p + ".running_mean"].astype(F32), sd[p + ".running_var"].astype(F32)
    scale = g / np.sqrt(rv + F32(1e-5))
    return scale, b - rm * scale


def bn(x, sd, p, relu=False):
    s, t = bn_scale_shift(sd, p)
    y = x * s.reshape(1, -1, 1, 1) + t.reshape(1, -1, 1, 1)
    return np.maximum(y, F32(0)) if relu else y


def conv_block_res(x, sd, p):
    """ConvBlockRes: (conv3x3 -> BN -> ReLU) x 2 plus identity / 1x1 shortcut (``:518-547``)."""
    y = bn(conv2d(x, sd[p + ".conv.0.weight"]), sd, p + ".conv.1", relu=True)
    y = bn(conv2d(y, sd[p + ".conv.3.weight"]), sd, p + ".conv.4", relu=True)
    if p + ".shortcut.weight" in sd:
        return y + conv2d(x, sd[p + ".shortcut.weight"], sd.get(p + ".shortcut.bias"), pad=0)
    return y + x


def conv_transpose2d(x, w):
    """3x3, stride 2, padding 1, output padding 1: zero insertion, flipped kernel (``:319-384``)."""
    _, C, H, W = x.shape
    up = np.zeros((1, C, 2 * H - 1, 2 * W - 1), dtype=F32)
    up[:, :, ::2, ::2] = x
    wf = np.ascontiguousarray(w.transpose(1, 0, 2, 3)[:, :, ::-1, ::-1])
    y = conv2d(up, wf, None, pad=1)
    out = np.zeros((1, wf.shape[0], 2 * H, 2 * W), dtype=F32)
    out[:, :, :y.shape[2], :y.shape[3]] = y
    return out


def avg_pool(x):
    B, C, H, W = x.shape
    return x.reshape(B, C, H // 2, 2, W // 2, 2).mean(axis=(3, 5))


def sigmoid(x):
    """``runtime/nn.py:520-523``."""
    return np.where(x >= 0, 1.0 / (1.0 + np.exp(-x)), np.exp(x) / (1.0 + np.exp(x)))


def bgru(x, sd):
    """Bidirectional one-layer GRU, gate order r, z, n (``runtime/models/rmvpe.py:393-442``)."""
    def run(xs, sfx):
        wi, wh = sd["fc.0.gru.weight_ih_l0" + sfx], sd["fc.0.gru.weight_hh_l0" + sfx]
        bi, bh = sd["fc.0.gru.bias_ih_l0" + sfx], sd["fc.0.gru.bias_hh_l0" + sfx]
        H = wh.shape[1]
        gx = xs @ wi.T + bi
        h = np.zeros(H, dtype=F32)
        out = np.empty((xs.shape[0], H), dtype=F32)
        with np.errstate(over="ignore", invalid="ignore"):
            for t in range(xs.shape[0]):
                gh = h @ wh.T + bh
                r = sigmoid(gx[t, :H] + gh[:H])
                z = sigmoid(gx[t, H:2 * H] + gh[H:2 * H])
                n = np.tanh(gx[t, 2 * H:] + r * gh[2 * H:])
                h = (1.0 - z) * n + z * h
                out[t] = h
        return out
    return np.concatenate([run(x, ""), run(x[::-1], "_reverse")[::-1]], axis=-1)


def _tap(taps, name, a):
    if taps is not None:
        taps[name] = np.array(a, dtype=F32, copy=True)


def salience(sd: dict, mel: np.ndarray, taps=None) -> np.ndarray:
    """``[128, F]`` log-mel -> ``[F, 360]`` salience (``mel2hidden``, ``:861-876``)."""
    nf = mel.shape[-1]
    npad = 32 * ((nf - 1) // 32 + 1) - nf
    x = np.pad(mel, ((0, 0), (0, npad)))[None, None].transpose(0, 1, 3, 2).astype(F32)  # [1,1,F',128]
    x = bn(x, sd, "unet.encoder.bn")
    skips = []
    for i in range(5):
        for j in range(4):
            x = conv_block_res(x, sd, f"unet.encoder.layers.{i}.conv.{j}")
        _tap(taps, f"enc{i}", x)
        skips.append(x)
        x = avg_pool(x)
    for i in range(4):
        for j in range(4):
            x = conv_block_res(x, sd, f"unet.intermediate.layers.{i}.conv.{j}")
    _tap(taps, "inter", x)
    for i in range(5):
        p = f"unet.decoder.layers.{i}"
        y = bn(conv_transpose2d(x, sd[p + ".conv1.0.weight"]), sd, p + ".conv1.1", relu=True)
        y = np.concatenate([y, skips[-1 - i]], axis=1)
        for j in range(4):
            y = conv_block_res(y, sd, f"{p}.conv2.{j}")
        x = y
        _tap(taps, f"dec{i}", x)
    x = conv2d(x, sd["cnn.weight"], sd["cnn.bias"], pad=1)  # [1,3,F',128]
    x = x.transpose(0, 2, 1, 3).reshape(1, x.shape[2], -1)  # [1,F',384]
    _tap(taps, "cnn", x[0])
    h = bgru(x[0], sd)
    _tap(taps, "gru", h)
    out = sigmoid(h @ sd["fc.1.weight"].T + sd["fc.1.bias"]).astype(F32)
    return out[:nf]


CENTS = np.pad(20 * np.arange(360) + 1997.3794084376191, (4, 4)).astype(F32)


def decode(sal: np.ndarray, thred: float = 0.03) -> np.ndarray:
    """Argmax, 9-bin local average of cents, f0 = 10 * 2^(cents/1200), 0 where
    the peak is <= thred (``runtime/models/rmvpe.py:899-925``)."""
    sal = np.asarray(sal, dtype=F32)
    F = sal.shape[0]
    c = np.argmax(sal, axis=1) + 4
    sp = np.pad(sal, ((0, 0), (4, 4)))
    cols = (c - 4)[:, None] + np.arange(9)[None, :]
    rows = np.arange(F)[:, None]
    ts, tc = sp[rows, cols], CENTS[cols]
    cents = np.sum(ts * tc, axis=1) / np.sum(ts, axis=1)
    cents[np.max(sp, axis=1) <= thred] = 0
    f0 = 10 * (2 ** (cents / 1200))
    f0[f0 == 10] = 0
    return f0


def infer(sd: dict, x: np.ndarray, thred: float = 0.03, taps=None) -> np.ndarray:
    """``[T]`` audio -> ``[F]`` f0 in Hz."""
    mel = log_mel(x)
    _tap(taps, "mel", mel)
    sal = salience(sd, mel, taps)
    _tap(taps, "salience", sal)
    return decode(sal, thred)
