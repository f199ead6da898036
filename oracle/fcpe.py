"""Oracle for the FCPE F0 estimator CPU path.

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``).  A numpy restatement of the
reference's numpy ``FCPE.infer`` (``runtime/models/fcpe.py:344-369``): the
log-mel front end (``:204-235``, ``_stft_frames`` ``:372-383``, the Slaney mel
filter bank of ``runtime/dsp/mel.py:118-146``), the input stack (``:237-255``),
six conv-only conformer layers (``:257-288``), the output norm and
weight-normalised projection with a sigmoid (``:290-302``) and the local
argmax decode (``:304-342``).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
SR, N_FFT, HOP, N_MELS = 16000, 1024, 160, 128


def _hz_to_mel(f):
    f = np.asarray(f, dtype=np.float64)
    mels = f / (200.0 / 3.0)
    if f.ndim:
        lt = f >= 1000.0
        mels[lt] = 15.0 + np.log(f[lt] / 1000.0) / (np.log(6.4) / 27.0)
    elif f >= 1000.0:
        mels = 15.0 + np.log(f / 1000.0) / (np.log(6.4) / 27.0)
    return mels


def _mel_to_hz(m):
    m = np.asarray(m, dtype=np.float64)
    f = (200.0 / 3.0) * m
    lt = m >= 15.0
    f[lt] = 1000.0 * np.exp((np.log(6.4) / 27.0) * (m[lt] - 15.0))
    return f


def mel_basis(fmin=0.0, fmax=8000.0):
    """Slaney mel filters with area normalisation (``runtime/dsp/mel.py:118-146``), float32."""
    n_bins = N_FFT // 2 + 1
    fftf = np.linspace(0.0, SR / 2.0, n_bins)
    mel_f = _mel_to_hz(np.linspace(float(_hz_to_mel(fmin)), float(_hz_to_mel(fmax)), N_MELS + 2))
    fdiff = np.diff(mel_f)
    ramps = np.subtract.outer(mel_f, fftf)
    w = np.zeros((N_MELS, n_bins))
    for i in range(N_MELS):
        w[i] = np.maximum(0.0, np.minimum(-ramps[i] / fdiff[i], ramps[i + 2] / fdiff[i + 1]))
    w *= (2.0 / (mel_f[2:N_MELS + 2] - mel_f[:N_MELS]))[:, None]
    return w.astype(F32)


def periodic_hann(n=N_FFT):
    t = np.arange(n, dtype=np.float64)
    return 0.5 - 0.5 * np.cos(2.0 * np.pi * t / n)


def log_mel(x):
    """``[T]`` -> ``[F, 128]``, F = T // 160 + 1 (``runtime/models/fcpe.py:204-235``)."""
    x = np.asarray(x, dtype=np.float64)
    T = x.shape[0]
    pl = (N_FFT - HOP) // 2
    pr = max((N_FFT - HOP + 1) // 2, N_FFT - T - pl)
    y = np.pad(x, (pl, pr), mode="reflect" if pr < T else "constant")
    nf = 1 + (y.shape[0] - N_FFT) // HOP
    idx = np.arange(N_FFT)[None, :] + HOP * np.arange(nf)[:, None]
    spec = np.fft.rfft(y[idx] * periodic_hann()[None, :], axis=1).T
    mag = np.sqrt(spec.real ** 2 + spec.imag ** 2 + 1e-9).astype(F32)
    mel = np.log(np.clip(mel_basis() @ mag, 1e-5, None)).astype(F32).T
    F = T // HOP + 1
    if F > mel.shape[0]:
        mel = np.concatenate([mel, mel[-1:]], axis=0)
    return mel[:F]


def sigmoid(x):
    with np.errstate(over="ignore", invalid="ignore"):
        return np.where(x >= 0, 1.0 / (1.0 + np.exp(-x)), np.exp(x) / (1.0 + np.exp(x)))


def conv1d_k(x, w, b, pad):
    """channels-last ``x [F, C_in]`` with ``w [O, C_in, K]`` -> ``[F, O]``."""
    F, _ = x.shape
    K = w.shape[2]
    xp = np.pad(x, ((pad, pad), (0, 0)))
    out = np.zeros((F, w.shape[0]), dtype=F32)
    for k in range(K):
        out += xp[k:k + F] @ w[:, :, k].T
    return out + b


def layer_norm(x, g, b, eps=1e-5):
    m = x.mean(-1, keepdims=True)
    v = x.var(-1, keepdims=True)
    return ((x - m) / np.sqrt(v + eps)) * g + b


def latent(sd, mel, taps=None):
    """``[F, 128]`` log-mel -> ``[F, 360]`` sigmoid salience."""
    def tap(name, a):
        if taps is not None:
            taps[name] = np.array(a, copy=True)

    h = conv1d_k(mel, sd["input_stack.0.weight"], sd["input_stack.0.bias"], 1)
    F = h.shape[0]
    hg = h.T.reshape(4, 128, F)                                      # GroupNorm(4), over channels x time
    m = hg.mean(axis=(1, 2), keepdims=True)
    v = hg.var(axis=(1, 2), keepdims=True)
    hg = (hg - m) / np.sqrt(v + 1e-5)
    h = (hg.reshape(512, F) * sd["input_stack.1.weight"][:, None] + sd["input_stack.1.bias"][:, None]).T
    h = np.where(h >= 0, h, 0.01 * h).astype(F32)
    x = conv1d_k(h, sd["input_stack.3.weight"], sd["input_stack.3.bias"], 1)
    tap("stack", x)
    for i in range(6):
        p = f"net.encoder_layers.{i}.conformer.net"
        xn = layer_norm(x, sd[p + ".0.weight"], sd[p + ".0.bias"])
        u = xn @ sd[p + ".2.weight"][:, :, 0].T + sd[p + ".2.bias"]
        g = u[:, :1024] * sigmoid(u[:, 1024:])                       # GLU
        gp = np.pad(g, ((15, 15), (0, 0)))
        wd = sd[p + ".4.conv.weight"][:, 0, :]                       # depthwise k31
        d = np.zeros_like(g)
        for k in range(31):
            d += gp[k:k + F] * wd[:, k]
        d = d + sd[p + ".4.conv.bias"]
        s = d * sigmoid(d)                                           # SiLU
        x = x + (s @ sd[p + ".6.weight"][:, :, 0].T + sd[p + ".6.bias"])
        tap(f"layer{i}", x)
    x = layer_norm(x, sd["norm.weight"], sd["norm.bias"])
    v_ = sd["output_proj.weight_v"]
    w = v_ / np.maximum(np.linalg.norm(v_, axis=1, keepdims=True), 1e-12) * sd["output_proj.weight_g"].reshape(-1)[:, None]
    lat = sigmoid(x @ w.T + sd["output_proj.bias"]).astype(F32)
    tap("latent", lat)
    return lat


def decode(lat, cent_table, threshold=0.006):
    """Local argmax decode (``runtime/models/fcpe.py:304-342``): f0 [F] Hz."""
    lat = np.asarray(lat, dtype=F32)
    conf = lat.max(axis=-1, keepdims=True)
    mi = lat.argmax(axis=-1)
    li = np.clip(np.arange(9)[None, :] + (mi[:, None] - 4), 0, lat.shape[1] - 1)
    cents = np.broadcast_to(cent_table[None, :], lat.shape)
    c = np.take_along_axis(cents, li, axis=-1)
    y = np.take_along_axis(lat, li, axis=-1)
    den = y.sum(axis=-1, keepdims=True)
    den = np.where(den == 0.0, np.float32(1e-30), den)
    dec = (c * y).sum(axis=-1, keepdims=True) / den
    dec = np.where(conf <= threshold, float("-inf"), dec)
    return (10.0 * np.power(2.0, dec / 1200.0))[:, 0].astype(F32)


def infer(sd, x, threshold=0.006, taps=None):
    """``[T]`` 16 kHz -> f0 ``[T // 160 + 1]``."""
    mel = log_mel(np.asarray(x, dtype=F32))
    if taps is not None:
        taps["mel"] = mel
    return decode(latent(sd, mel, taps), sd["cent_table"], threshold)
