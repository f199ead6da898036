"""Oracle for the pipeline's signal processing around the models.

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``): the checker for the device
DSP path, never part of it.  A numpy / pure-Python restatement of

* the 48 Hz high-pass ``signal.filtfilt(_BH, _AH, audio)``
  (``runtime/pipeline.py:49``, ``:765``).  ``filtfilt`` comes from scipy
  (``scipy.signal``, 1.18.1 in the environment the fixtures were made in;
  the reference pins only ``scipy>=1.13``).  Restated here from scipy's
  published algorithm: odd extension of ``padlen = 3 * max(len(a), len(b))``
  samples at each end, ``lfilter`` forward from ``lfilter_zi * x[0]``, then
  backward over the reversed output from ``lfilter_zi * y[-1]``; ``lfilter``
  is the direct-form-II-transposed recursion with coefficients normalised by
  ``a[0]``; ``lfilter_zi`` is scipy 1.18's closed form (cumulative sums of
  ``b - y_inf a`` from the last tap, ``y_inf = sum(b) / sum(a)``);
* the silence split (``runtime/pipeline.py:767-790``);
* the x2 feature interpolation (``runtime/nn.py:734-758``) and the protect
  blend (``runtime/pipeline.py:594-608``);
* ``change_rms`` with ``_rms_curve`` / ``_interp_linear_size``
  (``runtime/pipeline.py:164-235``);
* the peak-normalised int16 conversion (``runtime/pipeline.py:1208-1213``).

Pinned by ``tests/golden/dsp.npz``, made by running the reference's own
functions (``tests/golden/make_golden.py --only dsp``).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------- filtfilt
def lfilter_zi(b, a):
    """Steady-state initial state of ``lfilter`` for a unit step, in scipy
    1.18's closed form: ``y_inf = sum(b) / sum(a)`` and
    ``zi[k] = sum_{j>k} (b_j - y_inf a_j)``, summed from the last tap down."""
    b = np.atleast_1d(np.asarray(b, np.float64))
    a = np.atleast_1d(np.asarray(a, np.float64))
    if a[0] != 1:
        b, a = b / a[0], a / a[0]
    y_inf = np.sum(b) / np.sum(a)
    n = max(a.size, b.size)
    c = np.r_[b, np.zeros(n - b.size)] - y_inf * np.r_[a, np.zeros(n - a.size)]
    return np.flip(np.cumsum(np.flip(c)))[1:]


def lfilter(b, a, x, zi):
    """Direct-form-II-transposed IIR filter, float64, sequential (scipy's
    ``lfilter`` order: ``y = z0 + b0 x``; ``z_k = z_{k+1} + x b_{k+1} - y a_{k+1}``)."""
    b = np.asarray(b, np.float64)
    a = np.asarray(a, np.float64)
    n = max(a.size, b.size)
    bb = list(np.r_[b, np.zeros(n - b.size)] / a[0])
    aa = list(np.r_[a, np.zeros(n - a.size)] / a[0])
    z = [float(v) for v in zi]
    xs = np.asarray(x, np.float64).tolist()
    out = [0.0] * len(xs)
    for t, xv in enumerate(xs):
        y = z[0] + bb[0] * xv
        for k in range(n - 2):
            z[k] = z[k + 1] + xv * bb[k + 1] - y * aa[k + 1]
        z[n - 2] = xv * bb[n - 1] - y * aa[n - 1]
        out[t] = y
    return np.asarray(out, np.float64)


def odd_ext(x, n):
    """``[2 x0 - x[n..1], x, 2 x_last - x[-2..-n-1]]`` in the signal's dtype."""
    x = np.asarray(x)
    left = 2 * x[:1] - x[n:0:-1]
    right = 2 * x[-1:] - x[-2:-n - 2:-1]
    return np.concatenate([left, x, right])


def filtfilt(b, a, x):
    """``scipy.signal.filtfilt(b, a, x)`` with the default ``padtype='odd'``."""
    x = np.asarray(x)
    pl = 3 * max(len(a), len(b))
    if x.shape[0] <= pl:
        raise ValueError("the input must be longer than padlen")
    ext = odd_ext(x, pl)
    zi = lfilter_zi(b, a)
    y = lfilter(b, a, ext, zi * float(ext[0]))
    y = lfilter(b, a, y[::-1], zi * float(y[-1]))
    return y[::-1][pl:-pl].copy()


# ---------------------------------------------------------------- split
def split_points(audio, window, t_query, step):
    """Cut points of the silence split (``runtime/pipeline.py:767-790``): the
    160-sample absolute sums of the reflect-padded signal, accumulated in
    window order, and for every ``t = step, 2 step, ... < len(audio)`` the
    first minimum within ``t_query`` of ``t`` (empty windows skipped)."""
    audio = np.asarray(audio)
    pad = np.pad(audio, (window // 2, window // 2), mode="reflect")
    ap_abs = np.abs(pad)
    s = np.zeros_like(audio)
    for i in range(window):
        s += ap_abs[i:i - window]
    out = []
    for t in range(step, audio.shape[0], step):
        lo = max(0, t - t_query)
        hi = min(s.shape[0], t + t_query)
        seg = s[lo:hi]
        if seg.size == 0:
            continue
        out.append(lo + int(np.where(seg == seg.min())[0][0]))
    return out


# ---------------------------------------------------------------- features
def interpolate_linear(x, scale_factor=2, axis=-1):
    """``runtime.nn.interpolate_linear`` (``runtime/nn.py:734-758``):
    ``src = (i + 0.5) / scale - 0.5`` clipped to ``[0, L-1]``, ``frac`` in
    the array's dtype."""
    x = np.asarray(x)
    L = x.shape[axis]
    Lo = int(L * scale_factor)
    if Lo == L:
        return x.copy()
    src = (np.arange(Lo, dtype=np.float64) + 0.5) / float(scale_factor) - 0.5
    src = np.clip(src, 0.0, L - 1)
    lo = np.floor(src).astype(np.int64)
    hi = np.minimum(lo + 1, L - 1)
    frac = (src - lo).astype(x.dtype) if x.dtype != np.float64 else src - lo
    xm = np.moveaxis(x, axis, -1)
    out = xm[..., lo] * (1.0 - frac) + xm[..., hi] * frac
    return np.moveaxis(out, -1, axis)


def protect_blend(feats, feats0, pitchf, protect):
    """``feats * w + feats0 * (1 - w)``, ``w = 1`` where ``pitchf > 0`` and
    ``protect`` where ``pitchf < 1`` (``runtime/pipeline.py:604-608``)."""
    pitchff = np.asarray(pitchf).copy()
    pitchff[pitchf > 0] = 1
    pitchff[pitchf < 1] = protect
    pitchff = pitchff[..., None]
    return feats * pitchff + feats0 * (1 - pitchff)


def align_frames(arr, n):
    """Repeat the last frame or cut to ``n`` frames along axis 1
    (``runtime/pipeline.py:582-603``)."""
    m = arr.shape[1]
    if m < n:
        return np.concatenate([arr, np.repeat(arr[:, -1:], n - m, axis=1)], axis=1)
    return arr[:, :n]


# ---------------------------------------------------------------- rms mix
def rms_curve(x, sr):
    """``_rms_curve`` (``runtime/pipeline.py:195-211``): RMS of frames of
    ``sr//2*2`` samples every ``sr//2`` of the zero-padded signal, float32."""
    fl = sr // 2 * 2
    hop = sr // 2
    xp = np.pad(np.asarray(x, F32), (fl // 2, fl // 2), mode="constant")
    frames = np.lib.stride_tricks.sliding_window_view(xp, fl)[::hop]
    return np.sqrt(np.mean(frames.astype(F32) ** 2, axis=-1))[None, :].astype(F32)


def interp_linear_size(x, n_out):
    """``_interp_linear_size`` (``runtime/pipeline.py:214-235``) along the last axis."""
    x = np.asarray(x, np.float64)
    L = x.shape[-1]
    if n_out <= 0 or L == n_out:
        return x.astype(F32)
    src = (np.arange(n_out, dtype=np.float64) + 0.5) * (L / n_out) - 0.5
    src = np.clip(src, 0.0, L - 1)
    lo = np.floor(src).astype(np.int64)
    hi = np.minimum(lo + 1, L - 1)
    frac = src - lo
    return (x[..., lo] * (1.0 - frac) + x[..., hi] * frac).astype(F32)


def change_rms(data1, data2, sr1, sr2, rate):
    """``change_rms`` (``runtime/pipeline.py:164-192``)."""
    n = np.asarray(data2).shape[0]
    if n == 0:
        return np.asarray(data2, F32).copy()
    r1 = interp_linear_size(rms_curve(data1, int(sr1)), n)
    r2 = np.maximum(interp_linear_size(rms_curve(data2, int(sr2)), n), F32(1e-6))
    ratio = np.power(r1, 1.0 - rate) * np.power(r2, rate - 1.0)
    return np.asarray(data2, F32) * ratio.reshape(-1)


# ---------------------------------------------------------------- int16
def to_int16(audio):
    """Peak normalisation to 0.99 of full scale when the peak exceeds it, then
    truncation to int16 (``runtime/pipeline.py:1208-1213``)."""
    audio = np.asarray(audio, F32)
    audio_max = np.abs(audio).max() / 0.99
    max_int16 = 32768.0
    if audio_max > 1:
        max_int16 /= audio_max
    return (audio * max_int16).astype(np.int16)


# ---------------------------------------------------------------- pm f0
def f0_autocorrelation(x, sr, hop=160, f0_min=50.0, f0_max=1100.0, voicing_threshold=0.6, time_step=0.01):
    """``f0_autocorrelation`` (``runtime/dsp/f0.py:24-94``): per frame of ``win``
    samples (45 ms, at least three periods of ``f0_min``, odd) centred on
    ``i * hop``: mean removed, Hann window, autocorrelation through an rfft of
    ``nfft >= 2 win`` points, the first lag of the largest normalised value in
    ``[sr / f0_max, sr / f0_min]``; voiced above the threshold."""
    x = np.asarray(x, dtype=np.float64)
    if time_step is not None and time_step > 0:
        hop = int(round(sr * time_step))
    hop = max(1, int(hop))
    win = int(round(sr * 0.045))
    if f0_min > 0 and win < 3 * sr / f0_min:
        win = int(round(3 * sr / f0_min))
    if win % 2 == 0:
        win += 1
    n_frames = int(np.ceil(len(x) / hop))
    f0 = np.zeros(n_frames, dtype=F32)
    lag_min = max(1, int(round(sr / f0_max)))
    lag_max = min(int(round(sr / f0_min)), win - 1)
    nfft = 1 << int(np.ceil(np.log2(2 * win)))
    w = np.hanning(win)
    half = win // 2
    for i in range(n_frames):
        s = i * hop - half
        e = s + win
        if s >= 0 and e <= len(x):
            seg = x[s:e]
        else:
            seg = np.pad(x[max(s, 0):min(e, len(x))], (max(0, -s), max(0, e - len(x))))
        seg = seg - seg.mean()
        if float(np.max(np.abs(seg))) < 1e-7:
            continue
        X = np.fft.rfft(seg * w, n=nfft)
        r = np.fft.irfft(X * np.conj(X), n=nfft)[:win]
        if r[0] <= 0.0:
            continue
        rn = r / r[0]
        seg_r = rn[lag_min:lag_max + 1]
        k = int(np.argmax(seg_r)) + lag_min
        if seg_r[k - lag_min] > voicing_threshold:
            f0[i] = sr / k
    return f0


# ---------------------------------------------------------------- resample
def _kaiser_sinc(t, radius, beta=12.0):
    x = t / float(radius)
    with np.errstate(invalid="ignore", divide="ignore"):
        kaiser = np.where(np.abs(x) <= 1.0, np.i0(beta * np.sqrt(np.maximum(0.0, 1.0 - x * x))) / np.i0(beta), 0.0)
    return np.sinc(t) * kaiser


def resample(x, orig_sr, target_sr, method="fft"):
    """``resample`` (``runtime/dsp/resample.py:129-168``) for 1-D signals:
    ``fft`` interpolates the rfft spectrum at ``p_k = k n_in sr_out / (sr_in n_out)``
    with a 33-tap Kaiser-sinc (beta 12) over the edge-padded spectrum, zero past
    the source Nyquist, then irfft and ``* n_out / n_in`` (:41-78); ``sinc`` is
    the 25-tap time-domain kernel (:96-126); ``linear`` is ``np.interp`` on
    ``np.linspace(0, n_in - 1, n_out)`` (:81-93)."""
    x = np.asarray(x, dtype=np.float64)
    n_in = x.shape[-1]
    if orig_sr == target_sr:
        return x.copy().astype(F32)
    n_out = max(1, int(round(n_in * target_sr / orig_sr)))
    if method == "fft":
        X = np.fft.rfft(x, n=n_in)
        nbi, nbo = X.shape[-1], n_out // 2 + 1
        p = np.arange(nbo, dtype=np.float64) * (n_in * target_sr / (orig_sr * n_out))
        ok = p <= (nbi - 1)
        Y = np.zeros(nbo, dtype=np.complex128)
        if ok.any():
            radius, pad = 16, 17
            Xp = np.pad(X, (pad, pad), mode="edge")
            pp = p[ok] + pad
            base = np.floor(pp)[:, None].astype(np.int64) + np.arange(-radius, radius + 1)[None, :]
            kern = _kaiser_sinc(pp[:, None] - base.astype(np.float64), radius)
            Y[ok] = np.sum(Xp[base] * kern, axis=-1)
        y = np.fft.irfft(Y, n=n_out) * (n_out / n_in)
    elif method == "sinc":
        ratio = n_in / n_out
        pos = np.arange(n_out, dtype=np.float64) * ratio
        base = pos.astype(np.int64)
        y = np.zeros(n_out, dtype=np.float64)
        for k in range(-12, 13):
            idx = np.clip(base + k, 0, n_in - 1)
            y += np.take(x, idx) * _kaiser_sinc(pos - (base + k), 12)
    else:
        y = np.interp(np.linspace(0.0, n_in - 1, n_out), np.arange(n_in), x)
    return y.astype(F32)
