"""Pipeline signal processing on the device.

The steps ``runtime/pipeline.py`` runs in numpy / scipy around the models:
the 48 Hz high-pass ``filtfilt`` (``:49``, ``:765``), the silence split points
(``:767-790``), the x2 feature interpolation (``runtime/nn.py:734-758``), the
protect blend (``:594-608``), ``change_rms`` (``:164-235``) and the int16
conversion (``:1208-1213``).  Each call takes and returns numpy arrays; the
filter coefficients are designed on the host with the same scipy call as the
reference.

``patch_reference`` points ``runtime.pipeline``'s ``change_rms``,
``interpolate_linear`` and ``signal.filtfilt`` (through a proxy of the scipy
module bound in that module only) at these functions.
"""

from __future__ import annotations

import ctypes as C
import types
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, fptr, lib

__all__ = ["filtfilt", "highpass", "split_points", "interpolate_linear", "protect_blend", "change_rms", "to_int16",
           "f0_autocorrelation", "resample", "patch_reference"]


def _ctx(device: Optional[int] = None):
    return _lib.get_context(device)


def _dp(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def filtfilt(b, a, x) -> np.ndarray:
    """``scipy.signal.filtfilt(b, a, x)`` (padtype 'odd', method 'pad'), float64, 1-D."""
    b = np.ascontiguousarray(np.atleast_1d(np.asarray(b, dtype=np.float64)))
    a = np.ascontiguousarray(np.atleast_1d(np.asarray(a, dtype=np.float64)))
    x = np.asarray(x)
    x = np.ascontiguousarray(x, dtype=np.float32 if x.dtype == np.float32 else np.float64)
    if x.ndim != 1:
        raise ValueError(f"filtfilt on the device takes 1-D signals, got {x.shape}")
    y = np.empty(x.size, np.float64)
    check(lib.rvc_cuda_filtfilt(_ctx().handle, _dp(b), b.size, _dp(a), a.size, _dp(x), int(x.dtype == np.float32),
                                x.size, _dp(y)))
    return y


_HP = None


def highpass(audio) -> np.ndarray:
    """The pipeline's 5th-order 48 Hz Butterworth high-pass at 16 kHz, forward-backward."""
    global _HP
    if _HP is None:
        from scipy import signal  # noqa: PLC0415 - the same filter design call as the reference
        _HP = signal.butter(N=5, Wn=48, btype="high", fs=16000)
    return filtfilt(_HP[0], _HP[1], audio)


def split_points(audio, t_query: int, step: int, window: int = 160) -> list:
    """Cut points of the pipeline's silence split for ``t = step, 2 step, ... < len(audio)``:
    the first minimum of the ``window``-sample absolute sums within ``t_query`` of ``t``."""
    x = np.ascontiguousarray(np.asarray(audio, dtype=np.float64))
    n = x.size
    cap = max(1, (n - 1) // step if n > step else 1)
    out = np.empty(cap, np.int64)
    cnt = C.c_int64(0)
    check(lib.rvc_cuda_split_points(_ctx().handle, _dp(x), n, int(window), int(t_query), int(step), _dp(out), cap,
                                    C.byref(cnt)))
    return [int(v) for v in out[:cnt.value] if v >= 0]


def interpolate_linear(x, scale_factor=2, axis=-1):
    """``runtime.nn.interpolate_linear`` for float32 arrays (align_corners=False)."""
    x = np.asarray(x)
    if x.dtype != np.float32:
        raise ValueError("the device interpolate_linear takes float32 arrays")
    xm = np.moveaxis(x, axis, 0)
    L = xm.shape[0]
    rest = xm.shape[1:]
    Lo = int(L * scale_factor)
    if Lo == L:
        return x.copy()
    D = int(np.prod(rest)) if rest else 1
    src = np.ascontiguousarray(xm.reshape(L, D))
    out = np.empty((Lo, D), np.float32)
    check(lib.rvc_cuda_interp_linear(_ctx().handle, fptr(src), L, D, float(scale_factor), fptr(out), Lo))
    return np.moveaxis(out.reshape((Lo,) + rest), 0, axis)


def protect_blend(feats, feats0, pitchf, protect: float) -> np.ndarray:
    """``feats * w + feats0 * (1 - w)`` with ``w = protect`` where ``pitchf < 1`` else 1
    (feats / feats0 ``[1,P,D]``, pitchf ``[1,P]``)."""
    f = np.ascontiguousarray(np.asarray(feats, dtype=np.float32))
    f0 = np.ascontiguousarray(np.asarray(feats0, dtype=np.float32))
    pf = np.ascontiguousarray(np.asarray(pitchf, dtype=np.float32).reshape(-1))
    P, D = f.shape[-2], f.shape[-1]
    if f0.shape != f.shape or pf.size != P:
        raise ValueError("protect_blend: feats, feats0 and pitchf disagree in shape")
    out = np.empty_like(f)
    check(lib.rvc_cuda_protect(_ctx().handle, fptr(f), fptr(f0), fptr(pf), P, D, float(protect), fptr(out)))
    return out


def change_rms(data1, data2, sr1, sr2, rate):
    """``runtime.pipeline.change_rms(data1, data2, sr1, sr2, rate)``."""
    d1 = np.ascontiguousarray(np.asarray(data1, dtype=np.float32).reshape(-1))
    d2 = np.ascontiguousarray(np.asarray(data2, dtype=np.float32).reshape(-1))
    out = np.empty_like(d2)
    if d2.size:
        check(lib.rvc_cuda_change_rms(_ctx().handle, fptr(d1), d1.size, int(sr1), fptr(d2), d2.size, int(sr2),
                                      float(rate), fptr(out)))
    return out


def to_int16(audio) -> np.ndarray:
    """Peak-normalised int16 (peak at 0.99 of full scale when the signal exceeds it)."""
    x = np.ascontiguousarray(np.asarray(audio, dtype=np.float32).reshape(-1))
    y = np.empty(x.size, np.int16)
    if x.size:
        check(lib.rvc_cuda_to_int16(_ctx().handle, fptr(x), x.size, _dp(y)))
    return y


def f0_autocorrelation(x, sr, hop=160, f0_min=50.0, f0_max=1100.0, voicing_threshold=0.6, time_step=0.01):
    """``runtime.dsp.f0.f0_autocorrelation`` (``runtime/dsp/f0.py:24-94``): the
    frame / lag parameters and the Hann window are derived on the host exactly
    as there, the per-frame analysis runs on the device."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float64))
    if x.ndim != 1:
        raise ValueError(f"f0_autocorrelation needs a 1-D signal, got {x.ndim}-D")
    if time_step is not None and time_step > 0:
        hop = int(round(sr * time_step))
    hop = max(1, int(hop))
    win = int(round(sr * 0.045))
    if f0_min > 0 and win < 3 * sr / f0_min:
        win = int(round(3 * sr / f0_min))
    if win % 2 == 0:
        win += 1
    n_frames = int(np.ceil(len(x) / hop))
    lag_min = max(1, int(round(sr / f0_max)))
    lag_max = int(round(sr / f0_min))
    if lag_max >= win:
        lag_max = win - 1
    if lag_min > lag_max:
        raise ValueError("no valid lag between f0_max and f0_min inside the window")
    f0 = np.zeros(n_frames, dtype=np.float32)
    if n_frames and x.size:
        w = np.ascontiguousarray(np.hanning(win))
        check(lib.rvc_cuda_f0_autocorr(_ctx().handle, _dp(x), x.size, int(sr), hop, win, lag_min, lag_max, _dp(w),
                                       float(voicing_threshold), fptr(f0), n_frames))
    return f0


_RESAMPLE_METHODS = {"fft": 0, "linear": 1, "sinc": 2}


def resample(x, orig_sr, target_sr, method="fft"):
    """``runtime.dsp.resample.resample`` (``runtime/dsp/resample.py:129``) for
    1-D signals: float32 of length ``max(1, round(n * target_sr / orig_sr))``."""
    if orig_sr <= 0 or target_sr <= 0:
        raise ValueError("sample rates must be positive")
    if method not in _RESAMPLE_METHODS:
        raise ValueError(f"unsupported method: {method!r} (use 'fft', 'linear' or 'sinc')")
    x = np.asarray(x)
    if x.ndim != 1:
        raise ValueError(f"the device resample takes 1-D signals, got {x.ndim}-D")
    xx = np.ascontiguousarray(x, dtype=np.float32 if x.dtype == np.float32 else np.float64)
    if orig_sr == target_sr:
        return xx.astype(np.float32)
    n_in = xx.size
    n_out = max(1, int(round(n_in * target_sr / orig_sr)))
    y = np.empty(n_out, np.float32)
    if n_in == 0:
        raise ValueError("resample of an empty signal")
    check(lib.rvc_cuda_resample(_ctx().handle, _dp(xx), int(xx.dtype == np.float32), n_in, int(orig_sr),
                                int(target_sr), _RESAMPLE_METHODS[method], fptr(y), n_out))
    return y


# ---- device-pointer forms (asynchronous on the context's stream), used by the
# device-resident conversion in rvc_cuda.pipeline
def interpolate_device(ctx, d_x: int, L: int, D: int, scale: float, d_y: int, Lo: int):
    check(lib.rvc_cuda_interp_linear_device(ctx.handle, C.c_void_p(d_x), int(L), int(D), float(scale),
                                            C.c_void_p(d_y), int(Lo)))


def protect_device(ctx, d_feats: int, d_feats0: int, d_pitchf: int, P: int, D: int, protect: float, d_out: int):
    check(lib.rvc_cuda_protect_device(ctx.handle, C.c_void_p(d_feats), C.c_void_p(d_feats0), C.c_void_p(d_pitchf),
                                      int(P), int(D), float(protect), C.c_void_p(d_out)))


def change_rms_device(ctx, d1: int, n1: int, sr1: int, d2: int, n2: int, sr2: int, rate: float, d_out: int):
    check(lib.rvc_cuda_change_rms_device(ctx.handle, C.c_void_p(d1), int(n1), int(sr1), C.c_void_p(d2), int(n2),
                                         int(sr2), float(rate), C.c_void_p(d_out)))


def to_int16_device(ctx, d_x: int, n: int, d_y: int):
    check(lib.rvc_cuda_to_int16_device(ctx.handle, C.c_void_p(d_x), int(n), C.c_void_p(d_y)))


def patch_reference(pipeline_module=None):
    """Route ``runtime.pipeline``'s ``change_rms``, ``interpolate_linear``,
    ``resample``, ``signal.filtfilt`` and the pm f0 (``f0_autocorrelation``,
    imported there by name, ``runtime/pipeline.py:40``) to the device versions."""
    if pipeline_module is None:
        from runtime import pipeline as pipeline_module  # noqa: PLC0415
    if getattr(pipeline_module, "_rvc_cuda_patched_dsp", False):
        return pipeline_module
    scipy_signal = pipeline_module.signal
    proxy = types.SimpleNamespace(**{k: getattr(scipy_signal, k) for k in dir(scipy_signal) if not k.startswith("__")})

    def _filtfilt(b, a, x, *args, **kw):
        if args or kw:  # other padding modes are not on the device path
            raise ValueError("the device filtfilt supports the default padtype / method only")
        return filtfilt(b, a, x)

    proxy.filtfilt = _filtfilt
    pipeline_module._rvc_cuda_orig_signal = scipy_signal
    pipeline_module.signal = proxy
    pipeline_module._rvc_cuda_orig_change_rms = pipeline_module.change_rms
    pipeline_module.change_rms = change_rms
    pipeline_module._rvc_cuda_orig_interpolate_linear = pipeline_module.interpolate_linear
    pipeline_module.interpolate_linear = interpolate_linear
    if hasattr(pipeline_module, "resample"):
        pipeline_module._rvc_cuda_orig_resample = pipeline_module.resample
        pipeline_module.resample = resample
    if hasattr(pipeline_module, "f0_autocorrelation"):
        pipeline_module._rvc_cuda_orig_f0_autocorrelation = pipeline_module.f0_autocorrelation
        pipeline_module.f0_autocorrelation = f0_autocorrelation
    pipeline_module._rvc_cuda_patched_dsp = True
    return pipeline_module
