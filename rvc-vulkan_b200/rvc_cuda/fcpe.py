"""Model-level fast path for the FCPE F0 estimator.

``CudaFcpe`` keeps the contract of ``FCPE.infer`` (``runtime/models/fcpe.py:344``):
``[T]`` float32 16 kHz audio -> ``[F]`` float32 f0 in Hz, ``F = T // 160 + 1``,
``decoder_mode`` "local_argmax" (the pipeline's) or "argmax".  The whole model
(log-mel front end, input stack, six conv-only conformer layers,
weight-normalised projection, sigmoid, decode) runs in one library call per
batch of equal-length clips;
the convolutions and linears on tensor cores (BF16x3, fp32 accumulate).
Weights are the reference's checkpoint dict (``FCPE.W``) under its own keys.

``patch_reference`` replaces ``FCPE.infer`` on the class, so the pipeline's
``load_fcpe().infer(...)`` (``runtime/pipeline.py:452-462``) runs on the device.
"""

from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, fptr, lib

__all__ = ["CudaFcpe", "frames", "patch_reference"]

PRECISIONS = {"bf16x3": 0, "simt": 1}


def frames(T: int) -> int:
    """Frames for ``T`` samples (hop 160)."""
    return int(T) // 160 + 1


DECODER_MODES = {"local_argmax": 0, "argmax": 1}


class CudaFcpe:
    """Device-resident FCPE on one GPU (one library context)."""

    def __init__(self, weights: dict, device: Optional[int] = None, precision: str = "bf16x3"):
        p = os.environ.get("RVC_CUDA_PRECISION", precision)
        if p not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}")
        self.ctx = _lib.get_context(device)
        h = C.c_int64(0)
        check(lib.rvc_cuda_fcpe_create(self.ctx.handle, PRECISIONS[p], C.byref(h)))
        self.handle = int(h.value)
        for k, v in weights.items():
            t = np.ascontiguousarray(np.asarray(v, dtype=np.float32))
            shape = (C.c_int64 * max(1, t.ndim))(*t.shape)
            check(lib.rvc_cuda_fcpe_set_weight(self.handle, k.encode(), fptr(t), shape, t.ndim))
        check(lib.rvc_cuda_fcpe_finalize(self.handle))

    @classmethod
    def from_reference(cls, model, device: Optional[int] = None, precision: str = "bf16x3"):
        """Build from a loaded reference ``FCPE`` (its float32 checkpoint dict)."""
        return cls(model.W, device=device, precision=precision)

    def close(self):
        if getattr(self, "handle", 0):
            lib.rvc_cuda_fcpe_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def infer_batch(self, xb, threshold: float = 0.006, return_argmax: bool = False,
                    decoder_mode: str = "local_argmax"):
        """``xb [B,T]`` equal-length clips -> ``f0 [B,F]`` (and the latent argmax
        ``[B,F]`` int32 when ``return_argmax``); ``decoder_mode`` as in
        ``FCPE._decode`` (``runtime/models/fcpe.py:304-342``)."""
        if decoder_mode not in DECODER_MODES:
            raise ValueError(f"Unknown FCPE decoder mode: {decoder_mode}")
        xb = np.ascontiguousarray(np.asarray(xb, dtype=np.float32))
        if xb.ndim != 2 or xb.shape[1] < 1:
            raise ValueError(f"batch input must be [B, T] with T >= 1, got {xb.shape}")
        B, T = xb.shape
        F = frames(T)
        f0 = np.empty((B, F), np.float32)
        am = np.empty((B, F), np.int32)
        check(lib.rvc_cuda_fcpe_infer_mode(self.handle, B, T, fptr(xb), float(threshold),
                                           DECODER_MODES[decoder_mode], fptr(f0),
                                           am.ctypes.data_as(C.POINTER(C.c_int32))))
        return (f0, am) if return_argmax else f0

    def infer(self, x, sr: int = 16000, decoder_mode: str = "local_argmax", threshold: float = 0.006) -> np.ndarray:
        """``FCPE.infer``: ``[T]`` -> ``[F]`` Hz."""
        x = np.asarray(x, dtype=np.float32)
        if x.ndim != 1:
            raise ValueError(f"infer needs 1-D audio, got {x.ndim}-D")
        if sr != 16000:
            raise NotImplementedError(f"FCPE is defined at sr=16000, got sr={sr}; resample to 16 kHz first")
        return self.infer_batch(x[None, :], threshold, decoder_mode=decoder_mode)[0]

    # ---------------------------------------------------------------- debug
    def keep_taps(self, on: bool = True):
        check(lib.rvc_cuda_fcpe_keep_taps(self.handle, 1 if on else 0))

    def tap(self, name: str, shape) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.float32)
        check(lib.rvc_cuda_fcpe_tap(self.handle, name.encode(), fptr(out), out.size))
        return out.reshape(shape)


def patch_reference(fcpe_module=None, device: Optional[int] = None, precision: str = "bf16x3"):
    """Replace ``FCPE.infer`` on the class (one device model per instance)."""
    if fcpe_module is None:
        from runtime.models import fcpe as fcpe_module  # noqa: PLC0415
    cls = fcpe_module.FCPE
    if getattr(cls, "_rvc_cuda_patched", False):
        return cls

    def _model(self):
        m = self.__dict__.get("_rvc_cuda_model")
        if m is None:
            m = CudaFcpe(self.W, device=device, precision=precision)
            self.__dict__["_rvc_cuda_model"] = m
        return m

    def infer(self, x, sr=16000, decoder_mode="local_argmax", threshold=0.006):
        return _model(self).infer(x, sr=sr, decoder_mode=decoder_mode, threshold=threshold)

    cls._rvc_cuda_orig_infer = cls.infer
    cls.infer = infer
    cls._rvc_cuda_patched = True
    return cls
