"""Model-level fast path for the RMVPE F0 estimator.

``CudaRmvpe`` keeps the contract of ``RMVPE.infer_from_audio``
(``runtime/models/rmvpe.py:927``): ``[T]`` float32 16 kHz audio -> ``[F]``
float32 f0 in Hz, ``F = 1 + T // 160``.  The whole model (log-mel front end,
U-Net, BiGRU, linear + sigmoid, local-average decode) runs in one library call
per batch of equal-length clips, in fp32 (float64 for the STFT) so that the
salience argmax follows the reference.  Weights are the reference's checkpoint
dict (``RMVPE.W``) under its own keys.

``patch_reference`` replaces ``RMVPE.infer_from_audio`` on the class, so the
pipeline's ``load_rmvpe().infer_from_audio(...)`` (``runtime/pipeline.py:443-449``)
runs on the device unchanged.
"""

from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, fptr, lib

__all__ = ["CudaRmvpe", "frames", "patch_reference"]


def frames(T: int) -> int:
    """Frames for ``T`` samples (hop 160, centred STFT)."""
    F = C.c_int64(0)
    check(lib.rvc_cuda_rmvpe_frames(int(T), C.byref(F)))
    return int(F.value)


def max_lanes() -> int:
    """Concurrent f0 lanes of ``CudaRmvpe.infer_many`` (``RVC_CUDA_RMVPE_LANES``,
    default 4): each extra lane holds its own weight copy (~180 MB) and
    workspace, so the count is fixed rather than following the input."""
    n = int(os.environ.get("RVC_CUDA_RMVPE_LANES", "4"))
    if n < 1:
        raise ValueError(f"RVC_CUDA_RMVPE_LANES must be >= 1, got {n}")
    return n


class CudaRmvpe:
    """Device-resident RMVPE on one GPU (one library context)."""

    def __init__(self, weights: dict, device: Optional[int] = None, own_stream: bool = False):
        """``own_stream``: a private library context (stream and workspace) on the
        device, so f0 extraction can run concurrently with work on the shared
        context (the device pipeline overlaps it with HuBERT)."""
        if own_stream:
            dev = device if device is not None else int(os.environ.get("RVC_CUDA_DEVICE", "0"))
            self.ctx = _lib.Context(dev)
        else:
            self.ctx = _lib.get_context(device)
        self._weights = weights  # sibling lanes of infer_many are built from the same dict
        self._lanes = []
        h = C.c_int64(0)
        check(lib.rvc_cuda_rmvpe_create(self.ctx.handle, C.byref(h)))
        self.handle = int(h.value)
        for k, v in weights.items():
            if k.endswith("num_batches_tracked"):
                continue
            t = np.ascontiguousarray(np.asarray(v, dtype=np.float32))
            shape = (C.c_int64 * max(1, t.ndim))(*t.shape)
            check(lib.rvc_cuda_rmvpe_set_weight(self.handle, k.encode(), fptr(t), shape, t.ndim))
        check(lib.rvc_cuda_rmvpe_finalize(self.handle))

    @classmethod
    def from_reference(cls, model, device: Optional[int] = None):
        """Build from a loaded reference ``RMVPE`` (its float32 checkpoint dict)."""
        return cls(model.W, device=device)

    def close(self):
        for m in getattr(self, "_lanes", ()):
            m.close()
        self._lanes = []
        if getattr(self, "handle", 0):
            lib.rvc_cuda_rmvpe_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def infer_batch(self, xb, thred: float = 0.03, return_argmax: bool = False):
        """``xb [B,T]`` equal-length clips -> ``f0 [B,F]`` (and the salience
        argmax ``[B,F]`` int32 when ``return_argmax``)."""
        xb = np.ascontiguousarray(np.asarray(xb, dtype=np.float32))
        if xb.ndim != 2:
            raise ValueError(f"batch input must be [B, T], got {xb.shape}")
        B, T = xb.shape
        if T <= 512:
            raise ValueError(f"audio of {T} samples is too short (reflect padding needs > 512)")
        F = frames(T)
        f0 = np.empty((B, F), np.float32)
        am = np.empty((B, F), np.int32)
        check(lib.rvc_cuda_rmvpe_infer(self.handle, B, T, fptr(xb), float(thred), fptr(f0),
                                       am.ctypes.data_as(C.POINTER(C.c_int32))))
        return (f0, am) if return_argmax else f0

    def infer_from_audio(self, x, thred: float = 0.03) -> np.ndarray:
        """``RMVPE.infer_from_audio``: ``[T]`` -> ``[F]`` Hz."""
        x = np.asarray(x, dtype=np.float32)
        if x.ndim != 1:
            raise ValueError(f"infer_from_audio needs 1-D audio, got {x.ndim}-D")
        return self.infer_batch(x[None, :], thred)[0]

    def infer_many(self, xs, thred: float = 0.03):
        """f0 of several 1-D clips of any lengths, run concurrently on at most
        ``max_lanes()`` lanes (this model, then sibling models with their own
        context, stream and weight copy, built on first use and kept): clip
        ``i`` runs on lane ``i % lanes``, each lane's clips in order on one host
        thread.  Each result equals ``infer_from_audio`` of that clip (each clip
        is its own batch of one, as in the reference's per-segment calls), so
        the lane count changes the timing only."""
        xs = [np.asarray(x, dtype=np.float32) for x in xs]
        n = min(len(xs), max_lanes())
        if n <= 1:
            return [self.infer_from_audio(x, thred) for x in xs]
        while len(self._lanes) < n - 1:
            self._lanes.append(CudaRmvpe(self._weights, device=self.ctx.device, own_stream=True))
        lanes = [self] + self._lanes[:n - 1]

        def run_lane(j):
            return [(i, lanes[j].infer_from_audio(xs[i], thred)) for i in range(j, len(xs), n)]

        from concurrent.futures import ThreadPoolExecutor  # noqa: PLC0415
        out = [None] * len(xs)
        with ThreadPoolExecutor(max_workers=n, thread_name_prefix="rvc-rmvpe") as ex:
            for f in [ex.submit(run_lane, j) for j in range(n)]:
                for i, r in f.result():
                    out[i] = r
        return out

    # ---------------------------------------------------------------- debug
    def keep_taps(self, on: bool = True):
        check(lib.rvc_cuda_rmvpe_keep_taps(self.handle, 1 if on else 0))

    def tap(self, name: str, shape) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.float32)
        check(lib.rvc_cuda_rmvpe_tap(self.handle, name.encode(), fptr(out), out.size))
        return out.reshape(shape)


def patch_reference(rmvpe_module=None, device: Optional[int] = None):
    """Route ``RMVPE.infer_from_audio`` of the reference through ``CudaRmvpe``
    (one device model cached per ``RMVPE`` instance)."""
    if rmvpe_module is None:
        from runtime.models import rmvpe as rmvpe_module  # noqa: PLC0415
    cls = rmvpe_module.RMVPE
    if getattr(cls, "_rvc_cuda_patched", False):
        return cls

    def infer_from_audio(self, x, thred=0.03):
        m = self.__dict__.get("_rvc_cuda_model")
        if m is None:
            m = CudaRmvpe.from_reference(self, device=device)
            self.__dict__["_rvc_cuda_model"] = m
        return m.infer_from_audio(x, thred)

    cls._rvc_cuda_orig_infer_from_audio = cls.infer_from_audio
    cls.infer_from_audio = infer_from_audio
    cls._rvc_cuda_patched = True
    return cls
