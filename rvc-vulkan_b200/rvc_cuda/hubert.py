"""Model-level fast path for the HuBERT-base feature encoder.

``CudaHubert`` keeps the numpy-in / numpy-out contract of
``HubertEncoder.encode`` and ``encode_batch`` (``runtime/models/hubert.py:564``,
``:593``): ``x [1,T]`` float32 16 kHz (already layer-normed by the caller) ->
``[1,L,768]`` (version 2, last hidden state) or ``[1,L,256]`` (version 1,
layer 9 through ``final_proj``).  Weights are uploaded once under the
reference's state-dict keys; the positional conv's weight norm is folded on the
device (or taken pre-folded from ``_pos_conv_weight``, as
``HubertEncoder._load_and_prepare`` stores it, ``runtime/models/hubert.py:499-559``).

``patch_reference`` installs it on the reference class so ``runtime/pipeline.py``
and ``runtime/vc.py`` run unchanged.
"""

from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, fptr, lib

__all__ = ["CudaHubert", "out_len", "patch_reference", "HUBERT_KEYS"]

PRECISIONS = {"bf16x3": 0, "simt": 1}


def _keys() -> list:
    ks = [f"feature_extractor.conv_layers.{i}.conv.weight" for i in range(7)]
    ks += ["feature_extractor.conv_layers.0.layer_norm.weight", "feature_extractor.conv_layers.0.layer_norm.bias",
           "feature_projection.layer_norm.weight", "feature_projection.layer_norm.bias",
           "feature_projection.projection.weight", "feature_projection.projection.bias",
           "encoder.pos_conv_embed.conv.bias", "encoder.layer_norm.weight", "encoder.layer_norm.bias"]
    for i in range(12):
        p = f"encoder.layers.{i}."
        for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
            ks += [p + f"attention.{nm}.weight", p + f"attention.{nm}.bias"]
        ks += [p + "layer_norm.weight", p + "layer_norm.bias", p + "final_layer_norm.weight",
               p + "final_layer_norm.bias", p + "feed_forward.intermediate_dense.weight",
               p + "feed_forward.intermediate_dense.bias", p + "feed_forward.output_dense.weight",
               p + "feed_forward.output_dense.bias"]
    return ks


HUBERT_KEYS = tuple(_keys())
_POS_KEYS = (("_pos_conv_weight",),
             ("encoder.pos_conv_embed.conv.weight_g", "encoder.pos_conv_embed.conv.weight_v"),
             ("encoder.pos_conv_embed.conv.parametrizations.weight.original0",
              "encoder.pos_conv_embed.conv.parametrizations.weight.original1"))


def out_len(T: int) -> int:
    """Frames for ``T`` samples: conv strides 5,2,2,2,2,2,2 with kernels 10,3,3,3,3,2,2."""
    L = C.c_int64(0)
    check(lib.rvc_cuda_hubert_out_len(int(T), C.byref(L)))
    return int(L.value)


class CudaHubert:
    """Device-resident HuBERT-base encoder on one GPU (one library context)."""

    def __init__(self, sd: dict, device: Optional[int] = None, precision: str = "bf16x3"):
        self.ctx = _lib.get_context(device)
        p = os.environ.get("RVC_CUDA_PRECISION", precision)
        if p not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}")
        self.precision = p
        h = C.c_int64(0)
        check(lib.rvc_cuda_hubert_create(self.ctx.handle, PRECISIONS[p], C.byref(h)))
        self.handle = int(h.value)
        keys = list(HUBERT_KEYS)
        for group in _POS_KEYS:
            if all(k in sd for k in group):
                keys += list(group)
                break
        else:
            raise KeyError("HuBERT weights lack the positional conv (weight_g/weight_v or _pos_conv_weight)")
        self.has_final_proj = "final_proj.weight" in sd and "final_proj.bias" in sd
        if self.has_final_proj:
            keys += ["final_proj.weight", "final_proj.bias"]
        for k in keys:
            t = np.ascontiguousarray(np.asarray(sd[k], dtype=np.float32))
            shape = (C.c_int64 * max(1, t.ndim))(*t.shape)
            check(lib.rvc_cuda_hubert_set_weight(self.handle, k.encode(), fptr(t), shape, t.ndim))
        check(lib.rvc_cuda_hubert_finalize(self.handle))

    @classmethod
    def from_reference(cls, enc, device: Optional[int] = None, precision: str = "bf16x3"):
        """Build from a loaded reference ``HubertEncoder`` (its prepared state dict)."""
        return cls(enc._sd, device=device, precision=precision)

    def close(self):
        if getattr(self, "handle", 0):
            lib.rvc_cuda_hubert_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    # ---------------------------------------------------------------- encode
    def encode_equal(self, xb: np.ndarray, version: int = 2) -> np.ndarray:
        """``xb [B,T]`` equal-length chunks -> ``[B,L,768|256]`` in one call."""
        if version not in (1, 2):
            raise ValueError(f"version must be 1 or 2, got {version}")
        xb = np.ascontiguousarray(xb, dtype=np.float32)
        if xb.ndim != 2:
            raise ValueError(f"batch input must be [B,T], got {xb.shape}")
        B, T = xb.shape
        L = out_len(T)
        if L < 1:
            raise ValueError(f"input of {T} samples is too short for the HuBERT conv stack")
        out = np.empty((B, L, 256 if version == 1 else 768), np.float32)
        check(lib.rvc_cuda_hubert_encode(self.handle, B, T, fptr(xb), version, fptr(out)))
        return out

    def encode_device(self, d_x: int, B: int, T: int, version: int, d_out: int):
        """Device pointers (from this model's context): ``x [B,T]`` -> ``out [B,L,768|256]``,
        asynchronous on the context's stream."""
        check(lib.rvc_cuda_hubert_encode_device(self.handle, int(B), int(T), C.c_void_p(d_x), int(version),
                                                C.c_void_p(d_out)))

    def out_frames(self, T: int) -> int:
        """Feature frames of a ``T``-sample input."""
        return out_len(T)

    def encode(self, x: np.ndarray, version: int = 2) -> np.ndarray:
        """``HubertEncoder.encode``: ``[1,T]`` (or ``[T]``) -> ``[1,L,C]``."""
        if version not in (1, 2):
            raise ValueError(f"version must be 1 or 2, got {version}")
        x = np.asarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None, :]
        if x.ndim != 2 or x.shape[0] != 1:
            raise ValueError(f"input must be [1, T], got {x.shape}")
        return self.encode_equal(x, version)

    def encode_batch(self, xs, version: int = 2) -> list:
        """``HubertEncoder.encode_batch``: list of ``[1,T_i]`` -> list of
        ``[1,L_i,C]``.  Chunks of equal length share one batched call."""
        if version not in (1, 2):
            raise ValueError(f"version must be 1 or 2, got {version}")
        if isinstance(xs, np.ndarray):
            xs = [xs]
        xl = []
        for x in xs:
            x = np.asarray(x, dtype=np.float32)
            if x.ndim == 1:
                x = x[None, :]
            if x.ndim != 2 or x.shape[0] != 1:
                raise ValueError(f"batch input must be [1, T], got {x.shape}")
            xl.append(x)
        out: list = [None] * len(xl)
        by_len: dict = {}
        for i, x in enumerate(xl):
            by_len.setdefault(x.shape[1], []).append(i)
        for _, idx in by_len.items():
            ys = self.encode_equal(np.concatenate([xl[i] for i in idx], axis=0), version)
            for j, i in enumerate(idx):
                out[i] = ys[j:j + 1]
        return out

    # ---------------------------------------------------------------- debug
    def keep_taps(self, on: bool = True):
        check(lib.rvc_cuda_hubert_keep_taps(self.handle, 1 if on else 0))

    def tap(self, name: str, shape) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.float32)
        check(lib.rvc_cuda_hubert_tap(self.handle, name.encode(), fptr(out), out.size))
        return out.reshape(shape)


def patch_reference(hubert_module=None, device: Optional[int] = None, precision: str = "bf16x3"):
    """Route ``HubertEncoder.encode`` / ``encode_batch`` of the reference through
    ``CudaHubert``.  The class methods are replaced (``runtime/vc.py`` imports
    the loader by name); one device model is cached per encoder instance."""
    if hubert_module is None:
        from runtime.models import hubert as hubert_module  # noqa: PLC0415
    cls = hubert_module.HubertEncoder
    if getattr(cls, "_rvc_cuda_patched", False):
        return cls

    def _model(self):
        m = self.__dict__.get("_rvc_cuda_model")
        if m is None:
            m = CudaHubert.from_reference(self, device=device, precision=precision)
            self.__dict__["_rvc_cuda_model"] = m
        return m

    def encode(self, x, version=2):
        return _model(self).encode(x, version)

    def encode_batch(self, xs, version=2):
        return _model(self).encode_batch(xs, version)

    cls._rvc_cuda_orig_encode = cls.encode
    cls._rvc_cuda_orig_encode_batch = cls.encode_batch
    cls.encode = encode
    cls.encode_batch = encode_batch
    cls._rvc_cuda_patched = True
    return cls
