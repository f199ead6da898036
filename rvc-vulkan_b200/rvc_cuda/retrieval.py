"""Brute-force feature retrieval on the device (top-k L2 search + blend).

``CudaIndex`` holds an index ``[N,D]`` in device memory and serves the
reference's ``runtime.retrieval.search_l2`` contract (``runtime/retrieval.py:35-82``):
``(scores [F,k'] f32 ascending, indices [F,k'] i64)``, ``k' = min(k, N)``.
The distances come from a tensor-core GEMM; the k + 8 best candidates of each
query are then re-ranked with the exact float64 distance, so the returned
order does not depend on the GEMM's rounding (equal distances keep the lower
index first).  ``blend`` runs the pipeline's inverse-squared-distance blend
and mix (``runtime/pipeline.py:545-551``, ``:563-566``) on the device too.

``search_l2`` / ``weighted_blend`` here are drop-ins for the reference
functions: they keep one device index per index array (recognised by its
buffer, shape and a sample of its rows).  ``patch_reference`` installs them
in ``runtime.retrieval`` and ``runtime.pipeline``.
"""

from __future__ import annotations

import ctypes as C
import hashlib
import os
from collections import OrderedDict
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, fptr, iptr, lib

__all__ = ["CudaIndex", "search_l2", "weighted_blend", "patch_reference", "MAX_K"]

PRECISIONS = {"bf16x3": 0, "simt": 1}
MAX_K = 16
BLEND_MODES = {"pipeline": 0, "weighted": 1}


class CudaIndex:
    """Device-resident index ``[N,D]`` float32 on one GPU."""

    def __init__(self, db, device: Optional[int] = None, precision: str = "bf16x3"):
        db = np.ascontiguousarray(np.asarray(db, dtype=np.float32))
        if db.ndim != 2 or db.shape[0] < 1 or db.shape[1] < 1:
            raise ValueError(f"index must be a non-empty [N, D] array, got {db.shape}")
        p = os.environ.get("RVC_CUDA_PRECISION", precision)
        if p not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}")
        self.ctx = _lib.get_context(device)
        self.N, self.D = (int(s) for s in db.shape)
        h = C.c_int64(0)
        check(lib.rvc_cuda_index_create(self.ctx.handle, fptr(db), self.N, self.D, PRECISIONS[p], C.byref(h)))
        self.handle = int(h.value)

    def close(self):
        if getattr(self, "handle", 0):
            lib.rvc_cuda_index_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def _query(self, query) -> np.ndarray:
        q = np.ascontiguousarray(np.asarray(query, dtype=np.float32))
        if q.ndim != 2 or q.shape[1] != self.D:
            raise ValueError(f"queries must be [F, {self.D}], got {q.shape}")
        return q

    def search(self, query, k: int = 8):
        """``search_l2`` on this index: ``(scores [F,k'], indices [F,k'])``."""
        q = self._query(query)
        if not 1 <= int(k) <= MAX_K:
            raise ValueError(f"k must be in [1, {MAX_K}], got {k}")
        kk = min(int(k), self.N)
        F = q.shape[0]
        scores = np.empty((F, kk), np.float32)
        inds = np.empty((F, kk), np.int64)
        if F:
            check(lib.rvc_cuda_index_search(self.handle, fptr(q), F, self.D, int(k), fptr(scores), iptr(inds)))
        return scores, inds

    def blend(self, query, k: int = 8, mode: str = "pipeline", feats=None, index_rate: float = 1.0):
        """Retrieved-feature blend: ``sum_j w_j db[idx_j]`` with ``w = (1/score)^2``
        row-normalised (``mode="pipeline"``) or ``1/max(score,1e-6)^2``
        (``mode="weighted"``, ``weighted_blend``); with ``feats`` the result is
        ``blend * index_rate + feats * (1 - index_rate)``."""
        q = self._query(query)
        if mode not in BLEND_MODES:
            raise ValueError(f"mode must be one of {sorted(BLEND_MODES)}")
        if not 1 <= int(k) <= MAX_K:
            raise ValueError(f"k must be in [1, {MAX_K}], got {k}")
        F = q.shape[0]
        out = np.empty((F, self.D), np.float32)
        f = None
        if feats is not None:
            f = np.ascontiguousarray(np.asarray(feats, dtype=np.float32).reshape(F, self.D))
        if F:
            check(lib.rvc_cuda_index_blend(self.handle, fptr(q), F, self.D, int(k), BLEND_MODES[mode],
                                           float(index_rate), fptr(f) if f is not None else None, fptr(out)))
        return out


_cache: "OrderedDict[tuple, CudaIndex]" = OrderedDict()
_CACHE_MAX = 4


def _fingerprint(db: np.ndarray) -> tuple:
    n = db.shape[0]
    step = max(1, n // 64)
    h = hashlib.sha1(np.ascontiguousarray(db[::step]).tobytes()).hexdigest()
    return (db.__array_interface__["data"][0], db.shape, db.strides, h)


def _index_for(db) -> CudaIndex:
    db = np.asarray(db, dtype=np.float32)
    key = _fingerprint(db)
    m = _cache.get(key)
    if m is None:
        m = CudaIndex(db)
        _cache[key] = m
        while len(_cache) > _CACHE_MAX:
            _cache.popitem(last=False)
    else:
        _cache.move_to_end(key)
    return m


def search_l2(query, db, k: int = 8, chunk: int = 4096):
    """Drop-in for ``runtime.retrieval.search_l2`` (``chunk`` is accepted and
    ignored: the device search is not chunked by index rows)."""
    return _index_for(db).search(query, k)


def weighted_blend(query, db, k: int = 8):
    """Drop-in for ``runtime.retrieval.weighted_blend`` (``runtime/retrieval.py:85-108``)."""
    return _index_for(db).blend(query, k, mode="weighted")


def patch_reference(retrieval_module=None, pipeline_module=None):
    """Route the reference's brute-force search through the device index:
    ``runtime.retrieval.search_l2`` / ``weighted_blend`` (``FeatureIndex.search``
    looks ``search_l2`` up in that module) and ``runtime.pipeline.search_l2``
    (imported there by name, ``runtime/pipeline.py:44``)."""
    if retrieval_module is None:
        from runtime import retrieval as retrieval_module  # noqa: PLC0415
    if pipeline_module is None:
        try:
            from runtime import pipeline as pipeline_module  # noqa: PLC0415
        except Exception:  # noqa: BLE001 - pipeline needs scipy; retrieval alone still patches
            pipeline_module = None
    for mod in (retrieval_module, pipeline_module):
        if mod is None or getattr(mod, "_rvc_cuda_patched_retrieval", False):
            continue
        if hasattr(mod, "search_l2"):
            mod._rvc_cuda_orig_search_l2 = mod.search_l2
            mod.search_l2 = search_l2
        if hasattr(mod, "weighted_blend"):
            mod._rvc_cuda_orig_weighted_blend = mod.weighted_blend
            mod.weighted_blend = weighted_blend
        mod._rvc_cuda_patched_retrieval = True
    return retrieval_module
