"""Brute-force feature retrieval on the device (top-k L2 search + blend).

``CudaIndex`` holds an index ``[N,D]`` in device memory and serves the
reference's ``runtime.retrieval.search_l2`` contract (``runtime/retrieval.py:35-82``):
``(scores [F,k'] f32 ascending, indices [F,k'] i64)``, ``k' = min(k, N)``.
The distances come from a tensor-core GEMM; the k + 8 best candidates of each
query are then re-ranked with the exact float64 distance, so the returned
order does not depend on the GEMM's rounding (equal distances keep the lower
index first).  ``blend`` runs the pipeline's inverse-squared-distance blend
and mix (``runtime/pipeline.py:545-551``, ``:563-566``) on the device too.

With ``set_ivf`` the index also serves the inverted-file mode of
``runtime/ivf_index.py`` (``IVFIndex``): ``ivf_search`` is the pipeline's
strict per-row bucket search ``_ivf_strict_search``
(``runtime/pipeline.py:66-161``) and ``ivf_blend`` its blend
(``:523-527``): nearest centroids from the same exact search over the
centroids, then a bucket scan with exact float64 distances.

``search_l2`` / ``weighted_blend`` / ``ivf_strict_search`` here are drop-ins
for the reference functions: they keep one device index per index array
(recognised by its buffer, shape and a sample of its rows).
``patch_reference`` installs them in ``runtime.retrieval`` and
``runtime.pipeline``.
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

__all__ = ["CudaIndex", "search_l2", "weighted_blend", "ivf_strict_search", "patch_reference", "MAX_K"]

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
        self.nlist = 0
        self.nprobe = 1

    @classmethod
    def from_ivf(cls, ivf, device: Optional[int] = None, precision: str = "bf16x3"):
        """Device copy of an ``IVFIndex`` (``runtime/ivf_index.py:121``): its
        vectors, centroids, bucket assignments and default nprobe."""
        m = cls(np.asarray(ivf._vectors, dtype=np.float32), device=device, precision=precision)
        m.set_ivf(ivf.centroids, ivf._assignments, nprobe=getattr(ivf, "nprobe", 1) or 1)
        return m

    def set_ivf(self, centroids, assignments, nprobe: int = 1):
        """Inverted-file structure: ``centroids [nlist, D]`` and the bucket of
        every row, ``assignments [N]`` in ``[0, nlist)``."""
        c = np.ascontiguousarray(np.asarray(centroids, dtype=np.float32))
        a = np.ascontiguousarray(np.asarray(assignments, dtype=np.int64).reshape(-1))
        if c.ndim != 2 or c.shape[1] != self.D or c.shape[0] < 1:
            raise ValueError(f"centroids must be [nlist, {self.D}], got {c.shape}")
        if a.size != self.N:
            raise ValueError(f"assignments must hold {self.N} buckets, got {a.size}")
        check(lib.rvc_cuda_index_set_ivf(self.handle, fptr(c), c.shape[0], iptr(a)))
        self.nlist, self.nprobe = int(c.shape[0]), int(nprobe)

    def _nprobe(self, nprobe):
        if not self.nlist:
            raise ValueError("the index has no IVF structure (set_ivf first)")
        n = self.nprobe if nprobe is None else int(nprobe)
        if n < 1:
            raise ValueError("nprobe must be >= 1")
        return n

    def ivf_search(self, query, k: int = 8, nprobe: Optional[int] = None):
        """``_ivf_strict_search``: ``(scores [F,k], indices [F,k])``, inf / -1 past
        the rows of the probed buckets."""
        q = self._query(query)
        n = self._nprobe(nprobe)
        if not 1 <= int(k) <= MAX_K:
            raise ValueError(f"k must be in [1, {MAX_K}], got {k}")
        F = q.shape[0]
        scores = np.empty((F, int(k)), np.float32)
        inds = np.empty((F, int(k)), np.int64)
        if F:
            check(lib.rvc_cuda_index_ivf_search(self.handle, fptr(q), F, self.D, int(k), n, fptr(scores), iptr(inds)))
        return scores, inds

    def ivf_blend(self, query, k: int = 8, nprobe: Optional[int] = None, feats=None, index_rate: float = 1.0):
        """The pipeline's blend over ``ivf_search`` (``w = (1/score)^2``
        row-normalised), mixed as ``blend * index_rate + feats * (1 - index_rate)``
        when ``feats`` is given."""
        q = self._query(query)
        n = self._nprobe(nprobe)
        F = q.shape[0]
        out = np.empty((F, self.D), np.float32)
        f = None
        if feats is not None:
            f = np.ascontiguousarray(np.asarray(feats, dtype=np.float32).reshape(F, self.D))
        if F:
            check(lib.rvc_cuda_index_ivf_blend(self.handle, fptr(q), F, self.D, int(k), n, float(index_rate),
                                               fptr(f) if f is not None else None, fptr(out)))
        return out

    def blend_device(self, d_q: int, F: int, d_feats: int, index_rate: float, d_out: int, k: int = 8,
                     ivf: Optional[bool] = None, nprobe: Optional[int] = None):
        """The pipeline's blend + mix on device pointers (this index's context):
        ``q [F,D]``, ``feats [F,D]`` -> ``out [F,D]``; IVF search when the index
        has the structure (or ``ivf``), else brute force.  Asynchronous."""
        use_ivf = bool(self.nlist) if ivf is None else ivf
        if use_ivf:
            check(lib.rvc_cuda_index_ivf_blend_device(self.handle, C.c_void_p(d_q), int(F), self.D, int(k),
                                                      self._nprobe(nprobe), float(index_rate), C.c_void_p(d_feats),
                                                      C.c_void_p(d_out)))
        else:
            check(lib.rvc_cuda_index_blend_device(self.handle, C.c_void_p(d_q), int(F), self.D, int(k),
                                                  BLEND_MODES["pipeline"], float(index_rate), C.c_void_p(d_feats),
                                                  C.c_void_p(d_out)))

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


def _ivf_for(ivf) -> CudaIndex:
    vecs = np.asarray(ivf._vectors, dtype=np.float32)
    cen = np.asarray(ivf.centroids, dtype=np.float32)
    asg = np.asarray(ivf._assignments)
    key = ("ivf",) + _fingerprint(vecs) + (hashlib.sha1(cen.tobytes()).hexdigest(),
                                           hashlib.sha1(np.ascontiguousarray(asg).tobytes()).hexdigest())
    m = _cache.get(key)
    if m is None:
        m = CudaIndex(vecs)
        m.set_ivf(cen, asg, nprobe=getattr(ivf, "nprobe", 1) or 1)
        _cache[key] = m
        while len(_cache) > _CACHE_MAX:
            _cache.popitem(last=False)
    else:
        _cache.move_to_end(key)
    return m


def ivf_strict_search(index, query, k: int = 8, nprobe=None):
    """Drop-in for ``runtime.pipeline._ivf_strict_search`` (``runtime/pipeline.py:66-161``)
    with ``index`` an ``IVFIndex``: the same guards (IP metric refused, empty
    query, no IVF structure -> brute-force search), the search on the device."""
    if str(getattr(index, "metric", "L2")).upper() == "IP":
        raise NotImplementedError("retrieval with an inner-product (IP) index is not supported: the blend "
                                  "weights (1/score)^2 assume L2 distances")
    q = np.asarray(query, dtype=np.float32)
    if nprobe is None:
        nprobe = getattr(index, "nprobe", 1) or 1
    F = q.shape[0]
    if F == 0:
        return np.empty((0, k), dtype=np.float32), np.empty((0, k), dtype=np.int64)
    centroids = getattr(index, "centroids", None)
    vecs = np.asarray(getattr(index, "_vectors", None), dtype=np.float32)
    if centroids is None or np.asarray(centroids).shape[0] == 0 or getattr(index, "buckets", None) is None:
        return search_l2(q, vecs, k=k)
    return _ivf_for(index).ivf_search(q, k, nprobe)


def search_l2(query, db, k: int = 8, chunk: int = 4096):
    """Drop-in for ``runtime.retrieval.search_l2`` (``chunk`` is accepted and
    ignored: the device search is not chunked by index rows)."""
    return _index_for(db).search(query, k)


def weighted_blend(query, db, k: int = 8):
    """Drop-in for ``runtime.retrieval.weighted_blend`` (``runtime/retrieval.py:85-108``)."""
    return _index_for(db).blend(query, k, mode="weighted")


def patch_reference(retrieval_module=None, pipeline_module=None):
    """Route the reference's searches through the device index:
    ``runtime.retrieval.search_l2`` / ``weighted_blend`` (``FeatureIndex.search``
    looks ``search_l2`` up in that module), ``runtime.pipeline.search_l2``
    (imported there by name, ``runtime/pipeline.py:44``) and the IVF search
    ``runtime.pipeline._ivf_strict_search``."""
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
        if hasattr(mod, "_ivf_strict_search"):
            mod._rvc_cuda_orig_ivf_strict_search = mod._ivf_strict_search
            mod._ivf_strict_search = ivf_strict_search
        mod._rvc_cuda_patched_retrieval = True
    return retrieval_module
