"""Oracle for brute-force feature retrieval (top-k L2 search + blend).

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``).  A numpy restatement of the
reference's ``runtime.retrieval.search_l2`` (``runtime/retrieval.py:35-82``)
and of the pipeline's inverse-squared-distance blend
(``runtime/pipeline.py:545-551``, mixed into the features at ``:563-566``).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def search_l2(query, db, k=8, chunk=4096):
    """``||q||^2 + ||d||^2 - 2 q.d`` clamped at 0, the k smallest per query in
    ascending order, merged chunk by chunk (``runtime/retrieval.py:35-82``).
    Returns ``(scores [F,k'] f32, indices [F,k'] i64)`` with ``k' = min(k, N)``."""
    query = np.asarray(query, dtype=F32)
    db = np.asarray(db, dtype=F32)
    F = query.shape[0]
    N = db.shape[0]
    k = min(k, N)
    q2 = np.einsum("fd,fd->f", query, query)
    d2 = np.einsum("nd,nd->n", db, db)
    scores = np.full((F, k), np.inf, dtype=F32)
    inds = np.full((F, k), -1, dtype=np.int64)
    rows = np.arange(F)[:, None]
    for s in range(0, N, chunk):
        e = min(s + chunk, N)
        dist = q2[:, None] + d2[None, s:e] - 2.0 * (query @ db[s:e].T)
        np.maximum(dist, 0.0, out=dist)
        kb = min(k, e - s)
        part = np.argpartition(dist, kb - 1, axis=1)[:, :kb]
        ps = np.take_along_axis(dist, part, axis=1)
        o = np.argsort(ps, axis=1)
        part = np.take_along_axis(part, o, axis=1) + s
        ps = np.take_along_axis(ps, o, axis=1)
        merged = np.concatenate([scores, ps], axis=1)
        merged_i = np.concatenate([inds, part], axis=1)
        keep = np.argpartition(merged, k - 1, axis=1)[:, :k]
        keep = keep[rows, np.argsort(merged[rows, keep], axis=1)]
        scores = merged[rows, keep]
        inds = merged_i[rows, keep]
    return scores, inds


def blend(query, db, k=8):
    """Pipeline blend (``runtime/pipeline.py:545-551``): ``w = (1/score)^2``
    row-normalised (sum floored at 1e-12), ``sum_j w_j db[idx_j]``."""
    db = np.asarray(db, dtype=F32)
    sc, ix = search_l2(query, db, k=k)
    blk = db[ix]
    w = np.square(1.0 / sc)
    w /= np.maximum(w.sum(axis=1, keepdims=True), 1e-12)
    return np.sum(blk * w[:, :, None], axis=1)


def mix(feats, blended, index_rate):
    """``blend * index_rate + feats * (1 - index_rate)`` (``runtime/pipeline.py:563-566``)."""
    return blended * index_rate + np.asarray(feats, dtype=F32) * (1 - index_rate)
