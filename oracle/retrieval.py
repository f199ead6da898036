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


def ivf_buckets(assignments, nlist):
    """Row ids per bucket, stable (``IVFIndex._rebuild_buckets``,
    ``runtime/ivf_index.py:272-284``)."""
    a = np.asarray(assignments, dtype=np.int64)
    order = np.argsort(a, kind="stable")
    counts = np.bincount(a, minlength=nlist)
    return [b.astype(np.int64, copy=False) for b in np.split(order, np.cumsum(counts)[:-1])]


def ivf_strict_search(centroids, vecs, buckets, query, k=8, nprobe=1):
    """``_ivf_strict_search`` (``runtime/pipeline.py:66-161``): per query row
    the ``nprobe`` nearest centroids (fp32 ``q2 + c2 - 2 q.c``, clamped at 0;
    ``argmin`` for one probe, ``argpartition`` otherwise), then the k nearest
    rows of the union of those buckets (fp32 distances), padded with inf / -1."""
    query = np.asarray(query, dtype=F32)
    centroids = np.asarray(centroids, dtype=F32)
    vecs = np.asarray(vecs, dtype=F32)
    F = query.shape[0]
    q2 = np.einsum("fd,fd->f", query, query)
    c2 = np.einsum("nd,nd->n", centroids, centroids)
    dist = q2[:, None] + c2[None, :] - 2.0 * (query @ centroids.T)
    np.maximum(dist, 0.0, out=dist)
    nprobe = min(nprobe, centroids.shape[0])
    scores = np.full((F, k), np.inf, dtype=F32)
    inds = np.full((F, k), -1, dtype=np.int64)
    if nprobe == 1:
        top = np.argmin(dist, axis=1)
        d2 = np.einsum("nd,nd->n", vecs, vecs)
        for f in range(F):
            cand = buckets[top[f]]
            if cand.size == 0:
                continue
            kk = min(k, cand.size)
            d = q2[f] + d2[cand] - 2.0 * (query[f] @ vecs[cand].T)
            np.maximum(d, 0.0, out=d)
            if kk >= cand.size:
                order = np.argsort(d)
            else:
                p = np.argpartition(d, kk - 1)[:kk]
                order = p[np.argsort(d[p])]
            inds[f, :kk] = cand[order]
            scores[f, :kk] = d[order]
        return scores, inds
    top = np.argpartition(dist, nprobe - 1, axis=1)[:, :nprobe]
    for f in range(F):
        cand = np.concatenate([buckets[b] for b in top[f] if buckets[b].size] or [np.zeros(0, np.int64)])
        if cand.size == 0:
            continue
        s, ix = search_l2(query[f:f + 1], vecs[cand], k=min(k, cand.size))
        inds[f, :ix.shape[1]] = cand[ix[0]]
        scores[f, :s.shape[1]] = s[0]
    return scores, inds


def ivf_blend(vecs, scores, inds):
    """The pipeline's IVF blend (``runtime/pipeline.py:523-527``): rows by
    index (zero vectors for -1, ``IVFIndex.vectors_by_rows``), ``w = (1/score)^2``
    row-normalised, weighted sum."""
    vecs = np.asarray(vecs, dtype=F32)
    flat = inds.reshape(-1)
    blk = np.zeros((flat.size, vecs.shape[1]), dtype=F32)
    ok = flat >= 0
    blk[ok] = vecs[flat[ok]]
    blk = blk.reshape(inds.shape + (vecs.shape[1],))
    w = np.square(1.0 / scores)
    w /= np.maximum(w.sum(axis=1, keepdims=True), 1e-12)
    return np.sum(blk * w[:, :, None], axis=1)
