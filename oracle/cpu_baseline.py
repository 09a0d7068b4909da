"""Multithreaded exact CPU brute force: BLAS sgemm + partial selection.

TEST / BASELINE INFRASTRUCTURE ONLY (bench.py's cpu_baseline and
--impl reference legs).  The reference's own search path runs only on Apple
Metal and cannot execute on Linux, so the timed baseline is this CPU port of
its semantics, in the style of the reference's bench harness
(bench/bench.mm:134-156: all host threads, exact brute force), with the GEMM
form the reference uses on the GPU (src/FlatIndex.mm:85-104):
  L2  dist = max(0, ||q||^2 + ||x||^2 - 2 q.x)   (Distance.h:79-81)
  IP  score = q.x
then a per-query bounded top-k ordered by (distance, id): ties go to the
lowest id as in the reference's insertion scan (FlatIndex.mm:94-103).
numpy's matmul is the multithreaded BLAS sgemm (OpenBLAS); the selection of
each database block runs on a thread pool across queries.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

L2, IP = 0, 1


def _topk_rows(score_blk, ids0, k, best_s, best_i):
    """Merge a block of scores (larger = nearer) into running (m, k) lists,
    ordered by (score desc, id asc)."""
    m, nb = score_blk.shape
    kk = min(k, nb)
    part = np.argpartition(-score_blk, kk - 1, axis=1)[:, :kk]
    s = np.take_along_axis(score_blk, part, axis=1)
    kth = s.min(axis=1)
    # argpartition may keep a higher id among scores equal to the kk-th best;
    # redo those (rare) rows exactly so the lowest ids win.
    ties = np.nonzero((score_blk >= kth[:, None]).sum(axis=1) > kk)[0]
    for r in ties:
        idx = np.nonzero(score_blk[r] >= kth[r])[0]
        order = np.lexsort((idx, -score_blk[r, idx]))[:kk]
        part[r] = idx[order]
        s[r] = score_blk[r, part[r]]
    S = np.concatenate([best_s, s], axis=1)
    I = np.concatenate([best_i, part.astype(np.int64) + ids0], axis=1)
    order = np.lexsort((I, -S), axis=1)[:, :k]
    return np.take_along_axis(S, order, axis=1), np.take_along_axis(I, order, axis=1)


def search(db: np.ndarray, q: np.ndarray, k: int, metric: int = L2, block: int = 65536,
           threads: int | None = None, dnorm: np.ndarray | None = None):
    """Exact top-k; returns (ids int32 (m,k), dist float32 (m,k)) nearest-first."""
    threads = threads or os.cpu_count() or 1
    q = np.ascontiguousarray(q, np.float32)
    m = q.shape[0]
    n = db.shape[0]
    qn = np.einsum("ij,ij->i", q, q, dtype=np.float64).astype(np.float32)[:, None]
    if metric == L2 and dnorm is None:
        dnorm = np.einsum("ij,ij->i", db, db, dtype=np.float64).astype(np.float32)
    best_s = np.full((m, k), -np.inf, np.float32)
    best_i = np.full((m, k), -1, np.int64)
    qsplit = np.array_split(np.arange(m), threads)
    with ThreadPoolExecutor(threads) as pool:
        for j0 in range(0, n, block):
            j1 = min(n, j0 + block)
            g = q @ db[j0:j1].T                                   # BLAS sgemm
            if metric == L2:
                s = -np.maximum(0.0, qn + dnorm[j0:j1][None, :] - 2.0 * g)
            else:
                s = g
            s = s.astype(np.float32, copy=False)

            def work(rows, s=s, j0=j0):
                return rows, _topk_rows(s[rows], j0, k, best_s[rows], best_i[rows])

            for rows, (bs, bi) in pool.map(work, [r for r in qsplit if len(r)]):
                best_s[rows], best_i[rows] = bs, bi
    ids = np.where(np.isfinite(best_s), best_i, -1).astype(np.int32)
    dist = (-best_s if metric == L2 else best_s).astype(np.float32)
    return ids, dist
