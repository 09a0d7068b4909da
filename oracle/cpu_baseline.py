"""Multithreaded exact CPU brute force: BLAS sgemm + per-block top-k.

TEST / BASELINE INFRASTRUCTURE ONLY (bench.py's cpu_baseline and
--impl reference legs).  The reference's own search path runs only on Apple
Metal and cannot execute on Linux, so the timed baseline is this CPU port of
its semantics, in the style of the reference's bench harness
(bench/bench.mm:134-156: all host threads, exact brute force), with the GEMM
form the reference uses on the GPU (src/FlatIndex.mm:85-104):
  L2  dist = max(0, ||q||^2 + ||x||^2 - 2 q.x)   (Distance.h:79-81)
  IP  score = q.x
then a per-query top-k ordered by (distance, id): ties go to the lowest id as
in the reference's insertion scan (FlatIndex.mm:94-103).

The work runs on torch's CPU backend with every host thread: one fused GEMM
per database block (addmm: 2 q.x - ||x||^2, a multithreaded MKL/oneDNN sgemm)
and a multithreaded per-row top-(k + 8) of the block, merged into running
lists.  The 8 spare slots keep rows tied at the k-th place so that the final
(distance, id) ordering can give the tie to the lowest id; more than 8 rows
tied exactly at the k-th place would need more (none of the benchmark's
continuous random inputs comes close).
"""
from __future__ import annotations

import os

import numpy as np

L2, IP = 0, 1
SPARE = 8


def _torch(threads):
    import torch
    torch.set_num_threads(threads)
    return torch


class TopK:
    """Running exact top-k of fixed queries over database blocks fed in id order."""

    def __init__(self, q: np.ndarray, k: int, metric: int = L2, threads: int | None = None):
        self.torch = _torch(threads or os.cpu_count() or 1)
        self.q = np.ascontiguousarray(q, np.float32)
        self.qt = self.torch.from_numpy(self.q)
        self.k, self.metric = int(k), metric
        self.kk = self.k + SPARE
        m = self.q.shape[0]
        self.best_s = self.torch.full((m, 0), -float("inf"))
        self.best_i = self.torch.zeros((m, 0), dtype=self.torch.int64)

    def add(self, rows: np.ndarray, id0: int, dnorm: np.ndarray | None = None) -> None:
        torch = self.torch
        rows = np.ascontiguousarray(rows, np.float32)
        nb = rows.shape[0]
        if nb == 0:
            return
        x = torch.from_numpy(rows)
        if self.metric == L2:      # larger = nearer: 2 q.x - ||x||^2 (= ||q||^2 - dist)
            if dnorm is None:
                dnorm = np.einsum("ij,ij->i", rows, rows, dtype=np.float64).astype(np.float32)
            bias = torch.from_numpy(np.ascontiguousarray(dnorm, np.float32))
            s = torch.addmm(bias[None, :], self.qt, x.T, beta=-1.0, alpha=2.0)
        else:
            s = self.qt @ x.T
        v, i = torch.topk(s, min(self.kk, nb), dim=1)
        S = torch.cat([self.best_s, v], dim=1)
        I = torch.cat([self.best_i, i + id0], dim=1)
        if S.shape[1] > self.kk:
            v2, pos = torch.topk(S, self.kk, dim=1)
            self.best_s, self.best_i = v2, torch.gather(I, 1, pos)
        else:
            self.best_s, self.best_i = S, I

    def result(self):
        """(ids int32 (m,k), dist float32 (m,k)) nearest-first, (distance, id) order."""
        k, q = self.k, self.q
        S = self.best_s.numpy().astype(np.float64)
        I = self.best_i.numpy()
        if self.metric == L2:
            qn = np.einsum("ij,ij->i", q, q, dtype=np.float64).astype(np.float32)
            d = np.maximum(0.0, qn[:, None].astype(np.float64) - S).astype(np.float32)
            key = d
        else:
            d = S.astype(np.float32)
            key = -d
        order = np.lexsort((I, key), axis=1)[:, :k]
        ids = np.take_along_axis(I, order, axis=1).astype(np.int32)
        dist = np.take_along_axis(d, order, axis=1)
        pad = k - ids.shape[1]
        if pad > 0:
            ids = np.pad(ids, ((0, 0), (0, pad)), constant_values=-1)
            dist = np.pad(dist, ((0, 0), (0, pad)),
                          constant_values=np.inf if self.metric == L2 else -np.inf)
        return ids, dist


def search(db: np.ndarray, q: np.ndarray, k: int, metric: int = L2, block: int = 65536,
           threads: int | None = None, dnorm: np.ndarray | None = None):
    """Exact top-k; returns (ids int32 (m,k), dist float32 (m,k)) nearest-first."""
    t = TopK(q, k, metric, threads)
    for j0 in range(0, db.shape[0], block):
        j1 = min(db.shape[0], j0 + block)
        t.add(db[j0:j1], j0, None if dnorm is None else dnorm[j0:j1])
    return t.result()


def kmeans_assign(points: np.ndarray, cents: np.ndarray, threads: int | None = None,
                  block: int = 4096) -> np.ndarray:
    """Top-1 L2 assignment (argmin over centroids, lowest index on ties), the
    k-means step of src/Internal.h:321-359 as a BLAS brute force."""
    threads = threads or os.cpu_count() or 1
    torch = _torch(threads)
    points = np.ascontiguousarray(points, np.float32)
    cents = np.ascontiguousarray(cents, np.float32)
    ct = torch.from_numpy(cents)
    cb = torch.from_numpy(np.einsum("ij,ij->i", cents, cents, dtype=np.float64).astype(np.float32))
    out = np.empty(points.shape[0], np.int32)
    for a in range(0, points.shape[0], block):
        z = min(points.shape[0], a + block)
        dd = torch.addmm(cb[None, :], torch.from_numpy(points[a:z]), ct.T, beta=1.0, alpha=-2.0)
        out[a:z] = torch.argmin(dd, dim=1).numpy()
    return out
