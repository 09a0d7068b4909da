"""Exact oracle at the benchmarked sizes (10M-100M rows).

TEST INFRASTRUCTURE ONLY: the checker that tests/ and bench.py's parity leg
use at the configs' full sizes.  The product library never imports it.

The plain oracle (oracle.flat_search_f64, a single-threaded-per-query fp64 scan
in C) needs hours at 10M rows.  The classes here give the SAME answers in
seconds by screening first and proving that the screen lost nothing:

StreamingExact -- exact fp64 top-k (ties to the lowest id) of a fixed query
    set over a database that arrives in row blocks (each rank can feed only the
    rows it holds; merge_pools combines the ranks).  Per block:
      1. screen: S = 2 q.x - ||x||^2 (L2) or q.x (IP) in fp32 through a BLAS
         GEMM (torch on the CPU, all host threads);
      2. every row whose screen score can still reach the running k-th best
         exact score -- S + e >= L_k, e an a-priori bound on |S - exact| --
         is re-scored exactly in fp64 by mfo_score_pairs_f64 (the evaluation
         of mfo_flat_search_f64) and merged into a per-query pool;
      3. L_k = the k-th best exact score in the pool (a row whose upper bound
         is below it cannot enter the top-k: k pool rows are strictly better).
    The bound: |fl(q.x) - q.x| <= gamma_d * sum|q_i x_i| <= gamma_d ||q|| ||x||
    for any summation order (gamma_d = d u / (1 - d u), u = 2^-24), plus the
    rounding of ||x||^2 to fp32 and of the final subtraction; e takes twice
    that sum with X = the block's largest row norm.
    Reference semantics restated: src/Distance.h:26-81 (scores), the tie rule
    of src/FlatIndex.mm:272-281, nearest-first output (:406-418).

kmeans_assign_screened -- mfo_kmeans_assign_f32 (sequential fp32 sqL2,
    strict '<', src/CoarseQuantizer.mm:122-130) for many points against many
    centroids: an fp32 GEMM screen keeps every centroid whose sequential-fp32
    distance can still be the minimum (screen bound e plus the sequential
    sum's own relative error gamma_d), and mfo_kmeans_assign_cand re-runs the
    reference scan over exactly those, in ascending centroid order.

Both are pinned against the plain oracle in tests/test_oracle_scale.py.
"""
from __future__ import annotations

import numpy as np

import oracle as O

U = 2.0 ** -24


def _gamma(d: int) -> float:
    du = d * U
    return du / (1.0 - du)


def _torch():
    import torch
    return torch


def _f32_below(x: np.ndarray) -> np.ndarray:
    """Largest float32 values <= x (x float64; -inf stays -inf)."""
    f = x.astype(np.float32)
    up = f.astype(np.float64) > x
    f[up] = np.nextafter(f[up], np.float32(-np.inf))
    return f


def _f32_above(x: np.ndarray) -> np.ndarray:
    f = x.astype(np.float32)
    dn = f.astype(np.float64) < x
    f[dn] = np.nextafter(f[dn], np.float32(np.inf))
    return f


class StreamingExact:
    """Exact fp64 top-k of `q` over rows fed in blocks with add(rows, id0).

    metric: O.L2 / O.IP / O.COSINE (COSINE normalises queries and rows with
    the reference's normalizeRows, as the index stores them)."""

    def __init__(self, q: np.ndarray, k: int, metric: int = O.L2):
        q = np.ascontiguousarray(q, np.float32)
        if metric == O.COSINE:
            q = O.normalize_rows(q)
        self.metric = metric
        self.q = q
        self.m, self.dim = q.shape
        self.k = int(k)
        self.qn2 = np.einsum("ij,ij->i", q, q, dtype=np.float64)
        self.qnorm = np.sqrt(self.qn2)
        self.pool_id = [np.empty(0, np.int64) for _ in range(self.m)]
        self.pool_s = [np.empty(0, np.float64) for _ in range(self.m)]
        self.L = np.full(self.m, -np.inf)        # k-th best exact score in the pool
        self.rows_seen = 0
        self.rescored = 0
        self._qt = _torch().from_numpy(q)

    def add(self, rows: np.ndarray, id0: int) -> None:
        torch = _torch()
        rows = np.ascontiguousarray(rows, np.float32)
        if self.metric == O.COSINE:
            rows = O.normalize_rows(rows)
        b = rows.shape[0]
        if b == 0:
            return
        self.rows_seen += b
        xn2 = np.einsum("ij,ij->i", rows, rows, dtype=np.float64)
        xmax = float(np.sqrt(xn2.max()))
        g = _gamma(self.dim)
        xt = torch.from_numpy(rows)
        if self.metric == O.L2:
            bias = torch.from_numpy(xn2.astype(np.float32))
            S = torch.addmm(bias[None, :], self._qt, xt.T, beta=-1.0, alpha=2.0)
            # |S - (2 q.x - ||x||^2)| <= 2 g |q||x| + u ||x||^2 + u (2|q||x| + ||x||^2), doubled
            e = 2.0 * ((2 * g + 2 * U) * self.qnorm * xmax + 2 * U * xmax * xmax)
            off = self.qn2                          # exact score = S_exact - ||q||^2
        else:
            S = self._qt @ xt.T
            e = 2.0 * (g + U) * self.qnorm * xmax
            off = np.zeros(self.m)
        e = e + 1e-12 * (np.abs(off) + xmax * xmax + 1.0)
        thr = self.L + off - e                      # keep rows with S >= thr
        short = np.array([len(p) < self.k for p in self.pool_id])
        if short.any() and b >= self.k:
            # queries without k pooled rows yet: the block's own k-th best
            # screen score gives a lower bound (k rows score >= kth - e)
            rows_q = np.nonzero(short)[0]
            kth = torch.topk(S[torch.from_numpy(rows_q)], self.k, dim=1).values[:, -1].double().numpy()
            thr[rows_q] = np.maximum(thr[rows_q], kth - 2.0 * e[rows_q])
        thr32 = torch.from_numpy(_f32_below(thr))
        qi, ji = torch.nonzero(S >= thr32[:, None], as_tuple=True)
        qi = np.ascontiguousarray(qi.numpy(), np.int64)
        ji = np.ascontiguousarray(ji.numpy(), np.int64)
        if qi.size == 0:
            return
        ex = np.empty(qi.size, np.float64)
        O.lib().mfo_score_pairs_f64(rows, self.dim, self.metric, self.q, qi, ji, qi.size, ex)
        self.rescored += qi.size
        cuts = np.nonzero(np.diff(qi))[0] + 1
        for a, z in zip(np.r_[0, cuts], np.r_[cuts, qi.size]):
            r = int(qi[a])
            ids = np.concatenate([self.pool_id[r], ji[a:z] + id0])
            sc = np.concatenate([self.pool_s[r], ex[a:z]])
            if ids.size >= self.k:
                order = np.lexsort((ids, -sc))
                kth = sc[order[self.k - 1]]
                keep = sc >= kth
                ids, sc = ids[keep], sc[keep]
                self.L[r] = kth
            self.pool_id[r], self.pool_s[r] = ids, sc

    def pools(self):
        """Per-query (ids, exact scores) pools, for merging across ranks."""
        return self.pool_id, self.pool_s

    def result(self, pools=None):
        """(ids int32 (m, k), dist float32 (m, k)) nearest-first, like
        oracle.flat_search_f64; `pools` = merge_pools(...) of several ranks."""
        pid, ps = pools if pools is not None else (self.pool_id, self.pool_s)
        ids = np.full((self.m, self.k), -1, np.int32)
        empty = np.inf if self.metric == O.L2 else -np.inf
        dist = np.full((self.m, self.k), empty, np.float32)
        for r in range(self.m):
            if pid[r].size == 0:
                continue
            order = np.lexsort((pid[r], -ps[r]))[: self.k]
            n = order.size
            ids[r, :n] = pid[r][order]
            s = ps[r][order]
            dist[r, :n] = (-s if self.metric == O.L2 else s).astype(np.float32)
        return ids, dist


def merge_pools(pool_list):
    """Concatenate per-rank pools [(ids list, scores list), ...] per query."""
    m = len(pool_list[0][0])
    ids = [np.concatenate([p[0][r] for p in pool_list]) for r in range(m)]
    sc = [np.concatenate([p[1][r] for p in pool_list]) for r in range(m)]
    return ids, sc


def kmeans_assign_screened(points: np.ndarray, cents: np.ndarray, block: int = 4096) -> np.ndarray:
    """oracle.kmeans_assign_f32 at scale (same result, bit for bit)."""
    torch = _torch()
    points = np.ascontiguousarray(points, np.float32)
    cents = np.ascontiguousarray(cents, np.float32)
    n, d = points.shape
    cn2 = np.einsum("ij,ij->i", cents, cents, dtype=np.float64)
    cmax = float(np.sqrt(cn2.max()))
    ct = torch.from_numpy(cents)
    cb = torch.from_numpy(cn2.astype(np.float32))
    g = _gamma(d)
    gs = 1.01 * _gamma(d + 2)      # sequential fp32 sqL2: |seq - exact| <= gs * exact
    out = np.empty(n, np.int32)
    for a in range(0, n, block):
        z = min(n, a + block)
        p = points[a:z]
        pn2 = np.einsum("ij,ij->i", p, p, dtype=np.float64)
        pnorm = np.sqrt(pn2)
        # D = ||c||^2 - 2 p.c  (the point's own ||p||^2 dropped)
        D = torch.addmm(cb[None, :], torch.from_numpy(p), ct.T, beta=1.0, alpha=-2.0)
        e = 2.0 * ((2 * g + 2 * U) * pnorm * cmax + 2 * U * (cmax * cmax + pn2)) + 1e-12 * (pn2 + cmax * cmax + 1.0)
        dmin = D.min(dim=1).values.double().numpy()
        # upper bound of the best exact distance, then of its sequential value;
        # a centroid can win only if its sequential value's lower bound is <= that
        best_ub = np.maximum(dmin + e + pn2, 0.0) * (1.0 + gs)
        lim = best_ub / (1.0 - gs) - pn2 + e
        lim32 = torch.from_numpy(_f32_above(lim))
        qi, ci = torch.nonzero(D <= lim32[:, None], as_tuple=True)
        qi = qi.numpy().astype(np.int64)
        ci = np.ascontiguousarray(ci.numpy(), np.int32)
        ptr = np.zeros(z - a + 1, np.int64)
        np.cumsum(np.bincount(qi, minlength=z - a), out=ptr[1:])
        O.lib().mfo_kmeans_assign_cand(p, z - a, cents, d, ptr, ci, out[a:z])
    return out
