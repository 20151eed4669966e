"""Numpy restatement of the reference GraphKVCache (cluster-routed L2 tier).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each method cites the reference function it restates (``graph_cache.py`` of
the ``inference`` package).  The three regions are kept like the reference:
sinks (filled by absolute position), a recent ring, and ``n_clusters``
clusters of ``cluster_capacity`` slots, each with an online mean of its
tokens' layer-0 / head-0 keys as centroid.

Floating point.  Centroid updates are elementwise float32 operations, rounded
one at a time as torch does them (``(c * n + k) / (n + 1)`` and
``(c * n - k) / (n - 1)``), so they are exact.  Cosine similarities are
reductions whose order torch leaves open; this restatement sums in float64,
and the fixtures it is checked against are generated with every routing and
retrieval decision clear of its threshold or runner-up by a margin far above
float32 rounding, so any reduction order decides the same way.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import numpy as np


@dataclass
class ClusterGeometry:
    """Restates ``ClusterConfig`` (graph_cache.py:72-94)."""
    num_layers: int
    num_kv_heads: int
    head_dim: int
    n_clusters: int = 16
    cluster_capacity: int = 32
    sim_threshold: float = 0.3
    sink_size: int = 4
    recent_size: int = 128

    @property
    def cluster_budget(self) -> int:
        return self.n_clusters * self.cluster_capacity

    @property
    def total_budget(self) -> int:
        return self.sink_size + self.recent_size + self.cluster_budget


def cos_sim(q: np.ndarray, centroid: np.ndarray, count: int) -> float:
    """``_Cluster.cos_sim_to_query`` (graph_cache.py:136-144): -1 for an empty
    cluster, else the cosine of q and the centroid (norms clamped at 1e-6)."""
    if count == 0:
        return -1.0
    q = q.astype(np.float64)
    c = centroid.astype(np.float64)
    qs = max(float(np.sqrt((q * q).sum())), 1e-6)
    cs = max(float(np.sqrt((c * c).sum())), 1e-6)
    return float((q / qs * c / cs).sum())


class GraphOracle:
    """``GraphKVCache`` (graph_cache.py:218-495) over numpy arrays.

    K/V are ``[L, H, slots, D]`` in the cache dtype for each region;
    positions are int64 (-1 empty); cluster scores float32; centroids
    float32 ``[n_clusters, D]``."""

    def __init__(self, g: ClusterGeometry, dtype=np.float16):
        self.g, self.dtype = g, dtype
        L, H, D = g.num_layers, g.num_kv_heads, g.head_dim
        self.sink_k = np.zeros((L, H, g.sink_size, D), dtype)
        self.sink_v = np.zeros_like(self.sink_k)
        self.sink_pos = np.full(g.sink_size, -1, np.int64)
        self.sink_fill = 0
        self.rec_k = np.zeros((L, H, g.recent_size, D), dtype)
        self.rec_v = np.zeros_like(self.rec_k)
        self.rec_pos = np.full(g.recent_size, -1, np.int64)
        self.rec_ptr = 0
        self.rec_fill = 0
        C, cap = g.n_clusters, g.cluster_capacity
        self.cl_k = np.zeros((C, L, H, cap, D), dtype)
        self.cl_v = np.zeros_like(self.cl_k)
        self.cl_pos = np.full((C, cap), -1, np.int64)
        self.cl_score = np.zeros((C, cap), np.float32)
        self.cl_fill = np.zeros(C, np.int64)
        self.centroid = np.zeros((C, D), np.float32)
        self.c_count = np.zeros(C, np.int64)
        self.decisions: List[Tuple[int, int, int]] = []  # (position, cluster, evicted slot or -1)

    # graph_cache.py:146-186
    def _cluster_insert(self, c: int, k_tok: np.ndarray, v_tok: np.ndarray, position: int, score: float) -> int:
        cap = self.g.cluster_capacity
        evicted = -1
        if self.cl_fill[c] >= cap:
            fill = int(self.cl_fill[c])
            evicted = int(np.argmin(self.cl_score[c, :fill]))  # first index of the minimum
            old_key = self.cl_k[c, 0, 0, evicted].astype(np.float32)
            n = np.float32(self.c_count[c])
            if self.c_count[c] > 1:
                self.centroid[c] = (self.centroid[c] * n - old_key) / np.float32(n - 1)
                self.c_count[c] -= 1
            else:
                self.centroid[c] = 0
                self.c_count[c] = 0
            slot = evicted
        else:
            slot = int(self.cl_fill[c])
            self.cl_fill[c] += 1
        self.cl_k[c, :, :, slot] = k_tok.astype(self.dtype)
        self.cl_v[c, :, :, slot] = v_tok.astype(self.dtype)
        self.cl_pos[c, slot] = position
        self.cl_score[c, slot] = np.float32(score)
        new_key = self.cl_k[c, 0, 0, slot].astype(np.float32)
        n = np.float32(self.c_count[c])
        self.centroid[c] = (self.centroid[c] * n + new_key) / np.float32(n + 1)
        self.c_count[c] += 1
        return evicted

    # graph_cache.py:325-361
    def route(self, key00: np.ndarray) -> int:
        """Cluster for a displaced token whose layer-0 / head-0 key is key00."""
        g = self.g
        best_i, best_sim = -1, -2.0
        for i in range(g.n_clusters):
            sim = cos_sim(key00, self.centroid[i], int(self.c_count[i]))
            if sim > best_sim:
                best_sim, best_i = sim, i
        if best_sim < g.sim_threshold:
            empty = [i for i in range(g.n_clusters) if self.cl_fill[i] == 0]
            if empty:
                best_i = empty[0]
            else:
                best_i = int(min(range(g.n_clusters), key=lambda i: self.cl_fill[i]))
        return best_i

    def route_margin(self, key00: np.ndarray) -> float:
        """Distance of this routing decision from a tie or the threshold."""
        sims = sorted((cos_sim(key00, self.centroid[i], int(self.c_count[i])) for i in range(self.g.n_clusters)),
                      reverse=True)
        m = abs(sims[0] - self.g.sim_threshold)
        if len(sims) > 1 and sims[1] > -1.0:
            m = min(m, sims[0] - sims[1])
        return m

    # graph_cache.py:287-323
    def push(self, k_tok: np.ndarray, v_tok: np.ndarray, position: int, score: float = 0.0) -> None:
        """k_tok, v_tok: [L, H, D]."""
        g = self.g
        if position < g.sink_size and self.sink_fill < g.sink_size:
            s = self.sink_fill
            self.sink_k[:, :, s] = k_tok.astype(self.dtype)
            self.sink_v[:, :, s] = v_tok.astype(self.dtype)
            self.sink_pos[s] = position
            self.sink_fill += 1
            return
        ptr = self.rec_ptr
        if self.rec_pos[ptr] >= 0:
            old_k = self.rec_k[:, :, ptr].copy()
            old_v = self.rec_v[:, :, ptr].copy()
            old_pos = int(self.rec_pos[ptr])
            c = self.route(old_k[0, 0].astype(np.float32))
            ev = self._cluster_insert(c, old_k, old_v, old_pos, score)  # the current token's score
            self.decisions.append((old_pos, c, ev))
        self.rec_k[:, :, ptr] = k_tok.astype(self.dtype)
        self.rec_v[:, :, ptr] = v_tok.astype(self.dtype)
        self.rec_pos[ptr] = position
        self.rec_fill = min(self.rec_fill + 1, g.recent_size)
        self.rec_ptr = (ptr + 1) % g.recent_size

    # graph_cache.py:442-467
    def load_from_summary(self, k: np.ndarray, v: np.ndarray, scores: np.ndarray,
                          positions: Optional[np.ndarray] = None) -> None:
        """k, v: [L, H, T, D]; scores [T]."""
        self.__init__(self.g, self.dtype)
        T = k.shape[2]
        pos = np.arange(T) if positions is None else positions
        for t in range(T):
            self.push(k[:, :, t], v[:, :, t], int(pos[t]), float(scores[t]))

    # graph_cache.py:363-440
    def select(self, query_key: np.ndarray, threshold: Optional[float] = None,
               top_n: Optional[int] = None) -> np.ndarray:
        """Clusters retrieve() uses for query_key [H, D]."""
        g = self.g
        thresh = g.sim_threshold if threshold is None else threshold
        qm = query_key.astype(np.float32).mean(axis=0)
        sims = np.array([cos_sim(qm, self.centroid[i], int(self.c_count[i])) for i in range(g.n_clusters)])
        sel = np.zeros(g.n_clusters, bool)
        if top_n is not None:
            order = np.argsort(-sims, kind="stable")[:min(top_n, g.n_clusters)]
            sel[order] = True
        else:
            sel = sims >= thresh
            if not sel.any():
                sel[int(np.argmax(sims))] = True
        return sel

    def retrieve_positions(self, selected: np.ndarray) -> np.ndarray:
        """Token positions in the order retrieve() concatenates them: sinks in
        slot order, the recent ring by position, then each selected non-empty
        cluster by position."""
        parts = [self.sink_pos[:self.sink_fill]]
        rp = self.rec_pos[:self.rec_fill]
        parts.append(np.sort(rp))
        for i in range(self.g.n_clusters):
            if selected[i] and self.cl_fill[i] > 0:
                parts.append(np.sort(self.cl_pos[i, :self.cl_fill[i]]))
        return np.concatenate(parts) if parts else np.zeros(0, np.int64)

    def retrieve(self, query_key: np.ndarray, threshold: Optional[float] = None,
                 top_n: Optional[int] = None):
        """(per-layer (K, V) [H, F, D] lists, selected) like retrieve()."""
        sel = self.select(query_key, threshold, top_n)
        L = self.g.num_layers
        ks, vs = [], []
        for li in range(L):
            ro = np.argsort(self.rec_pos[:self.rec_fill])
            pk = [self.sink_k[li][:, :self.sink_fill], self.rec_k[li][:, ro]]
            pv = [self.sink_v[li][:, :self.sink_fill], self.rec_v[li][:, ro]]
            for i in range(self.g.n_clusters):
                if sel[i] and self.cl_fill[i] > 0:
                    o = np.argsort(self.cl_pos[i, :self.cl_fill[i]])
                    pk.append(self.cl_k[i, li][:, o])
                    pv.append(self.cl_v[i, li][:, o])
            ks.append(np.concatenate(pk, axis=1))
            vs.append(np.concatenate(pv, axis=1))
        return ks, vs, sel
