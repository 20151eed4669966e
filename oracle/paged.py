"""PagePool / KVAllocator / PagedSessionView / MultiSessionCache on the CPU.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates paged_cache.py:99-454 with numpy storage.  The one deliberate
difference: LRU time stamps come from a logical clock (one tick per
``allocate_page`` / ``touch``) instead of ``time.monotonic`` so that the
eviction order depends on call order alone.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np

PAGE_SIZE = 16


class OraclePagePool:
    """paged_cache.py:99-200: K/V [L, H, n_pages * 16, D]."""

    def __init__(self, n_pages, n_layers, n_heads, head_dim, dtype=np.float32, max_pps=64):
        self.n_pages = n_pages
        self.max_pps = max_pps
        shape = (n_layers, n_heads, n_pages * PAGE_SIZE, head_dim)
        self.K = np.zeros(shape, dtype)
        self.V = np.zeros(shape, dtype)

    def write_token(self, layer, page_id, slot, k_vec, v_vec):
        a = page_id * PAGE_SIZE + slot
        self.K[layer, :, a, :] = k_vec
        self.V[layer, :, a, :] = v_vec

    def gather_session(self, layer, page_ids: List[int], n_tokens: int):
        if not page_ids:
            e = np.zeros((self.K.shape[1], 0, self.K.shape[3]), self.K.dtype)
            return e, e
        idx = np.concatenate([np.arange(p * PAGE_SIZE, (p + 1) * PAGE_SIZE) for p in page_ids])
        idx = idx[:n_tokens]
        return self.K[layer][:, idx, :], self.V[layer][:, idx, :]


class OracleAllocator:
    """paged_cache.py:205-288 (LIFO free list, LRU session eviction)."""

    def __init__(self, n_pages, max_pps):
        self.max_pps = max_pps
        self.free: List[int] = list(range(n_pages))
        self.pages: Dict[str, List[int]] = {}
        self.atime: Dict[str, float] = {}
        self.ntok: Dict[str, int] = {}
        self.clock = 0.0

    def _tick(self):
        self.clock += 1.0
        return self.clock

    def _release(self, sid):
        self.free.extend(self.pages.pop(sid, []))
        self.atime.pop(sid, None)
        self.ntok.pop(sid, None)

    def allocate_page(self, sid) -> int:
        cur = len(self.pages.get(sid, []))
        if cur >= self.max_pps:
            raise RuntimeError(f"Session {sid!r} exceeded max pages ({self.max_pps})")
        if not self.free:
            if not self.pages:
                raise RuntimeError("PagePool exhausted and no sessions to evict")
            lru = min(self.atime, key=self.atime.__getitem__)
            self._release(lru)
        p = self.free.pop()
        self.pages.setdefault(sid, []).append(p)
        self.atime[sid] = self._tick()
        return p

    def touch(self, sid):
        if sid in self.atime:
            self.atime[sid] = self._tick()

    def utilization(self):
        used = sum(len(v) for v in self.pages.values())
        n = used + len(self.free)
        return used / n if n else 0.0


class OracleSessionView:
    """paged_cache.py:293-396 (append-only per-session page list)."""

    def __init__(self, sid, pool: OraclePagePool, alloc: OracleAllocator):
        self.sid, self.pool, self.alloc = sid, pool, alloc
        self.pages: List[int] = []
        self.n_tokens = 0
        self.importance: List[float] = []
        self.positions: List[int] = []

    def push(self, k, v, positions, importance):
        """k, v: [L, H, T, D]."""
        L = k.shape[0]
        for t in range(k.shape[2]):
            off = self.n_tokens % PAGE_SIZE
            if off == 0:
                self.pages.append(self.alloc.allocate_page(self.sid))
            page = self.pages[-1]
            for l in range(L):
                self.pool.write_token(l, page, off, k[l, :, t, :], v[l, :, t, :])
            self.n_tokens += 1
            self.positions.append(positions[t] if t < len(positions) else self.n_tokens - 1)
            self.importance.append(importance[t] if t < len(importance) else 0.0)
        self.alloc.ntok[self.sid] = self.n_tokens
        self.alloc.touch(self.sid)

    def gather(self, layer):
        return self.pool.gather_session(layer, self.pages, self.n_tokens)

    def top_importance_tokens(self, top_k):
        pairs = sorted(zip(self.importance, range(len(self.importance))), reverse=True)[:top_k]
        return [i for _, i in pairs], [x for x, _ in pairs]

    def reset(self):
        self.alloc._release(self.sid)
        self.pages, self.n_tokens, self.importance, self.positions = [], 0, [], []


class OracleMultiSession:
    """paged_cache.py:401-454."""

    def __init__(self, pool: OraclePagePool):
        self.pool = pool
        self.alloc = OracleAllocator(pool.n_pages, pool.max_pps)
        self.views: Dict[str, OracleSessionView] = {}

    def get_or_create(self, sid):
        if sid not in self.views:
            self.views[sid] = OracleSessionView(sid, self.pool, self.alloc)
        return self.views[sid]

    def reset(self, sid):
        v = self.views.pop(sid, None)
        if v:
            v.reset()

    def active_sessions(self):
        return list(self.alloc.pages.keys())
