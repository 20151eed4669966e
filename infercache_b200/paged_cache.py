"""Multi-session paged KV pool: PagePool, KVAllocator, PagedSessionView,
MultiSessionCache.

Same classes, signatures and error behaviour as the reference's
``paged_cache.py`` (paged_cache.py:71-454).  The pool tensors keep the
reference layout ``K, V [n_layers, n_heads, n_pages * 16, head_dim]`` with a
token addressed as ``page_id * 16 + slot`` (paged_cache.py:103-108, 156-157),
so the budgeted ``HierarchicalKVCache`` sessions and the append-only
``PagedSessionView`` sessions can share one pool.

What changes is where the bytes move: token writes and session gathers are
single kernel launches over all layers and tokens (``ic_page_write`` /
``ic_page_gather``) instead of per-token, per-layer Python indexing.  The
allocator stays on the host, as in the reference (a free list and an LRU map
under a lock, paged_cache.py:205-288).
"""
from __future__ import annotations

import contextlib
import heapq
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib

__all__ = ["PAGE_SIZE", "PagePool", "KVAllocator", "MultiSessionCache", "PagedSessionView",
           "PagedCacheConfig"]

PAGE_SIZE: int = 16


@dataclass
class PagedCacheConfig:
    """paged_cache.py:77-94."""
    n_pages: int = 512
    n_layers: int = 36
    n_heads: int = 8
    head_dim: int = 128
    dtype: torch.dtype = torch.float16
    device: str = "cuda"
    max_pages_per_session: int = 64

    @property
    def total_tokens(self) -> int:
        return self.n_pages * PAGE_SIZE

    def gpu_memory_mb(self) -> float:
        bytes_per_elem = 2 if self.dtype == torch.float16 else 4
        total = 2 * self.n_layers * self.n_heads * self.total_tokens * self.head_dim
        return total * bytes_per_elem / (1024 ** 2)


class PagePool:
    """Pre-allocated K/V tensors divided into 16-token pages (paged_cache.py:99-200)."""

    def __init__(self, cfg: PagedCacheConfig) -> None:
        self.cfg = cfg
        dev = torch.device(cfg.device)
        _lib.require_device(dev)
        _lib.dtype_code(cfg.dtype)
        total = cfg.n_pages * PAGE_SIZE
        self.K = torch.zeros(cfg.n_layers, cfg.n_heads, total, cfg.head_dim, dtype=cfg.dtype, device=dev)
        self.V = torch.zeros(cfg.n_layers, cfg.n_heads, total, cfg.head_dim, dtype=cfg.dtype, device=dev)
        self._c_pool = self.c_pool()

    @classmethod
    def build(cls, n_sessions: int, n_layers: int, n_heads: int, head_dim: int,
              avg_tokens_per_session: int = 256, dtype: torch.dtype = torch.float16,
              device: str = "cuda") -> "PagePool":
        """Size for n_sessions x avg tokens plus 25 % (paged_cache.py:125-152)."""
        tokens_needed = n_sessions * avg_tokens_per_session
        pages_needed = (tokens_needed + PAGE_SIZE - 1) // PAGE_SIZE
        pages_needed = int(pages_needed * 1.25)
        cfg = PagedCacheConfig(n_pages=pages_needed, n_layers=n_layers, n_heads=n_heads, head_dim=head_dim,
                               dtype=dtype, device=device,
                               max_pages_per_session=(avg_tokens_per_session * 4) // PAGE_SIZE + 4)
        return cls(cfg)

    @property
    def device(self) -> torch.device:
        return self.K.device

    def c_pool(self) -> _lib.ic_pool:
        c = self.cfg
        return _lib.ic_pool(k=self.K.data_ptr(), v=self.V.data_ptr(), pool_tokens=c.n_pages * PAGE_SIZE,
                            num_layers=c.n_layers, num_kv_heads=c.n_heads, head_dim=c.head_dim,
                            dtype=_lib.dtype_code(c.dtype))

    def _abs(self, page_id: int, slot: int) -> int:
        return page_id * PAGE_SIZE + slot

    def _page_ids(self, page_ids) -> torch.Tensor:
        """int32 page ids on the pool's device (a device tensor passes through)."""
        if isinstance(page_ids, torch.Tensor):
            return page_ids
        return torch.tensor(page_ids, dtype=torch.int32).to(self.device, non_blocking=True)

    def write_rows(self, page_ids: List[int], start_token: int, k: torch.Tensor, v: torch.Tensor,
                   layer_begin: int = 0) -> None:
        """Write k, v [L', H, T, D] as tokens start_token .. start_token+T-1 of
        the session whose pages are `page_ids`, layers layer_begin .. +L'."""
        k = k.to(self.device, self.cfg.dtype)
        v = v.to(self.device, self.cfg.dtype)
        # strided sources go to the kernel as they are (rows must be contiguous)
        if k.stride(-1) != 1 or k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        pid = self._page_ids(page_ids)
        a = _lib.ic_page_rows_args(pool=self._c_pool, page_ids=pid.data_ptr(), n_page_ids=len(page_ids),
                                   layer_begin=layer_begin, layer_end=layer_begin + k.shape[0],
                                   start_token=start_token, n_tokens=k.shape[2], k_buf=k.data_ptr(),
                                   v_buf=v.data_ptr(), stride_l=k.stride(0), stride_h=k.stride(1),
                                   stride_t=k.stride(2))
        _lib.call("ic_page_write", a)

    def write_token(self, layer: int, page_id: int, slot: int, k_vec: torch.Tensor,
                    v_vec: torch.Tensor) -> None:
        """paged_cache.py:159-170: k_vec, v_vec [n_heads, head_dim]."""
        with torch.no_grad():
            self.write_rows([page_id], slot, k_vec[None, :, None, :], v_vec[None, :, None, :], layer)

    def gather_rows(self, page_ids: List[int], n_tokens: int, layer_begin: int,
                    layer_end: int) -> Tuple[torch.Tensor, torch.Tensor]:
        c = self.cfg
        nl = layer_end - layer_begin
        K = torch.empty(nl, c.n_heads, n_tokens, c.head_dim, dtype=c.dtype, device=self.device)
        V = torch.empty_like(K)
        if n_tokens == 0 or nl == 0:
            return K, V
        pid = self._page_ids(page_ids)
        a = _lib.ic_page_rows_args(pool=self._c_pool, page_ids=pid.data_ptr(), n_page_ids=len(page_ids),
                                   layer_begin=layer_begin, layer_end=layer_end, start_token=0,
                                   n_tokens=n_tokens, k_buf=K.data_ptr(), v_buf=V.data_ptr(),
                                   stride_l=K.stride(0), stride_h=K.stride(1), stride_t=K.stride(2))
        _lib.call("ic_page_gather", a)
        return K, V

    def _rows_args(self, page_ids: torch.Tensor, n_page_ids: int, start: int, k: torch.Tensor, v: torch.Tensor,
                   layer_begin: int) -> _lib.ic_page_rows_args:
        return _lib.ic_page_rows_args(pool=self._c_pool, page_ids=page_ids.data_ptr(), n_page_ids=n_page_ids,
                                      layer_begin=layer_begin, layer_end=layer_begin + k.shape[0],
                                      start_token=start, n_tokens=k.shape[2], k_buf=k.data_ptr(),
                                      v_buf=v.data_ptr(), stride_l=k.stride(0), stride_h=k.stride(1),
                                      stride_t=k.stride(2))

    def _run_batches(self, name: str, descs: List[_lib.ic_page_rows_args]) -> None:
        step = _lib.IC_PAGE_BATCH_MAX
        for i in range(0, len(descs), step):
            _lib.call_batch(name, descs[i:i + step])

    def write_rows_many(self, items) -> None:
        """write_rows for several page lists, all layers from 0: items are
        (page_ids, start_token, k, v) with k, v [L, H, T, D]; one launch per
        IC_PAGE_BATCH_MAX items.  The page lists must not share pool rows."""
        descs, keep = [], []
        for page_ids, start, k, v in items:
            if k.shape[2] == 0:
                continue
            k = k.to(self.device, self.cfg.dtype)
            v = v.to(self.device, self.cfg.dtype)
            if k.stride(-1) != 1 or k.stride() != v.stride():
                k, v = k.contiguous(), v.contiguous()
            pid = self._page_ids(page_ids)
            keep.append((pid, k, v))
            descs.append(self._rows_args(pid, len(page_ids), start, k, v, 0))
        self._run_batches("ic_page_write_batch", descs)

    def gather_rows_many(self, items, out=None) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """gather_rows(page_ids, n_tokens, 0, n_layers) for several page lists:
        items are (page_ids, n_tokens); one launch per IC_PAGE_BATCH_MAX items.
        `out`, if given, holds a (K, V) pair per item to gather into: tensors of
        the pool's dtype and device, shape [n_layers, n_heads, n_tokens,
        head_dim], rows contiguous and 16-byte aligned."""
        c = self.cfg
        outs, descs = [], []
        for i, (page_ids, n) in enumerate(items):
            if out is None:
                K = torch.empty(c.n_layers, c.n_heads, n, c.head_dim, dtype=c.dtype, device=self.device)
                V = torch.empty_like(K)
            else:
                K, V = out[i]
                shape = (c.n_layers, c.n_heads, n, c.head_dim)
                for x in (K, V):
                    if tuple(x.shape) != shape or x.dtype != c.dtype or x.device != self.device or x.stride(-1) != 1:
                        raise ValueError(f"gather_rows_many: out[{i}] must be {shape} {c.dtype} on {self.device} "
                                         "with contiguous rows")
            outs.append((K, V))
            if n > 0:
                descs.append(self._rows_args(self._page_ids(page_ids), len(page_ids), 0, K, V, 0))
        self._run_batches("ic_page_gather_batch", descs)
        return outs

    def gather_session(self, layer: int, page_ids: List[int], n_tokens: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """K, V [n_heads, n_tokens, head_dim] (paged_cache.py:172-200)."""
        if len(page_ids) == 0:
            empty = torch.zeros(self.cfg.n_heads, 0, self.cfg.head_dim, dtype=self.cfg.dtype, device=self.device)
            return empty, empty
        n_tokens = min(n_tokens, len(page_ids) * PAGE_SIZE)
        K, V = self.gather_rows(page_ids, n_tokens, layer, layer + 1)
        return K[0], V[0]


@dataclass
class _Lease:
    """One session's hold on the pool: its pages in allocation order, the clock
    value of its last use and its creation rank (which orders equal clock
    values the way a dict of sessions in creation order would)."""
    pages: List[int] = field(default_factory=list)
    stamp: float = 0.0
    rank: int = 0


class KVAllocator:
    """Page allocator with least-recently-used session eviction
    (paged_cache.py:205-288).

    Free pages form a stack (an int32 array and a top index): the initial
    stack holds page ids 0 .. n-1 with n-1 on top, a released session's pages
    are pushed back in their allocation order, and an allocation takes the top
    page -- the reference's free-list order.  Each session with pages holds a
    ``_Lease``.  Eviction victims come from a heap of (last use, creation rank,
    session) entries; a touch pushes a new entry and the stale ones are
    skipped when they surface, so finding the least recently used session is
    O(log n) instead of a scan over all sessions.  Equal last-use values go to
    the earliest-created lease, as a minimum over a creation-ordered dict
    would.  ``clock`` replaces time.monotonic (tests pass a counter).  All
    methods hold one lock."""

    def __init__(self, n_pages: int, max_pages_per_session: int, clock=None) -> None:
        self.n_pages = int(n_pages)
        self.max_pages_per_session = int(max_pages_per_session)
        self._stack = np.arange(self.n_pages, dtype=np.int32)
        self._top = self.n_pages
        self._owner = np.full(self.n_pages, -1, dtype=np.int64)  # page -> creation rank of its lease
        self._leases: Dict[str, _Lease] = {}
        self._tokens: Dict[str, int] = {}
        self._lru: List[Tuple[float, int, str]] = []
        self._next_rank = 0
        self._now = clock or time.monotonic
        self._mu = threading.Lock()
        self.lru_evictions = 0

    # -- internals (lock held) --------------------------------------------------------
    def _stamp(self, session_id: str, lease: _Lease) -> None:
        lease.stamp = self._now()
        heapq.heappush(self._lru, (lease.stamp, lease.rank, session_id))
        if len(self._lru) > 4 * len(self._leases) + 64:  # drop stale heap entries now and then
            self._lru = [(lz.stamp, lz.rank, sid) for sid, lz in self._leases.items()]
            heapq.heapify(self._lru)

    def _drop(self, session_id: str) -> None:
        lease = self._leases.pop(session_id, None)
        self._tokens.pop(session_id, None)
        if lease is not None and lease.pages:
            n = len(lease.pages)
            self._stack[self._top:self._top + n] = lease.pages
            self._top += n
            self._owner[lease.pages] = -1

    def _victim(self) -> str:
        while self._lru:
            stamp, rank, sid = heapq.heappop(self._lru)
            lease = self._leases.get(sid)
            if lease is not None and lease.rank == rank and lease.stamp == stamp:
                return sid
        raise RuntimeError("PagePool exhausted and no sessions to evict")

    def _take(self, session_id: str) -> int:
        lease = self._leases.get(session_id)
        if lease is not None and len(lease.pages) >= self.max_pages_per_session:
            raise RuntimeError(f"Session {session_id!r} exceeded max pages ({self.max_pages_per_session})")
        if self._top == 0:
            if not self._leases:
                raise RuntimeError("PagePool exhausted and no sessions to evict")
            self._drop(self._victim())
            self.lru_evictions += 1
            lease = self._leases.get(session_id)
        if lease is None:
            lease = self._leases[session_id] = _Lease(rank=self._next_rank)
            self._next_rank += 1
        self._top -= 1
        page = int(self._stack[self._top])
        lease.pages.append(page)
        self._owner[page] = lease.rank
        self._stamp(session_id, lease)
        return page

    # -- the reference's interface -------------------------------------------------------
    def allocate_page(self, session_id: str) -> int:
        """One page for `session_id`; evicts the least recently used session when
        no page is free.  RuntimeError at the per-session cap or when nothing can
        be evicted."""
        with self._mu:
            return self._take(session_id)

    def allocate_pages(self, session_id: str, count: int) -> Tuple[List[int], Optional[RuntimeError]]:
        """``count`` consecutive allocate_page calls under one lock acquisition:
        the pages obtained before any failure, and that failure (or None)."""
        got: List[int] = []
        with self._mu:
            while len(got) < count:
                # pages that need neither an eviction nor pass the cap come off
                # the stack in one slice (the order consecutive takes give) with
                # one stamp: no victim is chosen in between, so the intermediate
                # stamps could not change any decision; the others one by one
                lease = self._leases.get(session_id)
                have = 0 if lease is None else len(lease.pages)
                fast = min(count - len(got), self.max_pages_per_session - have, self._top)
                if fast > 0:
                    if lease is None:
                        lease = self._leases[session_id] = _Lease(rank=self._next_rank)
                        self._next_rank += 1
                    pages = self._stack[self._top - fast:self._top][::-1]
                    self._top -= fast
                    self._owner[pages] = lease.rank
                    taken = pages.tolist()
                    lease.pages.extend(taken)
                    got.extend(taken)
                    self._stamp(session_id, lease)
                    continue
                try:
                    got.append(self._take(session_id))
                except RuntimeError as e:
                    return got, e
        return got, None

    def page_count(self, session_id: str) -> int:
        """How many pages `session_id` holds (len(pages_for(...)) without the copy)."""
        with self._mu:
            lease = self._leases.get(session_id)
            return 0 if lease is None else len(lease.pages)

    def holds(self, session_id: str, pages: List[int]) -> bool:
        """Whether every page in `pages` is leased to `session_id` now (O(len(pages)))."""
        if len(pages) == 0:
            return True
        with self._mu:
            lease = self._leases.get(session_id)
            return lease is not None and all(int(self._owner[p]) == lease.rank for p in pages)

    def touch(self, session_id: str) -> None:
        with self._mu:
            lease = self._leases.get(session_id)
            if lease is not None:
                self._stamp(session_id, lease)

    def release_session(self, session_id: str) -> None:
        with self._mu:
            self._drop(session_id)

    def set_token_count(self, session_id: str, n: int) -> None:
        with self._mu:
            self._tokens[session_id] = int(n)

    def get_token_count(self, session_id: str) -> int:
        with self._mu:
            return self._tokens.get(session_id, 0)

    def pages_for(self, session_id: str) -> List[int]:
        with self._mu:
            lease = self._leases.get(session_id)
            return list(lease.pages) if lease is not None else []

    def utilization(self) -> float:
        with self._mu:
            return (self.n_pages - self._top) / self.n_pages if self.n_pages else 0.0

    def active_sessions(self) -> List[str]:
        with self._mu:
            return list(self._leases)

    # -- additions ---------------------------------------------------------------------
    def free_pages(self) -> int:
        with self._mu:
            return self._top

    def free_list(self) -> List[int]:
        """The free pages bottom to top (the next allocation takes the last)."""
        with self._mu:
            return self._stack[:self._top].tolist()

    def fragmentation(self, page_size: int = PAGE_SIZE) -> float:
        """Allocated-but-empty token slots / allocated token slots, from the token
        counts the sessions report (set_token_count)."""
        with self._mu:
            held = sum(len(lz.pages) for lz in self._leases.values()) * page_size
            if held == 0:
                return 0.0
            used = sum(min(self._tokens.get(sid, 0), len(lz.pages) * page_size) for sid, lz in self._leases.items())
            return (held - used) / held


class PagedSessionView:
    """Append-only view of one session's pages (paged_cache.py:293-396).

    Token metadata lives in growable numpy arrays; a push allocates its pages
    in one allocator call and writes every layer and token in one kernel
    launch (``PagePool.write_rows``)."""

    def __init__(self, session_id: str, pool: PagePool, allocator: KVAllocator) -> None:
        self.session_id = session_id
        self._pool = pool
        self._alloc = allocator
        self._pages: List[int] = []
        self._n_tokens: int = 0
        self._pos = np.zeros(0, dtype=np.int64)
        self._imp = np.zeros(0, dtype=np.float64)
        self._lock = threading.Lock()
        # the page list mirrored on the pool's device, uploaded as it grows, so
        # writes and gathers pass a device pointer instead of re-sending the list
        self._dev_pages: Optional[torch.Tensor] = None
        self._dev_n = 0

    @property
    def n_tokens(self) -> int:
        return self._n_tokens

    def _device_pages(self):
        """The page list on the pool's device (its first len(self._pages) entries)."""
        n = len(self._pages)
        dev = getattr(self._pool, "device", None)
        if dev is None or not isinstance(dev, torch.device) or dev.type != "cuda":
            return self._pages
        if self._dev_pages is None or self._dev_pages.numel() < n:
            cap = max(64, 2 * n)
            grown = torch.empty(cap, dtype=torch.int32, device=dev)
            if self._dev_pages is not None and self._dev_n:
                grown[:self._dev_n].copy_(self._dev_pages[:self._dev_n])
            self._dev_pages = grown
        if self._dev_n < n:
            self._dev_pages[self._dev_n:n].copy_(torch.tensor(self._pages[self._dev_n:n], dtype=torch.int32),
                                                 non_blocking=True)
            self._dev_n = n
        return self._dev_pages[:n]

    def _grow(self, n: int) -> None:
        if n > self._pos.shape[0]:
            cap = max(n, 2 * self._pos.shape[0], 64)
            pos = np.zeros(cap, dtype=np.int64)
            imp = np.zeros(cap, dtype=np.float64)
            pos[:self._n_tokens] = self._pos[:self._n_tokens]
            imp[:self._n_tokens] = self._imp[:self._n_tokens]
            self._pos, self._imp = pos, imp

    def _reserve(self, n_new: int):
        """The allocation half of push (the caller holds the lock): pages for
        n_new more tokens, allocated in one call, in the reference's order.
        Returns (start, fit, err): tokens start .. start + fit - 1 fit the pages
        now held; err is the allocation error push raises once they are written."""
        start = self._n_tokens
        room = len(self._pages) * PAGE_SIZE - start
        need = max(0, -(-(n_new - room) // PAGE_SIZE)) if n_new > room else 0
        got, err = self._alloc.allocate_pages(self.session_id, need) if need else ([], None)
        self._pages.extend(got)
        fit = max(0, min(n_new, len(self._pages) * PAGE_SIZE - start))
        return start, fit, err

    def _record(self, start: int, fit: int, positions: List[int], importance: List[float]) -> None:
        """The token metadata of a push's written tokens; missing positions
        continue the token count, missing importance values are 0."""
        if fit <= 0:
            return
        self._grow(start + fit)
        npos, nimp = min(len(positions), fit), min(len(importance), fit)
        self._pos[start:start + npos] = np.asarray(positions[:npos], dtype=np.int64)
        self._pos[start + npos:start + fit] = np.arange(start + npos, start + fit, dtype=np.int64)
        self._imp[start:start + nimp] = np.asarray(importance[:nimp], dtype=np.float64)
        self._imp[start + nimp:start + fit] = 0.0
        self._n_tokens = start + fit

    def _commit(self) -> None:
        self._alloc.set_token_count(self.session_id, self._n_tokens)
        self._alloc.touch(self.session_id)

    def push(self, k_states: torch.Tensor, v_states: torch.Tensor, positions: List[int],
             importance: List[float]) -> None:
        """Write T tokens [n_layers, n_heads, T, head_dim] (paged_cache.py:330-363).

        A page is allocated whenever a token starts one, in the reference's
        order.  If an allocation fails, the tokens that fit in the pages
        obtained so far are still written and counted, as the reference's
        token-by-token loop does, and the error propagates.  Missing positions
        continue the token count; missing importance values are 0.
        """
        n_new = int(k_states.shape[2])
        with self._lock:
            start, fit, err = self._reserve(n_new)
            if fit > 0:
                self._pool.write_rows(self._device_pages(), start, k_states[:, :, :fit], v_states[:, :, :fit])
            self._record(start, fit, positions, importance)
            if err is not None:
                raise err
            self._commit()

    def gather(self, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return self._pool.gather_session(layer, self._device_pages(), self._n_tokens)

    def gather_all(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """K, V [n_layers, n_heads, n_tokens, head_dim] in one launch."""
        n = min(self._n_tokens, len(self._pages) * PAGE_SIZE)
        return self._pool.gather_rows(self._device_pages(), n, 0, self._pool.cfg.n_layers)

    def to_hf_past_key_values(self, device: str = None):
        K, V = self.gather_all()
        if device is not None:
            K, V = K.to(device), V.to(device)
        return [(K[l][None], V[l][None]) for l in range(K.shape[0])]

    def top_importance_tokens(self, top_k: int) -> Tuple[List[int], List[float]]:
        """Token indices and importance of the top_k tokens: highest importance
        first, equal importance by higher index first (the order of a
        descending sort of (importance, index) pairs)."""
        n = self._n_tokens
        if n == 0:
            return [], []
        imp = self._imp[:n]
        order = np.lexsort((np.arange(n), imp))[::-1][:max(0, top_k)]
        return order.tolist(), imp[order].tolist()

    def reset(self) -> None:
        """Give the pages back and forget every token."""
        with self._lock:
            self._alloc.release_session(self.session_id)
            self._pages, self._n_tokens = [], 0
            self._dev_n = 0
            self._pos = np.zeros(0, dtype=np.int64)
            self._imp = np.zeros(0, dtype=np.float64)


class MultiSessionCache:
    """Session views over one PagePool with one shared allocator
    (paged_cache.py:401-454)."""

    def __init__(self, pool: PagePool, clock=None) -> None:
        self._pool = pool
        self.allocator = KVAllocator(pool.cfg.n_pages, pool.cfg.max_pages_per_session, clock=clock)
        self._sessions: Dict[str, PagedSessionView] = {}
        self._mu = threading.Lock()

    @property
    def _alloc(self) -> KVAllocator:
        return self.allocator

    def get_or_create(self, session_id: str) -> PagedSessionView:
        with self._mu:
            view = self._sessions.get(session_id)
            if view is None:
                view = self._sessions[session_id] = PagedSessionView(session_id, self._pool, self.allocator)
            return view

    def reset(self, session_id: str) -> None:
        with self._mu:
            view = self._sessions.pop(session_id, None)
        if view is not None:
            view.reset()

    def reset_all(self) -> None:
        for sid in self.sessions():
            self.reset(sid)

    def push_many(self, session_ids: List[str], k_states, v_states) -> List[Optional[Exception]]:
        """PagedSessionView.push of k_states[i], v_states[i] ([n_layers,
        n_heads, T, head_dim]) to session_ids[i] for every i, positions and
        importance left to their defaults, with the writes in one launch per
        IC_PAGE_BATCH_MAX sessions.  The allocator sees exactly the calls of
        consecutive push calls in list order (allocation, token count, touch);
        a session whose pages a later allocation of the same call evicted is
        not written, as its rows may already belong to another session (a
        write goes ahead only when every page it touches is still leased to its
        session, which keeps the call's writes on disjoint rows).  Returns the
        error each push would have raised (None when it completed)."""
        if len(set(session_ids)) != len(session_ids):
            raise ValueError("push_many: a session may appear once per call")
        views = [self.get_or_create(sid) for sid in session_ids]
        errors: List[Optional[Exception]] = []
        writes = []
        with contextlib.ExitStack() as locks:
            for view in sorted(views, key=lambda x: x.session_id):
                locks.enter_context(view._lock)
            for i, view in enumerate(views):
                k, v = k_states[i], v_states[i]
                start, fit, err = view._reserve(int(k.shape[2]))
                if fit > 0:
                    writes.append((view, start, k[:, :, :fit], v[:, :, :fit]))
                view._record(start, fit, [], [])
                if err is None:
                    view._commit()
                errors.append(err)
            live = []
            for vw, start, k, v in writes:
                touched = vw._pages[start // PAGE_SIZE:(start + int(k.shape[2]) - 1) // PAGE_SIZE + 1]
                if self.allocator.holds(vw.session_id, touched):
                    live.append((vw._device_pages(), start, k, v))
            self._pool.write_rows_many(live)
        return errors

    def gather_many(self, session_ids: List[str], out=None) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """PagedSessionView.gather_all of several sessions, in one launch per
        IC_PAGE_BATCH_MAX sessions: [(K, V)] with K, V [n_layers, n_heads,
        n_tokens, head_dim] in list order (written into `out`'s pairs when
        given: see PagePool.gather_rows_many)."""
        items = []
        for sid in session_ids:
            view = self.get_or_create(sid)
            n = min(view._n_tokens, len(view._pages) * PAGE_SIZE)
            items.append((view._device_pages(), n))
        return self._pool.gather_rows_many(items, out)

    def gathered_tokens(self, session_id: str) -> int:
        """The token count gather_all / gather_many return for `session_id`."""
        view = self.get_or_create(session_id)
        return min(view._n_tokens, len(view._pages) * PAGE_SIZE)

    def sessions(self) -> List[str]:
        """Ids of every view created and not reset (with or without pages)."""
        with self._mu:
            return list(self._sessions)

    def utilization(self) -> float:
        return self.allocator.utilization()

    def active_sessions(self) -> List[str]:
        return self.allocator.active_sessions()

    def pool_info(self) -> dict:
        """Pool size and use, with the reference's keys."""
        c = self._pool.cfg
        return dict(total_pages=c.n_pages, total_tokens=c.total_tokens, gpu_memory_mb=c.gpu_memory_mb(),
                    utilization="%.1f%%" % (100.0 * self.utilization()),
                    active_sessions=len(self.active_sessions()))
