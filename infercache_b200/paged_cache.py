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

import threading
import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

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

    def _page_ids(self, page_ids: List[int]) -> torch.Tensor:
        return torch.tensor(page_ids, dtype=torch.int32).to(self.device, non_blocking=True)

    def write_rows(self, page_ids: List[int], start_token: int, k: torch.Tensor, v: torch.Tensor,
                   layer_begin: int = 0) -> None:
        """Write k, v [L', H, T, D] as tokens start_token .. start_token+T-1 of
        the session whose pages are `page_ids`, layers layer_begin .. +L'."""
        k = k.to(self.device, self.cfg.dtype).contiguous()
        v = v.to(self.device, self.cfg.dtype).contiguous()
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

    def gather_session(self, layer: int, page_ids: List[int], n_tokens: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """K, V [n_heads, n_tokens, head_dim] (paged_cache.py:172-200)."""
        if not page_ids:
            empty = torch.zeros(self.cfg.n_heads, 0, self.cfg.head_dim, dtype=self.cfg.dtype, device=self.device)
            return empty, empty
        n_tokens = min(n_tokens, len(page_ids) * PAGE_SIZE)
        K, V = self.gather_rows(page_ids, n_tokens, layer, layer + 1)
        return K[0], V[0]


class KVAllocator:
    """Thread-safe LIFO free-list page allocator with LRU session eviction
    (paged_cache.py:205-288).  ``clock`` replaces time.monotonic when given."""

    def __init__(self, n_pages: int, max_pages_per_session: int, clock=None) -> None:
        self._max_pps = max_pages_per_session
        self._lock = threading.Lock()
        self._free_list: List[int] = list(range(n_pages))
        self._session_pages: Dict[str, List[int]] = {}
        self._session_atime: Dict[str, float] = {}
        self._session_ntok: Dict[str, int] = {}
        self._clock = clock or time.monotonic
        self.lru_evictions = 0

    def _evict_lru(self) -> None:
        if not self._session_pages:
            raise RuntimeError("PagePool exhausted and no sessions to evict")
        lru_session = min(self._session_atime, key=self._session_atime.__getitem__)
        self._release_locked(lru_session)
        self.lru_evictions += 1

    def _release_locked(self, session_id: str) -> None:
        pages = self._session_pages.pop(session_id, [])
        self._free_list.extend(pages)
        self._session_atime.pop(session_id, None)
        self._session_ntok.pop(session_id, None)

    def allocate_page(self, session_id: str) -> int:
        with self._lock:
            cur_pages = len(self._session_pages.get(session_id, []))
            if cur_pages >= self._max_pps:
                raise RuntimeError(f"Session {session_id!r} exceeded max pages ({self._max_pps})")
            if not self._free_list:
                self._evict_lru()
            page_id = self._free_list.pop()
            self._session_pages.setdefault(session_id, []).append(page_id)
            self._session_atime[session_id] = self._clock()
            return page_id

    def touch(self, session_id: str) -> None:
        with self._lock:
            if session_id in self._session_atime:
                self._session_atime[session_id] = self._clock()

    def release_session(self, session_id: str) -> None:
        with self._lock:
            self._release_locked(session_id)

    def set_token_count(self, session_id: str, n: int) -> None:
        with self._lock:
            self._session_ntok[session_id] = n

    def get_token_count(self, session_id: str) -> int:
        with self._lock:
            return self._session_ntok.get(session_id, 0)

    def pages_for(self, session_id: str) -> List[int]:
        with self._lock:
            return list(self._session_pages.get(session_id, []))

    def utilization(self) -> float:
        with self._lock:
            total_pages = sum(len(v) for v in self._session_pages.values())
            n_pages = total_pages + len(self._free_list)
            return total_pages / n_pages if n_pages else 0.0

    def active_sessions(self) -> List[str]:
        with self._lock:
            return list(self._session_pages.keys())

    def free_pages(self) -> int:
        with self._lock:
            return len(self._free_list)


class PagedSessionView:
    """Append-only view of one session's pages (paged_cache.py:293-396)."""

    def __init__(self, session_id: str, pool: PagePool, allocator: KVAllocator) -> None:
        self.session_id = session_id
        self._pool = pool
        self._alloc = allocator
        self._pages: List[int] = []
        self._n_tokens: int = 0
        self._importance: List[float] = []
        self._positions: List[int] = []
        self._lock = threading.Lock()

    @property
    def n_tokens(self) -> int:
        return self._n_tokens

    def push(self, k_states: torch.Tensor, v_states: torch.Tensor, positions: List[int],
             importance: List[float]) -> None:
        """Write T tokens [n_layers, n_heads, T, head_dim] (paged_cache.py:330-363).

        Pages are allocated in the reference's order (one whenever a token
        starts a page).  If an allocation raises, the tokens that fit in the
        pages obtained so far are still written and counted, as in the
        reference's token-by-token loop, and the error propagates.
        """
        n_new = k_states.shape[2]
        with self._lock:
            start = self._n_tokens
            fit = 0
            err: Optional[BaseException] = None
            for t in range(n_new):
                if (start + t) % PAGE_SIZE == 0:
                    try:
                        self._pages.append(self._alloc.allocate_page(self.session_id))
                    except RuntimeError as e:
                        err = e
                        break
                fit += 1
            if fit:
                self._pool.write_rows(self._pages, start, k_states[:, :, :fit], v_states[:, :, :fit])
            for t in range(fit):
                self._n_tokens += 1
                self._positions.append(positions[t] if t < len(positions) else self._n_tokens - 1)
                self._importance.append(importance[t] if t < len(importance) else 0.0)
            if err is not None:
                raise err
            self._alloc.set_token_count(self.session_id, self._n_tokens)
            self._alloc.touch(self.session_id)

    def gather(self, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return self._pool.gather_session(layer, self._pages, self._n_tokens)

    def gather_all(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """K, V [n_layers, n_heads, n_tokens, head_dim] in one launch."""
        n = min(self._n_tokens, len(self._pages) * PAGE_SIZE)
        return self._pool.gather_rows(self._pages, n, 0, self._pool.cfg.n_layers)

    def to_hf_past_key_values(self, device: str = None):
        K, V = self.gather_all()
        if device is not None:
            K, V = K.to(device), V.to(device)
        return [(K[l][None], V[l][None]) for l in range(K.shape[0])]

    def top_importance_tokens(self, top_k: int) -> Tuple[List[int], List[float]]:
        if not self._importance:
            return [], []
        pairs = sorted(zip(self._importance, range(len(self._importance))), reverse=True)
        top_pairs = pairs[:top_k]
        return [p for _, p in top_pairs], [imp for imp, _ in top_pairs]

    def reset(self) -> None:
        with self._lock:
            self._alloc.release_session(self.session_id)
            self._pages = []
            self._n_tokens = 0
            self._importance = []
            self._positions = []


class MultiSessionCache:
    """All PagedSessionViews sharing one PagePool (paged_cache.py:401-454)."""

    def __init__(self, pool: PagePool, clock=None) -> None:
        self._pool = pool
        self._alloc = KVAllocator(pool.cfg.n_pages, pool.cfg.max_pages_per_session, clock=clock)
        self._views: Dict[str, PagedSessionView] = {}
        self._lock = threading.Lock()

    def get_or_create(self, session_id: str) -> PagedSessionView:
        with self._lock:
            if session_id not in self._views:
                self._views[session_id] = PagedSessionView(session_id, self._pool, self._alloc)
            return self._views[session_id]

    def reset(self, session_id: str) -> None:
        with self._lock:
            view = self._views.pop(session_id, None)
        if view:
            view.reset()

    def reset_all(self) -> None:
        with self._lock:
            sessions = list(self._views.keys())
        for sid in sessions:
            self.reset(sid)

    def utilization(self) -> float:
        return self._alloc.utilization()

    def active_sessions(self) -> List[str]:
        return self._alloc.active_sessions()

    def pool_info(self) -> dict:
        cfg = self._pool.cfg
        return {
            "total_pages": cfg.n_pages,
            "total_tokens": cfg.total_tokens,
            "gpu_memory_mb": cfg.gpu_memory_mb(),
            "utilization": f"{self.utilization() * 100:.1f}%",
            "active_sessions": len(self.active_sessions()),
        }
