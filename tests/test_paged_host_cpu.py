"""Host bookkeeping of the paged cache on the CPU: KVAllocator and the
allocation order of PagedSessionView.push / MultiSessionCache against the
reference's own trace (tests/golden/paged_trace.npz, produced by the
reference's classes).  The page pool itself is replaced by a recorder: its
device copies are covered by the GPU test of the same trace."""
import json

import numpy as np
import pytest
import torch

import specs
from infercache_b200.paged_cache import KVAllocator, MultiSessionCache, PagedCacheConfig


class RecordingPool:
    """Stands in for PagePool: records the rows each push writes."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.writes = []

    def write_rows(self, page_ids, start_token, k, v, layer_begin=0):
        self.writes.append((list(page_ids), start_token, k.shape[2]))

    def gather_session(self, layer, page_ids, n_tokens):
        return None, None


def _msc():
    sp = specs.PAGED
    cfg = PagedCacheConfig(n_pages=sp["n_pages"], n_layers=sp["layers"], n_heads=sp["heads"], head_dim=sp["d"],
                           dtype=torch.float32, device="cpu", max_pages_per_session=sp["max_pps"])
    ticks = iter(range(1, 10 ** 6))
    return MultiSessionCache(RecordingPool(cfg), clock=lambda: float(next(ticks)))


def test_allocation_trace_matches_reference(golden):
    g = golden("paged_trace")
    msc = _msc()
    for i, op in enumerate(specs.paged_ops()):
        err = ""
        try:
            if op[0] == "push":
                _, sid, n, seed = op
                kk, vv = specs.paged_tokens(n, seed)
                view = msc.get_or_create(sid)
                view.push(kk, vv, positions=list(range(view.n_tokens, view.n_tokens + n)),
                          importance=[float(x) for x in np.linspace(0, 1, n)])
            elif op[0] == "reset":
                msc.reset(op[1])
            elif op[0] == "touch":
                msc._alloc.touch(op[1])
        except RuntimeError as e:
            err = str(e)
        assert err == str(g["errors"][i]), (i, op, err)
        pages = {s: msc._alloc.pages_for(s) for s in sorted(msc.active_sessions())}
        assert pages == json.loads(str(g["pages"][i])), (i, op)
        assert msc._alloc._free_list == json.loads(str(g["free"][i])), (i, op)
        assert abs(msc.utilization() - float(g["util"][i])) < 1e-12


def test_partial_push_on_cap_keeps_what_fits():
    """A push that hits the per-session cap writes the tokens that fit in the
    pages obtained so far, counts them, and raises (the reference's
    token-by-token loop, paged_cache.py:330-363)."""
    msc = _msc()
    sp = specs.PAGED
    view = msc.get_or_create("S")
    n = sp["max_pps"] * 16 + 5
    kk = torch.zeros(sp["layers"], sp["heads"], n, sp["d"])
    with pytest.raises(RuntimeError, match="exceeded max pages"):
        view.push(kk, kk, positions=list(range(n)), importance=[0.0] * n)
    assert view.n_tokens == sp["max_pps"] * 16
    assert msc._pool.writes[-1][2] == sp["max_pps"] * 16
    assert len(msc._alloc.pages_for("S")) == sp["max_pps"]


def test_allocator_lifo_lru_and_exhaustion():
    ticks = iter(range(1, 100))
    a = KVAllocator(4, 3, clock=lambda: float(next(ticks)))
    assert [a.allocate_page("x") for _ in range(2)] == [3, 2]  # LIFO pop from the end
    assert a.allocate_page("y") == 1
    a.touch("x")                                              # y is now least recently used
    assert a.allocate_page("z") == 0
    assert a.allocate_page("z") == 1                          # pool empty: y evicted (LRU)
    assert a.active_sessions() == ["x", "z"] and a.lru_evictions == 1
    assert abs(a.utilization() - 1.0) < 1e-12
    a.release_session("x")
    assert a.free_pages() == 2 and a.pages_for("x") == []
    c = KVAllocator(8, 2)
    c.allocate_page("s")
    c.allocate_page("s")
    with pytest.raises(RuntimeError, match="exceeded max pages"):
        c.allocate_page("s")
    b = KVAllocator(0, 4)
    with pytest.raises(RuntimeError, match="PagePool exhausted and no sessions to evict"):
        b.allocate_page("s")
