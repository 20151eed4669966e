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

    def write_rows_many(self, items):
        for page_ids, start_token, k, v in items:
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
                msc.allocator.touch(op[1])
        except RuntimeError as e:
            err = str(e)
        assert err == str(g["errors"][i]), (i, op, err)
        pages = {s: msc.allocator.pages_for(s) for s in sorted(msc.active_sessions())}
        assert pages == json.loads(str(g["pages"][i])), (i, op)
        assert msc.allocator.free_list() == json.loads(str(g["free"][i])), (i, op)
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
    assert len(msc.allocator.pages_for("S")) == sp["max_pps"]


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


def test_allocator_matches_oracle_on_random_ops():
    """Random allocations, touches and releases over a small pool: the same
    pages, free-stack order, active sessions, utilization and errors as the
    oracle's restatement of the reference allocator (paged_cache.py:205-288)."""
    import random
    from oracle.paged import OracleAllocator
    rng = random.Random(5)
    for trial in range(20):
        n_pages, cap = rng.randint(1, 24), rng.randint(1, 8)
        oa = OracleAllocator(n_pages, cap)
        ticks = iter(range(1, 10 ** 6))
        ka = KVAllocator(n_pages, cap, clock=lambda: float(next(ticks)))
        sids = [f"s{i}" for i in range(rng.randint(1, 6))]
        for step in range(300):
            op, sid = rng.random(), rng.choice(sids)
            if op < 0.7:
                res = []
                for a in (oa, ka):
                    try:
                        res.append(a.allocate_page(sid))
                    except RuntimeError as e:
                        res.append(str(e))
                assert res[0] == res[1], (trial, step, res)
            elif op < 0.85:
                oa.touch(sid)
                ka.touch(sid)
            else:
                oa._release(sid)
                ka.release_session(sid)
            assert ka.free_list() == oa.free, (trial, step)
            assert ka.active_sessions() == list(oa.pages), (trial, step)
            for s in sids:
                assert ka.pages_for(s) == oa.pages.get(s, [])
            assert abs(ka.utilization() - oa.utilization()) < 1e-12


def test_lru_equal_clock_values_evict_earliest_created():
    """With a clock that does not advance, the victim is the session created
    first among those holding pages (a minimum over a creation-ordered map)."""
    a = KVAllocator(3, 4, clock=lambda: 7.0)
    a.allocate_page("x")
    a.allocate_page("y")
    a.allocate_page("z")
    a.touch("x")
    assert a.allocate_page("w") == 2      # x (created first) is evicted; its page 2 is reused
    assert a.active_sessions() == ["y", "z", "w"] and a.lru_evictions == 1
    a.release_session("y")                # page 1 back on the stack
    assert a.allocate_page("x") == 1      # x comes back as a new, latest-created lease
    assert a.allocate_page("v") == 0      # no free page: z, the earliest-created holder, goes
    assert a.allocate_page("u") == 2      # then w
    assert a.active_sessions() == ["x", "v", "u"] and a.lru_evictions == 3


def test_fragmentation_and_batched_allocation():
    a = KVAllocator(10, 4)
    got, err = a.allocate_pages("s", 3)
    assert got == [9, 8, 7] and err is None
    a.set_token_count("s", 33)                       # 48 slots held, 33 used
    assert abs(a.fragmentation() - 15 / 48) < 1e-12
    got, err = a.allocate_pages("s", 3)              # cap 4: one more, then the cap error
    assert got == [6] and "exceeded max pages" in str(err)


def test_top_importance_tokens_order_matches_oracle():
    from oracle.paged import OracleAllocator, OracleMultiSession, OraclePagePool
    sp = specs.PAGED
    msc = _msc()
    view = msc.get_or_create("S")
    imp = [0.5, 0.25, 0.5, 1.0, 0.0, 0.25, 1.0, 0.5]
    kk = torch.zeros(sp["layers"], sp["heads"], len(imp), sp["d"])
    view.push(kk, kk, positions=list(range(len(imp))), importance=imp)
    pairs = sorted(zip(imp, range(len(imp))), reverse=True)
    for k in (0, 3, 8, 20):
        idx, vals = view.top_importance_tokens(k)
        assert idx == [i for _, i in pairs[:k]] and vals == [x for x, _ in pairs[:k]]


class _GatherPool(RecordingPool):
    """RecordingPool whose gathers return shape-only tensors."""

    def gather_rows(self, page_ids, n_tokens, layer_begin, layer_end):
        c = self.cfg
        K = torch.empty(layer_end - layer_begin, c.n_heads, n_tokens, c.head_dim, device="meta")
        return K, K

    def gather_rows_many(self, items, out=None):
        if out is not None:
            return out
        return [self.gather_rows(p, n, 0, self.cfg.n_layers) for p, n in items]


def test_paged_stress_host_logic_matches_oracle_allocator():
    """The config-5 driver (bench.paged_stress) on the host with a recording
    pool: Poisson-like arrivals into a pool far smaller than the sessions
    need, so the allocator evicts least-recently-used sessions; every
    allocation, error and the final free list agree with the oracle's
    allocator replaying the recorded trace, evicted sessions are dropped, and
    every surviving session decodes its 8 steps."""
    import random
    import bench
    cfg = PagedCacheConfig(n_pages=60, n_layers=2, n_heads=2, head_dim=8, dtype=torch.float32, device="cpu",
                           max_pages_per_session=30)
    ticks = iter(range(1, 10 ** 9))
    msc = MultiSessionCache(_GatherPool(cfg), clock=lambda: float(next(ticks)))
    rec = bench._RecordingAllocator(msc.allocator)
    msc.allocator = rec
    rng = random.Random(4)
    t, trace = 0.0, []
    for i in range(40):
        t += rng.expovariate(1 / 5.0)
        trace.append((i, rng.randint(10, 300), t))
    src = torch.zeros(2, 2, 400, 8)
    r = bench.paged_stress(msc, trace, 8, src, src, tick_timer=lambda fn: (fn(), 4.0)[1])
    assert r["lru_evictions"] > 0 and r["dropped_by_lru"] > 0
    assert r["decode_tokens"] >= 8 * (40 - r["dropped_by_lru"] - 5)
    assert 0.0 <= r["fragmentation_mean"] <= r["fragmentation_max"] < 1.0
    assert bench.replay_on_oracle(rec.ops, 60, 30, rec.inner.free_list())
    assert msc.allocator.free_pages() == 60  # every session departed or was dropped


def _small_msc(n_pages, max_pps):
    cfg = PagedCacheConfig(n_pages=n_pages, n_layers=1, n_heads=1, head_dim=8, dtype=torch.float32, device="cpu",
                           max_pages_per_session=max_pps)
    ticks = iter(range(1, 10 ** 6))
    return MultiSessionCache(RecordingPool(cfg), clock=lambda: float(next(ticks)))


def test_push_many_matches_consecutive_pushes():
    """push_many makes the allocator calls of consecutive pushes in list order:
    the same pages, free list, token counts, LRU victims and errors after every
    call; its writes are those of the pushes, less the ones whose pages were
    evicted by a later allocation of the same call."""
    rng = np.random.default_rng(7)
    seq, bat = _small_msc(24, 5), _small_msc(24, 5)
    sids = [f"s{i}" for i in range(7)]
    for call in range(30):
        pick = list(rng.choice(sids, size=int(rng.integers(1, 6)), replace=False))
        lens = [int(rng.integers(0, 40)) for _ in pick]
        ks = [torch.zeros(1, 1, n, 8) for n in lens]
        errs_seq = []
        for sid, k in zip(pick, ks):
            try:
                seq.get_or_create(sid).push(k, k, positions=[], importance=[])
                errs_seq.append(None)
            except RuntimeError as e:
                errs_seq.append(str(e))
        errs_bat = [None if e is None else str(e) for e in bat.push_many(pick, ks, ks)]
        assert errs_bat == errs_seq, call
        assert seq.allocator.free_list() == bat.allocator.free_list(), call
        for sid in sids:
            assert seq.allocator.pages_for(sid) == bat.allocator.pages_for(sid), (call, sid)
            assert seq.allocator.get_token_count(sid) == bat.allocator.get_token_count(sid)
            assert seq.get_or_create(sid).n_tokens == bat.get_or_create(sid).n_tokens
        assert seq.allocator.lru_evictions == bat.allocator.lru_evictions
        if rng.random() < 0.2:
            gone = str(rng.choice(sids))
            seq.reset(gone)
            bat.reset(gone)
    assert seq.allocator.lru_evictions > 0
    # every batched write is one of the consecutive pushes' writes, on pages leased at the time
    assert set(map(lambda w: (tuple(w[0]), w[1], w[2]), bat._pool.writes)) <= \
        set(map(lambda w: (tuple(w[0]), w[1], w[2]), seq._pool.writes))


def test_push_many_skips_writes_to_pages_evicted_in_the_same_call():
    """Two sessions hold four of five pages; in one push_many call the first
    appends into its last page, then the second takes the free page (which
    makes it the most recently used) and, for a second page, evicts the first:
    the first session's write is dropped, the second's kept."""
    msc = _small_msc(5, 4)
    z = torch.zeros(1, 1, 24, 8)
    msc.push_many(["A", "B"], [z, z], [z, z])
    assert len(msc.allocator.pages_for("A")) == 2 and len(msc.allocator.pages_for("B")) == 2
    msc._pool.writes.clear()
    one = torch.zeros(1, 1, 1, 8)
    more = torch.zeros(1, 1, 25, 8)
    errs = msc.push_many(["A", "B"], [one, more], [one, more])
    assert errs == [None, None]
    assert msc.allocator.pages_for("A") == [] and msc.allocator.lru_evictions == 1
    assert len(msc.allocator.pages_for("B")) == 4
    assert [w[1:] for w in msc._pool.writes] == [(24, 25)]


def test_push_many_rejects_repeated_sessions():
    msc = _small_msc(4, 4)
    z = torch.zeros(1, 1, 1, 8)
    with pytest.raises(ValueError):
        msc.push_many(["A", "A"], [z, z], [z, z])


def test_allocator_page_count_and_holds():
    ticks = iter(range(1, 100))
    a = KVAllocator(4, 3, clock=lambda: float(next(ticks)))
    a.allocate_page("x")
    a.allocate_page("x")
    a.allocate_page("y")
    assert a.page_count("x") == 2 and a.page_count("y") == 1 and a.page_count("z") == 0
    assert a.holds("x", a.pages_for("x")) and not a.holds("x", a.pages_for("y")) and a.holds("x", [])
    a.touch("x")
    a.allocate_page("z")
    gone = a.pages_for("y")
    a.allocate_page("z")                     # evicts y; its page goes to z
    assert not a.holds("y", gone) and a.holds("z", gone) and a.page_count("y") == 0
    a.release_session("x")
    assert not a.holds("x", [3]) and a.page_count("x") == 0


def test_allocate_pages_matches_consecutive_allocate_page_on_oracle():
    """allocate_pages (free pages taken in slices between evictions) against
    the oracle's allocate_page called count times: the same pages in the same
    order, the same error at the same point, the same free stack and holders,
    over random counts that cross the per-session cap and empty the pool."""
    import random
    from oracle.paged import OracleAllocator
    rng = random.Random(9)
    for trial in range(30):
        n_pages, cap = rng.randint(1, 40), rng.randint(1, 12)
        oa = OracleAllocator(n_pages, cap)
        ticks = iter(range(1, 10 ** 6))
        ka = KVAllocator(n_pages, cap, clock=lambda: float(next(ticks)))
        sids = [f"s{i}" for i in range(rng.randint(1, 5))]
        for step in range(200):
            sid, r = rng.choice(sids), rng.random()
            if r < 0.6:
                count = rng.randint(0, 15)
                want, werr = [], ""
                for _ in range(count):
                    try:
                        want.append(oa.allocate_page(sid))
                    except RuntimeError as e:
                        werr = str(e)
                        break
                got, err = ka.allocate_pages(sid, count)
                assert (got, str(err) if err else "") == (want, werr), (trial, step)
            elif r < 0.8:
                oa.touch(sid)
                ka.touch(sid)
            else:
                oa._release(sid)
                ka.release_session(sid)
            assert ka.free_list() == oa.free, (trial, step)
            assert ka.active_sessions() == list(oa.pages), (trial, step)
            for x in sids:
                assert ka.pages_for(x) == oa.pages.get(x, [])
                assert ka.holds(x, ka.pages_for(x))
