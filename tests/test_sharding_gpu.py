"""Moving a session between SessionBatches (the rebalance path) on one
B200: export -> import reproduces the session exactly, and both copies
decode identically afterwards (index work exact, outputs bit-identical)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _batch(S, seed):
    from infercache_b200 import CacheConfig, SessionBatch
    cfg = CacheConfig(num_layers=3, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=16, important_size=40,
                      dtype=torch.float16, decay=0.99)
    b = SessionBatch(cfg, S, "cuda:0")
    g = torch.Generator(device="cuda").manual_seed(seed)
    for s in range(S):
        T = 150 + 10 * s
        pkv = tuple((torch.randn(1, 2, T, 128, generator=g, device="cuda").half(),
                     torch.randn(1, 2, T, 128, generator=g, device="cuda").half()) for _ in range(3))
        b.load_prompt(s, pkv, torch.rand(T, generator=g, device="cuda"))
    return b


def _decode(b, steps, seed, start):
    g = torch.Generator(device="cuda").manual_seed(seed)
    S, outs = b.num_sessions, []
    for i in range(steps):
        q = torch.randn(3, S, 16, 128, generator=g, device="cuda").half()
        k = torch.randn(3, S, 2, 128, generator=g, device="cuda").half()
        v = torch.randn(3, S, 2, 128, generator=g, device="cuda").half()
        outs.append(b.step(q, k, v, torch.full((S,), start + i, dtype=torch.int64, device="cuda")).clone())
    return outs


def test_export_import_roundtrip_then_identical_decoding():
    from infercache_b200.sharding import export_session, import_session
    a = _batch(4, seed=1)
    _decode(a, 30, seed=2, start=400)  # move the session mid-stream (ring wrapped, L2 evicting)
    dst = _batch(6, seed=3)
    st = export_session(a, 2)
    import_session(dst, 5, st)
    st2 = export_session(dst, 5)
    for key in st:
        assert torch.equal(st[key], st2[key]), key
    # one-session batches continue identically from either copy
    from infercache_b200 import SessionBatch
    one_a = SessionBatch(a.cfg, 1, "cuda:0")
    one_b = SessionBatch(a.cfg, 1, "cuda:0")
    import_session(one_a, 0, st)
    import_session(one_b, 0, st2)
    oa = _decode(one_a, 25, seed=9, start=430)
    ob = _decode(one_b, 25, seed=9, start=430)
    for x, y in zip(oa, ob):
        assert torch.equal(x, y)
    for key in ("positions", "importance", "occupied", "ctrl", "counters"):
        assert torch.equal(getattr(one_a, key), getattr(one_b, key)), key
    one_a.check_device_status()


def test_host_stepper_matches_eager_steps():
    """SessionBatch.host_stepper (pinned host buffers, one CUDA graph per step)
    produces the same outputs and cache state as eager steps."""
    a = _batch(3, seed=11)
    b = _batch(3, seed=11)
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(3, 3, 16, 128, generator=g, device="cuda").half()
    k = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    v = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    pos = torch.full((3,), 500, dtype=torch.int64, device="cuda")
    oh = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    st = b.host_stepper(q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory(), oh, pos)
    for i in range(20):
        ref = a.step(q, k, v, torch.full((3,), 500 + i, dtype=torch.int64, device="cuda"))
        st.run(sync=True)
        assert torch.equal(oh, ref.cpu())
    assert int(pos[0]) == 520
    for key in ("positions", "importance", "occupied", "ctrl", "counters"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key


def test_pipelined_host_stepper_matches_eager_steps():
    """The pipelined stepper (output copies on a copy stream, two host
    buffers) delivers every step's output intact."""
    a = _batch(3, seed=13)
    b = _batch(3, seed=13)
    g = torch.Generator(device="cuda").manual_seed(6)
    q = torch.randn(3, 3, 16, 128, generator=g, device="cuda").half()
    k = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    v = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    pos = torch.full((3,), 700, dtype=torch.int64, device="cuda")
    ohs = tuple(torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2))
    st = b.host_stepper(q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory(), ohs, pos)
    refs = [a.step(q, k, v, torch.full((3,), 700 + i, dtype=torch.int64, device="cuda")).cpu() for i in range(12)]
    for i in range(12):
        idx = st.run()
        assert idx == i % 2
        if i % 3 == 2:  # read back some steps right away, let others overlap
            st.wait(idx)
            assert torch.equal(ohs[idx], refs[i])
    st.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(ohs[1], refs[11]) and torch.equal(ohs[0], refs[10])
    for key in ("positions", "importance", "occupied", "ctrl", "counters"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key


def test_packed_input_host_stepper_matches_eager_steps():
    """q / k / v as views of one pinned block: one upload per step, same
    outputs and cache state as eager steps."""
    a = _batch(3, seed=19)
    b = _batch(3, seed=19)
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(3, 3, 16, 128, generator=g, device="cuda").half()
    k = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    v = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    block = torch.empty(q.numel() + k.numel() + v.numel(), dtype=torch.float16).pin_memory()
    qh = block[:q.numel()].view(q.shape)
    kh = block[q.numel():q.numel() + k.numel()].view(k.shape)
    vh = block[q.numel() + k.numel():].view(v.shape)
    qh.copy_(q.cpu()); kh.copy_(k.cpu()); vh.copy_(v.cpu())
    pos = torch.full((3,), 600, dtype=torch.int64, device="cuda")
    ohs = tuple(torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2))
    st = b.host_stepper(qh, kh, vh, ohs, pos)
    assert st.packed_inputs
    for i in range(8):
        ref = a.step(q, k, v, torch.full((3,), 600 + i, dtype=torch.int64, device="cuda")).cpu()
        idx = st.run()
        st.wait(idx)
        assert torch.equal(ohs[idx], ref), i
    for key in ("positions", "importance", "occupied", "ctrl", "counters"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key


def test_zero_copy_host_stepper_matches_eager_steps():
    """The stepper whose kernels read and write the pinned host buffers
    directly (zero_copy) gives the same outputs and cache state as eager
    steps."""
    a = _batch(3, seed=17)
    b = _batch(3, seed=17)
    g = torch.Generator(device="cuda").manual_seed(8)
    q = torch.randn(3, 3, 16, 128, generator=g, device="cuda").half()
    k = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    v = torch.randn(3, 3, 2, 128, generator=g, device="cuda").half()
    pos = torch.full((3,), 900, dtype=torch.int64, device="cuda")
    ohs = tuple(torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2))
    st = b.host_stepper(q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory(), ohs, pos,
                        zero_copy=True)
    assert st.zero_copy
    refs = [a.step(q, k, v, torch.full((3,), 900 + i, dtype=torch.int64, device="cuda")).cpu() for i in range(10)]
    for i in range(10):
        idx = st.run()
        st.wait(idx)
        assert torch.equal(ohs[idx], refs[i]), i
    st.synchronize()
    torch.cuda.synchronize()
    for key in ("positions", "importance", "occupied", "ctrl", "counters"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key
    b.check_device_status()


def test_state_dict_round_trip_and_async_stats():
    """HierarchicalKVCache.state_dict / load_state_dict through host memory,
    and the asynchronous stats readback."""
    import io
    from infercache_b200 import CacheConfig, HierarchicalKVCache
    cfg = CacheConfig(num_layers=2, num_kv_heads=2, head_dim=128, sink_size=2, recent_size=6, important_size=9,
                      dtype=torch.float16)
    a = HierarchicalKVCache(cfg, "cuda:0")
    g = torch.Generator(device="cuda").manual_seed(3)
    pkv = tuple((torch.randn(1, 2, 40, 128, generator=g, device="cuda").half(),
                 torch.randn(1, 2, 40, 128, generator=g, device="cuda").half()) for _ in range(2))
    a.load_from_hf_output(pkv, torch.rand(40, generator=g, device="cuda"))
    for i in range(15):
        a.step(torch.randn(2, 8, 128, generator=g, device="cuda").half(),
               torch.randn(2, 2, 128, generator=g, device="cuda").half(),
               torch.randn(2, 2, 128, generator=g, device="cuda").half(), 40 + i)
    buf = io.BytesIO()
    torch.save(a.state_dict(), buf)
    b = HierarchicalKVCache(cfg, "cuda:0")
    b.load_state_dict(torch.load(io.BytesIO(buf.getvalue())))
    assert torch.equal(a.positions, b.positions) and torch.equal(a.importance, b.importance)
    assert torch.equal(a.occupied, b.occupied) and torch.equal(a.K, b.K) and torch.equal(a.V, b.V)
    assert a.stats == b.stats
    rb = a.batch.stats_async()
    assert rb.result()[0] == a.stats
