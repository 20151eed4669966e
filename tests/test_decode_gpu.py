"""Parity of the CUDA decode path (kernels A and B, tier fill, gathers) with
the oracle and with the reference's golden fixtures.  Every call goes
through the C ABI via the package's classes."""
import numpy as np
import pytest
import torch

import specs
from gpu_protocol import compare_state, make_gpu_cache, run_c1, run_small
from oracle.hier_cache import OracleCache, TierGeometry, decode_step
from oracle.summary import tier_fill
from tolerances import elem_close, rows_close, rows_err

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)


def test_c1_full_protocol(golden):
    """4096-token single-layer fp32 decode: every step's output within 1e-5
    of the oracle, every push event identical, final slot state identical;
    and the same against the reference's own run."""
    cache, oc, events, keep, worst = run_c1(check_every=512)
    g = golden("c1_decode")
    assert np.array_equal(events, g["events"])
    assert cache.stats.total_evictions == 801
    # decisions whose two smallest L2 scores lay within 1e-6 relative: one in the
    # oracle's run; the GPU's sums differ in the last bits, so its count may
    # differ by one while every event above still matches
    assert oc.near_ties == 1 and abs(cache.stats.near_ties - oc.near_ties) <= 1
    pos = cache.positions.cpu().numpy()
    assert np.array_equal(pos, g["positions"])
    assert np.array_equal(cache.occupied.cpu().numpy(), g["occupied"])
    assert elem_close(cache.importance.cpu().numpy(), g["importance"], 1e-5)
    for i, s in enumerate(g["keep_steps"]):
        assert rows_close(keep[int(s)], g["o_keep"][i], 1e-5), s
    assert worst < 1e-5
    cache.batch.check_device_status()


@pytest.mark.parametrize("name", list(specs.SMALL))
def test_small_protocol(golden, name):
    """Primed multi-layer decode (fp32, fp16, GQA 7:1, short prompt)."""
    cache, oc, outs, events = run_small(name)
    g = golden(f"small_decode_{name}")
    rtol = 1e-5 if specs.SMALL[name]["dtype"] == "float32" else 1e-3
    assert np.array_equal(events, g["events"])
    assert rows_close(outs, g["o"], rtol)
    assert np.array_equal(cache.positions.cpu().numpy(), g["positions"])
    cache.batch.check_device_status()


@pytest.mark.parametrize("variant", [0, 3, 5])
def test_wide_budget_vs_oracle(variant):
    """Budget 2048 (4/512/1532) with 28/4 heads: the lean kernel then runs
    eight warp pipelines, one CTA per SM (AUTO), and the streaming kernel."""
    cache, oc, outs, events = run_small("c3_budget", out_dtype=torch.float16, variant=variant)
    cache.batch.check_device_status()


@pytest.mark.parametrize("name", ["f16", "g7"])
@pytest.mark.parametrize("variant", [1, 2, 3, 4, 5])
def test_small_protocol_variants(name, variant):
    """Every kernel-A implementation (CUDA cores; tensor cores with one
    cluster per group; tensor cores streaming a group per CTA; four warp
    pipelines per group; a cluster of CTAs over slot chunks merged through
    distributed shared memory) against the oracle."""
    cache, oc, outs, events = run_small(name, variant=variant)
    cache.batch.check_device_status()


@pytest.mark.parametrize("name", ["f16", "g7", "short_prompt"])
def test_small_protocol_bf16(name):
    """bf16 caches (tensor-core kernel) against the oracle on bf16-rounded inputs."""
    cache, oc, outs, events = run_small(name, dtype="bfloat16")
    cache.batch.check_device_status()


@pytest.mark.parametrize("name", list(specs.TIER))
def test_tier_fill_exact(golden, name):
    """load_from_hf_output slot placement is bit-exact with the reference."""
    sp = specs.TIER[name]
    g = golden(f"tier_fill_{name}")
    scores, positions = specs.tier_inputs(name)
    T = scores.shape[0]
    cache = make_gpu_cache(1, 1, 128, sp["sink"], sp["recent"], sp["important"], torch.float32)
    # K row of token t holds t, so the slot -> token map can be read back
    kk = torch.arange(T, dtype=torch.float32)[None, None, :, None].expand(1, 1, T, 128).contiguous()
    cache.load_from_hf_output(((kk, kk),), scores, positions=positions)
    assert np.array_equal(cache.positions.cpu().numpy(), g["positions"])
    assert np.array_equal(cache.importance.cpu().numpy(), g["importance"])
    assert np.array_equal(cache.occupied.cpu().numpy(), g["occupied"])
    Kl = cache.K[0, 0, :, 0].cpu()
    tok = torch.where(cache.occupied.cpu(), Kl.long(), torch.full_like(Kl.long(), -1))
    assert np.array_equal(tok.numpy(), g["slot_token"])
    st = cache.stats
    assert [st.sink_fill, st.recent_fill, cache._recent_ptr, st.important_fill] == list(g["fills"])
    assert [st.total_tokens_seen, st.total_evictions] == list(g["counters"])


def test_tier_fill_batch_random_ties():
    """Many sessions primed at once, heavy ties, vs the oracle tier fill."""
    from infercache_b200 import CacheConfig, SessionBatch
    from infercache_b200 import _lib
    cfg = CacheConfig(num_layers=1, num_kv_heads=1, head_dim=128, sink_size=4, recent_size=64,
                      important_size=300, dtype=torch.float16)
    S, T = 12, 3000
    b = SessionBatch(cfg, S, "cuda:0")
    g = torch.Generator().manual_seed(21)
    scores = (torch.rand(S, T, generator=g) * 50).round() / 50
    positions = torch.stack([torch.randperm(T + 500, generator=g)[:T] for _ in range(S)])
    slot_token = torch.empty((S, cfg.total_budget), dtype=torch.int32, device="cuda")
    sc, ps = scores.cuda().contiguous(), positions.cuda().contiguous()
    a = _lib.ic_tier_fill_args(tiers=b._c_tiers, sess=b._c_sess, session0=0, n=S, T=T, scores=sc.data_ptr(),
                               positions=ps.data_ptr(), slot_token=slot_token.data_ptr())
    _lib.call("ic_tier_fill", a)
    st = slot_token.cpu().numpy()
    for s in range(S):
        r = tier_fill(scores[s].numpy(), positions[s].numpy(), 4, 64, 300)
        assert np.array_equal(st[s], r["slot_token"]), s
        assert np.array_equal(b.positions[s].cpu().numpy(), r["positions"]), s
        assert int(b.counters[s, 1]) == r["counters"][1]


def test_batch_sessions_vs_oracle():
    """Several sessions in one launch, each checked against its own oracle."""
    from infercache_b200 import CacheConfig, SessionBatch
    L, Hq, Hkv, D = 2, 16, 2, 128
    sink, recent, imp = 4, 16, 12
    S, T0, steps = 5, 60, 90
    cfg = CacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, sink_size=sink, recent_size=recent,
                      important_size=imp, decay=0.99, dtype=torch.float16)
    b = SessionBatch(cfg, S, "cuda:0")
    geo = TierGeometry(L, Hkv, D, sink, recent, imp)
    g = torch.Generator().manual_seed(5)
    ocs = []
    for s in range(S):
        T = T0 + 7 * s
        pk = torch.randn(L, Hkv, T, D, generator=g).half()
        pv = torch.randn(L, Hkv, T, D, generator=g).half()
        sc = torch.rand(T, generator=g)
        b.load_prompt(s, tuple((pk[l][None], pv[l][None]) for l in range(L)), sc)
        oc = OracleCache(geo, np.float16)
        oc.load_from_hf_output(pk.float().numpy(), pv.float().numpy(), sc.numpy())
        ocs.append((oc, T))
    q = torch.randn(steps, L, S, Hq, D, generator=g).half()
    k = torch.randn(steps, L, S, Hkv, D, generator=g).half()
    v = torch.randn(steps, L, S, Hkv, D, generator=g).half()
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    for t in range(steps):
        pos = torch.tensor([ocs[s][1] + t for s in range(S)], dtype=torch.int64, device="cuda")
        o = b.step(qd[t], kd[t], vd[t], pos, out_dtype=torch.float32).cpu().numpy()
        ev = b.events.cpu().numpy()
        for s in range(S):
            oc, T = ocs[s]
            oo, e = decode_step(oc, q[t, :, s].float().numpy(), k[t, :, s].float().numpy(),
                                v[t, :, s].float().numpy(), T + t, 0.99)
            assert rows_close(o[:, s], oo, 1e-3), (t, s, rows_err(o[:, s], oo))
            assert tuple(ev[s]) == e.as_tuple(), (t, s)
    for s in range(S):
        oc, _ = ocs[s]
        assert np.array_equal(b.positions[s].cpu().numpy(), oc.positions)
        assert elem_close(b.importance[s].cpu().numpy(), oc.importance, 1e-3)
    b.check_device_status()


@pytest.mark.parametrize("variant", [2, 3, 4, 5])
def test_config2_full_size(variant):
    """The bench workload at full size: 36 layers, 16 sessions, 16/2 heads,
    budget 4/256/780, fp16, 2048-token prompts.  Session 0 is checked against
    the oracle step by step; all sessions are checked for invariants; a second
    run from the same state reproduces every output bit for bit."""
    from infercache_b200 import CacheConfig, SessionBatch
    L, Hq, Hkv, D, S, T, steps = 36, 16, 2, 128, 16, 2048, 6
    cfg = CacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, sink_size=4, recent_size=256,
                      important_size=780, decay=0.99, dtype=torch.float16)
    g = torch.Generator().manual_seed(1)
    prompts = []

    def build():
        b = SessionBatch(cfg, S, "cuda:0")
        b.kernel_variant = variant
        for s in range(S):
            b.load_prompt(s, tuple((prompts[s][0][l][None].cuda(), prompts[s][1][l][None].cuda())
                                   for l in range(L)), prompts[s][2])
        return b

    for s in range(S):
        prompts.append((torch.randn(L, Hkv, T, D, generator=g).half(), torch.randn(L, Hkv, T, D, generator=g).half(),
                        torch.rand(T, generator=g)))
    q = torch.randn(steps, L, S, Hq, D, generator=g).half()
    k = torch.randn(steps, L, S, Hkv, D, generator=g).half()
    v = torch.randn(steps, L, S, Hkv, D, generator=g).half()
    b1 = build()
    oc = OracleCache(TierGeometry(L, Hkv, D, 4, 256, 780), np.float16)
    oc.load_from_hf_output(prompts[0][0].float().numpy(), prompts[0][1].float().numpy(), prompts[0][2].numpy())
    outs = []
    for t in range(steps):
        o = b1.step(q[t].cuda(), k[t].cuda(), v[t].cuda(), [T + t] * S)
        outs.append(o.clone())
        oo, e = decode_step(oc, q[t, :, 0].float().numpy(), k[t, :, 0].float().numpy(),
                            v[t, :, 0].float().numpy(), T + t, 0.99)
        assert rows_close(o[:, 0].float().cpu().numpy(), oo, 1e-3), t
        assert tuple(b1.events[0].tolist()) == e.as_tuple(), t
    assert np.array_equal(b1.positions[0].cpu().numpy(), oc.positions)
    # invariants on every session
    ntot = cfg.total_budget + 1
    for s in range(S):
        rows = b1.slot_table[s].cpu()
        assert rows.unique().numel() == ntot, "slot table is no longer a permutation of the session's rows"
        pos = b1.positions[s].cpu()
        assert bool(b1.occupied[s].all())
        ring = pos[4:260]
        assert sorted(ring.tolist())[-steps:] == [T + t for t in range(steps)]
        assert pos.unique().numel() == cfg.total_budget
        assert bool((b1.importance[s] >= 0).all())
    # determinism
    b2 = build()
    for t in range(steps):
        o = b2.step(q[t].cuda(), k[t].cuda(), v[t].cuda(), [T + t] * S)
        assert torch.equal(o, outs[t]), t
    assert torch.equal(b1.importance, b2.importance)
    assert torch.equal(b1.slot_table, b2.slot_table)
    b1.check_device_status()


def test_config2_full_size_grouped():
    """The bench workload at full size (36 layers, 16 sessions, budget 1040,
    2048-token prompts) stepped as 8 session ranges on their own streams, from
    device buffers (GroupedStepper) and from host buffers (GroupedHostStepper):
    outputs and metadata bit-identical to the same steps of the whole batch."""
    from infercache_b200 import CacheConfig, SessionBatch
    L, Hq, Hkv, D, S, T = 36, 16, 2, 128, 16, 2048
    cfg = CacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, sink_size=4, recent_size=256,
                      important_size=780, decay=0.99, dtype=torch.float16)
    dev = torch.device("cuda", 0)

    def build():
        gd = torch.Generator(device=dev).manual_seed(5)
        b = SessionBatch(cfg, S, dev)
        for s in range(S):
            pk = torch.randn(L, 1, Hkv, T, D, generator=gd, device=dev).half()
            pv = torch.randn(L, 1, Hkv, T, D, generator=gd, device=dev).half()
            b.load_prompt(s, tuple((pk[l], pv[l]) for l in range(L)), torch.rand(T, generator=gd, device=dev))
        return b

    gd = torch.Generator(device=dev).manual_seed(6)
    q = torch.randn(L, S, Hq, D, generator=gd, device=dev).half()
    k = torch.randn(L, S, Hkv, D, generator=gd, device=dev).half()
    v = torch.randn(L, S, Hkv, D, generator=gd, device=dev).half()
    bs = [build() for _ in range(3)]
    pos = [torch.full((S,), T, dtype=torch.int64, device=dev) for _ in range(3)]
    outs = [torch.empty_like(q) for _ in range(3)]
    for b, p_, o in zip(bs, pos, outs):
        b.step(q, k, v, p_, out=o, advance_positions=True)
    gs = bs[1].grouped_stepper(q, k, v, outs[1], pos[1], groups=8, steps_per_graph=4)
    gh = bs[2].grouped_host_stepper(pos[2], num_q_heads=Hq, groups=8)
    gh.load_inputs(q.cpu(), k.cpu(), v.cpu())
    gs.run(2)
    gh.run(8)
    for _ in range(8):
        bs[0].step(q, k, v, pos[0], out=outs[0], advance_positions=True)
    gh.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0].cpu(), gh.outputs())
    for b in bs[1:]:
        for key in ("positions", "importance", "occupied", "slot_table", "ctrl", "counters", "events", "mass"):
            assert torch.equal(getattr(bs[0], key), getattr(b, key)), key
    assert pos[0].tolist() == [T + 9] * S and torch.equal(pos[0], pos[1]) and torch.equal(pos[0], pos[2])
    for b in bs:
        b.check_device_status()


def test_step_advancing_positions_in_kernel():
    """advance_positions: kernel B adds one to every session's position after
    reading it; steps driven that way match steps given explicit positions."""
    from infercache_b200 import CacheConfig, SessionBatch
    cfg = CacheConfig(num_layers=2, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=8, important_size=12,
                      decay=0.99, dtype=torch.float16)
    g = torch.Generator().manual_seed(23)
    pk = torch.randn(2, 2, 2, 50, 128, generator=g).half()
    pv = torch.randn(2, 2, 2, 50, 128, generator=g).half()
    sc = torch.rand(50, generator=g)
    bs = []
    for _ in range(2):
        b = SessionBatch(cfg, 2, "cuda:0")
        for s in range(2):
            b.load_prompt(s, tuple((pk[l][s][None].cuda(), pv[l][s][None].cuda()) for l in range(2)), sc)
        bs.append(b)
    q = torch.randn(6, 2, 2, 16, 128, generator=g).half().cuda()
    k = torch.randn(6, 2, 2, 2, 128, generator=g).half().cuda()
    v = torch.randn(6, 2, 2, 2, 128, generator=g).half().cuda()
    pos = torch.tensor([50, 70], dtype=torch.int64, device="cuda")
    for t in range(6):
        o1 = bs[0].step(q[t], k[t], v[t], [50 + t, 70 + t])
        o2 = bs[1].step(q[t], k[t], v[t], pos, advance_positions=True)
        assert torch.equal(o1, o2), t
    assert pos.tolist() == [56, 76]
    for key in ("positions", "importance", "occupied", "slot_table", "counters"):
        assert torch.equal(getattr(bs[0], key), getattr(bs[1], key)), key
    with pytest.raises(ValueError):
        bs[1].step(q[0], k[0], v[0], [1, 2], advance_positions=True)


@pytest.mark.parametrize("groups", [1, 2, 3, 5])
def test_grouped_stepper_matches_steps(groups):
    """Session ranges on their own streams and graphs (GroupedStepper) give
    bit-identical outputs and metadata to the same steps of the whole batch."""
    from infercache_b200 import CacheConfig, SessionBatch
    S, L, T = 5, 2, 60
    cfg = CacheConfig(num_layers=L, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=8, important_size=12,
                      decay=0.99, dtype=torch.float16)
    g = torch.Generator().manual_seed(31)
    pk = torch.randn(L, S, 2, T, 128, generator=g).half()
    pv = torch.randn(L, S, 2, T, 128, generator=g).half()
    sc = torch.rand(T, generator=g)
    bs = []
    for _ in range(2):
        b = SessionBatch(cfg, S, "cuda:0")
        for s in range(S):
            b.load_prompt(s, tuple((pk[l][s][None].cuda(), pv[l][s][None].cuda()) for l in range(L)), sc)
        bs.append(b)
    q = torch.randn(L, S, 16, 128, generator=g).half().cuda()
    k = torch.randn(L, S, 2, 128, generator=g).half().cuda()
    v = torch.randn(L, S, 2, 128, generator=g).half().cuda()
    pos0 = torch.arange(T, T + S, dtype=torch.int64, device="cuda")
    pos1 = pos0.clone()
    o0 = torch.empty_like(q)
    o1 = torch.empty_like(q)
    bs[0].step(q, k, v, pos0, out=o0, advance_positions=True)  # kernels configured before capture
    bs[1].step(q, k, v, pos1, out=o1, advance_positions=True)
    st = bs[1].grouped_stepper(q, k, v, o1, pos1, groups=groups, steps_per_graph=2)
    assert len(st.ranges) == groups and st.launches_per_step == groups * (L + 1)
    st.run(3)
    for _ in range(6):
        bs[0].step(q, k, v, pos0, out=o0, advance_positions=True)
    torch.cuda.synchronize()
    assert torch.equal(o0, o1)
    assert torch.equal(pos0, pos1) and pos1.tolist() == list(range(T + 7, T + 7 + S))
    for key in ("positions", "importance", "occupied", "slot_table", "ctrl", "counters", "events", "mass"):
        assert torch.equal(getattr(bs[0], key), getattr(bs[1], key)), key


@pytest.mark.parametrize("groups", [1, 3, 5])
def test_grouped_host_stepper_matches_steps(groups):
    """Session ranges driven from range-major pinned host buffers on their own
    streams (GroupedHostStepper) give the outputs and metadata of the same
    steps run through SessionBatch.step, bit for bit."""
    from infercache_b200 import CacheConfig, SessionBatch
    S, L, T = 5, 2, 60
    cfg = CacheConfig(num_layers=L, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=8, important_size=12,
                      decay=0.99, dtype=torch.float16)
    g = torch.Generator().manual_seed(37)
    pk = torch.randn(L, S, 2, T, 128, generator=g).half()
    pv = torch.randn(L, S, 2, T, 128, generator=g).half()
    sc = torch.rand(T, generator=g)
    bs = []
    for _ in range(2):
        b = SessionBatch(cfg, S, "cuda:0")
        for s in range(S):
            b.load_prompt(s, tuple((pk[l][s][None].cuda(), pv[l][s][None].cuda()) for l in range(L)), sc)
        bs.append(b)
    q = torch.randn(L, S, 16, 128, generator=g).half()
    k = torch.randn(L, S, 2, 128, generator=g).half()
    v = torch.randn(L, S, 2, 128, generator=g).half()
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    pos0 = torch.arange(T, T + S, dtype=torch.int64, device="cuda")
    pos1 = pos0.clone()
    o0 = torch.empty_like(qd)
    bs[0].step(qd, kd, vd, pos0, out=o0, advance_positions=True)
    bs[1].step(qd, kd, vd, pos1, out=torch.empty_like(qd), advance_positions=True)
    gh = bs[1].grouped_host_stepper(pos1, num_q_heads=16, groups=groups)
    assert len(gh.ranges) == groups
    assert gh.h2d_bytes == (q.numel() + k.numel() + v.numel()) * 2 and gh.d2h_bytes == q.numel() * 2
    gh.load_inputs(q, k, v)
    gh.run(4)
    gh.synchronize()
    for _ in range(4):
        bs[0].step(qd, kd, vd, pos0, out=o0, advance_positions=True)
    torch.cuda.synchronize()
    assert torch.equal(gh.outputs(), o0.cpu())
    assert torch.equal(pos0, pos1)
    for key in ("positions", "importance", "occupied", "slot_table", "ctrl", "counters", "events", "mass"):
        assert torch.equal(getattr(bs[0], key), getattr(bs[1], key)), key


def test_grouped_stepper_rejects_bad_arguments():
    from infercache_b200 import CacheConfig, SessionBatch
    cfg = CacheConfig(num_layers=1, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=8, important_size=12,
                      dtype=torch.float16)
    b = SessionBatch(cfg, 2, "cuda:0")
    q = torch.zeros(1, 2, 16, 128, dtype=torch.float16, device="cuda")
    kv = torch.zeros(1, 2, 2, 128, dtype=torch.float16, device="cuda")
    pos = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        b.grouped_stepper(q, kv, kv, torch.empty_like(q), pos, groups=3)
    with pytest.raises(ValueError):
        b.grouped_stepper(q, kv, kv, torch.empty_like(q), pos.int(), groups=1)
    with pytest.raises(ValueError):
        b.grouped_stepper(q.float(), kv, kv, torch.empty_like(q), pos, groups=1)


def test_cluster_sizes_agree():
    """8- and 16-CTA clusters differ only in float summation order."""
    from infercache_b200 import CacheConfig, SessionBatch
    cfg = CacheConfig(num_layers=2, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=256,
                      important_size=780, dtype=torch.float16)
    g = torch.Generator().manual_seed(3)
    T = 1500
    pk = torch.randn(2, 2, T, 128, generator=g).half()
    sc = torch.rand(T, generator=g)
    q = torch.randn(2, 3, 16, 128, generator=g).half().cuda()
    kv = torch.randn(2, 3, 2, 128, generator=g).half().cuda()
    res = []
    for cl in (8, 16):
        b = SessionBatch(cfg, 3, "cuda:0")
        b.cluster_size = cl
        for s in range(3):
            b.load_prompt(s, tuple((pk[l][None], pk[l][None]) for l in range(2)), sc)
        o = b.step(q, kv, kv, [T] * 3, out_dtype=torch.float32)
        res.append((o.cpu().numpy(), b.events.cpu().numpy(), b.importance.cpu().numpy()))
    assert rows_close(res[0][0], res[1][0], 1e-5)
    assert np.array_equal(res[0][1], res[1][1])
    assert elem_close(res[0][2], res[1][2], 1e-5)


def test_push_reference_path():
    """The reference-compatible push(key, value, position, attn_weights): mean
    over (layers, heads, queries) added in position order, no decay."""
    L, Hkv, D = 2, 2, 128
    cache = make_gpu_cache(L, Hkv, D, 2, 5, 4, torch.float32)
    geo = TierGeometry(L, Hkv, D, 2, 5, 4)
    oc = OracleCache(geo, np.float32)
    g = torch.Generator().manual_seed(11)
    T = 14
    pk = torch.randn(L, Hkv, T, D, generator=g)
    sc = torch.rand(T, generator=g)
    cache.load_from_hf_output(tuple((pk[l][None], pk[l][None]) for l in range(L)), sc)
    oc.load_from_hf_output(pk.numpy(), pk.numpy(), sc.numpy())
    for t in range(40):
        kk = torch.randn(L, Hkv, 1, D, generator=g)
        F = int(cache.occupied.sum())
        w = None
        if t % 5 != 4:   # every fifth push carries no weights (the shipped two_pass loop)
            w = torch.rand(L, Hkv, 2, F + (t % 3) - 1, generator=g)  # widths F-1, F, F+1
        cache.push(kk, kk, position=T + t, attn_weights=w)
        e = oc.push(kk[:, :, 0].numpy(), kk[:, :, 0].numpy(), T + t, None if w is None else w.numpy())
        assert cache.last_event() == e.as_tuple(), t
        compare_state(cache, oc, 1e-6, f"push {t}")
    # to_hf export and position ids
    hf = cache.to_hf_past_key_values()
    ref = oc.to_hf_past_key_values()
    from infercache_b200.cache_safety import normalise_kv
    for (K, V), (Ko, Vo) in zip(normalise_kv(hf), ref):
        assert np.array_equal(K.cpu().numpy(), Ko)
        assert np.array_equal(V.cpu().numpy(), Vo)
    assert np.array_equal(cache.get_position_ids_for_cache().cpu().numpy(), oc.get_position_ids_for_cache())
    cache.reset()
    assert cache.current_fill == 0 and not bool(cache.occupied.any())
    assert float(cache.K.abs().sum()) == 0.0


def test_evict_kernel_ties_exact():
    """Kernel B alone on crafted scores: equal minima are evicted lowest slot
    first, a displaced score equal to the minimum is rejected, and the update
    is importance * decay + mass / div with each step rounded."""
    from infercache_b200 import CacheConfig, SessionBatch
    from infercache_b200 import _lib
    cfg = CacheConfig(num_layers=3, num_kv_heads=2, head_dim=128, sink_size=2, recent_size=3,
                      important_size=6, decay=0.5, dtype=torch.float16)
    b = SessionBatch(cfg, 2, "cuda:0")
    B = cfg.total_budget
    # session 0: L2 full with a tied minimum at slots 7 and 9; ring slot 2 holds score 3
    imp = torch.tensor([[9., 9., 3., 5., 5., 8., 4., 2., 6., 2., 7.],
                        [9., 9., 1., 5., 5., 8., 4., 2., 6., 2., 7.]])
    b.importance.copy_(imp)
    b.occupied.fill_(True)
    b.positions.copy_(torch.arange(B).repeat(2, 1) + 100)
    b.ctrl[:, _lib.IC_CTRL_RECENT_FILL] = 3
    b.ctrl[:, _lib.IC_CTRL_IMPORTANT_FILL] = 6
    b.ctrl[:, _lib.IC_CTRL_RECENT_PTR] = 2
    b.mass.zero_()
    rows0 = b.slot_table.clone()
    b.evict([500, 501], decay=1.0)
    ev = b.events.cpu().tolist()
    # session 0: score 3 > min 2 at slot 7 (first of the tie) -> evict slot 7
    assert ev[0] == [3, 102, 7, 107]
    # session 1: score 1 <= min 2 -> reject, target is still the first minimum
    assert ev[1] == [4, 102, 7, -1]
    # both decisions rested on an exact tie of the two smallest L2 scores
    assert b.counters[:, _lib.IC_CNT_NEAR_TIES].tolist() == [1, 1]
    assert b.stats(0).near_ties == 1
    st = b.slot_table.cpu()
    assert st[0, 7] == rows0[0, 2] and st[0, 2] == rows0[0, B] and st[0, B] == rows0[0, 7]
    assert st[1, 2] == rows0[1, B] and st[1, B] == rows0[1, 2]
    assert b.positions[0, 2].item() == 500 and b.positions[0, 7].item() == 102
    # decay + mass arithmetic on one session, rounded step by step: the layer
    # columns [S, Hkv, slot, layer] summed in layer order, then the heads
    g = torch.Generator().manual_seed(2)
    m = torch.rand(2, 2, B + 1, 3, generator=g)
    mcol = m.to("cuda").contiguous()
    before = b.importance.clone()
    npos = torch.tensor([600, 601], device="cuda")
    e = _lib.ic_evict_args(tiers=b._c_tiers, sess=b._c_sess, mass=mcol.data_ptr(), mass_heads=2, mass_layers=3,
                           mass_div=6.0, decay=0.75, pdl=0, new_pos=npos.data_ptr(), events=b.events.data_ptr())
    _lib.call("ic_evict_update", e)
    torch.cuda.synchronize()
    mn = m.numpy()
    heads = [((mn[:, hh, :B, 0] + mn[:, hh, :B, 1]) + mn[:, hh, :B, 2]).astype(np.float32) for hh in range(2)]
    want = (before.cpu().numpy() * np.float32(0.75)).astype(np.float32) + \
           ((heads[0] + heads[1]) / np.float32(6.0)).astype(np.float32)
    got = b.importance.cpu().numpy()
    ev2 = b.events.cpu().numpy()
    mask = np.ones_like(got, bool)
    for s in range(2):
        mask[s, 3] = False  # slot 3 is the new ring slot of this step (reset to 0)
        if ev2[s, 0] in (2, 3):  # promotion target now holds the displaced score
            mask[s, ev2[s, 2]] = False
            assert got[s, ev2[s, 2]] == want[s, 3]
    assert np.array_equal(got[mask], want.astype(np.float32)[mask])


@pytest.mark.parametrize("ml,mh", [(1, 4), (1, 8), (5, 3), (8, 2)])
def test_evict_mass_layouts(ml, mh):
    """Kernel B's importance update for each mass layout it handles: one column
    per KV head (the decode step's; loads batched per thread), columns of a few
    layers, and many layers (a separate wide update kernel first), over a budget
    of more than two slots per thread: importance * decay + (sum over layers in
    order, then heads in order) / div, each step rounded, on every occupied slot
    but the ones the step rewrites."""
    from infercache_b200 import CacheConfig, SessionBatch
    from infercache_b200 import _lib
    cfg = CacheConfig(num_layers=2, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=64,
                      important_size=1100, decay=0.9, dtype=torch.float16)
    S = 3
    b = SessionBatch(cfg, S, "cuda:0")
    B = cfg.total_budget
    g = torch.Generator().manual_seed(40 + ml)
    imp = torch.rand(S, B, generator=g) + 0.5
    occ = torch.rand(S, B, generator=g) < 0.9
    b.importance.copy_(imp)
    b.occupied.copy_(occ)
    b.positions.copy_(torch.arange(B).repeat(S, 1) + 10)
    b.ctrl[:, _lib.IC_CTRL_RECENT_FILL] = cfg.recent_size
    b.ctrl[:, _lib.IC_CTRL_IMPORTANT_FILL] = cfg.important_size
    b.ctrl[:, _lib.IC_CTRL_RECENT_PTR] = 7
    m = torch.rand(S, mh, B + 1, ml, generator=g)
    mcol = m.to("cuda").contiguous()
    npos = torch.arange(S, device="cuda", dtype=torch.int64) + 5000
    div = float(ml * mh)
    e = _lib.ic_evict_args(tiers=b._c_tiers, sess=b._c_sess, mass=mcol.data_ptr(), mass_heads=mh, mass_layers=ml,
                           mass_div=div, decay=0.9, pdl=0, new_pos=npos.data_ptr(), events=b.events.data_ptr())
    _lib.call("ic_evict_update", e)
    torch.cuda.synchronize()
    b.check_device_status()
    mn = m.numpy()
    tot = None
    for hh in range(mh):
        acc = mn[:, hh, :B, 0].astype(np.float32)
        for l in range(1, ml):
            acc = (acc + mn[:, hh, :B, l]).astype(np.float32)
        tot = acc if tot is None else (tot + acc).astype(np.float32)
    want = ((imp.numpy() * np.float32(0.9)).astype(np.float32) + (tot / np.float32(div)).astype(np.float32))
    want = np.where(occ.numpy(), want.astype(np.float32), imp.numpy())
    got = b.importance.cpu().numpy()
    ev = b.events.cpu().numpy()
    mask = np.ones_like(got, bool)
    for s_ in range(S):
        mask[s_, 7] = False  # the ring slot the step rewrites
        if ev[s_, 0] in (2, 3):
            mask[s_, ev[s_, 2]] = False
            assert got[s_, ev[s_, 2]] == want[s_, 7]
    assert np.array_equal(got[mask], want[mask])


def test_paged_trace_gpu(golden):
    """MultiSessionCache / KVAllocator / PagePool against the reference trace."""
    import json
    from infercache_b200 import MultiSessionCache, PagePool, PagedCacheConfig
    sp = specs.PAGED
    g = golden("paged_trace")
    ticks = iter(range(1, 10 ** 6))
    cfg = PagedCacheConfig(n_pages=sp["n_pages"], n_layers=sp["layers"], n_heads=sp["heads"], head_dim=sp["d"],
                           dtype=torch.float32, device="cuda:0", max_pages_per_session=sp["max_pps"])
    msc = MultiSessionCache(PagePool(cfg), clock=lambda: float(next(ticks)))
    gathers = []
    for i, op in enumerate(specs.paged_ops()):
        err = ""
        try:
            if op[0] == "push":
                _, sid, n, seed = op
                kk, vv = specs.paged_tokens(n, seed)
                view = msc.get_or_create(sid)
                view.push(kk, vv, positions=list(range(view.n_tokens, view.n_tokens + n)),
                          importance=[float(x) for x in np.linspace(0, 1, n)])
            elif op[0] == "gather":
                K, V = msc.get_or_create(op[1]).gather(op[2])
                gathers.append(np.concatenate([K.cpu().numpy().ravel(), V.cpu().numpy().ravel()]))
            elif op[0] == "reset":
                msc.reset(op[1])
            elif op[0] == "touch":
                msc.allocator.touch(op[1])
        except RuntimeError as e:
            err = str(e)
        assert err == str(g["errors"][i]), (i, op)
        pages = {s: msc.allocator.pages_for(s) for s in sorted(msc.active_sessions())}
        assert pages == json.loads(str(g["pages"][i])), (i, op)
        assert abs(msc.utilization() - float(g["util"][i])) < 1e-12
    assert np.array_equal(np.concatenate(gathers), g["gathers"])


def test_batched_page_push_and_gather_match_per_session_calls():
    """MultiSessionCache.push_many / gather_many (one launch per 32 sessions)
    against push / gather_all session by session on a second pool: the same
    allocator state and gathered bytes after every call, over 40 sessions (two
    launches per call), empty pushes and sessions, and one-token decode pushes.
    The prompts overfill the pool, so later sessions of the first call evict
    earlier ones (already pushed in that call); a third of the rest then leave,
    so the decode calls evict nobody (a session evicted before its own push in
    the same call would write stale pages in the per-session loop)."""
    from infercache_b200 import MultiSessionCache, PagePool, PagedCacheConfig
    rng = np.random.default_rng(11)

    def make():
        cfg = PagedCacheConfig(n_pages=160, n_layers=3, n_heads=2, head_dim=128, dtype=torch.float16,
                               device="cuda:0", max_pages_per_session=12)
        ticks = iter(range(1, 10 ** 6))
        return MultiSessionCache(PagePool(cfg), clock=lambda: float(next(ticks)))

    seq, bat = make(), make()
    sids = [f"s{i}" for i in range(40)]
    g = torch.Generator(device="cuda:0").manual_seed(5)
    for call in range(8):
        lens = [0 if i == 3 else (int(rng.integers(40, 120)) if call == 0 else int(rng.integers(0, 3)))
                for i in range(len(sids))]
        ks = [torch.randn(3, 2, n, 128, generator=g, device="cuda:0").half() for n in lens]
        vs = [torch.randn(3, 2, n, 128, generator=g, device="cuda:0").half() for n in lens]
        errs = []
        for sid, k, v in zip(sids, ks, vs):
            try:
                seq.get_or_create(sid).push(k, v, positions=[], importance=[])
                errs.append(None)
            except RuntimeError as e:
                errs.append(str(e))
        got = [None if e is None else str(e) for e in bat.push_many(sids, ks, vs)]
        assert got == errs, call
        assert seq.allocator.free_list() == bat.allocator.free_list(), call
        live = [sid for sid in sids if seq.allocator.pages_for(sid)]
        for sid in sids:
            assert seq.allocator.pages_for(sid) == bat.allocator.pages_for(sid), (call, sid)
        many = bat.gather_many(live)
        if call % 2:  # into caller buffers carved from one flat tensor
            flat = torch.full((sum(2 * K.numel() + 128 for K, _ in many),), 7.0, dtype=torch.float16,
                              device="cuda:0")
            outs, off = [], 0
            for K, _ in many:
                pair = []
                for _ in range(2):
                    pair.append(flat[off:off + K.numel()].view(K.shape))
                    off = (off + K.numel() + 63) // 64 * 64
                outs.append(tuple(pair))
            many = bat.gather_many(live, out=outs)
            assert all(a is b for pr, pb in zip(many, outs) for a, b in zip(pr, pb))
        for sid, (K, V) in zip(live, many):
            K0, V0 = seq.get_or_create(sid).gather_all()
            assert torch.equal(K, K0) and torch.equal(V, V0), (call, sid)
        gone = [s_ for s_ in sids if s_ not in live] + (live[::3] if call == 0 else [])
        for sid in gone:  # evicted sessions start again, as the stress workload's do
            seq.reset(sid)
            bat.reset(sid)
        if call == 0:
            evictions = bat.allocator.lru_evictions
            assert evictions > 0
    assert bat.allocator.lru_evictions == evictions
    torch.cuda.synchronize()


def _random_spec(i):
    r = np.random.default_rng(1000 + i)
    hkv = int(r.integers(1, 3))
    return dict(layers=int(r.integers(1, 3)), hq=hkv * int(r.integers(1, 9)), hkv=hkv, d=128,
                sink=int(r.integers(0, 5)), recent=int(r.integers(1, 13)), important=int(r.integers(1, 21)),
                prompt=int(r.integers(1, 61)), steps=30, decay=float(r.choice([0.99, 0.9, 1.0])),
                dtype=["float32", "float16"][i % 2], seed=2000 + i)


@pytest.mark.parametrize("i", range(12))
def test_random_small_configs_vs_oracle(i):
    """Small random tier geometries (empty sink, ring of one, importance tier
    of one, prompts shorter than the budget, ties in the prompt scores, decay 1)
    through the fused step: events exact, outputs and importance within the
    dtype's tolerance, every step."""
    cache, oc, outs, events = run_small(_random_spec(i), out_dtype=torch.float32)
    cache.batch.check_device_status()


def _c2_prompts(L, Hkv, D, S, T, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(L, Hkv, T, D, generator=g).half(), torch.randn(L, Hkv, T, D, generator=g).half(),
             torch.rand(T, generator=g)) for _ in range(S)], g


@pytest.mark.parametrize("variant,knob", [(0, 0), (5, 8), (5, 14)])
def test_attend_layer_at_a_time_vs_oracle(variant, knob):
    """One layer at a time, as a decoder forward calls it (attend per layer,
    q of a layer only after the previous layer: no inputs_ready), which runs
    the slot-split kernel (a cluster of CTAs merging through distributed shared
    memory, cluster_size = knob): the bench
    workload's shapes (36 layers, 16 sessions, 16/2 heads, budget 4/256/780,
    fp16, 2048-token prompts).  Session 0 against the oracle step by step;
    every session against the one-cluster-per-group kernel (events equal,
    outputs and importance within 1e-3); a second run reproduces every output
    bit for bit (the chunks are merged in chunk order)."""
    from infercache_b200 import CacheConfig, SessionBatch
    from infercache_b200 import _lib
    L, Hq, Hkv, D, S, T, steps = 36, 16, 2, 128, 16, 2048, 4
    cfg = CacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, sink_size=4, recent_size=256,
                      important_size=780, decay=0.99, dtype=torch.float16)
    prompts, g = _c2_prompts(L, Hkv, D, S, T, 7)
    q = torch.randn(steps, L, S, Hq, D, generator=g).half().cuda()
    k = torch.randn(steps, L, S, Hkv, D, generator=g).half().cuda()
    v = torch.randn(steps, L, S, Hkv, D, generator=g).half().cuda()

    def build(variant):
        b = SessionBatch(cfg, S, "cuda:0")
        b.kernel_variant = variant
        if variant == _lib.IC_DECODE_TENSOR_SPLIT:
            b.cluster_size = knob
        for s in range(S):
            b.load_prompt(s, tuple((prompts[s][0][l][None].cuda(), prompts[s][1][l][None].cuda())
                                   for l in range(L)), prompts[s][2])
        return b

    def run(b, oc=None):
        outs, evs = [], []
        for t in range(steps):
            o = torch.empty(L, S, Hq, D, dtype=torch.float16, device="cuda:0")
            for l in range(L):
                b.attend(l, q[t, l], k[t, l], v[t, l], out=o[l])
            b.evict([T + t] * S)
            outs.append(o)
            evs.append(b.events.clone())
            if oc is not None:
                oo, e = decode_step(oc, q[t, :, 0].float().cpu().numpy(), k[t, :, 0].float().cpu().numpy(),
                                    v[t, :, 0].float().cpu().numpy(), T + t, 0.99)
                assert rows_close(o[:, 0].float().cpu().numpy(), oo, 1e-3), t
                assert tuple(b.events[0].tolist()) == e.as_tuple(), t
        return outs, evs

    b1 = build(variant)
    oc = OracleCache(TierGeometry(L, Hkv, D, 4, 256, 780), np.float16)
    oc.load_from_hf_output(prompts[0][0].float().numpy(), prompts[0][1].float().numpy(), prompts[0][2].numpy())
    outs1, evs1 = run(b1, oc)
    assert np.array_equal(b1.positions[0].cpu().numpy(), oc.positions)
    assert elem_close(b1.importance[0].cpu().numpy(), oc.importance, 1e-3)
    b1.check_device_status()
    # the cluster kernel on the same steps
    b2 = build(_lib.IC_DECODE_TENSOR_CORES)
    outs2, evs2 = run(b2)
    for t in range(steps):
        assert rows_close(outs1[t].float().cpu().numpy(), outs2[t].float().cpu().numpy(), 1e-3), t
        assert torch.equal(evs1[t], evs2[t]), t
    assert torch.equal(b1.slot_table, b2.slot_table)
    assert elem_close(b1.importance.cpu().numpy(), b2.importance.cpu().numpy(), 1e-3)
    # bit-for-bit reproducible
    b3 = build(variant)
    outs3, _ = run(b3)
    for t in range(steps):
        assert torch.equal(outs1[t], outs3[t]), t
    assert torch.equal(b1.importance, b3.importance)
    b3.check_device_status()


@pytest.mark.parametrize("dtype,hq,S,recent,important,T", [
    ("float16", 32, 16, 256, 780, 1200), ("bfloat16", 32, 16, 256, 780, 1200),
    ("float16", 16, 8, 512, 1532, 2200), ("bfloat16", 32, 8, 512, 1532, 2200)])
def test_attend_split_default_geometry_two_head_blocks(dtype, hq, S, recent, important, T):
    """The slot-split kernel's default geometry (the fewest CTAs per group that
    fit with 64 CTAs or more; two 16-slot blocks per warp, one CTA per SM): at
    budget 1040 with 32 groups and 16 query heads per KV head (two n = 8
    blocks), and at budget 2048 with 16 groups (6 CTAs per group of eleven
    warps; 7 with two head blocks, whose shared memory rules 6 out), fp16 and
    bf16: outputs (fp32) within 1e-3 of the one-cluster-per-group kernel,
    identical events, slot tables and positions, importance within 1e-3, and a
    second run bit for bit."""
    from infercache_b200 import CacheConfig, SessionBatch
    from infercache_b200 import _lib
    L, Hq, Hkv, D, steps = 4, hq, 2, 128, 3
    dt = torch.float16 if dtype == "float16" else torch.bfloat16
    cfg = CacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, sink_size=4, recent_size=recent,
                      important_size=important, decay=0.99, dtype=dt)
    g = torch.Generator().manual_seed(21)
    prompts = [(torch.randn(L, Hkv, T, D, generator=g).to(dt), torch.randn(L, Hkv, T, D, generator=g).to(dt),
                torch.rand(T, generator=g)) for _ in range(S)]
    q = torch.randn(steps, L, S, Hq, D, generator=g).to(dt).cuda()
    k = torch.randn(steps, L, S, Hkv, D, generator=g).to(dt).cuda()
    v = torch.randn(steps, L, S, Hkv, D, generator=g).to(dt).cuda()

    def run(variant):
        b = SessionBatch(cfg, S, "cuda:0")
        b.kernel_variant = variant
        for s_ in range(S):
            b.load_prompt(s_, tuple((prompts[s_][0][l][None].cuda(), prompts[s_][1][l][None].cuda())
                                    for l in range(L)), prompts[s_][2])
        outs, evs = [], []
        for t in range(steps):
            o = torch.empty(L, S, Hq, D, dtype=torch.float32, device="cuda:0")
            for l in range(L):
                b.attend(l, q[t, l], k[t, l], v[t, l], out=o[l])
            b.evict([T + t] * S)
            outs.append(o)
            evs.append(b.events.clone())
        torch.cuda.synchronize()
        b.check_device_status()
        return b, outs, evs

    b1, outs1, evs1 = run(_lib.IC_DECODE_AUTO)
    b2, outs2, evs2 = run(_lib.IC_DECODE_TENSOR_CORES)
    for t in range(steps):
        assert rows_close(outs1[t].cpu().numpy(), outs2[t].cpu().numpy(), 1e-3), t
        assert torch.equal(evs1[t], evs2[t]), t
    assert torch.equal(b1.slot_table, b2.slot_table) and torch.equal(b1.positions, b2.positions)
    assert elem_close(b1.importance.cpu().numpy(), b2.importance.cpu().numpy(), 1e-3)
    b3, outs3, _ = run(_lib.IC_DECODE_AUTO)
    for t in range(steps):
        assert torch.equal(outs1[t], outs3[t]), t
    assert torch.equal(b1.importance, b3.importance)


def run_small_attend(sp, dtype, variant=0):
    """run_small with each step taken layer by layer through attend()."""
    from gpu_protocol import TORCH_DT
    dt = TORCH_DT[dtype]
    pk, pv, scores, q, k, v = specs.small_inputs(sp)
    pk, pv, q, k, v = (t.to(dt).float() for t in (pk, pv, q, k, v))
    cache = make_gpu_cache(sp["layers"], sp["hkv"], sp["d"], sp["sink"], sp["recent"], sp["important"], dt,
                           sp["decay"])
    cache.batch.kernel_variant = variant
    oc = OracleCache(TierGeometry(sp["layers"], sp["hkv"], sp["d"], sp["sink"], sp["recent"], sp["important"]),
                     np.float32)
    cache.load_from_hf_output(tuple((pk[l][None].to(dt), pv[l][None].to(dt)) for l in range(sp["layers"])), scores)
    oc.load_from_hf_output(pk.numpy(), pv.numpy(), scores.numpy())
    T = pk.shape[2]
    qd, kd, vd = q.to(dt).cuda(), k.to(dt).cuda(), v.to(dt).cuda()
    outs, events = [], []
    for s in range(sp["steps"]):
        o = torch.stack([cache.attend(l, qd[s, l], kd[s, l], vd[s, l], out_dtype=torch.float32)
                         for l in range(sp["layers"])])
        cache.evict(T + s)
        oo, ev = decode_step(oc, q[s].numpy(), k[s].numpy(), v[s].numpy(), T + s, sp["decay"])
        g = o.float().cpu().numpy()
        assert rows_close(g, oo, 1e-3), f"output differs at step {s}: {rows_err(g, oo)}"
        assert cache.last_event() == ev.as_tuple(), s
        compare_state(cache, oc, 1e-3, f"step {s}")
        outs.append(g)
        events.append(cache.last_event())
    return cache, oc, np.stack(outs), np.array(events, np.int64)


@pytest.mark.parametrize("variant", [0, 5])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("hq", [8, 32])
def test_attend_split_kernel_small(dtype, hq, variant):
    """The slot-split kernel layer at a time on a small primed cache, with 4
    and 16 query heads per KV head (one and two n = 8 blocks), fp16 and bf16,
    against the oracle on inputs rounded to the cache dtype."""
    sp = dict(specs.SMALL["f16"])
    sp.update(hq=hq, hkv=2)
    cache, oc, outs, events = run_small_attend(sp, dtype, variant)
    cache.batch.check_device_status()


def test_device_timeout_is_reported_and_context_survives():
    """A bounded device-side wait that runs out (ic_wait_probe: an mbarrier
    phase nothing completes, 50 ms limit) sets IC_DEVFLAG_TIMEOUT; the host
    maps it to IC_ERR_DEVICE_TIMEOUT; the context stays usable, so after the
    flag is cleared the cache decodes and checks clean."""
    import ctypes
    from infercache_b200 import _lib
    cache = make_gpu_cache(2, 2, 128, 2, 5, 4, torch.float16)
    b = cache.batch
    lib = _lib.load()
    rc = lib.ic_wait_probe(ctypes.c_void_p(b.dev_status.data_ptr()), 50_000_000,
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.IC_OK
    torch.cuda.synchronize()
    assert int(b.dev_status.item()) & _lib.IC_DEVFLAG_TIMEOUT
    with pytest.raises(_lib.InferCacheError) as ei:
        b.check_device_status()
    assert ei.value.status == _lib.IC_ERR_DEVICE_TIMEOUT
    b.dev_status.zero_()
    g = torch.Generator().manual_seed(4)
    pk = torch.randn(2, 2, 12, 128, generator=g).half()
    cache.load_from_hf_output(tuple((pk[l][None], pk[l][None]) for l in range(2)), torch.rand(12, generator=g))
    q = torch.randn(2, 4, 128, generator=g).half().cuda()
    kv = torch.randn(2, 2, 128, generator=g).half().cuda()
    o = cache.step(q, kv, kv, 12)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    b.check_device_status()


def test_batched_append_matches_per_session_push():
    """SessionBatch.append (every session's token in one launch, kernel B
    without a boost) leaves exactly the state of the reference-compatible
    push(key, value, position) without weights called session by session,
    over enough steps that ring tokens are dropped for a zero score."""
    from infercache_b200 import CacheConfig, SessionBatch
    cfg = CacheConfig(num_layers=3, num_kv_heads=2, head_dim=128, sink_size=2, recent_size=6, important_size=5,
                      dtype=torch.float16)
    S, L = 4, 3
    g = torch.Generator().manual_seed(21)
    pk = torch.randn(L, 2, 30, 128, generator=g).half()
    sc = torch.rand(30, generator=g)
    batches = [SessionBatch(cfg, S, "cuda:0") for _ in range(2)]
    for b in batches:
        for s in range(S):
            b.load_prompt(s, tuple((pk[l][None], pk[l][None]) for l in range(L)), sc)
    for t in range(12):
        k = torch.randn(L, S, 2, 128, generator=g).half()
        v = torch.randn(L, S, 2, 128, generator=g).half()
        batches[0].append(k.cuda(), v.cuda(), [30 + t] * S)
        for s in range(S):
            batches[1].push(s, k[:, s, :, None, :], v[:, s, :, None, :], 30 + t)
        assert torch.equal(batches[0].events, batches[1].events), t
    a, b = batches
    for name in ("slot_table", "positions", "importance", "occupied", "ctrl", "counters"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    for s in range(S):
        Ka, Va = a.gather(s)
        Kb, Vb = b.gather(s)
        assert torch.equal(Ka, Kb) and torch.equal(Va, Vb)
    a.check_device_status()


@pytest.mark.parametrize("variant", [0, 5])
def test_attend_split_kernel_partly_filled(variant):
    """The slot-split kernel on a cache whose prompt (5 tokens) is shorter than
    its budget: empty slots in every tier while it fills, against the oracle."""
    sp = dict(specs.SMALL["short_prompt"])
    cache, oc, outs, events = run_small_attend(sp, "float16", variant)
    cache.batch.check_device_status()
