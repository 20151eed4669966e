"""TwoPassEngine over the fixed-budget cache with a small random-weight
Qwen2-shaped model (head_dim 128), on a B200.

* attention-mass summary pass (kernel C inside the model's prefill) against
  the reference's formula applied to eager ``output_attentions`` tensors, for
  layer 0 (identical inputs on both sides): relative 2e-3 for scores >= 1e-4,
  absolute 2e-7 below (the eager probabilities are fp16-rounded, so the
  reference itself carries absolute errors of the fp16 quantum); summed over
  all layers: relative 1e-2 — deeper layers see hidden states from two
  different fp16 forward paths (eager vs kernel C), which differ by ~1e-3;
* fused decode (kernel A as the model's attention + kernel B) against the
  reference's DynamicCache loop: identical greedy tokens and identical cache
  state (fp32 model, exact index work);
* the short-prompt direct path against a plain Hugging Face greedy loop;
* both decode paths against the reference's own TwoPassEngine (fixture made
  by running it on the CPU), and the memory engine's save / load calls on the
  cache against the oracle.
"""
import numpy as np
import pytest
import torch


pytestmark = pytest.mark.gpu


from specs import CharTokenizer, tiny_qwen2


def tiny_model(dtype, seed=0, layers=3):
    """specs.tiny_qwen2 (built on the CPU from the seed) on the GPU in `dtype`."""
    return tiny_qwen2(seed, layers).to("cuda", dtype).eval()


def cache_cfg(model, dtype, sink=4, recent=16, important=40):
    from infercache_b200 import CacheConfig
    c = model.config
    return CacheConfig(num_layers=c.num_hidden_layers, num_kv_heads=c.num_key_value_heads, head_dim=128,
                       sink_size=sink, recent_size=recent, important_size=important, dtype=dtype)


PROMPT = "".join(chr(33 + (i * 37) % 90) for i in range(300))


def reference_attention_mass(model, ids, all_layers, layer_idx):
    """two_pass.py:104-137 on eager attention tensors."""
    prev = model.config._attn_implementation
    model.config._attn_implementation = "eager"
    try:
        with torch.no_grad():
            out = model(ids, output_attentions=True, use_cache=False)
    finally:
        model.config._attn_implementation = prev
    atts = out.attentions if all_layers else (out.attentions[layer_idx % len(out.attentions)],)
    imp = None
    for a in atts:
        r = a[0].float().sum(dim=(0, 1))
        imp = r if imp is None else imp + r
    return (imp / imp.sum()).cpu().numpy(), out.logits.float()


@pytest.mark.parametrize("all_layers,layer,rtol", [(False, 0, 2e-3), (True, -1, 1e-2)])
def test_summary_pass_attention_mass(all_layers, layer, rtol):
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    model = tiny_model(torch.float16)
    tok = CharTokenizer(512)
    eng = TwoPassEngine(model, tok, cache_cfg(model, torch.float16),
                        TwoPassConfig(use_hidden_importance=False, all_layers_importance=all_layers,
                                      importance_layer=layer))
    ids = tok.encode(PROMPT, return_tensors="pt").cuda()
    res = eng.summary_pass(ids)
    ref, ref_logits = reference_attention_mass(model, ids, all_layers, layer)
    assert res.seq_len == ids.shape[1]
    got = res.importance_scores.numpy().astype(np.float64)
    err = np.abs(got - ref)
    big = ref >= 1e-4
    assert np.all(err[big] <= rtol * ref[big]), float((err[big] / ref[big]).max())
    assert np.all(err[~big] <= 2e-7), float(err[~big].max())
    # the model's own output through kernel C matches the eager forward
    err = (res.last_logits.float() - ref_logits[0, -1].cpu()).abs().max() / ref_logits[0, -1].abs().max()
    assert float(err) < 2e-2
    # priming places the top-scored tokens exactly as the oracle would
    from oracle.summary import tier_fill
    eng._prime_cache(res)
    tf = tier_fill(res.importance_scores.numpy(), None, 4, 16, 40)
    assert np.array_equal(eng._cache.positions.cpu().numpy(), tf["positions"])
    assert np.array_equal(eng._cache.occupied.cpu().numpy(), tf["occupied"])


def test_fused_decode_matches_dynamic_cache_loop():
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    model = tiny_model(torch.float32, seed=1)
    tok = CharTokenizer(512)
    outs = {}
    for path in ("dynamic_cache", "fused"):
        eng = TwoPassEngine(model, tok, cache_cfg(model, torch.float32),
                            TwoPassConfig(temperature=0.0, max_new_tokens=48, decode_path=path))
        ids = eng.generate_ids(PROMPT)
        c = eng._cache
        outs[path] = (ids, c.positions.cpu().numpy(), c.occupied.cpu().numpy(), c.importance.cpu().numpy(),
                      c.stats.total_evictions)
    a, b = outs["dynamic_cache"], outs["fused"]
    assert a[0] == b[0], "greedy tokens differ"
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])
    assert a[4] == b[4]
    assert len(a[0]) == 48


def test_attention_mode_fused_generation_runs():
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    model = tiny_model(torch.bfloat16, seed=2)
    tok = CharTokenizer(512)
    eng = TwoPassEngine(model, tok, cache_cfg(model, torch.bfloat16),
                        TwoPassConfig(temperature=0.7, top_k=50, top_p=0.9, max_new_tokens=40,
                                      use_hidden_importance=False, decode_importance=True))
    torch.manual_seed(0)
    text = eng.generate(PROMPT)
    assert len(text) == 40
    st = eng._cache.stats
    assert st.current_fill == eng._cache.total_budget
    pieces = list(eng.stream_generate(PROMPT))
    assert len(pieces) == 40
    eng.reset_cache()
    assert eng._cache.current_fill == 0


def test_direct_path_matches_plain_loop():
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    model = tiny_model(torch.float32, seed=3)
    tok = CharTokenizer(512)
    eng = TwoPassEngine(model, tok, cache_cfg(model, torch.float32),
                        TwoPassConfig(temperature=0.0, max_new_tokens=12))
    prompt = PROMPT[:60]
    got = eng.generate_ids(prompt)
    ids = tok.encode(prompt, return_tensors="pt").cuda()
    want, past = [], None
    with torch.no_grad():
        cur = ids
        for _ in range(12):
            o = model(cur, past_key_values=past, use_cache=True)
            nxt = int(o.logits[0, -1].argmax())
            want.append(nxt)
            past, cur = o.past_key_values, torch.tensor([[nxt]], device="cuda")
    assert got == want


@pytest.mark.parametrize("path", ["fused", "dynamic_cache"])
def test_matches_reference_two_pass_engine(golden, path):
    """Against the reference's own TwoPassEngine (fixture twopass_ref.npz, made
    by running it on the CPU: tests/golden/make_twopass_golden.py): the same
    tiny fp32 model (weights regenerated from the seed), prompt, budget and
    greedy sampling give the same 48 tokens (the fixture's smallest top-2
    logit margin, ~1e-2, is far above the fp32 differences between the two
    devices), the same retained positions and eviction count, importance
    within 1e-5 per position, and -- primed from the reference's own summary
    scores -- the reference's slot layout exactly."""
    import specs
    from infercache_b200 import CacheConfig
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    g = golden("twopass_ref")
    sp = specs.TWOPASS
    model = specs.tiny_qwen2(sp["seed"], sp["layers"], sp["vocab"]).to("cuda")
    ccfg = CacheConfig(num_layers=sp["layers"], num_kv_heads=1, head_dim=128, sink_size=sp["sink"],
                       recent_size=sp["recent"], important_size=sp["important"], dtype=torch.float32)
    eng = TwoPassEngine(model, specs.CharTokenizer(sp["vocab"]), ccfg,
                        TwoPassConfig(temperature=0.0, max_new_tokens=sp["max_new_tokens"], decode_path=path))
    ids = eng.generate_ids(specs.TWOPASS_PROMPT)
    assert ids == g["ids"].tolist()
    c = eng._cache
    pos, ref_pos = c.positions.cpu().numpy(), g["positions"]
    assert np.array_equal(c.occupied.cpu().numpy(), g["occupied"])
    # sinks and the recent ring slot by slot; the importance tier as a set of
    # positions: its slot order records which near-equal priming score went
    # first, and those scores are hidden-state norms computed on two devices
    ring_end = sp["sink"] + sp["recent"]
    assert np.array_equal(pos[:ring_end], ref_pos[:ring_end])
    assert sorted(pos[ring_end:].tolist()) == sorted(ref_pos[ring_end:].tolist())
    imp = dict(zip(pos.tolist(), c.importance.cpu().numpy().tolist()))
    ref_imp = dict(zip(ref_pos.tolist(), g["importance"].tolist()))
    for p_, x in ref_imp.items():
        assert abs(imp[p_] - x) <= 1e-5 * max(abs(x), 1e-30), p_
    assert c.stats.total_evictions == int(g["evictions"])
    # primed from the reference's own summary scores, the slot layout is exact
    res = eng.summary_pass(torch.tensor([specs.CharTokenizer(sp["vocab"]).encode(specs.TWOPASS_PROMPT)]))
    res.importance_scores = torch.from_numpy(g["prime_scores"])
    eng._prime_cache(res)
    assert np.array_equal(eng._cache.positions.cpu().numpy(), g["prime_positions"])


def test_memory_engine_save_load_round_trip():
    """The cache-side calls of the reference's PersistentMemoryEngine
    (memory_engine.py:406-410, 434-440) on the new cache: after generation the
    occupied slots' positions and importance are read through the public
    tensors (occupied.nonzero, positions[idx], importance[idx]); a later turn
    re-primes a cache from the stored tokens, sorted by position, through
    load_from_hf_output with explicit, non-contiguous positions.  The primed
    state must equal the oracle's load of the same tokens."""
    import specs
    from infercache_b200 import CacheConfig, HierarchicalKVCache
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    from oracle.hier_cache import OracleCache, TierGeometry
    sp = specs.TWOPASS
    model = specs.tiny_qwen2(sp["seed"], sp["layers"], sp["vocab"]).to("cuda")
    ccfg = CacheConfig(num_layers=sp["layers"], num_kv_heads=1, head_dim=128, sink_size=sp["sink"],
                       recent_size=sp["recent"], important_size=sp["important"], dtype=torch.float32)
    eng = TwoPassEngine(model, specs.CharTokenizer(sp["vocab"]), ccfg, TwoPassConfig(temperature=0.0, max_new_tokens=24))
    eng.generate_ids(specs.TWOPASS_PROMPT)
    cache = eng._cache
    # _save_turn: what it reads
    occ_idx = cache.occupied.nonzero(as_tuple=True)[0]
    positions = cache.positions[occ_idx].tolist()
    importances = cache.importance[occ_idx].tolist()
    assert len(positions) == cache.total_budget and len(set(positions)) == len(positions)
    # keep the tokens above a threshold, as min_importance does, then the load path
    keep = [(p, i) for p, i in zip(positions, importances) if i >= 1e-4] or list(zip(positions, importances))
    keep.sort(key=lambda r: r[0])
    pos = [p for p, _ in keep]
    imp = [i for _, i in keep]
    g = torch.Generator().manual_seed(8)
    L, n = sp["layers"], len(pos)
    k = torch.randn(L, 1, n, 128, generator=g)
    v = torch.randn(L, 1, n, 128, generator=g)
    fresh = HierarchicalKVCache(ccfg, device="cuda")
    fresh.load_from_hf_output(tuple((k[l][None], v[l][None]) for l in range(L)),
                              importance_scores=torch.tensor(imp, dtype=torch.float32),
                              positions=torch.tensor(pos, dtype=torch.long))
    oc = OracleCache(TierGeometry(L, 1, 128, sp["sink"], sp["recent"], sp["important"]), np.float32)
    oc.load_from_hf_output(k.numpy(), v.numpy(), np.array(imp, np.float32), positions=np.array(pos, np.int64))
    assert np.array_equal(fresh.positions.cpu().numpy(), oc.positions)
    assert np.array_equal(fresh.occupied.cpu().numpy(), oc.occupied)
    assert np.array_equal(fresh.importance.cpu().numpy(), oc.importance)
    K, V = fresh.K.cpu().numpy(), fresh.V.cpu().numpy()
    occ = oc.occupied
    assert np.array_equal(K[:, :, occ], oc.K[:, :, occ]) and np.array_equal(V[:, :, occ], oc.V[:, :, occ])
    # and the saved state of the restored cache reads back the same way
    idx2 = fresh.occupied.nonzero(as_tuple=True)[0]
    assert sorted(fresh.positions[idx2].tolist()) == sorted(oc.positions[occ].tolist())
