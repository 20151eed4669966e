"""Generate golden fixtures by running the reference implementation itself.

Run in a container that has the reference checked out (read-only is fine):

    INFERCACHE_REF=/path/to/infercache python tests/golden/make_golden.py

The reference is a flat Python package that imports itself as ``inference``;
this script links it into a temporary directory under that name and imports
it.  Every fixture is produced by the reference's own classes and functions
(``HierarchicalKVCache``, ``_attention_mass``, ``PagePool`` / ``KVAllocator``
/ ``MultiSessionCache``) driven by the seeded harnesses below; inputs are
regenerated from their seeds by the tests, so only outputs are stored.

Fixtures (all small):
  c1_decode.npz     single-layer fp32 decode, 16/2 heads, D=128, budget
                    4/256/780, 4096 tokens from seed 0: every push event,
                    per-step output checksums, outputs and importance at a few
                    steps, final slot state.
  small_decode_*.npz multi-layer decode after a primed prompt (tiny budget so
                    every tier transition happens), fp32 and fp16, full
                    per-step outputs and importance.
  tier_fill_*.npz   ``load_from_hf_output`` slot placement for several prompt
                    shapes, with ties, short prompts and permuted positions.
  attn_mass.npz     ``_attention_mass`` of a causal bf16-rounded GQA prompt
                    (T=2048, 16/2 heads) and the tier fill it induces.
  paged_trace.npz   a seeded alloc / push / gather / reset / LRU trace.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import specs  # noqa: E402  (seeded input generators shared with the tests)


def import_reference():
    ref = os.environ.get("INFERCACHE_REF", "/root/reference")
    d = tempfile.mkdtemp(prefix="icref_")
    os.symlink(ref, os.path.join(d, "inference"))
    sys.path.insert(0, d)
    import inference  # noqa: F401
    from inference import hierarchical_cache, two_pass, paged_cache
    return hierarchical_cache, two_pass, paged_cache


HC, TP, PC = import_reference()
EV_NONE, EV_DROP, EV_FILL, EV_EVICT, EV_REJECT = 0, 1, 2, 3, 4


class EventTap:
    """Wraps a reference cache's ``_maybe_promote_to_l2`` to record what each
    push did to the displaced ring token (instrumentation only; the wrapped
    method runs unchanged)."""

    def __init__(self, cache):
        self.cache = cache
        self.last = None
        orig = cache._maybe_promote_to_l2
        cfg = cache.cfg

        def tapped(slot):
            c = self.cache
            score = float(c.importance[slot].item())
            dpos = int(c.positions[slot].item())
            fill0 = c._important_fill
            ev0 = c._stats.total_evictions
            target = -1
            if score > 0 and fill0 >= cfg.important_size:
                target = c._l2_min_slot()
                epos_before = int(c.positions[target].item())
            orig(slot)
            if score <= 0:
                self.last = (EV_DROP, dpos, -1, -1)
            elif fill0 < cfg.important_size:
                self.last = (EV_FILL, dpos, cfg.important_start + fill0, -1)
            elif c._stats.total_evictions > ev0:
                self.last = (EV_EVICT, dpos, target, epos_before)
            else:
                self.last = (EV_REJECT, dpos, target, -1)

        cache._maybe_promote_to_l2 = tapped

    def push(self, *a, **kw):
        self.last = (EV_NONE, -1, -1, -1)
        self.cache.push(*a, **kw)
        return self.last


def ref_decode_step(cache, tap, q, k, v, position, decay, kv_dtype):
    """The decode protocol on a reference cache (torch, float32 compute).

    q: [L, Hq, D]; k, v: [L, Hkv, D].  Gathers the occupied slots in
    position order, appends the new token, attends with scale D**-0.5, sums
    the probabilities over the query heads of each KV group, decays the
    importance of occupied slots and pushes with that mass.
    """
    cfg = cache.cfg
    L, Hkv, D = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    G = q.shape[1] // Hkv
    occ = cache.occupied.nonzero(as_tuple=True)[0]
    ss = occ[cache.positions[occ].argsort()]
    outs, masses = [], []
    for l in range(L):
        K = torch.cat([cache.K[l][:, ss, :].float(), k[l][:, None, :].to(kv_dtype).float()], 1)
        V = torch.cat([cache.V[l][:, ss, :].float(), v[l][:, None, :].to(kv_dtype).float()], 1)
        qq = q[l].float().view(Hkv, G, D)
        p = (torch.einsum("hgd,hfd->hgf", qq, K) * (D ** -0.5)).softmax(-1)
        outs.append(torch.einsum("hgf,hfd->hgd", p, V).reshape(Hkv * G, D))
        masses.append(p.sum(1))
    w = torch.stack(masses)[:, :, None, :]          # [L, Hkv, 1, F+1]
    cache.importance[cache.occupied] *= decay
    ev = tap.push(k[:, :, None, :].to(kv_dtype), v[:, :, None, :].to(kv_dtype),
                  position=position, attn_weights=w)
    return torch.stack(outs), ev


def slot_state(cache):
    return dict(positions=cache.positions.numpy().copy(),
                importance=cache.importance.numpy().copy(),
                occupied=cache.occupied.numpy().copy(),
                fills=np.array([cache._sink_fill, cache._recent_fill,
                                cache._recent_ptr, cache._important_fill], np.int64),
                counters=np.array([cache._stats.total_tokens_seen,
                                   cache._stats.total_evictions], np.int64))


# ---------------------------------------------------------------------------
def gen_c1(perturb=0.0):
    sp = specs.C1
    q, k, v = specs.c1_inputs()
    cfg = HC.CacheConfig(num_layers=1, num_kv_heads=sp["hkv"], head_dim=sp["d"],
                         sink_size=sp["sink"], recent_size=sp["recent"],
                         important_size=sp["important"], dtype=torch.float32)
    c = HC.HierarchicalKVCache(cfg, device="cpu")
    tap = EventTap(c)
    s0 = sp["sink"]
    c.load_from_hf_output(((k[:s0].transpose(0, 1)[None], v[:s0].transpose(0, 1)[None]),),
                          torch.zeros(s0))
    gen = torch.Generator().manual_seed(12345)
    events, sums, abssums = [], [], []
    o_keep, imp_keep = {}, {}
    keep = set(sp["keep_steps"])
    for s in range(s0, sp["n"]):
        o, ev = ref_decode_step_perturbed(c, tap, q[s][None], k[s][None], v[s][None], s,
                                          sp["decay"], perturb, gen)
        events.append(ev)
        sums.append(float(o.double().sum()))
        abssums.append(float(o.double().abs().sum()))
        if s in keep:
            o_keep[s] = o[0].numpy().copy()
            imp_keep[s] = c.importance.numpy().copy()
    return dict(events=np.array(events, np.int64), o_sum=np.array(sums), o_abssum=np.array(abssums),
                keep_steps=np.array(sorted(keep), np.int64),
                o_keep=np.stack([o_keep[s] for s in sorted(keep)]),
                imp_keep=np.stack([imp_keep[s] for s in sorted(keep)]),
                **slot_state(c))


def ref_decode_step_perturbed(cache, tap, q, k, v, position, decay, perturb, gen):
    if perturb == 0.0:
        return ref_decode_step(cache, tap, q, k, v, position, decay, torch.float32)
    # Same protocol with the mass multiplied by (1 + perturb * N(0,1)): used
    # only to show that the eviction sequence does not hinge on last-ulp
    # differences in the mass.
    orig_push = tap.push

    def noisy_push(kk, vv, position, attn_weights):
        w = attn_weights * (1 + perturb * torch.randn(attn_weights.shape, generator=gen))
        return orig_push(kk, vv, position=position, attn_weights=w)

    tap.push = noisy_push
    try:
        return ref_decode_step(cache, tap, q, k, v, position, decay, torch.float32)
    finally:
        tap.push = orig_push


def gen_small(name):
    sp = specs.SMALL[name]
    kv_dtype = getattr(torch, sp["dtype"])
    pk, pv, scores, q, k, v = specs.small_inputs(name)
    cfg = HC.CacheConfig(num_layers=sp["layers"], num_kv_heads=sp["hkv"], head_dim=sp["d"],
                         sink_size=sp["sink"], recent_size=sp["recent"],
                         important_size=sp["important"], dtype=kv_dtype)
    c = HC.HierarchicalKVCache(cfg, device="cpu")
    tap = EventTap(c)
    T = pk.shape[2]
    pkv = tuple((pk[l][None].to(kv_dtype), pv[l][None].to(kv_dtype)) for l in range(sp["layers"]))
    c.load_from_hf_output(pkv, scores)
    prime = slot_state(c)
    outs, imps, poss, evs = [], [], [], []
    for s in range(sp["steps"]):
        o, ev = ref_decode_step(c, tap, q[s], k[s], v[s], T + s, sp["decay"], kv_dtype)
        outs.append(o.numpy())
        imps.append(c.importance.numpy().copy())
        poss.append(c.positions.numpy().copy())
        evs.append(ev)
    return dict(o=np.stack(outs), importance_steps=np.stack(imps), positions_steps=np.stack(poss),
                events=np.array(evs, np.int64),
                prime_positions=prime["positions"], prime_importance=prime["importance"],
                prime_fills=prime["fills"], prime_counters=prime["counters"],
                **slot_state(c))


def gen_tier_fill(name):
    sp = specs.TIER[name]
    scores, positions = specs.tier_inputs(name)
    cfg = HC.CacheConfig(num_layers=1, num_kv_heads=1, head_dim=8, sink_size=sp["sink"],
                         recent_size=sp["recent"], important_size=sp["important"],
                         dtype=torch.float32)
    c = HC.HierarchicalKVCache(cfg, device="cpu")
    T = scores.shape[0]
    # K carries the token index so the slot -> token map can be read back.
    tok = torch.arange(T, dtype=torch.float32)
    kk = tok[None, None, :, None].expand(1, 1, T, 8).contiguous()
    c.load_from_hf_output(((kk, kk),), scores, positions=positions)
    slot_token = torch.where(c.occupied, c.K[0, 0, :, 0].long(), torch.full_like(c.positions, -1))
    return dict(slot_token=slot_token.numpy(), **slot_state(c))


def gen_attn_mass():
    sp = specs.AMASS
    q, k, v = specs.amass_inputs()           # bf16-rounded, float32 tensors [Hq|Hkv, T, D]
    Hq, T, D = q.shape
    G = Hq // k.shape[0]
    kx = k.repeat_interleave(G, 0)
    s = torch.einsum("htd,hsd->hts", q, kx) * (D ** -0.5)
    mask = torch.ones(T, T, dtype=torch.bool).triu(1)
    s.masked_fill_(mask, float("-inf"))
    P = s.softmax(-1)
    imp = TP._attention_mass((P[None],), all_layers=False, layer_idx=-1)
    colsum = P.sum(dim=(0, 1))
    cfg = HC.CacheConfig(num_layers=1, num_kv_heads=1, head_dim=8, sink_size=sp["sink"],
                         recent_size=sp["recent"], important_size=sp["important"],
                         dtype=torch.float32)
    c = HC.HierarchicalKVCache(cfg, device="cpu")
    tok = torch.arange(T, dtype=torch.float32)
    kk = tok[None, None, :, None].expand(1, 1, T, 8).contiguous()
    c.load_from_hf_output(((kk, kk),), imp)
    slot_token = torch.where(c.occupied, c.K[0, 0, :, 0].long(), torch.full_like(c.positions, -1))
    return dict(scores=imp.numpy(), colsum=colsum.numpy(), slot_token=slot_token.numpy(),
                **slot_state(c))


class LogicalClock:
    """Stands in for the ``time`` module inside the reference's paged_cache so
    that LRU order is a function of call order only."""

    def __init__(self):
        self.t = 0.0

    def monotonic(self):
        self.t += 1.0
        return self.t


def gen_paged():
    sp = specs.PAGED
    PC.time = LogicalClock()
    cfg = PC.PagedCacheConfig(n_pages=sp["n_pages"], n_layers=sp["layers"], n_heads=sp["heads"],
                              head_dim=sp["d"], dtype=torch.float32, device="cpu",
                              max_pages_per_session=sp["max_pps"])
    pool = PC.PagePool(cfg)
    msc = PC.MultiSessionCache(pool)
    ops = specs.paged_ops()
    log_pages, log_free, log_util, errors = [], [], [], []
    gathers = []
    for op in ops:
        kind = op[0]
        err = ""
        try:
            if kind == "push":
                _, sid, n, seed = op
                kk, vv = specs.paged_tokens(n, seed)
                view = msc.get_or_create(sid)
                view.push(kk, vv, positions=list(range(view.n_tokens, view.n_tokens + n)),
                          importance=[float(x) for x in np.linspace(0, 1, n)])
            elif kind == "gather":
                _, sid, layer = op
                view = msc.get_or_create(sid)
                K, V = view.gather(layer)
                gathers.append(np.concatenate([K.numpy().ravel(), V.numpy().ravel()]))
            elif kind == "reset":
                msc.reset(op[1])
            elif kind == "touch":
                msc._alloc.touch(op[1])
        except RuntimeError as e:
            err = str(e)
        errors.append(err)
        log_pages.append(json.dumps({s: msc._alloc.pages_for(s) for s in sorted(msc.active_sessions())}))
        log_free.append(json.dumps(list(msc._alloc._free_list)))
        log_util.append(msc.utilization())
    return dict(pages=np.array(log_pages), free=np.array(log_free), util=np.array(log_util),
                errors=np.array(errors),
                gathers=np.concatenate(gathers) if gathers else np.zeros(0, np.float32),
                gather_sizes=np.array([g.size for g in gathers], np.int64))


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    manifest = {}
    out = gen_c1()
    np.savez_compressed(HERE / "c1_decode.npz", **out)
    noisy = gen_c1(perturb=1e-6)
    stable = bool(np.array_equal(noisy["events"], out["events"]))
    manifest["c1_decode"] = dict(evictions=int(out["counters"][1]),
                                 events_stable_under_mass_noise_1e6=stable)
    for name in specs.SMALL:
        np.savez_compressed(HERE / f"small_decode_{name}.npz", **gen_small(name))
    for name in specs.TIER:
        r = gen_tier_fill(name)
        np.savez_compressed(HERE / f"tier_fill_{name}.npz", **r)
        manifest[f"tier_fill_{name}"] = dict(evictions=int(r["counters"][1]))
    np.savez_compressed(HERE / "attn_mass.npz", **gen_attn_mass())
    np.savez_compressed(HERE / "paged_trace.npz", **gen_paged())
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
