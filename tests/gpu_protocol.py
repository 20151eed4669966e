"""Drivers that run the decode protocol through the CUDA path and through the
oracle on the same seeded inputs (shared by the GPU tests and smoke())."""
from __future__ import annotations

import numpy as np
import torch

import specs
from oracle.hier_cache import OracleCache, TierGeometry, decode_step
from tolerances import elem_close, rows_close, rows_err

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
NP_DT = {"float32": np.float32, "float16": np.float16}


def make_gpu_cache(layers, hkv, d, sink, recent, important, dtype, decay=0.99):
    from infercache_b200 import CacheConfig, HierarchicalKVCache
    cfg = CacheConfig(num_layers=layers, num_kv_heads=hkv, head_dim=d, sink_size=sink,
                      recent_size=recent, important_size=important, decay=decay, dtype=dtype)
    return HierarchicalKVCache(cfg, device="cuda:0")


def gpu_state(cache):
    return (cache.positions.cpu().numpy(), cache.importance.cpu().numpy(),
            cache.occupied.cpu().numpy())


def compare_state(cache, oc: OracleCache, rtol, where=""):
    pos, imp, occ = gpu_state(cache)
    assert np.array_equal(pos, oc.positions), f"positions differ {where}"
    assert np.array_equal(occ, oc.occupied), f"occupancy differs {where}"
    assert elem_close(imp, oc.importance, rtol), f"importance differs {where}"
    st = cache.stats
    assert (st.sink_fill, st.recent_fill, st.important_fill) == (oc.sink_fill, oc.recent_fill, oc.important_fill), where
    assert (st.total_tokens_seen, st.total_evictions) == (oc.total_tokens_seen, oc.total_evictions), where
    assert cache._recent_ptr == oc.recent_ptr, where


def run_c1(steps=None, check_every=1):
    """Single-layer fp32 decode of 4096 tokens (seed 0), GPU vs oracle per step.
    Returns (events, outputs at keep steps, max normwise output error)."""
    sp = specs.C1
    q, k, v = specs.c1_inputs()
    n = sp["n"] if steps is None else min(sp["n"], sp["sink"] + steps)
    cache = make_gpu_cache(1, sp["hkv"], sp["d"], sp["sink"], sp["recent"], sp["important"], torch.float32,
                           sp["decay"])
    geo = TierGeometry(1, sp["hkv"], sp["d"], sp["sink"], sp["recent"], sp["important"])
    oc = OracleCache(geo, np.float32)
    s0 = sp["sink"]
    cache.load_from_hf_output(((k[:s0].transpose(0, 1)[None], v[:s0].transpose(0, 1)[None]),), torch.zeros(s0))
    oc.load_from_hf_output(k[:s0].numpy().transpose(1, 0, 2)[None], v[:s0].numpy().transpose(1, 0, 2)[None],
                           np.zeros(s0, np.float32))
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    events, keep, worst = [], {}, 0.0
    keep_steps = set(sp["keep_steps"])
    for s in range(s0, n):
        o = cache.step(qd[s][None], kd[s][None], vd[s][None], s)
        oo, ev = decode_step(oc, q[s][None].numpy(), k[s][None].numpy(), v[s][None].numpy(), s, sp["decay"])
        g = o.cpu().numpy()
        worst = max(worst, rows_err(g, oo))
        assert rows_close(g, oo, 1e-5), f"output differs at step {s}: {rows_err(g, oo)}"
        gev = cache.last_event()
        assert gev == ev.as_tuple(), f"event differs at step {s}: gpu {gev} oracle {ev.as_tuple()}"
        events.append(gev)
        if s in keep_steps:
            keep[s] = g[0]
        if check_every and (s % check_every == 0 or s == n - 1):
            compare_state(cache, oc, 1e-5, f"at step {s}")
    return cache, oc, np.array(events, np.int64), keep, worst


def run_small(name, out_dtype=torch.float32, variant=0, dtype=None):
    """Primed multi-layer decode of one SMALL spec, GPU vs oracle per step.

    variant: kernel A implementation (0 auto, 1 CUDA cores, 2 tensor cores).
    dtype: override the spec's cache dtype ("bfloat16": the oracle then holds
    the bf16-rounded values in float32 storage, which is exact)."""
    sp = dict(name if isinstance(name, dict) else (specs.SMALL[name] if name in specs.SMALL else specs.WIDE[name]))
    base_dt = sp["dtype"]
    if dtype is not None:
        sp["dtype"] = dtype
    dt = TORCH_DT[sp["dtype"]]
    rtol = 1e-5 if sp["dtype"] == "float32" else 1e-3
    pk, pv, scores, q, k, v = specs.small_inputs(name if not isinstance(name, dict) else sp)
    if dtype is not None and dtype != base_dt:
        pk, pv, q, k, v = (t.to(dt).float() for t in (pk, pv, q, k, v))
    cache = make_gpu_cache(sp["layers"], sp["hkv"], sp["d"], sp["sink"], sp["recent"], sp["important"], dt,
                           sp["decay"])
    cache.batch.kernel_variant = variant
    geo = TierGeometry(sp["layers"], sp["hkv"], sp["d"], sp["sink"], sp["recent"], sp["important"])
    oc = OracleCache(geo, NP_DT.get(sp["dtype"], np.float32))
    pkv = tuple((pk[l][None].to(dt), pv[l][None].to(dt)) for l in range(sp["layers"]))
    cache.load_from_hf_output(pkv, scores)
    oc.load_from_hf_output(pk.numpy(), pv.numpy(), scores.numpy())
    compare_state(cache, oc, 0.0, "after priming")
    T = pk.shape[2]
    outs, events = [], []
    qd, kd, vd = q.to(dt).cuda(), k.to(dt).cuda(), v.to(dt).cuda()
    for s in range(sp["steps"]):
        o = cache.step(qd[s], kd[s], vd[s], T + s, out_dtype=out_dtype)
        oo, ev = decode_step(oc, q[s].numpy(), k[s].numpy(), v[s].numpy(), T + s, sp["decay"])
        g = o.float().cpu().numpy()
        assert rows_close(g, oo, rtol), f"{name}: output differs at step {s}: {rows_err(g, oo)}"
        gev = cache.last_event()
        assert gev == ev.as_tuple(), f"{name}: event differs at step {s}: gpu {gev} oracle {ev.as_tuple()}"
        compare_state(cache, oc, rtol, f"{name} step {s}")
        outs.append(g)
        events.append(gev)
    return cache, oc, np.stack(outs), np.array(events, np.int64)
