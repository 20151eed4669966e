"""Fixture from the reference's own TwoPassEngine (two_pass.py:142-434).

    INFERCACHE_REF=/path/to/infercache python tests/golden/make_twopass_golden.py

Runs the reference engine on the CPU with the tiny fp32 Qwen2-shaped model of
``specs.tiny_qwen2`` (weights regenerated from the seed by the tests), the
character tokenizer and greedy sampling, in its default hidden-state
importance mode: summary pass, cache priming (load_from_hf_output), then the
decode loop (to_hf_past_key_values, model forward, push of the new token).
Stores the generated token ids, the cache's final positions / occupancy /
importance and eviction count, each step's margin between the two largest
logits (so a test can see how far every greedy choice is from a tie), and the
summary pass's importance scores with the slot layout they primed.
"""
from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import specs  # noqa: E402


def main():
    ref = os.environ.get("INFERCACHE_REF", "/root/reference")
    d = tempfile.mkdtemp(prefix="icref_")
    os.symlink(ref, os.path.join(d, "inference"))
    sys.path.insert(0, d)
    from inference.hierarchical_cache import CacheConfig
    from inference.two_pass import TwoPassConfig, TwoPassEngine

    sp = specs.TWOPASS
    model = specs.tiny_qwen2(sp["seed"], sp["layers"], sp["vocab"])
    tok = specs.CharTokenizer(sp["vocab"])
    ccfg = CacheConfig(num_layers=sp["layers"], num_kv_heads=1, head_dim=128, sink_size=sp["sink"],
                       recent_size=sp["recent"], important_size=sp["important"], dtype=torch.float32)
    eng = TwoPassEngine(model, tok, ccfg, TwoPassConfig(temperature=0.0, max_new_tokens=sp["max_new_tokens"]),
                        device="cpu")
    margins = []
    orig = eng._sample

    def sample(logits, generated):
        top = torch.topk(logits.float(), 2).values
        margins.append(float(top[0] - top[1]))
        return orig(logits, generated)

    eng._sample = sample
    primed = {}
    orig_prime = eng._prime_cache

    def prime(summary):
        orig_prime(summary)
        primed["scores"] = summary.importance_scores.numpy().copy()
        primed["positions"] = eng._cache.positions.numpy().copy()

    eng._prime_cache = prime
    ids = eng.generate_ids(specs.TWOPASS_PROMPT)
    c = eng._cache
    out = dict(ids=np.array(ids, np.int64), positions=c.positions.numpy().copy(),
               occupied=c.occupied.numpy().copy(), importance=c.importance.numpy().copy(),
               evictions=np.array(c._stats.total_evictions, np.int64), margins=np.array(margins, np.float32),
               prime_scores=primed["scores"], prime_positions=primed["positions"])
    np.savez_compressed(HERE / "twopass_ref.npz", **out)
    print("tokens", len(ids), "evictions", int(out["evictions"]), "min logit margin", float(min(margins)))


if __name__ == "__main__":
    main()
