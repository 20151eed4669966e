"""Seeded input generators shared by ``make_golden.py`` and the tests.

Only seeds and shapes live here; fixture files hold the reference's outputs.
Inputs come from ``torch.Generator`` (CPU, deterministic across machines with
the same torch build), drawn in a fixed order.
"""
from __future__ import annotations

import numpy as np
import torch

# Single-layer fp32 decode, the correctness workload: 1 session, 16/2 heads,
# head_dim 128, budget 4/256/780, 4096 tokens from seed 0, decay 0.99.
C1 = dict(n=4096, hq=16, hkv=2, d=128, sink=4, recent=256, important=780, decay=0.99,
          keep_steps=[4, 5, 100, 259, 260, 261, 1000, 1035, 1036, 1037, 2048, 4095])


def c1_inputs():
    sp = C1
    g = torch.Generator().manual_seed(0)
    q = torch.randn(sp["n"], sp["hq"], sp["d"], generator=g)
    k = torch.randn(sp["n"], sp["hkv"], sp["d"], generator=g)
    v = torch.randn(sp["n"], sp["hkv"], sp["d"], generator=g)
    return q, k, v


# Multi-layer decode after a primed prompt.  Tiny budgets make every tier
# transition (ring wrap, L2 fill, L2 eviction, rejection) happen in few steps.
SMALL = {
    "f32": dict(layers=2, hq=4, hkv=2, d=128, sink=2, recent=5, important=4, prompt=24,
                steps=60, decay=0.99, dtype="float32", seed=7),
    "f16": dict(layers=3, hq=8, hkv=2, d=128, sink=2, recent=6, important=5, prompt=30,
                steps=60, decay=0.99, dtype="float16", seed=8),
    "g7": dict(layers=2, hq=14, hkv=2, d=128, sink=4, recent=8, important=6, prompt=40,
               steps=50, decay=0.99, dtype="float16", seed=9),
    "short_prompt": dict(layers=2, hq=4, hkv=2, d=128, sink=3, recent=6, important=4, prompt=5,
                         steps=40, decay=0.99, dtype="float32", seed=10),
}


# Wider shapes checked against the oracle only (the oracle is pinned by the
# SMALL fixtures): the Qwen2.5-7B-shaped budget 2048 (4/512/1532) with 28/4
# heads on two layers.
WIDE = {
    "c3_budget": dict(layers=2, hq=28, hkv=4, d=128, sink=4, recent=512, important=1532, prompt=2600,
                      steps=8, decay=0.99, dtype="float16", seed=12),
}


def small_inputs(name):
    """Prompt K/V [L, Hkv, T, D], prompt scores [T] (rounded to 0.05 so that
    ties occur), and per-step q [S, L, Hq, D], k/v [S, L, Hkv, D]."""
    sp = name if isinstance(name, dict) else (SMALL[name] if name in SMALL else WIDE[name])
    g = torch.Generator().manual_seed(sp["seed"])
    L, T, S, D = sp["layers"], sp["prompt"], sp["steps"], sp["d"]
    pk = torch.randn(L, sp["hkv"], T, D, generator=g)
    pv = torch.randn(L, sp["hkv"], T, D, generator=g)
    scores = (torch.rand(T, generator=g) * 20).round() / 20
    q = torch.randn(S, L, sp["hq"], D, generator=g)
    k = torch.randn(S, L, sp["hkv"], D, generator=g)
    v = torch.randn(S, L, sp["hkv"], D, generator=g)
    dt = getattr(torch, sp["dtype"])
    # Inputs are rounded to the cache dtype up front so that every
    # implementation sees identical values.
    return pk.to(dt).float(), pv.to(dt).float(), scores, q.to(dt).float(), k.to(dt).float(), v.to(dt).float()


# Tier fill by load_from_hf_output.
TIER = {
    "c2_prompt": dict(sink=4, recent=256, important=780, T=2048, seed=11, ties=1e-3, perm=False),
    "c3_prompt": dict(sink=4, recent=512, important=1532, T=8192, seed=12, ties=1e-3, perm=False),
    "short": dict(sink=4, recent=256, important=780, T=100, seed=13, ties=0.0, perm=False),
    "permuted": dict(sink=4, recent=64, important=100, T=600, seed=14, ties=1e-2, perm=True),
    "tiny": dict(sink=2, recent=3, important=4, T=30, seed=15, ties=0.25, perm=False),
}


def tier_inputs(name):
    sp = TIER[name]
    g = torch.Generator().manual_seed(sp["seed"])
    T = sp["T"]
    scores = torch.rand(T, generator=g)
    if sp["ties"] > 0:
        scores = (scores / sp["ties"]).round() * sp["ties"]
    if sp["perm"]:
        positions = torch.randperm(T + T // 2, generator=g)[:T].long()
    else:
        positions = torch.arange(T, dtype=torch.long)
    return scores.float(), positions


# _attention_mass of a causal GQA prompt (bf16-rounded inputs, fp32 math).
AMASS = dict(T=2048, hq=16, hkv=2, d=128, seed=3, sink=4, recent=256, important=780)


def amass_inputs():
    sp = AMASS
    g = torch.Generator().manual_seed(sp["seed"])
    q = torch.randn(sp["hq"], sp["T"], sp["d"], generator=g).bfloat16().float()
    k = torch.randn(sp["hkv"], sp["T"], sp["d"], generator=g).bfloat16().float()
    v = torch.randn(sp["hkv"], sp["T"], sp["d"], generator=g).bfloat16().float()
    return q, k, v


# Paged pool trace: 12 pages of 16 tokens, 2 layers x 2 heads x 8 dims.
PAGED = dict(n_pages=12, layers=2, heads=2, d=8, max_pps=6)


def paged_ops():
    return [
        ("push", "A", 20, 1),
        ("push", "B", 40, 2),
        ("gather", "A", 0),
        ("push", "C", 50, 3),
        ("push", "A", 30, 4),
        ("gather", "A", 1),
        ("touch", "B"),
        ("push", "D", 33, 5),          # pool exhausted: LRU eviction
        ("gather", "B", 1),
        ("gather", "D", 0),
        ("reset", "C"),
        ("push", "E", 16, 6),
        ("push", "A", 60, 7),          # exceeds the per-session page cap
        ("gather", "E", 1),
        ("push", "B", 1, 8),
        ("reset", "A"),
        ("push", "F", 70, 9),
        ("gather", "F", 1),
    ]


def paged_tokens(n, seed):
    sp = PAGED
    g = torch.Generator().manual_seed(100 + seed)
    k = torch.randn(sp["layers"], sp["heads"], n, sp["d"], generator=g)
    v = torch.randn(sp["layers"], sp["heads"], n, sp["d"], generator=g)
    return k, v


# Graph (cluster-routed) cache.  Layer-0 / head-0 keys are drawn around a few
# random directions so that tokens form clusters; the other heads and layers
# are plain noise.  Positions are the token indices.
GRAPH = {
    "push": dict(L=3, H=2, D=128, n_clusters=4, cap=6, sink=4, recent=8, threshold=0.3, T=120, n_dirs=5,
                 seed=31),
    "load": dict(L=2, H=2, D=128, n_clusters=6, cap=5, sink=4, recent=16, threshold=0.3, T=200, n_dirs=4,
                 seed=32),
    "wide": dict(L=4, H=4, D=128, n_clusters=16, cap=32, sink=4, recent=128, threshold=0.3, T=1500, n_dirs=12,
                 seed=34),
}
# retrieve() cases: (threshold or None, top_n or None)
GRAPH_QUERIES = [(None, None), (0.6, None), (0.95, None), (None, 1), (None, 3)]


def graph_inputs(name):
    sp = GRAPH[name]
    g = torch.Generator().manual_seed(sp["seed"])
    L, H, D, T = sp["L"], sp["H"], sp["D"], sp["T"]
    dirs = torch.randn(sp["n_dirs"], D, generator=g)
    dirs = dirs / dirs.norm(dim=1, keepdim=True)
    which = torch.randint(0, sp["n_dirs"], (T,), generator=g)
    k = torch.randn(L, H, T, D, generator=g)
    k[0, 0] = dirs[which] * 4.0 + torch.randn(T, D, generator=g) * 0.7
    v = torch.randn(L, H, T, D, generator=g)
    scores = torch.rand(T, generator=g)
    nq = len(GRAPH_QUERIES)
    qdir = torch.randint(0, sp["n_dirs"], (nq,), generator=g)
    queries = dirs[qdir][:, None, :] * 3.0 + torch.randn(nq, H, D, generator=g) * 0.8
    return k.half(), v.half(), scores, queries


# Two-pass engine comparator: a tiny random-weight Qwen2-shaped decoder
# (head_dim 128) built on the CPU from a seed, a deterministic character
# tokenizer, a 300-character prompt (two-pass path: longer than the summary
# threshold) and a 4/16/40 budget so tokens are evicted while decoding.
TWOPASS = dict(seed=1, layers=3, sink=4, recent=16, important=40, max_new_tokens=48, vocab=512)


class CharTokenizer:
    eos_token_id = None
    unk_token_id = 0

    def __init__(self, vocab=512):
        self.vocab = vocab
        self.vocab_size = vocab

    def encode(self, text, return_tensors=None, add_special_tokens=False):
        ids = [(ord(c) * 7) % self.vocab for c in text]
        return torch.tensor([ids]) if return_tensors == "pt" else ids

    def decode(self, ids, skip_special_tokens=False):
        return "".join(chr(32 + int(i) % 90) for i in ids)


def tiny_qwen2(seed=0, layers=3, vocab=512):
    """fp32 on the CPU; q / k projections scaled up so attention is peaked."""
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                      num_attention_heads=2, num_key_value_heads=1, max_position_embeddings=4096,
                      rope_theta=10000.0, tie_word_embeddings=True)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    m = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if ("q_proj" in n or "k_proj" in n) and p.dim() == 2:
                p.mul_(4.0)
    return m.eval()


TWOPASS_PROMPT = "".join(chr(33 + (i * 37) % 90) for i in range(300))
