"""Hugging Face plumbing of the attention integration, on the CPU.

The registered implementation routes each attention call to the active
context; here the contexts are plain-PyTorch stand-ins for kernels C and A,
so the test checks what transformers hands them (post-RoPE q / k / v shapes,
layer indices, the pass-through cache during decode) and that a forward
through them reproduces the model's own SDPA forward.
"""
import torch
import torch.nn.functional as F

from infercache_b200 import hf_attention


def tiny_model(layers=2):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=128, hidden_size=256, intermediate_size=256, num_hidden_layers=layers,
                      num_attention_heads=2, num_key_value_heads=1, max_position_embeddings=512)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def _gqa(q, k, v, causal):
    G = q.shape[1] // k.shape[1]
    return F.scaled_dot_product_attention(q, k.repeat_interleave(G, 1), v.repeat_interleave(G, 1),
                                          is_causal=causal)


class PrefillStandIn:
    def __init__(self):
        self.seen = []
        self.kv = {}

    def attend(self, module, q, k, v, scaling):
        self.seen.append((module.layer_idx, tuple(q.shape), tuple(k.shape)))
        self.kv[module.layer_idx] = (k, v)
        return _gqa(q, k, v, True).transpose(1, 2)


class DecodeStandIn:
    """Keeps each layer's K/V itself, as the fixed-budget cache does."""

    def __init__(self, kv):
        self.kv = dict(kv)

    def attend(self, module, q, k, v, scaling):
        assert q.shape[2] == 1 and k.shape[2] == 1  # the pass-through cache hands over the new token only
        pk, pv = self.kv[module.layer_idx]
        k_all, v_all = torch.cat([pk, k], 2), torch.cat([pv, v], 2)
        self.kv[module.layer_idx] = (k_all, v_all)
        return _gqa(q, k_all, v_all, False).transpose(1, 2)


def test_prefill_and_decode_route_through_context():
    m = tiny_model()
    ids = torch.randint(0, 128, (1, 40))
    with torch.no_grad():
        ref = m(ids, use_cache=True)
        pre = PrefillStandIn()
        with hf_attention.active(m, pre):
            got = m(ids, use_cache=True)
        assert m.config._attn_implementation == "sdpa"  # restored
        assert [s[0] for s in pre.seen] == [0, 1]
        assert pre.seen[0][1] == (1, 2, 40, 128) and pre.seen[0][2] == (1, 1, 40, 128)
        assert torch.allclose(got.logits, ref.logits, atol=1e-5, rtol=1e-4)

        # one decode step: reference with the model's DynamicCache, ours through the pass-through cache
        nxt = torch.tensor([[int(ref.logits[0, -1].argmax())]])
        pos = torch.tensor([[40]])
        ref2 = m(nxt, past_key_values=ref.past_key_values, position_ids=pos, use_cache=True)
        dec = DecodeStandIn(pre.kv)
        with hf_attention.active(m, dec):
            got2 = m(nxt, past_key_values=hf_attention.pass_through_cache(), position_ids=pos, use_cache=True)
        assert torch.allclose(got2.logits, ref2.logits, atol=1e-5, rtol=1e-4)


def test_no_context_defers_to_sdpa():
    m = tiny_model(1)
    ids = torch.randint(0, 128, (1, 17))
    with torch.no_grad():
        ref = m(ids).logits
        hf_attention.register()
        m.config._attn_implementation = hf_attention.ATTN_IMPLEMENTATION
        try:
            got = m(ids).logits
        finally:
            m.config._attn_implementation = "sdpa"
    assert torch.allclose(got, ref, atol=1e-5, rtol=1e-4)


def test_two_pass_config_defaults_match_reference():
    """two_pass.py:55-90 defaults."""
    from infercache_b200.two_pass import TwoPassConfig
    c = TwoPassConfig()
    assert (c.summary_threshold, c.max_new_tokens, c.temperature, c.top_p, c.top_k, c.repetition_penalty,
            c.use_hidden_importance, c.all_layers_importance, c.importance_layer) == \
        (128, 256, 1.0, 0.95, 0, 1.0, True, False, -1)


def test_sampling_rules():
    """two_pass.py:251-279: repetition penalty, greedy at temperature 0, top-k / top-p masks."""
    from infercache_b200.two_pass import TwoPassConfig, TwoPassEngine
    eng = TwoPassEngine.__new__(TwoPassEngine)
    eng.cfg = TwoPassConfig(temperature=0.0)
    logits = torch.tensor([1.0, 3.0, 2.0, -1.0])
    assert eng._sample(logits, []) == 1
    eng.cfg = TwoPassConfig(temperature=0.0, repetition_penalty=4.0)
    assert eng._sample(logits, [1]) == 2  # 3 / 4 < 2
    eng.cfg = TwoPassConfig(temperature=1.0, top_k=1, top_p=1.0)
    assert all(eng._sample(logits, []) == 1 for _ in range(20))
    eng.cfg = TwoPassConfig(temperature=1.0, top_k=0, top_p=0.5)
    big = torch.tensor([10.0, 0.0, 0.0, 0.0])
    assert all(eng._sample(big, []) == 0 for _ in range(20))
