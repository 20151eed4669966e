"""Two-pass inference over the fixed-budget cache (drop-in for two_pass.py).

Same classes, fields and methods as the reference (TwoPassConfig :55-90,
SummaryResult :93-100, TwoPassEngine :142-434):

1. ``summary_pass`` runs the model over the prompt once and scores every
   token — by the last hidden state's L2 norm (``use_hidden_importance``,
   the reference default) or by received attention mass.  The attention-mass
   mode runs each layer's attention through kernel C (``hf_attention``), so it
   needs no eager backend and no [H, T, T] tensors.
2. ``_prime_cache`` fills the cache's tiers from the prompt's K/V (kernel D).
3. ``_generate_two_pass`` decodes token by token.  ``decode_path="fused"``
   runs each step's attention as kernel A over the cache (no per-step
   ``DynamicCache``) and then the eviction update (kernel B);
   ``"dynamic_cache"`` is the reference's loop (to_hf_past_key_values, model
   forward, push of the new K/V).  Both push the new token at position
   ``cur_pos + 1`` with no attention weights, as the reference does
   (two_pass.py:326-336); ``decode_importance=True`` instead feeds each step's
   received mass back into the importance scores (decayed by the cache's
   ``decay``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, List, Optional

import torch

from . import hf_attention
from .cache_safety import normalise_kv
from .hierarchical_cache import CacheConfig, HierarchicalKVCache


@dataclass
class TwoPassConfig:
    summary_threshold: int = 128
    max_new_tokens: int = 256
    temperature: float = 1.0
    top_p: float = 0.95
    top_k: int = 0
    repetition_penalty: float = 1.0
    use_hidden_importance: bool = True
    all_layers_importance: bool = False
    importance_layer: int = -1
    # decode step: "fused" (kernel A as the model's attention) or "dynamic_cache"
    decode_path: str = "fused"
    # feed each decode step's received attention mass into the importance
    decode_importance: bool = False


@dataclass
class SummaryResult:
    importance_scores: torch.Tensor   # [seq_len] float32, CPU
    past_key_values: object
    last_logits: torch.Tensor         # [vocab] CPU
    seq_len: int
    hidden_states: Optional[torch.Tensor] = None


class TwoPassEngine:
    """Wraps a Hugging Face causal LM (Qwen2-style attention modules)."""

    def __init__(self, model, tokenizer, cache_cfg: CacheConfig, cfg: Optional[TwoPassConfig] = None,
                 device: str = "cuda"):
        self.model = model
        self.tokenizer = tokenizer
        self.cache_cfg = cache_cfg
        self.cfg = cfg or TwoPassConfig()
        if self.cfg.decode_path not in ("fused", "dynamic_cache"):
            raise ValueError(f"decode_path must be 'fused' or 'dynamic_cache', got {self.cfg.decode_path!r}")
        self.device = torch.device(device)
        self._cache = HierarchicalKVCache(cache_cfg, device=self.device)

    # ---- pass 1 ------------------------------------------------------------------------
    @torch.inference_mode()
    def summary_pass(self, input_ids: torch.Tensor) -> SummaryResult:
        ids = input_ids.to(self.device)
        if self.cfg.use_hidden_importance:
            out = self.model(ids, output_attentions=False, output_hidden_states=True, use_cache=True)
            h = out.hidden_states[-1][0].float()
            importance = h.norm(dim=-1)
            total = importance.sum()
            importance = (importance / total if total > 1e-9 else importance).cpu()
            hidden = out.hidden_states[-1].detach().cpu()
        else:
            ctx = hf_attention.SummaryContext(self.model.config.num_hidden_layers,
                                              self.cfg.all_layers_importance, self.cfg.importance_layer)
            with hf_attention.active(self.model, ctx):
                out = self.model(ids, output_attentions=False,
                                 output_hidden_states=self.cfg.all_layers_importance, use_cache=True)
            importance = ctx.importance().float().cpu()
            hidden = out.hidden_states[-1].detach().cpu() if out.hidden_states is not None else None
        return SummaryResult(importance_scores=importance, past_key_values=out.past_key_values,
                             last_logits=out.logits[0, -1].detach().cpu(), seq_len=ids.shape[1],
                             hidden_states=hidden)

    def _prime_cache(self, summary: SummaryResult) -> None:
        self._cache.reset()
        self._cache.load_from_hf_output(past_key_values=summary.past_key_values,
                                        importance_scores=summary.importance_scores,
                                        positions=torch.arange(summary.seq_len, dtype=torch.long))

    # ---- sampling (two_pass.py:251-279) ------------------------------------------------------
    def _sample(self, logits: torch.Tensor, generated: List[int]) -> int:
        cfg = self.cfg
        logits = logits.float().clone()
        if cfg.repetition_penalty != 1.0 and generated:
            for tok in set(generated):
                logits[tok] = logits[tok] / cfg.repetition_penalty if logits[tok] > 0 \
                    else logits[tok] * cfg.repetition_penalty
        if cfg.temperature < 1e-4:
            return int(logits.argmax(-1).item())
        logits /= cfg.temperature
        if cfg.top_k > 0:
            kth = logits.topk(cfg.top_k).values[-1]
            logits[logits < kth] = float("-inf")
        if cfg.top_p < 1.0:
            srt, idx = logits.sort(descending=True)
            probs = srt.softmax(-1)
            drop = (probs.cumsum(-1) - probs) > cfg.top_p
            logits[idx[drop]] = float("-inf")
        return int(logits.softmax(-1).multinomial(1).item())

    # ---- pass 2 ---------------------------------------------------------------------------
    def _decode_step_fused(self, token: int, cur_pos: int):
        b = self._cache.batch
        ctx = hf_attention.DecodeContext(b)
        with hf_attention.active(self.model, ctx):
            out = self.model(torch.tensor([[token]], device=self.device),
                             past_key_values=hf_attention.pass_through_cache(),
                             position_ids=torch.tensor([[cur_pos]], device=self.device, dtype=torch.long),
                             use_cache=True)
        if self.cfg.decode_importance:
            b.evict([cur_pos + 1])
        else:
            b.evict([cur_pos + 1], decay=1.0, use_mass=False)
        return out.logits[0, -1]

    def _decode_step_dynamic(self, token: int, cur_pos: int):
        past_kv = self._cache.to_hf_past_key_values(device=self.device)
        out = self.model(torch.tensor([[token]], device=self.device), past_key_values=past_kv,
                         position_ids=torch.tensor([[cur_pos]], device=self.device, dtype=torch.long),
                         use_cache=True)
        new_pkv = normalise_kv(out.past_key_values)
        new_k = torch.stack([new_pkv[l][0][0, :, -1, :] for l in range(len(new_pkv))], dim=0).unsqueeze(2)
        new_v = torch.stack([new_pkv[l][1][0, :, -1, :] for l in range(len(new_pkv))], dim=0).unsqueeze(2)
        self._cache.push(new_k, new_v, position=cur_pos + 1)
        return out.logits[0, -1]

    @torch.inference_mode()
    def _generate_two_pass(self, input_ids: torch.Tensor, eos_token_id: Optional[int]) -> List[int]:
        summary = self.summary_pass(input_ids)
        self._prime_cache(summary)
        generated: List[int] = []
        logits = summary.last_logits.to(self.device)
        T = summary.seq_len
        step_fn = self._decode_step_fused if self.cfg.decode_path == "fused" else self._decode_step_dynamic
        for step in range(self.cfg.max_new_tokens):
            next_id = self._sample(logits, generated)
            generated.append(next_id)
            if eos_token_id is not None and next_id == eos_token_id:
                break
            if len(generated) >= self.cfg.max_new_tokens:
                break
            logits = step_fn(next_id, T + step)
        self._cache.batch.check_device_status()
        return generated

    @torch.inference_mode()
    def _generate_direct(self, input_ids: torch.Tensor, eos_token_id: Optional[int]) -> List[int]:
        generated: List[int] = []
        past_kv = None
        cur = input_ids.to(self.device)
        for _ in range(self.cfg.max_new_tokens):
            out = self.model(cur, past_key_values=past_kv, use_cache=True)
            logits = out.logits[0, -1]
            next_id = self._sample(logits, generated)
            generated.append(next_id)
            if eos_token_id is not None and next_id == eos_token_id:
                break
            past_kv = out.past_key_values
            cur = torch.tensor([[next_id]], device=self.device)
        return generated

    # ---- public API ---------------------------------------------------------------------------
    def generate_ids(self, prompt: str, max_new_tokens: Optional[int] = None,
                     eos_token_id: Optional[int] = None) -> List[int]:
        if max_new_tokens is not None:
            self.cfg.max_new_tokens = max_new_tokens
        if eos_token_id is None:
            eos_token_id = getattr(self.tokenizer, "eos_token_id", None)
        ids = self.tokenizer.encode(prompt, return_tensors="pt")
        if ids.shape[1] > self.cfg.summary_threshold:
            return self._generate_two_pass(ids, eos_token_id)
        return self._generate_direct(ids, eos_token_id)

    def generate(self, prompt: str, **kwargs) -> str:
        return self.tokenizer.decode(self.generate_ids(prompt, **kwargs), skip_special_tokens=True)

    def stream_generate(self, prompt: str, eos_token_id: Optional[int] = None) -> Iterator[str]:
        if eos_token_id is None:
            eos_token_id = getattr(self.tokenizer, "eos_token_id", None)
        ids = self.tokenizer.encode(prompt, return_tensors="pt")
        gen = (self._generate_two_pass(ids, eos_token_id) if ids.shape[1] > self.cfg.summary_threshold
               else self._generate_direct(ids, eos_token_id))
        for tok in gen:
            yield self.tokenizer.decode([tok], skip_special_tokens=False)

    def reset_cache(self) -> None:
        self._cache.reset()
