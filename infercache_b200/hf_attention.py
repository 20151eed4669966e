"""The cache's kernels as a Hugging Face attention implementation.

transformers routes every attention call of a decoder (Qwen2, Llama, ...)
through ``ALL_ATTENTION_FUNCTIONS[config._attn_implementation]`` with the
post-RoPE query [B, Hq, T, D] and the key / value the model's cache object
returned.  Registering ``ATTN_IMPLEMENTATION`` lets the two-pass engine run:

* the summary pass (prefill) through kernel C: causal attention output plus
  the received attention mass per key, accumulated over the layers that
  ``_attention_mass`` reads (two_pass.py:104-137) — no [H, T, T] attention
  tensor and no eager backend;
* each decode step through kernel A: the step's query attends over the
  fixed-budget cache plus the new token (which it appends), so the compact
  ``DynamicCache`` the reference rebuilds every step
  (two_pass.py:312-321) is never built.

Outside an active context the implementation defers to PyTorch SDPA, so a
model left configured with it still runs normally.
"""
from __future__ import annotations

import contextlib
import threading
from typing import Optional

import torch

ATTN_IMPLEMENTATION = "infercache_b200"

_state = threading.local()
_registered = False


def _current():
    return getattr(_state, "ctx", None)


def _attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    ctx = _current()
    if ctx is None:
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        return sdpa_attention_forward(module, query, key, value, attention_mask, scaling=scaling,
                                      dropout=dropout, **kwargs)
    return ctx.attend(module, query, key, value, scaling), None


def _no_mask(*args, **kwargs):
    # both contexts apply causality themselves
    return None


def register() -> str:
    """Register the implementation with transformers (idempotent)."""
    global _registered
    if not _registered:
        from transformers import AttentionInterface
        from transformers.masking_utils import AttentionMaskInterface
        AttentionInterface.register(ATTN_IMPLEMENTATION, _attention)
        AttentionMaskInterface.register(ATTN_IMPLEMENTATION, _no_mask)
        _registered = True
    return ATTN_IMPLEMENTATION


@contextlib.contextmanager
def active(model, ctx):
    """Run ``model`` with this implementation and ``ctx`` handling its attention."""
    register()
    cfg = model.config
    prev_impl = cfg._attn_implementation
    prev_ctx = _current()
    cfg._attn_implementation = ATTN_IMPLEMENTATION
    _state.ctx = ctx
    try:
        yield ctx
    finally:
        _state.ctx = prev_ctx
        cfg._attn_implementation = prev_impl


class SummaryContext:
    """Prefill: causal attention through kernel C, received mass accumulated
    over the selected layers (all, or ``layer_idx % num_layers``)."""

    def __init__(self, num_layers: int, all_layers: bool, layer_idx: int = -1):
        self.num_layers = num_layers
        self.all_layers = all_layers
        self.layer = layer_idx % num_layers
        self.colsum: Optional[torch.Tensor] = None
        self.status: Optional[torch.Tensor] = None

    def attend(self, module, query, key, value, scaling):
        from .summary import summary_score
        if query.shape[0] != 1:
            raise ValueError("the summary pass scores one prompt at a time (batch 1)")
        if self.status is None:
            self.status = torch.zeros(1, dtype=torch.int32, device=query.device)
        want = self.all_layers or module.layer_idx == self.layer
        res = summary_score(query, key, value, scale=scaling, with_mass=want,
                            colsum=self.colsum if want else None,
                            accumulate=want and self.colsum is not None, normalise=False,
                            status=self.status, check_status=False)
        if want:
            self.colsum = res.colsum
        return res.out.transpose(1, 2)

    def importance(self) -> torch.Tensor:
        """colsum / total (two_pass.py:135-137), float32 [T] on the device."""
        if self.status is not None and int(self.status.item()):
            from . import _lib
            raise _lib.InferCacheError(_lib.IC_ERR_DEVICE_TIMEOUT, "summary pass: device-side wait timed out")
        imp = self.colsum[0]
        total = imp.sum()
        return imp / total if float(total) > 1e-9 else imp


class DecodeContext:
    """One decode step of every session of a ``SessionBatch``: each layer's
    attention is kernel A over the session's retained slots plus the new
    token; the caller runs the eviction update after the forward."""

    def __init__(self, batch):
        self.batch = batch
        self.out: Optional[torch.Tensor] = None

    def attend(self, module, query, key, value, scaling):
        b = self.batch
        S, Hq, T, D = query.shape
        if T != 1:
            raise ValueError("decode context: one new token per session per step")
        if self.out is None or self.out.shape != (b.cfg.num_layers, S, Hq, D) or self.out.dtype != query.dtype:
            self.out = torch.empty((b.cfg.num_layers, S, Hq, D), dtype=query.dtype, device=query.device)
        o = self.out[module.layer_idx]
        b.attend(module.layer_idx, query[:, :, 0].contiguous(), key[:, :, -1].contiguous(),
                 value[:, :, -1].contiguous(), out=o)
        return o[:, None]


def pass_through_cache(config=None):
    """A transformers cache that stores nothing: ``update`` hands the step's
    new key / value straight to the attention (the fixed-budget cache keeps
    them)."""
    from transformers import DynamicCache

    class _PassThrough(DynamicCache):
        def update(self, key_states, value_states, layer_idx, *args, **kwargs):
            return key_states, value_states

        def get_seq_length(self, layer_idx: int = 0) -> int:
            return 0

    return _PassThrough()
