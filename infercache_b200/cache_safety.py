"""HF past_key_values normalisation at the cache boundary.

``normalise_kv`` accepts the formats the reference accepts
(cache_safety.py:73-162): None, a tuple / list of (K, V) pairs, a
transformers >= 4.36 ``Cache`` with ``.layers[i].keys / .values``, an older
``DynamicCache`` with ``key_cache / value_cache``, anything with
``to_legacy_cache()``, and an iterable of (K, V, ...) items.  It returns a
tuple of (K, V) with K, V [batch, Hkv, T, D], or None when empty, and raises
TypeError for anything else.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

LegacyKV = Tuple[Tuple[torch.Tensor, torch.Tensor], ...]


def normalise_kv(past_key_values) -> Optional[LegacyKV]:
    if past_key_values is None:
        return None
    if isinstance(past_key_values, (tuple, list)):
        if len(past_key_values) == 0:
            return None
        first = past_key_values[0]
        if isinstance(first, (tuple, list)) and len(first) >= 2:
            return tuple((item[0], item[1]) for item in past_key_values)
        raise TypeError(f"past_key_values is a {type(past_key_values).__name__} whose first element has "
                        f"type {type(first).__name__} -- expected a (K, V) pair.")
    layers = getattr(past_key_values, "layers", None)
    if layers is not None:
        try:
            out = tuple((l.keys, l.values) for l in layers
                        if getattr(l, "is_initialized", False) and getattr(l, "keys", None) is not None)
            return out if out else None
        except Exception:
            pass
    kc = getattr(past_key_values, "key_cache", None)
    vc = getattr(past_key_values, "value_cache", None)
    if kc is not None and vc is not None:
        try:
            return tuple(zip(kc, vc)) if len(kc) > 0 else None
        except TypeError:
            pass
    to_legacy = getattr(past_key_values, "to_legacy_cache", None)
    if to_legacy is not None:
        try:
            r = to_legacy()
            if r is not None and len(r) > 0:
                return tuple(r)
        except Exception:
            pass
    try:
        items = list(past_key_values)
        if items and isinstance(items[0], (tuple, list)) and len(items[0]) >= 2:
            return tuple((it[0], it[1]) for it in items)
    except Exception:
        pass
    raise TypeError(f"Cannot normalise past_key_values of type {type(past_key_values).__name__}. "
                    "Expected a DynamicCache (transformers>=4.36), or legacy tuple/list of (K, V) pairs.")


def kv_seq_len(past_key_values) -> int:
    """Sequence length held by a (possibly unnormalised) cache (cache_safety.py:167-195)."""
    if past_key_values is None:
        return 0
    if hasattr(past_key_values, "get_seq_length"):
        try:
            return past_key_values.get_seq_length()
        except Exception:
            pass
    if hasattr(past_key_values, "key_cache"):
        kc = past_key_values.key_cache
        return kc[0].shape[2] if kc and hasattr(kc[0], "shape") else 0
    if isinstance(past_key_values, (tuple, list)) and len(past_key_values) > 0:
        first = past_key_values[0]
        if isinstance(first, (tuple, list)) and hasattr(first[0], "shape"):
            return first[0].shape[2]
    return 0


def to_dynamic_cache(layers_kv):
    """Build a transformers DynamicCache pre-populated with per-layer (K, V)
    (the construction of hierarchical_cache.py:335-348); a tuple when
    transformers is unavailable."""
    try:
        from transformers.cache_utils import DynamicCache, DynamicLayer
    except ImportError:
        return tuple(layers_kv)
    cache = DynamicCache()
    for K, V in layers_kv:
        layer = DynamicLayer()
        layer.dtype = K.dtype
        layer.device = K.device
        layer.keys = K
        layer.values = V
        layer.is_initialized = True
        cache.layers.append(layer)
    return cache
