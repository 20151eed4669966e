"""Summary-pass importance scoring and tier fill, restated on the CPU.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

* ``attention_mass``: ``_attention_mass`` (two_pass.py:104-137) for one layer
  of causal GQA attention: received[j] = sum_h sum_i P[h, i, j], normalised
  by the total.  The reference materialises P [H, T, T]; this restatement
  walks query chunks so T = 8192 stays within a few hundred MB.
* ``tier_fill``: the slot placement of ``load_from_hf_output``
  (hierarchical_cache.py:179-237 with ``_try_insert_important`` :390-418),
  metadata only: it returns which token each slot holds.
"""
from __future__ import annotations

from typing import Optional

import numpy as np


def causal_softmax_rows(q: np.ndarray, k: np.ndarray, i0: int, scale: float) -> np.ndarray:
    """P rows i0 .. i0+n-1 of causal softmax(q k^T * scale) for one head.

    q: [n, D] (rows i0..), k: [T, D].  Returns float32 [n, T] with zeros above
    the diagonal.
    """
    n = q.shape[0]
    T = k.shape[0]
    s = (q.astype(np.float32) @ k.astype(np.float32).T) * np.float32(scale)
    cols = np.arange(T)[None, :]
    rows = (i0 + np.arange(n))[:, None]
    s = np.where(cols <= rows, s, -np.inf).astype(np.float32)
    m = s.max(axis=1, keepdims=True)
    e = np.exp(s - m)
    return (e / e.sum(axis=1, keepdims=True)).astype(np.float32)


def attention_mass(q: np.ndarray, k: np.ndarray, scale: Optional[float] = None,
                   chunk: int = 512):
    """q: [Hq, T, D]; k: [Hkv, T, D] (GQA: query head h reads KV head h // G).

    Returns (colsum float64 [T], importance float32 [T]) where importance is
    colsum / sum(colsum) as in two_pass.py:135-137.
    """
    Hq, T, D = q.shape
    Hkv = k.shape[0]
    G = Hq // Hkv
    if scale is None:
        scale = D ** -0.5
    colsum = np.zeros(T, np.float64)
    for h in range(Hq):
        kh = k[h // G]
        for i0 in range(0, T, chunk):
            P = causal_softmax_rows(q[h, i0:i0 + chunk], kh, i0, scale)
            colsum += P.sum(axis=0, dtype=np.float64)
    imp = colsum.astype(np.float32)
    total = imp.sum(dtype=np.float32)
    if total > 1e-9:
        imp = (imp / total).astype(np.float32)
    return colsum, imp


def tier_fill(scores: np.ndarray, positions: Optional[np.ndarray], sink: int, recent: int,
              important: int) -> dict:
    """Slot placement of ``load_from_hf_output`` for a prompt of T tokens.

    Returns slot_token [B] (token index per slot, -1 = empty), positions [B],
    importance [B], occupied [B], fills (sink, recent, recent_ptr, important)
    and counters (tokens seen, L2 replacements).
    """
    scores = np.asarray(scores, np.float32)
    T = scores.shape[0]
    if positions is None:
        positions = np.arange(T, dtype=np.int64)
    B = sink + recent + important
    slot_token = np.full(B, -1, np.int64)
    pos_out = np.full(B, -1, np.int64)
    imp = np.zeros(B, np.float32)
    occ = np.zeros(B, bool)
    sink_fill = recent_fill = imp_fill = 0
    evictions = 0
    l2s = sink + recent

    def place(slot, tok):
        slot_token[slot] = tok
        pos_out[slot] = positions[tok]
        imp[slot] = scores[tok]
        occ[slot] = True

    for tok in range(T):
        pos = int(positions[tok])
        if pos < sink and sink_fill < sink:
            place(sink_fill, tok)
            sink_fill += 1
            continue
        if T - tok <= recent:
            if recent_fill < recent:
                place(sink + recent_fill, tok)
                recent_fill += 1
            continue
        if imp_fill < important:
            place(l2s + imp_fill, tok)
            imp_fill += 1
        else:
            e = l2s + int(np.argmin(imp[l2s:l2s + imp_fill]))
            if scores[tok] > imp[e]:
                place(e, tok)
                evictions += 1
    return dict(slot_token=slot_token, positions=pos_out, importance=imp, occupied=occ,
                fills=np.array([sink_fill, recent_fill, sink, imp_fill], np.int64),
                counters=np.array([T, evictions], np.int64))
