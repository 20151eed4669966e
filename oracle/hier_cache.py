"""Numpy restatement of the reference HierarchicalKVCache and its decode protocol.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each method cites the reference function it restates
(``hierarchical_cache.py`` of the ``inference`` package).  Storage mirrors the
reference: K/V ``[L, Hkv, budget, D]`` in the cache dtype, and per-slot
``positions`` (int64, -1 = empty), ``importance`` (float32) and ``occupied``
(bool).  All importance arithmetic is float32, like the reference's CPU
tensors.

Floating-point reduction order.  The reference leaves summation order to
torch.  This restatement fixes one order, the same one the CUDA kernels use,
so that the two agree to the last few ulps:

* received mass of a slot in one layer = sum over the query heads of its KV
  group, g = 0 .. G-1 in order;
* the boost of one decode step = (sum over KV heads h of (sum over layers l
  in order)) / (L * Hkv * Q), which is the mean ``_boost_importance`` takes
  (hierarchical_cache.py:435-438).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np

# Event kinds recorded for every push (one per session-step).
EV_NONE = 0      # ring slot was empty: nothing displaced
EV_DROP = 1      # displaced token had score <= 0 and was dropped
EV_FILL = 2      # displaced token copied into a free L2 slot
EV_EVICT = 3     # displaced token replaced the L2 minimum
EV_REJECT = 4    # displaced token scored <= the L2 minimum and was dropped


@dataclass
class TierGeometry:
    """Restates ``CacheConfig`` (hierarchical_cache.py:67-93)."""
    num_layers: int
    num_kv_heads: int
    head_dim: int
    sink_size: int = 4
    recent_size: int = 256
    important_size: int = 252

    @property
    def total_budget(self) -> int:
        return self.sink_size + self.recent_size + self.important_size

    @property
    def recent_start(self) -> int:
        return self.sink_size

    @property
    def important_start(self) -> int:
        return self.sink_size + self.recent_size


@dataclass
class Event:
    kind: int
    displaced_pos: int = -1
    target_slot: int = -1
    evicted_pos: int = -1

    def as_tuple(self) -> Tuple[int, int, int, int]:
        return (self.kind, self.displaced_pos, self.target_slot, self.evicted_pos)


class OracleCache:
    """Restates ``HierarchicalKVCache`` (hierarchical_cache.py:109-477)."""

    def __init__(self, geo: TierGeometry, kv_dtype=np.float32):
        self.geo = geo
        self.kv_dtype = np.dtype(kv_dtype)
        B = geo.total_budget
        shape = (geo.num_layers, geo.num_kv_heads, B, geo.head_dim)
        self.K = np.zeros(shape, self.kv_dtype)
        self.V = np.zeros(shape, self.kv_dtype)
        self.positions = np.full(B, -1, np.int64)
        self.importance = np.zeros(B, np.float32)
        self.occupied = np.zeros(B, bool)
        self.reset()

    # -- reset (hierarchical_cache.py:362-378) ------------------------------
    def reset(self) -> None:
        self.K[...] = 0
        self.V[...] = 0
        self.positions[:] = -1
        self.importance[:] = 0
        self.occupied[:] = False
        self.sink_fill = 0
        self.recent_fill = 0
        self.recent_ptr = self.geo.recent_start
        self.important_fill = 0
        self.step = 0
        self.total_tokens_seen = 0
        self.total_evictions = 0
        self.near_ties = 0  # L2 decisions whose two smallest scores were within 1e-6 relative
        self.events: List[Event] = []

    @property
    def current_fill(self) -> int:
        return self.sink_fill + self.recent_fill + self.important_fill

    # -- helpers ------------------------------------------------------------
    def sorted_slots(self) -> np.ndarray:
        """Occupied slots ordered by position (hierarchical_cache.py:320-323)."""
        occ = np.nonzero(self.occupied)[0]
        order = np.argsort(self.positions[occ], kind="stable")
        return occ[order]

    def _write_kv(self, slot: int, k_tok: np.ndarray, v_tok: np.ndarray) -> None:
        """``_write_kv`` (hierarchical_cache.py:382-388): k_tok is [L, Hkv, D]."""
        self.K[:, :, slot, :] = k_tok.astype(self.kv_dtype)
        self.V[:, :, slot, :] = v_tok.astype(self.kv_dtype)

    def _l2_min_slot(self) -> int:
        """First-index argmin over the filled L2 slice (:420-425)."""
        s = self.geo.important_start
        return s + int(np.argmin(self.importance[s:s + self.important_fill]))

    # -- bulk load (hierarchical_cache.py:179-237, 390-418) ----------------
    def load_from_hf_output(self, k_tokens: np.ndarray, v_tokens: np.ndarray,
                            scores: np.ndarray,
                            positions: Optional[np.ndarray] = None) -> None:
        """k_tokens/v_tokens: [L, Hkv, T, D]; scores: [T] float32."""
        self.reset()
        g = self.geo
        T = k_tokens.shape[2]
        if positions is None:
            positions = np.arange(T, dtype=np.int64)
        scores = np.asarray(scores, np.float32)
        for tok in range(T):
            pos = int(positions[tok])
            score = scores[tok]
            if pos < g.sink_size and self.sink_fill < g.sink_size:
                slot = self.sink_fill
                self._write_kv(slot, k_tokens[:, :, tok], v_tokens[:, :, tok])
                self.positions[slot] = pos
                self.importance[slot] = score
                self.occupied[slot] = True
                self.sink_fill += 1
                continue
            if T - tok <= g.recent_size:
                if self.recent_fill < g.recent_size:
                    slot = g.recent_start + self.recent_fill
                    self._write_kv(slot, k_tokens[:, :, tok], v_tokens[:, :, tok])
                    self.positions[slot] = pos
                    self.importance[slot] = score
                    self.occupied[slot] = True
                    self.recent_fill += 1
                continue
            self._try_insert_important(k_tokens[:, :, tok], v_tokens[:, :, tok],
                                       score, pos)
        self.total_tokens_seen += T

    def _try_insert_important(self, k_tok, v_tok, score, pos) -> None:
        """``_try_insert_important`` (:390-418); KLL feeding omitted (it never
        influences a decision: ``threshold`` is never called)."""
        g = self.geo
        if self.important_fill < g.important_size:
            slot = g.important_start + self.important_fill
            self.important_fill += 1
        else:
            slot = self._l2_min_slot()
            if not (score > self.importance[slot]):
                return
            self.total_evictions += 1
        self._write_kv(slot, k_tok, v_tok)
        self.positions[slot] = pos
        self.importance[slot] = score
        self.occupied[slot] = True

    # -- push (hierarchical_cache.py:241-294) ------------------------------
    def push(self, k_tok: np.ndarray, v_tok: np.ndarray, position: int,
             attn_weights: Optional[np.ndarray] = None) -> Event:
        """k_tok/v_tok: [L, Hkv, D]; attn_weights: [L, Hkv, Q, F'] or [L, Hkv, F']."""
        g = self.geo
        self.step += 1
        if attn_weights is not None:
            self._boost_importance(attn_weights)
        slot = self.recent_ptr
        ev = Event(EV_NONE)
        if self.occupied[slot]:
            ev = self._maybe_promote_to_l2(slot)
        self._write_kv(slot, k_tok, v_tok)
        self.positions[slot] = position
        self.importance[slot] = 0.0
        self.occupied[slot] = True
        self.recent_fill = min(self.recent_fill + 1, g.recent_size)
        self.recent_ptr = g.recent_start + (self.recent_ptr - g.recent_start + 1) % g.recent_size
        self.total_tokens_seen += 1
        self.events.append(ev)
        return ev

    def _boost_importance(self, w: np.ndarray) -> None:
        """``_boost_importance`` (:427-446): mean over (layers, heads, queries),
        added to occupied slots in position order; extra columns are dropped."""
        w = np.asarray(w, np.float32)
        if w.ndim == 3:
            w = w[:, :, None, :]
        L, H, Q, F = w.shape
        acc_h = []
        for h in range(H):
            acc = w[0, h, 0].copy()
            for qi in range(1, Q):
                acc = acc + w[0, h, qi]
            for l in range(1, L):
                for qi in range(Q):
                    acc = acc + w[l, h, qi]
            acc_h.append(acc)
        total = acc_h[0]
        for h in range(1, H):
            total = total + acc_h[h]
        agg = (total / np.float32(L * H * Q)).astype(np.float32)
        ss = self.sorted_slots()
        n = min(agg.shape[0], ss.shape[0])
        self.importance[ss[:n]] = self.importance[ss[:n]] + agg[:n]

    def _maybe_promote_to_l2(self, recent_slot: int) -> Event:
        """``_maybe_promote_to_l2`` (:448-477)."""
        g = self.geo
        score = self.importance[recent_slot]
        dpos = int(self.positions[recent_slot])
        if score <= 0.0:
            return Event(EV_DROP, dpos)
        if self.important_fill < g.important_size:
            target = g.important_start + self.important_fill
            self.important_fill += 1
            kind, epos = EV_FILL, -1
        else:
            target = self._l2_min_slot()
            s0 = g.important_start
            l2 = np.asarray(self.importance[s0:s0 + self.important_fill], np.float32)
            if l2.shape[0] > 1:
                lo = np.float32(self.importance[target])
                runner = np.min(np.delete(l2, target - s0))
                if float(runner) - float(lo) <= 1e-6 * abs(float(lo)):
                    self.near_ties += 1
            if not (score > self.importance[target]):
                return Event(EV_REJECT, dpos, target, -1)
            kind, epos = EV_EVICT, int(self.positions[target])
            self.total_evictions += 1
        self.K[:, :, target, :] = self.K[:, :, recent_slot, :]
        self.V[:, :, target, :] = self.V[:, :, recent_slot, :]
        self.positions[target] = dpos
        self.importance[target] = score
        self.occupied[target] = True
        return Event(kind, dpos, target, epos)

    # -- export (hierarchical_cache.py:297-360) ----------------------------
    def to_hf_past_key_values(self):
        if not self.occupied.any():
            return None
        ss = self.sorted_slots()
        return [(self.K[l][:, ss, :][None], self.V[l][:, ss, :][None])
                for l in range(self.geo.num_layers)]

    def get_position_ids_for_cache(self) -> np.ndarray:
        return np.sort(self.positions[self.occupied])


# ---------------------------------------------------------------------------
# Decode protocol: one decode step of one session over all layers.
# ---------------------------------------------------------------------------

def attend_group(q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float):
    """GQA decode attention in float32.

    q: [Hq, D]; K, V: [Hkv, F, D].  Returns o [Hq, D] and p [Hkv, G, F].
    Scores are (q . k) * scale; softmax is exp(s - max) / sum.
    """
    Hkv, F, D = K.shape
    G = q.shape[0] // Hkv
    qh = q.astype(np.float32).reshape(Hkv, G, D)
    s = np.matmul(qh, K.astype(np.float32).transpose(0, 2, 1)) * np.float32(scale)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    p = e / e.sum(axis=-1, keepdims=True)
    o = np.matmul(p, V.astype(np.float32))
    return o.reshape(Hkv * G, D).astype(np.float32), p.astype(np.float32)


def group_mass(p: np.ndarray) -> np.ndarray:
    """Received mass per key summed over the query heads of each KV group,
    g = 0 .. G-1 in order.  p: [Hkv, G, F] -> [Hkv, F]."""
    acc = p[:, 0, :].copy()
    for gi in range(1, p.shape[1]):
        acc = acc + p[:, gi, :]
    return acc


def decode_step(cache: OracleCache, q: np.ndarray, k: np.ndarray, v: np.ndarray,
                position: int, decay: float, scale: Optional[float] = None):
    """One step of the decode protocol on one session.

    q: [L, Hq, D]; k, v: [L, Hkv, D] (already in the cache dtype).
    1. gather the occupied slots in position order and append the new token;
    2. attend (per layer) and take the group-summed received mass;
    3. decay the importance of every occupied slot (importance *= decay);
    4. ``push`` with the mass as ``attn_weights`` (the push drops the new
       token's own column: hierarchical_cache.py:445).
    Returns (o [L, Hq, D] float32, Event).
    """
    g = cache.geo
    if scale is None:
        scale = g.head_dim ** -0.5
    ss = cache.sorted_slots()
    L = g.num_layers
    outs = []
    weights = []
    for l in range(L):
        K = np.concatenate([cache.K[l][:, ss, :], k[l][:, None, :].astype(cache.kv_dtype)], axis=1)
        V = np.concatenate([cache.V[l][:, ss, :], v[l][:, None, :].astype(cache.kv_dtype)], axis=1)
        o, p = attend_group(q[l], K, V, scale)
        outs.append(o)
        weights.append(group_mass(p))
    w = np.stack(weights)[:, :, None, :]            # [L, Hkv, 1, F+1]
    occ = cache.occupied
    cache.importance[occ] = cache.importance[occ] * np.float32(decay)
    ev = cache.push(k, v, position, w)
    return np.stack(outs), ev
