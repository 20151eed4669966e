"""Fixed-budget hierarchical KV cache on the B200.

Same tiers and semantics as the reference's ``hierarchical_cache.py``:
``[0, sink)`` attention sinks, ``[sink, sink+recent)`` the recent ring,
``[sink+recent, budget)`` the scored L2 pool with first-index-argmin
eviction (hierarchical_cache.py:6-48, 67-93).

Two classes:

* ``SessionBatch`` -- S sessions whose K/V live in one ``PagePool`` and whose
  slot metadata (positions, importance, occupancy, fill pointers, counters)
  lives on the GPU.  Its verbs are the decode hot path, all sessions per
  launch:
    ``attend(layer, q, k, v)``  kernel A: append + paged gather + GQA decode
                                attention + received mass, one layer;
    ``evict(positions)``        kernel B: decayed importance + mass,
                                promotion / eviction, ring advance;
    ``step(q, k, v, pos)``      every layer then ``evict``;
    ``gather(session)``         position-ordered K/V export.
* ``HierarchicalKVCache`` -- the reference's single-session class with the
  same constructor and methods (``push``, ``load_from_hf_output``,
  ``to_hf_past_key_values``, ``get_position_ids_for_cache``, ``reset``,
  ``stats``, ``current_fill``, ``total_budget`` and the public
  ``K / V / positions / importance / occupied`` tensors), backed by a
  one-session ``SessionBatch``.

Each logical slot maps to a pool row through a per-session slot table with
one extra entry, the staging row.  A decode step writes the new token's K/V
into the staging row of every layer; ``evict`` then rotates slot-table
entries so the staging row becomes the ring slot and a promoted token's row
moves to its L2 slot.  Promotion therefore copies no K/V (the reference
copies all layers, hierarchical_cache.py:461-462, 472-473).

There is no CPU path: construction requires an sm_100 device and the built
library.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .cache_safety import normalise_kv, to_dynamic_cache
from .paged_cache import PAGE_SIZE, PagedCacheConfig, PagePool

__all__ = ["CacheConfig", "CacheStats", "SessionBatch", "HostStepper", "HierarchicalKVCache", "_normalise_past_kv"]


@dataclass
class CacheConfig:
    """hierarchical_cache.py:67-93.  ``decay`` multiplies the importance of
    every occupied slot once per fused decode step (``SessionBatch.evict``);
    ``evict_quantile`` and ``kll_k`` are accepted for compatibility and
    unused (the reference never reads the quantile sketch either)."""
    num_layers: int
    num_kv_heads: int
    head_dim: int
    sink_size: int = 4
    recent_size: int = 256
    important_size: int = 252
    evict_quantile: float = 0.15
    decay: float = 0.99
    kll_k: int = 128
    dtype: torch.dtype = torch.float16

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
class CacheStats:
    """hierarchical_cache.py:98-105."""
    total_tokens_seen: int = 0
    total_evictions: int = 0
    current_fill: int = 0
    sink_fill: int = 0
    recent_fill: int = 0
    important_fill: int = 0
    total_promotions: int = 0  # tokens moved from the recent ring into the importance tier
    # eviction decisions whose two smallest importance-tier scores were within
    # 1e-6 relative: decisions that float summation order could flip
    near_ties: int = 0


def _check_cfg(cfg: CacheConfig) -> None:
    if cfg.recent_size < 1:
        raise ValueError("recent_size must be >= 1 (the ring advances modulo recent_size)")
    if cfg.sink_size < 0 or cfg.important_size < 0:
        raise ValueError("tier sizes must be >= 0")
    if not (0.0 < cfg.decay <= 1.0):
        raise ValueError(f"decay must be in (0, 1], got {cfg.decay}")


class SessionBatch:
    """S fixed-budget sessions on one GPU, one PagePool, device-resident metadata."""

    def __init__(self, cfg: CacheConfig, num_sessions: int, device="cuda",
                 pool: Optional[PagePool] = None, session_pages: Optional[Sequence[Sequence[int]]] = None):
        _check_cfg(cfg)
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        _lib.require_device(dev)
        self.cfg = cfg
        self.device = dev
        self.num_sessions = S = int(num_sessions)
        B = cfg.total_budget
        ntot = B + 1
        self.pages_per_session = -(-ntot // PAGE_SIZE)
        if pool is None:
            pool = PagePool(PagedCacheConfig(n_pages=max(1, S) * self.pages_per_session, n_layers=cfg.num_layers,
                                             n_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, dtype=cfg.dtype,
                                             device=str(dev), max_pages_per_session=self.pages_per_session))
            session_pages = [list(range(i * self.pages_per_session, (i + 1) * self.pages_per_session))
                             for i in range(S)]
        elif session_pages is None:
            raise ValueError("session_pages is required with a shared pool")
        pc = pool.cfg
        if (pc.n_layers, pc.n_heads, pc.head_dim, pc.dtype) != (cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, cfg.dtype):
            raise ValueError("pool geometry / dtype does not match the cache config")
        self.pool = pool
        self.session_pages = [list(p) for p in session_pages]
        rows = []
        for pages in self.session_pages:
            if len(pages) < self.pages_per_session:
                raise ValueError(f"each session needs {self.pages_per_session} pages")
            r = [p * PAGE_SIZE + o for p in pages for o in range(PAGE_SIZE)][:ntot]
            rows.append(r)
        self.slot_table = torch.tensor(rows, dtype=torch.int32).reshape(S, ntot).to(dev)
        self.positions = torch.full((S, B), -1, dtype=torch.int64, device=dev)
        self.importance = torch.zeros((S, B), dtype=torch.float32, device=dev)
        self.occupied = torch.zeros((S, B), dtype=torch.bool, device=dev)
        self.ctrl = torch.zeros((S, _lib.IC_CTRL_WORDS), dtype=torch.int32, device=dev)
        self.ctrl[:, _lib.IC_CTRL_RECENT_PTR] = cfg.recent_start
        self.counters = torch.zeros((S, _lib.IC_COUNTER_WORDS), dtype=torch.int64, device=dev)
        self.dev_status = torch.zeros(1, dtype=torch.int32, device=dev)
        # received mass of each slot per KV head, summed over the step's layers in layer order
        self.mass = torch.zeros((S, cfg.num_kv_heads, ntot), dtype=torch.float32, device=dev)
        self.events = torch.full((S, 4), -1, dtype=torch.int64, device=dev)
        self._pos_buf = torch.zeros(S, dtype=torch.int64, device=dev)
        self.scale = cfg.head_dim ** -0.5
        self.cluster_size = 0
        self.kernel_variant = _lib.IC_DECODE_AUTO

        self._c_tiers = _lib.ic_tiers(cfg.sink_size, cfg.recent_size, cfg.important_size, B)
        self._c_sess = _lib.ic_sessions(num_sessions=S, slot_table=self.slot_table.data_ptr(),
                                        positions=self.positions.data_ptr(), importance=self.importance.data_ptr(),
                                        occupied=self.occupied.data_ptr(), ctrl=self.ctrl.data_ptr(),
                                        counters=self.counters.data_ptr(), dev_status=self.dev_status.data_ptr())
        self._c_pool = pool.c_pool()
        self._dec = _lib.ic_decode_args(pool=self._c_pool, tiers=self._c_tiers, sess=self._c_sess,
                                        mass=self.mass.data_ptr(), scale=self.scale)
        self._ev = _lib.ic_evict_args(tiers=self._c_tiers, sess=self._c_sess, mass=self.mass.data_ptr(),
                                      mass_heads=cfg.num_kv_heads, mass_layers=1,
                                      mass_div=float(cfg.num_layers * cfg.num_kv_heads),
                                      decay=cfg.decay, new_pos=self._pos_buf.data_ptr(),
                                      events=self.events.data_ptr())
        # programmatic dependent launch between the step's kernels
        self.pdl = True
        self._step = _lib.ic_step_args(layer0=self._dec, evict=self._ev)

    # ---- hot path -------------------------------------------------------------------
    def attend(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """Kernel A for one layer: q [S, Hq, D], k / v [S, Hkv, D] in the cache
        dtype, contiguous, on this device.  Returns out [S, Hq, D].  The first
        layer of a step must be layer 0 (it starts the step's mass sum)."""
        cfg = self.cfg
        S = self.num_sessions
        if q.dim() != 3 or q.shape[0] != S or q.shape[2] != cfg.head_dim:
            raise ValueError(f"q must be [S={S}, Hq, {cfg.head_dim}], got {tuple(q.shape)}")
        if tuple(k.shape) != (S, cfg.num_kv_heads, cfg.head_dim) or k.shape != v.shape:
            raise ValueError(f"k / v must be [{S}, {cfg.num_kv_heads}, {cfg.head_dim}]")
        for t in (q, k, v):
            if t.dtype != cfg.dtype or t.device != self.device or not t.is_contiguous():
                raise ValueError("q / k / v must be contiguous tensors of the cache dtype on the cache device")
        Hq = q.shape[1]
        od = out_dtype or cfg.dtype
        if out is None:
            out = torch.empty((S, Hq, cfg.head_dim), dtype=od, device=self.device)
        elif out.shape != q.shape or not out.is_contiguous() or out.device != self.device:
            raise ValueError("out must be a contiguous [S, Hq, D] tensor on the cache device")
        d = self._dec
        self._prepare_decode(d, Hq)
        d.layer = layer
        d.q = q.data_ptr()
        d.k_new = k.data_ptr()
        d.v_new = v.data_ptr()
        d.out = out.data_ptr()
        d.out_dtype = _lib.dtype_code(out.dtype)
        d.inputs_ready = 0
        _lib.call("ic_decode_layer", d)
        return out

    def _prepare_decode(self, d: "_lib.ic_decode_args", Hq: int) -> None:
        """Set the launch options of one decode call on `d`."""
        d.num_q_heads = Hq
        d.cluster_size = self.cluster_size
        d.kernel_variant = self.kernel_variant
        d.pdl = 1 if self.pdl else 0

    def evict(self, positions, decay: Optional[float] = None, use_mass: bool = True) -> None:
        """Kernel B once per step after the last layer.  positions: [S] int64
        (tensor on this device, or a sequence of ints) of the decoded tokens.
        ``use_mass=False`` skips the importance boost (a push without attention
        weights, hierarchical_cache.py:259-261)."""
        pos = self._positions_arg(positions)
        e = self._ev
        e.new_pos = pos.data_ptr()
        e.decay = self.cfg.decay if decay is None else float(decay)
        e.mass = self.mass.data_ptr() if use_mass else 0
        e.mass_heads = self.cfg.num_kv_heads
        e.mass_layers = 1
        e.mass_div = float(self.cfg.num_layers * self.cfg.num_kv_heads)
        e.pdl = 1 if self.pdl else 0
        e.advance_pos = 0
        _lib.call("ic_evict_update", e)
        self._keep = pos  # keep alive until the launch is consumed

    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions,
             out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
             advance_positions: bool = False) -> torch.Tensor:
        """One decode step of every session in one C call (``ic_decode_step``):
        q [L, S, Hq, D], k / v [L, S, Hkv, D] contiguous in the cache dtype;
        positions [S] of the decoded tokens.  Returns out [L, S, Hq, D].
        ``advance_positions`` (positions an int64 tensor on this device): the
        eviction kernel adds one to each session's position once it has read
        it, so consecutive steps need no separate increment launch."""
        cfg = self.cfg
        L, S, D = cfg.num_layers, self.num_sessions, cfg.head_dim
        if q.dim() != 4 or q.shape[0] != L or q.shape[1] != S or q.shape[3] != D:
            raise ValueError(f"q must be [L={L}, S={S}, Hq, {D}], got {tuple(q.shape)}")
        if tuple(k.shape) != (L, S, cfg.num_kv_heads, D) or k.shape != v.shape:
            raise ValueError(f"k / v must be [{L}, {S}, {cfg.num_kv_heads}, {D}]")
        for t in (q, k, v):
            if t.dtype != cfg.dtype or t.device != self.device or not t.is_contiguous():
                raise ValueError("q / k / v must be contiguous tensors of the cache dtype on the cache device")
        Hq = q.shape[2]
        if out is None:
            out = torch.empty(q.shape, dtype=out_dtype or cfg.dtype, device=self.device)
        elif out.shape != q.shape or not out.is_contiguous() or out.device != self.device:
            raise ValueError("out must be a contiguous [L, S, Hq, D] tensor on the cache device")
        pos = self._positions_arg(positions)
        st = self._step
        d = st.layer0
        self._prepare_decode(d, Hq)
        d.q = q.data_ptr()
        d.k_new = k.data_ptr()
        d.v_new = v.data_ptr()
        d.out = out.data_ptr()
        d.out_dtype = _lib.dtype_code(out.dtype)
        st.evict.pdl = 1 if self.pdl else 0
        if advance_positions and not (isinstance(positions, torch.Tensor) and positions.device == self.device
                                      and positions.dtype == torch.int64 and positions.is_contiguous()):
            raise ValueError("advance_positions needs positions as a contiguous int64 tensor on the cache device")
        st.evict.advance_pos = 1 if advance_positions else 0
        st.q_layer_stride = S * Hq * D
        st.kv_layer_stride = S * cfg.num_kv_heads * D
        st.out_layer_stride = S * Hq * D
        st.evict.new_pos = pos.data_ptr()
        st.evict.decay = cfg.decay
        _lib.call("ic_decode_step", st)
        self._keep = pos
        return out

    def _step_raw(self, q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, num_q_heads: int,
                  out_dtype: torch.dtype, pos: torch.Tensor) -> None:
        """``step`` on raw device addresses of contiguous [L, S, H, D] buffers
        in the cache dtype (e.g. mapped pinned host memory), advancing the
        positions; no checks."""
        cfg = self.cfg
        S, D = self.num_sessions, cfg.head_dim
        st = self._step
        d = st.layer0
        self._prepare_decode(d, num_q_heads)
        d.q, d.k_new, d.v_new, d.out = q_ptr, k_ptr, v_ptr, out_ptr
        d.out_dtype = _lib.dtype_code(out_dtype)
        st.evict.pdl = 1 if self.pdl else 0
        st.evict.advance_pos = 1
        st.q_layer_stride = S * num_q_heads * D
        st.kv_layer_stride = S * cfg.num_kv_heads * D
        st.out_layer_stride = S * num_q_heads * D
        st.evict.new_pos = pos.data_ptr()
        st.evict.decay = cfg.decay
        _lib.call("ic_decode_step", st)
        self._keep = pos

    def host_stepper(self, q_host: torch.Tensor, k_host: torch.Tensor, v_host: torch.Tensor,
                     out_host, positions: torch.Tensor, zero_copy: bool = False) -> "HostStepper":
        """A decode step from pinned host buffers, captured once as a CUDA graph
        (see ``HostStepper``)."""
        return HostStepper(self, q_host, k_host, v_host, out_host, positions, zero_copy=zero_copy)

    def grouped_stepper(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                        positions: torch.Tensor, groups: int = 8, steps_per_graph: int = 4) -> "GroupedStepper":
        """Decode steps of every session with the sessions split into
        ``groups`` ranges on their own streams (see ``GroupedStepper``)."""
        return GroupedStepper(self, q, k, v, out, positions, groups=groups, steps_per_graph=steps_per_graph)

    def grouped_host_stepper(self, positions: torch.Tensor, num_q_heads: int, groups: int = 8) -> "GroupedHostStepper":
        """Decode steps driven from pinned host buffers, the sessions split into
        ``groups`` ranges on their own streams (see ``GroupedHostStepper``)."""
        return GroupedHostStepper(self, positions, num_q_heads, groups=groups)

    def _positions_arg(self, positions) -> torch.Tensor:
        if isinstance(positions, torch.Tensor) and positions.device == self.device and positions.dtype == torch.int64:
            return positions.contiguous()
        pos = torch.as_tensor(positions, dtype=torch.int64).reshape(self.num_sessions)
        self._pos_buf.copy_(pos, non_blocking=True)
        return self._pos_buf

    # ---- reference-compatible push (per session) --------------------------------------
    def push(self, session: int, key_states: torch.Tensor, value_states: torch.Tensor, position: int,
             attn_weights: Optional[torch.Tensor] = None) -> None:
        """hierarchical_cache.py:241-294 for one session of the batch:
        key_states [L, Hkv, 1, D]; attn_weights [L, Hkv, Q, F'] or [L, Hkv, F']
        (position-ordered, averaged over L, Hkv, Q).  No importance decay."""
        cfg = self.cfg
        sub = self._sub(session)
        k = key_states.to(self.device, cfg.dtype)[:, :, 0, :].contiguous()
        v = value_states.to(self.device, cfg.dtype)[:, :, 0, :].contiguous()
        if k.shape != (cfg.num_layers, cfg.num_kv_heads, cfg.head_dim):
            raise ValueError("key_states must be [num_layers, num_kv_heads, 1, head_dim]")
        a = _lib.ic_append_args(pool=self._c_pool, tiers=self._c_tiers, sess=sub, k=k.data_ptr(), v=v.data_ptr(),
                                stride_s=0, stride_l=k.stride(0), stride_h=k.stride(1))
        _lib.call("ic_append_staging", a)
        mass = None
        if attn_weights is not None:
            w = attn_weights.to(self.device, torch.float32)
            if w.dim() == 3:
                w = w[:, :, None, :]
            w = w.contiguous()
            Lw, Hw, Qw, F = w.shape
            srt, fill = self._sort(sub)
            mass = torch.empty((1, cfg.total_budget + 1), dtype=torch.float32, device=self.device)
            b = _lib.ic_boost_args(tiers=self._c_tiers, num_sessions=1, L=Lw, H=Hw, Q=Qw, width=F,
                                   weights=w.data_ptr(), sorted_slots=srt.data_ptr(), fill=fill.data_ptr(),
                                   mass_out=mass.data_ptr())
            _lib.call("ic_boost_sorted", b)
        pos = torch.tensor([int(position)], dtype=torch.int64).to(self.device, non_blocking=True)
        e = _lib.ic_evict_args(tiers=self._c_tiers, sess=sub, mass=_lib.ptr(mass), mass_heads=1, mass_layers=1,
                               mass_div=1.0,
                               decay=1.0, new_pos=pos.data_ptr(),
                               events=self.events[session:].data_ptr())
        _lib.call("ic_evict_update", e)
        self._keep = (k, v, mass, pos)

    def append(self, k: torch.Tensor, v: torch.Tensor, positions) -> None:
        """The new token of every session appended at once, without attention:
        k / v [L, S, Hkv, D] (any float dtype, on any device), positions [S].
        One staging-row write over all sessions and layers, then kernel B with
        no importance boost and no decay -- for every session what the
        reference's ``push(key, value, position)`` without ``attn_weights``
        does (hierarchical_cache.py:241-294), e.g. the two-pass loop's push
        (two_pass.py:326-336)."""
        cfg = self.cfg
        S = self.num_sessions
        want = (cfg.num_layers, S, cfg.num_kv_heads, cfg.head_dim)
        if tuple(k.shape) != want or k.shape != v.shape:
            raise ValueError(f"k / v must be [L, S, Hkv, D] = {list(want)}")
        k = k.to(self.device, cfg.dtype)
        v = v.to(self.device, cfg.dtype)
        if k.stride(-1) != 1 or k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        a = _lib.ic_append_args(pool=self._c_pool, tiers=self._c_tiers, sess=self._c_sess, k=k.data_ptr(),
                                v=v.data_ptr(), stride_s=k.stride(1), stride_l=k.stride(0), stride_h=k.stride(2))
        _lib.call("ic_append_staging", a)
        pos = self._positions_arg(positions)
        e = self._ev
        e.new_pos = pos.data_ptr()
        e.decay = 1.0
        e.mass = 0
        e.mass_heads = cfg.num_kv_heads
        e.mass_layers = 1
        e.mass_div = 1.0
        e.pdl = 0
        e.advance_pos = 0
        _lib.call("ic_evict_update", e)
        self._keep = (k, v, pos)

    # ---- priming, export, reset ------------------------------------------------------------
    def load_prompt(self, session: int, past_key_values, importance_scores: torch.Tensor,
                    positions: Optional[torch.Tensor] = None) -> None:
        """load_from_hf_output (hierarchical_cache.py:179-237) for one session."""
        cfg = self.cfg
        pkv = normalise_kv(past_key_values)
        if pkv is None:
            raise TypeError("past_key_values is empty")
        T = pkv[0][0].shape[2]
        self.reset([session], zero_kv=True)
        sub = self._sub(session)
        scores = importance_scores.to(self.device, torch.float32).reshape(1, T).contiguous()
        pos = None
        if positions is not None:
            pos = positions.to(self.device, torch.int64).reshape(1, T).contiguous()
        slot_token = torch.empty((1, cfg.total_budget), dtype=torch.int32, device=self.device)
        a = _lib.ic_tier_fill_args(tiers=self._c_tiers, sess=sub, session0=0, n=1, T=T,
                                   scores=scores.data_ptr(), positions=_lib.ptr(pos),
                                   slot_token=slot_token.data_ptr())
        _lib.call("ic_tier_fill", a)
        keep = []
        for li in range(min(cfg.num_layers, len(pkv))):
            K, V = pkv[li]
            Ks = K[0].to(self.device)
            Vs = V[0].to(self.device)
            if Ks.stride(-1) != 1 or Vs.stride(-1) != 1 or Ks.stride() != Vs.stride():
                Ks, Vs = Ks.contiguous(), Vs.contiguous()
            src_dt = _lib.dtype_code(Ks.dtype)
            Vs = Vs.to(Ks.dtype)
            la = _lib.ic_load_layer_args(pool=self._c_pool, tiers=self._c_tiers, sess=sub, session=0, layer=li,
                                         slot_token=slot_token.data_ptr(), k_src=Ks.data_ptr(), v_src=Vs.data_ptr(),
                                         stride_h=Ks.stride(0), stride_t=Ks.stride(1), src_dtype=src_dt, T=T)
            _lib.call("ic_load_layer", la)
            keep.append((Ks, Vs))
        self._keep = (keep, scores, pos, slot_token)
        return slot_token

    def _sort(self, sub=None):
        sub = sub if sub is not None else self._c_sess
        n = sub.num_sessions
        srt = torch.empty((n, self.cfg.total_budget), dtype=torch.int32, device=self.device)
        fill = torch.empty(n, dtype=torch.int32, device=self.device)
        _lib.call("ic_sort_slots", _lib.ic_sort_args(tiers=self._c_tiers, sess=sub, sorted_slots=srt.data_ptr(),
                                                     fill=fill.data_ptr()))
        return srt, fill

    def sorted_slots(self, session: int) -> torch.Tensor:
        """Occupied slots of `session` in position order (int64, on device)."""
        srt, fill = self._sort(self._sub(session))
        return srt[0, : int(fill[0].item())].long()

    def gather(self, session: int, slots: Optional[torch.Tensor] = None, layers: Optional[Tuple[int, int]] = None):
        """K, V [L', Hkv, n, D] of `slots` (default: occupied slots in position
        order) of one session."""
        cfg = self.cfg
        if slots is None:
            slots = self.sorted_slots(session)
        sl = slots.to(self.device, torch.int32).contiguous()
        lb, le = layers if layers is not None else (0, cfg.num_layers)
        n = sl.numel()
        K = torch.empty((le - lb, cfg.num_kv_heads, n, cfg.head_dim), dtype=cfg.dtype, device=self.device)
        V = torch.empty_like(K)
        if n:
            a = _lib.ic_gather_args(pool=self._c_pool, tiers=self._c_tiers, sess=self._c_sess, session=session, n=n,
                                    slots=sl.data_ptr(), layer_begin=lb, layer_end=le, k_out=K.data_ptr(),
                                    v_out=V.data_ptr())
            _lib.call("ic_gather_slots", a)
        return K, V

    def reset(self, sessions: Optional[Sequence[int]] = None, zero_kv: bool = True) -> None:
        if sessions is None:
            sessions = range(self.num_sessions)
        for s in sessions:
            a = _lib.ic_reset_args(pool=self._c_pool, tiers=self._c_tiers, sess=self._c_sess, session0=int(s), n=1,
                                   zero_kv=1 if zero_kv else 0)
            _lib.call("ic_reset_sessions", a)

    # ---- host views -----------------------------------------------------------------------------
    def _sub(self, s: int) -> _lib.ic_sessions:
        """ic_sessions for the single session row s."""
        if not 0 <= s < self.num_sessions:
            raise IndexError(s)
        return self._range_sessions(s, s + 1)

    def _range_sessions(self, s0: int, s1: int) -> _lib.ic_sessions:
        """ic_sessions for the session rows s0 .. s1 - 1."""
        return _lib.ic_sessions(num_sessions=s1 - s0, slot_table=self.slot_table[s0].data_ptr(),
                                positions=self.positions[s0].data_ptr(), importance=self.importance[s0].data_ptr(),
                                occupied=self.occupied[s0].data_ptr(), ctrl=self.ctrl[s0].data_ptr(),
                                counters=self.counters[s0].data_ptr(), dev_status=self.dev_status.data_ptr())

    @staticmethod
    def _stats_from(c, n) -> CacheStats:
        sf, rf, imf = c[_lib.IC_CTRL_SINK_FILL], c[_lib.IC_CTRL_RECENT_FILL], c[_lib.IC_CTRL_IMPORTANT_FILL]
        return CacheStats(total_tokens_seen=n[_lib.IC_CNT_TOKENS_SEEN], total_evictions=n[_lib.IC_CNT_EVICTIONS],
                          current_fill=sf + rf + imf, sink_fill=sf, recent_fill=rf, important_fill=imf,
                          total_promotions=n[_lib.IC_CNT_PROMOTIONS], near_ties=n[_lib.IC_CNT_NEAR_TIES])

    def stats(self, session: int) -> CacheStats:
        return self._stats_from(self.ctrl[session].tolist(), self.counters[session].tolist())

    def stats_async(self) -> "StatsReadback":
        """Every session's counters copied to pinned host memory behind the
        work already queued on the current stream, without synchronising;
        ``.result()`` waits for the copy and returns one CacheStats per session."""
        return StatsReadback(self)

    def export_session(self, session: int) -> dict:
        """One session's complete state (K/V of every slot and layer, positions,
        importance, occupancy, tier counters) as device tensors."""
        from .sharding import export_session
        return export_session(self, session)

    def import_session(self, session: int, state: dict) -> None:
        """Load a state from ``export_session`` into session row `session`."""
        from .sharding import import_session
        import_session(self, session, state)

    def check_device_status(self) -> None:
        """Raise if a kernel reported a bounded-wait timeout or a bad row."""
        st = int(self.dev_status.item())
        if st & _lib.IC_DEVFLAG_TIMEOUT:
            raise _lib.InferCacheError(_lib.IC_ERR_DEVICE_TIMEOUT, "a device-side wait timed out")
        if st & _lib.IC_DEVFLAG_BAD_ROW:
            raise _lib.InferCacheError(_lib.IC_ERR_CORRUPT_TABLE, "slot table or ring state out of range")


class StatsReadback:
    """Asynchronous copy of a SessionBatch's control words and counters."""

    def __init__(self, batch: "SessionBatch"):
        self._ctrl = torch.empty(batch.ctrl.shape, dtype=batch.ctrl.dtype).pin_memory()
        self._cnt = torch.empty(batch.counters.shape, dtype=batch.counters.dtype).pin_memory()
        self._ctrl.copy_(batch.ctrl, non_blocking=True)
        self._cnt.copy_(batch.counters, non_blocking=True)
        self._event = torch.cuda.Event()
        self._event.record(torch.cuda.current_stream(batch.device))

    def ready(self) -> bool:
        return self._event.query()

    def result(self) -> List[CacheStats]:
        self._event.synchronize()
        return [SessionBatch._stats_from(c, n) for c, n in zip(self._ctrl.tolist(), self._cnt.tolist())]


class GroupedStepper:
    """Decode steps of every session of a batch, the sessions split into
    ``groups`` contiguous ranges, each range's ``steps_per_graph`` steps
    captured as its own CUDA graph (``ic_decode_step`` on that range, the
    eviction kernel advancing the positions) and replayed on its own stream.

    Within one stream the GPU drains at every step boundary: the eviction
    kernel needs the step's last layer complete and the next step's first
    layer needs the eviction.  Session ranges are independent, so ranges on
    separate streams fill each other's drains.  Every kernel works per
    session, so the results are bit-identical to ``SessionBatch.step``.

    q / k / v / out: contiguous [L, S, H, D] device tensors in the cache dtype
    (fixed: the graphs hold their addresses), positions: contiguous int64 [S]
    on the device, advanced by one per step.  ``run(n)`` queues n replays
    (n * steps_per_graph steps of every session) behind the work on the
    current stream and makes the current stream wait for them; the streams
    join only there, so queue many replays in one call.
    """

    def __init__(self, batch: SessionBatch, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                 positions: torch.Tensor, groups: int = 8, steps_per_graph: int = 4):
        cfg = batch.cfg
        L, S, D, Hkv = cfg.num_layers, batch.num_sessions, cfg.head_dim, cfg.num_kv_heads
        if q.dim() != 4 or q.shape[0] != L or q.shape[1] != S or q.shape[3] != D:
            raise ValueError(f"q must be [L={L}, S={S}, Hq, {D}], got {tuple(q.shape)}")
        if tuple(k.shape) != (L, S, Hkv, D) or k.shape != v.shape:
            raise ValueError(f"k / v must be [{L}, {S}, {Hkv}, {D}]")
        if out.shape != q.shape:
            raise ValueError("out must have q's shape")
        for t in (q, k, v, out):
            if t.dtype != cfg.dtype or t.device != batch.device or not t.is_contiguous():
                raise ValueError("q / k / v / out must be contiguous tensors of the cache dtype on the cache device")
        if not (isinstance(positions, torch.Tensor) and positions.device == batch.device
                and positions.dtype == torch.int64 and positions.is_contiguous() and positions.numel() == S):
            raise ValueError("positions must be a contiguous int64 [S] tensor on the cache device")
        if not 1 <= int(groups) <= S or int(steps_per_graph) < 1:
            raise ValueError("need 1 <= groups <= sessions and steps_per_graph >= 1")
        self.batch, self.groups, self.steps_per_graph = batch, int(groups), int(steps_per_graph)
        self._keep = (q, k, v, out, positions)
        Hq = q.shape[2]
        esz = q.element_size()
        bounds = [S * g // self.groups for g in range(self.groups + 1)]
        self.ranges = [(bounds[g], bounds[g + 1]) for g in range(self.groups)]
        self._args = []
        for s0, s1 in self.ranges:
            d = _lib.ic_decode_args(pool=batch._c_pool, tiers=batch._c_tiers, sess=batch._range_sessions(s0, s1),
                                    mass=batch.mass[s0].data_ptr(), scale=batch.scale)
            batch._prepare_decode(d, Hq)
            d.q = q.data_ptr() + s0 * Hq * D * esz
            d.k_new = k.data_ptr() + s0 * Hkv * D * esz
            d.v_new = v.data_ptr() + s0 * Hkv * D * esz
            d.out = out.data_ptr() + s0 * Hq * D * esz
            d.out_dtype = _lib.dtype_code(out.dtype)
            e = _lib.ic_evict_args(tiers=batch._c_tiers, sess=batch._range_sessions(s0, s1),
                                   mass=batch.mass[s0].data_ptr(), mass_heads=Hkv, mass_layers=1,
                                   mass_div=float(L * Hkv), decay=cfg.decay, pdl=1 if batch.pdl else 0,
                                   advance_pos=1, new_pos=positions[s0].data_ptr(), events=batch.events[s0].data_ptr())
            self._args.append(_lib.ic_step_args(layer0=d, q_layer_stride=S * Hq * D, kv_layer_stride=S * Hkv * D,
                                                out_layer_stride=S * Hq * D, evict=e))
        dev = batch.device
        self.streams = [torch.cuda.Stream(device=dev) for _ in self.ranges]
        self.graphs = []
        self._replay = None
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        for a in self._args:
            g = torch.cuda.CUDAGraph()
            # relaxed: a kernel's first launch may set its shared-memory attribute
            with torch.cuda.graph(g, stream=cap, capture_error_mode="relaxed"):
                for _ in range(self.steps_per_graph):
                    _lib.call("ic_decode_step", a)
            self.graphs.append(g)
        torch.cuda.current_stream(dev).wait_stream(cap)

    @property
    def launches_per_step(self) -> int:
        """Kernel launches per step of every session (layers + eviction, per range)."""
        return self.groups * (self.batch.cfg.num_layers + 1)

    def run(self, replays: int = 1) -> None:
        cur = torch.cuda.current_stream(self.batch.device)
        for s in self.streams:
            s.wait_stream(cur)
        if self._replay is None:
            self._replay = _GraphReplay(self.graphs, self.streams, self.batch.device)
        self._replay(int(replays))
        for s in self.streams:
            cur.wait_stream(s)


class _GraphReplay:
    """Replays CUDA graphs, graph i on stream i, `rounds` times over, in one
    library call (ic_graph_replay): a grouped stepper's many small launches
    then cost no interpreter call each.  Holds the graphs, so their
    executables stay alive."""

    def __init__(self, graphs, streams, device) -> None:
        self.graphs, self.streams, self.device = list(graphs), list(streams), torch.device(device)
        n = len(self.graphs)
        self._execs = (ctypes.c_void_p * n)(*[int(g.raw_cuda_graph_exec()) for g in self.graphs])
        self._strms = (ctypes.c_void_p * n)(*[int(st.cuda_stream) for st in self.streams])

    def __call__(self, rounds: int) -> None:
        if rounds <= 0:
            return
        lib = _lib.load()
        with torch.cuda.device(self.device):  # the launches run on the graphs' device
            _lib.raise_for(lib.ic_graph_replay(self._execs, self._strms, len(self.graphs), int(rounds)),
                           "ic_graph_replay")


class GroupedHostStepper:
    """Decode steps of every session driven from pinned host memory, the
    sessions split into ``groups`` contiguous ranges that each run on their
    own stream: per range and step, one upload of the range's q / k / v, its
    ``ic_decode_step`` (all layers + eviction, positions advanced by one) and
    one download of its output, captured as one CUDA graph.

    Ranges do not wait for one another, so one range's copies and its
    step-boundary drain overlap the other ranges' decode kernels (at 16
    sessions x 36 layers, 8 ranges: ~1.5x ``HostStepper``).  Results are
    bit-identical to ``SessionBatch.step``.

    The host buffers are range-major so each range moves in one copy each
    way: ``q_host[g]`` [L, S_g, Hq, D], ``k_host[g]`` / ``v_host[g]`` [L, S_g,
    Hkv, D] (back to back in one pinned block per range) and ``out_host[g]``
    [L, S_g, Hq, D], in the cache dtype; ``load_inputs`` / ``outputs`` convert
    from / to [L, S, H, D].  ``run(n)`` queues n steps of every range; the
    copies read and write the host buffers while the steps run, so change the
    inputs or read the outputs only after ``synchronize()``.  positions: int64
    [S] on the device.
    """

    def __init__(self, batch: SessionBatch, positions: torch.Tensor, num_q_heads: int, groups: int = 8):
        cfg = batch.cfg
        L, S, D, Hkv, Hq = cfg.num_layers, batch.num_sessions, cfg.head_dim, cfg.num_kv_heads, int(num_q_heads)
        if not (isinstance(positions, torch.Tensor) and positions.device == batch.device
                and positions.dtype == torch.int64 and positions.is_contiguous() and positions.numel() == S):
            raise ValueError("positions must be a contiguous int64 [S] tensor on the cache device")
        if Hq < 1 or Hq % Hkv:
            raise ValueError("num_q_heads must be a positive multiple of num_kv_heads")
        if not 1 <= int(groups) <= S:
            raise ValueError("need 1 <= groups <= sessions")
        self.batch, self.groups, self.positions = batch, int(groups), positions
        dev, dt = batch.device, cfg.dtype
        bounds = [S * g // self.groups for g in range(self.groups + 1)]
        self.ranges = [(bounds[g], bounds[g + 1]) for g in range(self.groups)]
        self.q_host, self.k_host, self.v_host, self.out_host = [], [], [], []
        self._dev = []
        self.streams = [torch.cuda.Stream(device=dev) for _ in self.ranges]
        self.graphs = []
        self._replay = None
        self.h2d_bytes = self.d2h_bytes = 0
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        esz = torch.empty(0, dtype=dt).element_size()
        for s0, s1 in self.ranges:
            Sg = s1 - s0
            nq, nk = L * Sg * Hq * D, L * Sg * Hkv * D
            hb = torch.empty(nq + 2 * nk, dtype=dt).pin_memory()
            db = torch.empty(nq + 2 * nk, dtype=dt, device=dev)
            od = torch.empty(L, Sg, Hq, D, dtype=dt, device=dev)
            oh = torch.empty(L, Sg, Hq, D, dtype=dt).pin_memory()
            self.q_host.append(hb[:nq].view(L, Sg, Hq, D))
            self.k_host.append(hb[nq:nq + nk].view(L, Sg, Hkv, D))
            self.v_host.append(hb[nq + nk:].view(L, Sg, Hkv, D))
            self.out_host.append(oh)
            self.h2d_bytes += hb.numel() * esz
            self.d2h_bytes += oh.numel() * esz
            d = _lib.ic_decode_args(pool=batch._c_pool, tiers=batch._c_tiers, sess=batch._range_sessions(s0, s1),
                                    mass=batch.mass[s0].data_ptr(), scale=batch.scale)
            batch._prepare_decode(d, Hq)
            d.q, d.k_new, d.v_new = db.data_ptr(), db.data_ptr() + nq * esz, db.data_ptr() + (nq + nk) * esz
            d.out = od.data_ptr()
            d.out_dtype = _lib.dtype_code(dt)
            e = _lib.ic_evict_args(tiers=batch._c_tiers, sess=batch._range_sessions(s0, s1),
                                   mass=batch.mass[s0].data_ptr(), mass_heads=Hkv, mass_layers=1,
                                   mass_div=float(L * Hkv), decay=cfg.decay, pdl=1 if batch.pdl else 0,
                                   advance_pos=1, new_pos=positions[s0].data_ptr(), events=batch.events[s0].data_ptr())
            a = _lib.ic_step_args(layer0=d, q_layer_stride=Sg * Hq * D, kv_layer_stride=Sg * Hkv * D,
                                  out_layer_stride=Sg * Hq * D, evict=e)
            gr = torch.cuda.CUDAGraph()
            # relaxed: the first launch of each kernel may set its shared-memory limit
            with torch.cuda.graph(gr, stream=cap, capture_error_mode="relaxed"):
                db.copy_(hb, non_blocking=True)
                _lib.call("ic_decode_step", a)
                oh.copy_(od, non_blocking=True)
            self.graphs.append(gr)
            self._dev.append((hb, db, od, a))
        torch.cuda.current_stream(dev).wait_stream(cap)

    def load_inputs(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        """Copy [L, S, Hq, D] / [L, S, Hkv, D] tensors into the range-major
        host buffers (host-side; call after ``synchronize()``)."""
        for (s0, s1), qh, kh, vh in zip(self.ranges, self.q_host, self.k_host, self.v_host):
            qh.copy_(q[:, s0:s1])
            kh.copy_(k[:, s0:s1])
            vh.copy_(v[:, s0:s1])

    def outputs(self) -> torch.Tensor:
        """The last step's output as one [L, S, Hq, D] host tensor (after ``synchronize()``)."""
        return torch.cat(self.out_host, dim=1)

    def run(self, steps: int = 1) -> None:
        cur = torch.cuda.current_stream(self.batch.device)
        for s in self.streams:
            s.wait_stream(cur)
        if self._replay is None:
            self._replay = _GraphReplay(self.graphs, self.streams, self.batch.device)
        self._replay(int(steps))
        for s in self.streams:
            cur.wait_stream(s)

    def synchronize(self) -> None:
        for s in self.streams:
            s.synchronize()


class HostStepper:
    """One decode step of every session of a ``SessionBatch`` driven from host
    memory: copy q / k / v from pinned host buffers, run ``ic_decode_step``
    (all layers + eviction), advance each session's position by one and copy
    the output back to pinned host memory -- the device part captured once as
    a CUDA graph, so a step costs one graph launch on the host.

    q_host [L, S, Hq, D], k_host / v_host [L, S, Hkv, D] and the output
    buffers [L, S, Hq, D] are pinned tensors of the cache dtype; positions is
    an int64 [S] tensor on the device (the position of each session's next
    decoded token).

    ``out_host`` is one tensor, or a pair for a pipelined stepper: the copy of
    step i's output to ``out_host[i % 2]`` then runs on a copy stream while
    step i + 1 computes.  ``run()`` returns the index of the buffer receiving
    this step's output; ``wait(index)`` (or ``synchronize()``) makes it
    readable.

    When q_host, k_host and v_host lie back to back in one pinned block (one
    dtype), the step uploads the block with a single copy.

    ``zero_copy`` makes the decode kernels read q / k / v from, and write the
    output to, the pinned host buffers themselves (mapped host memory over
    PCIe): no staging copies and no copy launches, at the price of PCIe
    latency inside every layer's kernel.  (Measured at 16 sessions x 36
    layers: 0.250 ms per step against 0.222 ms staged.  Copies on a second
    stream do not overlap the step either: run beside the decode kernels, a
    2.36 MB upload took 176 us instead of 51 us and slowed the step by 93 us.)"""

    def __init__(self, batch: "SessionBatch", q_host: torch.Tensor, k_host: torch.Tensor, v_host: torch.Tensor,
                 out_host, positions: torch.Tensor, zero_copy: bool = False):
        outs = tuple(out_host) if isinstance(out_host, (tuple, list)) else (out_host,)
        if len(outs) not in (1, 2):
            raise ValueError("out_host must be a tensor or a pair of tensors")
        for name, t in (("q_host", q_host), ("k_host", k_host), ("v_host", v_host)) + \
                tuple((f"out_host[{i}]", o) for i, o in enumerate(outs)):
            if t.device.type != "cpu" or not t.is_pinned() or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous pinned host tensor")
        if positions.device != batch.device or positions.dtype != torch.int64 or positions.numel() != batch.num_sessions:
            raise ValueError("positions must be an int64 [S] tensor on the cache device")
        self.batch = batch
        self.q_host, self.k_host, self.v_host, self.out_host = q_host, k_host, v_host, outs
        self.positions = positions
        self.pipelined = len(outs) == 2
        self.zero_copy = bool(zero_copy)
        dev = batch.device
        if self.zero_copy:
            cfg = batch.cfg
            L, S = cfg.num_layers, batch.num_sessions
            Hq = q_host.shape[2] if q_host.dim() == 4 else -1
            if (q_host.dim() != 4 or tuple(q_host.shape[:2]) != (L, S) or q_host.shape[3] != cfg.head_dim or
                    tuple(k_host.shape) != (L, S, cfg.num_kv_heads, cfg.head_dim) or k_host.shape != v_host.shape):
                raise ValueError("q_host [L, S, Hq, D], k_host / v_host [L, S, Hkv, D] expected")
            for t in (q_host, k_host, v_host):
                if t.dtype != cfg.dtype:
                    raise ValueError("q_host / k_host / v_host must be in the cache dtype")
            for o in outs:
                if o.shape != q_host.shape:
                    raise ValueError("out_host must be shaped like q_host")
            self.h2d_bytes = sum(t.numel() * t.element_size() for t in (q_host, k_host, v_host))
            self.d2h_bytes = outs[0].numel() * outs[0].element_size()
            qd, kd, vd = (_lib.host_device_pointer(t) for t in (q_host, k_host, v_host))
            ods = [_lib.host_device_pointer(o) for o in outs]
            cap = torch.cuda.Stream(device=dev)
            cap.wait_stream(torch.cuda.current_stream(dev))
            self.graphs = []
            for k in range(len(outs)):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=cap, capture_error_mode="relaxed"):
                    batch._step_raw(qd, kd, vd, ods[k], Hq, outs[k].dtype, positions)
                self.graphs.append(gr)
            self.graph = self.graphs[0]
            self._copy = None
            self._computed = [torch.cuda.Event() for _ in outs]
            self._copied = self._computed
            self._used = [False] * len(outs)
            self._next = 0
            return
        # q, k and v back to back in one host block (same dtype): one upload of
        # the block into a device block with the same layout
        nq, nk, nv = q_host.numel(), k_host.numel(), v_host.numel()
        esz = q_host.element_size()
        self.packed_inputs = (q_host.dtype == k_host.dtype == v_host.dtype and
                              k_host.data_ptr() == q_host.data_ptr() + nq * esz and
                              v_host.data_ptr() == k_host.data_ptr() + nk * esz)
        if self.packed_inputs:
            block = torch.empty(nq + nk + nv, dtype=q_host.dtype, device=dev)
            self._q = block[:nq].view(q_host.shape)
            self._k = block[nq:nq + nk].view(k_host.shape)
            self._v = block[nq + nk:].view(v_host.shape)
            host_block = torch.empty(0, dtype=q_host.dtype).set_(
                q_host.untyped_storage(), q_host.storage_offset(), (nq + nk + nv,), (1,))
        else:
            self._q = torch.empty(q_host.shape, dtype=q_host.dtype, device=dev)
            self._k = torch.empty(k_host.shape, dtype=k_host.dtype, device=dev)
            self._v = torch.empty(v_host.shape, dtype=v_host.dtype, device=dev)
        self._o = [torch.empty(o.shape, dtype=o.dtype, device=dev) for o in outs]
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in (q_host, k_host, v_host))
        self.d2h_bytes = outs[0].numel() * outs[0].element_size()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        self.graphs = []
        for k in range(len(outs)):
            gr = torch.cuda.CUDAGraph()
            # relaxed: the first launch of each kernel may set its shared-memory limit
            with torch.cuda.graph(gr, stream=cap, capture_error_mode="relaxed"):
                if self.packed_inputs:
                    block.copy_(host_block, non_blocking=True)
                else:
                    self._q.copy_(q_host, non_blocking=True)
                    self._k.copy_(k_host, non_blocking=True)
                    self._v.copy_(v_host, non_blocking=True)
                batch.step(self._q, self._k, self._v, positions, out=self._o[k], advance_positions=True)
                if not self.pipelined:
                    outs[0].copy_(self._o[0], non_blocking=True)
            self.graphs.append(gr)
        self.graph = self.graphs[0]
        self._copy = torch.cuda.Stream(device=dev)
        self._computed = [torch.cuda.Event() for _ in outs]
        self._copied = [torch.cuda.Event() for _ in outs]
        self._used = [False] * len(outs)
        self._next = 0

    def run(self, sync: bool = False) -> int:
        k = self._next
        main = torch.cuda.current_stream(self.batch.device)
        if self.zero_copy:
            self.graphs[k].replay()  # the kernels write out_host[k] themselves
            self._computed[k].record(main)
            self._used[k] = True
            if self.pipelined:
                self._next = 1 - k
            if sync:
                self.wait(k)
            return k
        if self.pipelined and self._used[k]:
            main.wait_event(self._copied[k])  # the device output buffer has been read
        self.graphs[k].replay()
        if self.pipelined:
            self._computed[k].record(main)
            self._copy.wait_event(self._computed[k])
            with torch.cuda.stream(self._copy):
                self.out_host[k].copy_(self._o[k], non_blocking=True)
            self._copied[k].record(self._copy)
            self._used[k] = True
            self._next = 1 - k
        if sync:
            self.wait(k)
        return k

    def wait(self, index: int = 0) -> None:
        """Block the host until out_host[index] holds its step's output."""
        if self.pipelined or self.zero_copy:
            self._copied[index].synchronize()
        else:
            torch.cuda.current_stream(self.batch.device).synchronize()

    def synchronize(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make `stream` (default: the current one) wait for every pending
        output copy, without blocking the host."""
        st = stream or torch.cuda.current_stream(self.batch.device)
        if self.pipelined or self.zero_copy:
            for k, used in enumerate(self._used):
                if used:
                    st.wait_event(self._copied[k])


class HierarchicalKVCache:
    """Single-session drop-in for the reference class (hierarchical_cache.py:109-477)."""

    def __init__(self, cfg: CacheConfig, device=None):
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        if self.device.type != "cuda":
            raise ValueError("HierarchicalKVCache runs on the GPU only (no CPU path)")
        self._b = SessionBatch(cfg, 1, self.device)
        self.device = self._b.device

    # public tensors of the reference, device-resident views of session 0
    @property
    def positions(self) -> torch.Tensor:
        return self._b.positions[0]

    @property
    def importance(self) -> torch.Tensor:
        return self._b.importance[0]

    @property
    def occupied(self) -> torch.Tensor:
        return self._b.occupied[0]

    @property
    def K(self) -> torch.Tensor:
        """[L, Hkv, budget, D] by logical slot (a gathered copy)."""
        return self._b.gather(0, torch.arange(self.cfg.total_budget, device=self.device))[0]

    @property
    def V(self) -> torch.Tensor:
        return self._b.gather(0, torch.arange(self.cfg.total_budget, device=self.device))[1]

    @property
    def batch(self) -> SessionBatch:
        return self._b

    @property
    def total_budget(self) -> int:
        return self.cfg.total_budget

    @property
    def current_fill(self) -> int:
        return self.stats.current_fill

    @property
    def stats(self) -> CacheStats:
        return self._b.stats(0)

    @property
    def _recent_ptr(self) -> int:
        return int(self._b.ctrl[0, _lib.IC_CTRL_RECENT_PTR].item())

    @property
    def _important_fill(self) -> int:
        return int(self._b.ctrl[0, _lib.IC_CTRL_IMPORTANT_FILL].item())

    def last_event(self) -> Tuple[int, int, int, int]:
        """(kind, displaced position, target slot, evicted position) of the last push."""
        return tuple(self._b.events[0].tolist())

    def load_from_hf_output(self, past_key_values, importance_scores: torch.Tensor,
                            positions: Optional[torch.Tensor] = None) -> None:
        self._b.load_prompt(0, past_key_values, importance_scores, positions)

    def push(self, key_states: torch.Tensor, value_states: torch.Tensor, position: int,
             attn_weights: Optional[torch.Tensor] = None) -> None:
        self._b.push(0, key_states, value_states, position, attn_weights)

    # fused decode verbs for one session
    def attend(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """q [Hq, D], k / v [Hkv, D] -> o [Hq, D]."""
        return self._b.attend(layer, q[None], k[None], v[None], out_dtype=out_dtype)[0]

    def evict(self, position: int, decay: Optional[float] = None) -> None:
        self._b.evict([position], decay)

    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, position: int,
             out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """q [L, Hq, D], k / v [L, Hkv, D] -> o [L, Hq, D]."""
        return self._b.step(q[:, None], k[:, None], v[:, None], [position], out_dtype=out_dtype)[:, 0]

    def to_hf_past_key_values(self, device: Optional[torch.device] = None):
        """Occupied slots in position order, one (K, V) [1, Hkv, F, D] per layer
        (hierarchical_cache.py:297-351); None when empty."""
        slots = self._b.sorted_slots(0)
        if slots.numel() == 0:
            return None
        K, V = self._b.gather(0, slots)
        dev = device or self.device
        layers = [(K[l][None].to(dev), V[l][None].to(dev)) for l in range(self.cfg.num_layers)]
        return to_dynamic_cache(layers)

    def get_position_ids_for_cache(self) -> torch.Tensor:
        slots = self._b.sorted_slots(0)
        return self.positions[slots]

    def reset(self) -> None:
        self._b.reset([0], zero_kv=True)

    def state_dict(self) -> dict:
        """The cache's complete state on the host (K/V of every slot and layer,
        positions, importance, occupancy, tier pointers and counters), so a
        session can be saved with torch.save and restored later or elsewhere."""
        return {k: v.cpu() for k, v in self._b.export_session(0).items()}

    def load_state_dict(self, state: dict) -> None:
        self._b.import_session(0, state)


def _normalise_past_kv(past_key_values):
    return normalise_kv(past_key_values)
