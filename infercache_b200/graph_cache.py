"""Graph (cluster-routed) KV cache on the GPU: drop-in for the reference's
``ClusterConfig`` / ``GraphKVCache`` / ``MultiClusterCache``
(graph_cache.py:72-540).

Three regions, as in the reference: attention sinks (filled by absolute
position), a recent ring, and ``n_clusters`` clusters of
``cluster_capacity`` tokens.  A token leaving the ring joins the cluster whose
centroid (the running mean of its members' layer-0 / head-0 keys) is most
cosine-similar to its own layer-0 / head-0 key, or, below ``sim_threshold``,
the first empty (else least filled) cluster; a full cluster evicts its
lowest-scored member.  ``retrieve`` returns the sinks, the ring in position
order and the clusters whose centroid matches the head-mean query.

Everything lives on the device in one slot store (``ic_graph_state``): a
push of one token, or a bulk ``load_from_summary`` of a whole prompt, is one
routing launch (the sequential decisions, on the layer-0 / head-0 keys only)
plus a parallel copy of every layer's and head's K/V rows; ``retrieve`` is
one selection launch plus one row gather each for K and V over all layers.
There is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from . import _lib

__all__ = ["ClusterConfig", "GraphKVCache", "MultiClusterCache"]


@dataclass
class ClusterConfig:
    """graph_cache.py:72-94."""
    num_layers: int
    num_kv_heads: int
    head_dim: int
    n_clusters: int = 16
    cluster_capacity: int = 32
    sim_threshold: float = 0.3
    sink_size: int = 4
    recent_size: int = 128
    dtype: torch.dtype = torch.float16

    @property
    def cluster_budget(self) -> int:
        return self.n_clusters * self.cluster_capacity

    @property
    def total_budget(self) -> int:
        return self.sink_size + self.recent_size + self.cluster_budget


class GraphKVCache:
    """graph_cache.py:218-495, device-resident."""

    def __init__(self, cfg: ClusterConfig, device=None):
        self.cfg = cfg
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type != "cuda":
            raise ValueError("GraphKVCache runs on the GPU only (no CPU path)")
        _lib.require_device(dev)
        if cfg.head_dim != 128:
            raise ValueError("GraphKVCache: head_dim must be 128")
        self.device = dev
        L, H, D, C, cap = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, cfg.n_clusters, cfg.cluster_capacity
        NS = cfg.total_budget
        self.K = torch.zeros((L, H, NS, D), dtype=cfg.dtype, device=dev)
        self.V = torch.zeros_like(self.K)
        self.positions = torch.full((NS,), -1, dtype=torch.int64, device=dev)
        self.scores = torch.zeros(C * cap, dtype=torch.float32, device=dev)
        self.centroid = torch.zeros((C, D), dtype=torch.float32, device=dev)
        self.cl_fill = torch.zeros(C, dtype=torch.int32, device=dev)
        self.c_count = torch.zeros(C, dtype=torch.int32, device=dev)
        self.ctrl = torch.zeros(3, dtype=torch.int32, device=dev)
        self._slot_src = torch.empty(NS, dtype=torch.int32, device=dev)
        self._slots = torch.empty(NS, dtype=torch.int32, device=dev)
        self._count = torch.zeros(1, dtype=torch.int32, device=dev)
        self._selected = torch.zeros(C, dtype=torch.uint8, device=dev)
        self._pos1 = torch.zeros(1, dtype=torch.int64, device=dev)    # a single push's position and score,
        self._score1 = torch.zeros(1, dtype=torch.float32, device=dev)  # set on the device (no host copy)
        self._state = _lib.ic_graph_state(
            k=self.K.data_ptr(), v=self.V.data_ptr(), positions=self.positions.data_ptr(),
            scores=self.scores.data_ptr(), centroid=self.centroid.data_ptr(), cl_fill=self.cl_fill.data_ptr(),
            c_count=self.c_count.data_ptr(), ctrl=self.ctrl.data_ptr(), num_layers=L, num_kv_heads=H, head_dim=D,
            dtype=_lib.dtype_code(cfg.dtype), sink_size=cfg.sink_size, recent_size=cfg.recent_size, n_clusters=C,
            cluster_capacity=cap, sim_threshold=float(cfg.sim_threshold))
        self._keep = None

    # ---- slot views -------------------------------------------------------------------
    @property
    def n_clusters(self) -> int:
        return self.cfg.n_clusters

    def _cluster_slice(self, c: int) -> slice:
        s0 = self.cfg.sink_size + self.cfg.recent_size + c * self.cfg.cluster_capacity
        return slice(s0, s0 + self.cfg.cluster_capacity)

    @property
    def active_cluster_count(self) -> int:
        return int((self.cl_fill > 0).sum())

    # ---- insertion ----------------------------------------------------------------------
    def _push_many(self, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
                   scores: Optional[torch.Tensor], reset: bool) -> None:
        """k, v: [L, H, T, D]; positions int64 [T]; scores float [T] or None."""
        cfg = self.cfg
        k = k.to(self.device, cfg.dtype).contiguous()
        v = v.to(self.device, cfg.dtype).contiguous()
        if k.dim() != 4 or tuple(k.shape[:2]) != (cfg.num_layers, cfg.num_kv_heads) or k.shape[3] != cfg.head_dim \
                or k.shape != v.shape:
            raise ValueError(f"key / value states must be [{cfg.num_layers}, {cfg.num_kv_heads}, T, "
                             f"{cfg.head_dim}], got {tuple(k.shape)} / {tuple(v.shape)}")
        T = k.shape[2]
        pos = positions.to(self.device, torch.int64).reshape(T).contiguous()
        sc = None if scores is None else scores.to(self.device, torch.float32).reshape(T).contiguous()
        a = _lib.ic_graph_push_args(g=self._state, k_src=k.data_ptr(), v_src=v.data_ptr(), stride_l=k.stride(0),
                                    stride_h=k.stride(1), stride_t=k.stride(2), positions=pos.data_ptr(),
                                    scores=0 if sc is None else sc.data_ptr(), slot_src=self._slot_src.data_ptr(),
                                    T=T, reset=1 if reset else 0)
        _lib.call("ic_graph_push", a)
        self._keep = (k, v, pos, sc)  # alive until the launches are consumed

    def push(self, key_states: torch.Tensor, value_states: torch.Tensor, position: int,
             score: float = 0.0) -> None:
        """graph_cache.py:287-323: key_states / value_states [L, H, 1, D]."""
        self._pos1.fill_(int(position))
        self._score1.fill_(float(score))
        self._push_many(key_states, value_states, self._pos1, self._score1, reset=False)

    def load_from_summary(self, past_key_values, importance_scores: torch.Tensor,
                          positions: Optional[torch.Tensor] = None) -> None:
        """graph_cache.py:442-467: reset, then push every token of a summary-pass
        KV snapshot with its importance score, in one routing launch."""
        from .hierarchical_cache import _normalise_past_kv
        pkv = _normalise_past_kv(past_key_values)
        T = pkv[0][0].shape[2]
        k = torch.stack([pkv[li][0][0] for li in range(len(pkv))])
        v = torch.stack([pkv[li][1][0] for li in range(len(pkv))])
        pos = torch.arange(T, dtype=torch.int64) if positions is None else positions
        self._push_many(k, v, pos, importance_scores, reset=True)

    # ---- retrieval ----------------------------------------------------------------------
    def retrieve(self, query_key: torch.Tensor, threshold: Optional[float] = None,
                 top_n_clusters: Optional[int] = None, device: Optional[torch.device] = None):
        """graph_cache.py:363-440: (per-layer (K, V) [1, H, F, D] tuple or None,
        selected bool [n_clusters])."""
        cfg = self.cfg
        q = query_key.to(self.device, torch.float32).reshape(cfg.num_kv_heads, cfg.head_dim).contiguous()
        thresh = cfg.sim_threshold if threshold is None else float(threshold)
        a = _lib.ic_graph_select_args(g=self._state, query=q.data_ptr(), threshold=thresh,
                                      top_n=int(top_n_clusters) if top_n_clusters is not None else 0,
                                      selected=self._selected.data_ptr(), slots=self._slots.data_ptr(),
                                      count=self._count.data_ptr())
        _lib.call("ic_graph_select", a)
        F = int(self._count.item())
        selected = self._selected.to(torch.bool).cpu()
        if F == 0:
            return None, selected
        idx = self._slots[:F].to(torch.int64)
        dev = device or self.device
        # one row gather per store over all (layer, head) planes
        LH, NS = cfg.num_layers * cfg.num_kv_heads, cfg.total_budget
        K = torch.empty((cfg.num_layers, cfg.num_kv_heads, F, cfg.head_dim), dtype=cfg.dtype, device=self.device)
        V = torch.empty_like(K)
        for src, dst in ((self.K, K), (self.V, V)):
            ga = _lib.ic_index_rows_args(src=src.data_ptr(), out=dst.data_ptr(), idx=idx.data_ptr(),
                                         stride_h=NS * cfg.head_dim, stride_n=cfg.head_dim, H=LH, N=NS, F=F,
                                         D=cfg.head_dim, dtype=_lib.dtype_code(cfg.dtype))
            _lib.call("ic_index_rows", ga)
        K, V = K.to(dev), V.to(dev)
        return tuple((K[li][None], V[li][None]) for li in range(cfg.num_layers)), selected

    def retrieve_positions(self, query_key: torch.Tensor, threshold: Optional[float] = None,
                           top_n_clusters: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Positions of the tokens ``retrieve`` returns, in its order, and the selection."""
        cfg = self.cfg
        q = query_key.to(self.device, torch.float32).reshape(cfg.num_kv_heads, cfg.head_dim).contiguous()
        thresh = cfg.sim_threshold if threshold is None else float(threshold)
        a = _lib.ic_graph_select_args(g=self._state, query=q.data_ptr(), threshold=thresh,
                                      top_n=int(top_n_clusters) if top_n_clusters is not None else 0,
                                      selected=self._selected.data_ptr(), slots=self._slots.data_ptr(),
                                      count=self._count.data_ptr())
        _lib.call("ic_graph_select", a)
        F = int(self._count.item())
        return self.positions[self._slots[:F].to(torch.int64)], self._selected.to(torch.bool).cpu()

    # ---- reset / diagnostics --------------------------------------------------------------
    def reset(self) -> None:
        """graph_cache.py:469-479."""
        self.K.zero_()
        self.V.zero_()
        self.positions.fill_(-1)
        self.scores.zero_()
        self.centroid.zero_()
        self.cl_fill.zero_()
        self.c_count.zero_()
        self.ctrl.zero_()

    def cluster_summary(self) -> List[dict]:
        """graph_cache.py:481-492."""
        fill = self.cl_fill.cpu().tolist()
        norms = self.centroid.norm(dim=1).cpu().tolist()
        sc = self.scores.view(self.cfg.n_clusters, self.cfg.cluster_capacity).cpu()
        return [{"id": i, "fill": fill[i], "capacity": self.cfg.cluster_capacity, "centroid_norm": float(norms[i]),
                 "mean_score": float(sc[i, :fill[i]].mean()) if fill[i] > 0 else 0.0}
                for i in range(self.cfg.n_clusters)]


class MultiClusterCache:
    """graph_cache.py:497-540: one GraphKVCache per domain."""

    _DOMAINS = ("code", "qa", "language")

    def __init__(self, cfg: ClusterConfig, device=None):
        self._caches = {d: GraphKVCache(cfg, device=device) for d in self._DOMAINS}
        self._active = "language"

    def activate_domain(self, domain: str) -> None:
        if domain not in self._DOMAINS:
            raise ValueError(f"Unknown domain '{domain}'. Choose from {self._DOMAINS}")
        self._active = domain

    @property
    def active_cache(self) -> GraphKVCache:
        return self._caches[self._active]

    def get(self, domain: str) -> GraphKVCache:
        return self._caches[domain]

    def reset_all(self) -> None:
        for c in self._caches.values():
            c.reset()

    def summary(self) -> dict:
        return {domain: cache.cluster_summary() for domain, cache in self._caches.items()}
