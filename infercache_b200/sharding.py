"""Sessions sharded across GPUs: one process per GPU, no collective on the
decode path.

Sessions are independent (each owns its slot table, metadata and pages), so a
fleet of N sessions is partitioned across ranks and every rank runs its own
``SessionBatch`` on its own GPU.  What crosses ranks is host bookkeeping and,
optionally, whole sessions when one GPU's pool runs short:

* ``shard_sessions`` / ``ShardMap``: which rank owns which global session.
* ``max_over_ranks``: timing reductions (the only collective the bench uses).
* ``export_session`` / ``import_session``: one session's complete state
  (K/V of every logical slot and layer, positions, importance, occupancy,
  tier counters) as a dict of tensors, and back into a free session row.
* ``send_session`` / ``recv_session``: that dict over ``torch.distributed``
  point-to-point (NCCL between GPUs, gloo on CPU), with a deadline: a peer
  that never sends raises ``SessionTransferError`` instead of hanging.
* ``PeerMonitor``: heartbeats in the process group's key-value store, so a
  rank learns on the host, between steps, that a peer stopped.
"""
from __future__ import annotations

import time
from datetime import timedelta
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

STATE_KEYS = ("k", "v", "positions", "importance", "occupied", "ctrl", "counters")


class SessionTransferError(RuntimeError):
    pass


def shard_sessions(n_sessions: int, world: int, rank: int, mode: str = "contiguous") -> List[int]:
    """Global session ids owned by `rank` out of `n_sessions` over `world` ranks."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if mode == "contiguous":
        base, extra = divmod(n_sessions, world)
        start = rank * base + min(rank, extra)
        return list(range(start, start + base + (1 if rank < extra else 0)))
    if mode == "round_robin":
        return list(range(rank, n_sessions, world))
    raise ValueError(f"unknown shard mode {mode!r}")


class ShardMap:
    """Global session id <-> (rank, local index)."""

    def __init__(self, n_sessions: int, world: int, mode: str = "contiguous"):
        self.n_sessions, self.world, self.mode = n_sessions, world, mode
        self._owner: Dict[int, Tuple[int, int]] = {}
        self._local: List[List[int]] = []
        for r in range(world):
            ids = shard_sessions(n_sessions, world, r, mode)
            self._local.append(ids)
            for i, g in enumerate(ids):
                self._owner[g] = (r, i)

    def owner(self, session: int) -> Tuple[int, int]:
        return self._owner[session]

    def local_sessions(self, rank: int) -> List[int]:
        return list(self._local[rank])

    def move(self, session: int, dst_rank: int, dst_local: int) -> None:
        """Record that `session` now lives at (dst_rank, dst_local)."""
        r, i = self._owner[session]
        self._local[r][i] = -1
        while len(self._local[dst_rank]) <= dst_local:
            self._local[dst_rank].append(-1)
        self._local[dst_rank][dst_local] = session
        self._owner[session] = (dst_rank, dst_local)


def max_over_ranks(value: float, device: Optional[torch.device] = None) -> float:
    """Max of a host scalar over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- session state ------------------------------------------------------------------------
def session_state_like(cfg, device) -> Dict[str, torch.Tensor]:
    """Empty buffers with the shapes of one session's exported state."""
    from . import _lib
    B = cfg.total_budget
    kv = (cfg.num_layers, cfg.num_kv_heads, B, cfg.head_dim)
    return {"k": torch.empty(kv, dtype=cfg.dtype, device=device), "v": torch.empty(kv, dtype=cfg.dtype, device=device),
            "positions": torch.empty(B, dtype=torch.int64, device=device),
            "importance": torch.empty(B, dtype=torch.float32, device=device),
            "occupied": torch.empty(B, dtype=torch.uint8, device=device),
            "ctrl": torch.empty(_lib.IC_CTRL_WORDS, dtype=torch.int32, device=device),
            "counters": torch.empty(_lib.IC_COUNTER_WORDS, dtype=torch.int64, device=device)}


def export_session(batch, session: int) -> Dict[str, torch.Tensor]:
    """Complete state of one session of a SessionBatch (device tensors)."""
    B = batch.cfg.total_budget
    K, V = batch.gather(session, torch.arange(B, device=batch.device))
    return {"k": K, "v": V, "positions": batch.positions[session].clone(),
            "importance": batch.importance[session].clone(),
            "occupied": batch.occupied[session].to(torch.uint8), "ctrl": batch.ctrl[session].clone(),
            "counters": batch.counters[session].clone()}


def import_session(batch, session: int, state: Dict[str, torch.Tensor]) -> None:
    """Write an exported state into session row `session` of `batch`: K/V of
    every logical slot through the tier-fill copy kernel, then the metadata."""
    from . import _lib
    cfg = batch.cfg
    like = session_state_like(cfg, batch.device)
    for k in STATE_KEYS:
        if tuple(state[k].shape) != tuple(like[k].shape):
            raise ValueError(f"state[{k!r}] has shape {tuple(state[k].shape)}, expected {tuple(like[k].shape)}")
    batch.reset([session], zero_kv=True)
    sub = batch._sub(session)
    ident = torch.arange(cfg.total_budget, dtype=torch.int32, device=batch.device)[None]
    K = state["k"].to(batch.device, cfg.dtype)
    V = state["v"].to(batch.device, cfg.dtype)
    for li in range(cfg.num_layers):
        Ks, Vs = K[li].contiguous(), V[li].contiguous()
        la = _lib.ic_load_layer_args(pool=batch._c_pool, tiers=batch._c_tiers, sess=sub, session=0, layer=li,
                                     slot_token=ident.data_ptr(), k_src=Ks.data_ptr(), v_src=Vs.data_ptr(),
                                     stride_h=Ks.stride(0), stride_t=Ks.stride(1),
                                     src_dtype=_lib.dtype_code(Ks.dtype), T=cfg.total_budget)
        _lib.call("ic_load_layer", la)
    batch.positions[session].copy_(state["positions"])
    batch.importance[session].copy_(state["importance"])
    batch.occupied[session].copy_(state["occupied"].bool())
    batch.ctrl[session].copy_(state["ctrl"])
    batch.counters[session].copy_(state["counters"])
    batch._keep = (K, V, ident)


def send_session(state: Dict[str, torch.Tensor], dst: int, timeout_s: float = 30.0, group=None) -> None:
    """Send an exported state to rank `dst` (tensors in STATE_KEYS order)."""
    works = [dist.isend(state[k].contiguous(), dst, group=group) for k in STATE_KEYS]
    _wait_all(works, timeout_s, f"send to rank {dst}")


def recv_session(like: Dict[str, torch.Tensor], src: int, timeout_s: float = 30.0,
                 group=None) -> Dict[str, torch.Tensor]:
    """Receive a state from rank `src` into buffers shaped like `like`."""
    out = {k: torch.empty_like(like[k]) for k in STATE_KEYS}
    works = [dist.irecv(out[k], src, group=group) for k in STATE_KEYS]
    _wait_all(works, timeout_s, f"receive from rank {src}")
    return out


def _wait_all(works, timeout_s: float, what: str) -> None:
    deadline = time.monotonic() + timeout_s
    for w in works:
        left = max(0.0, deadline - time.monotonic())
        try:
            ok = w.wait(timeout=timedelta(seconds=left))
        except RuntimeError as e:  # gloo / NCCL raise on timeout or a dead peer
            raise SessionTransferError(f"{what} failed: {e}") from e
        if ok is False:
            raise SessionTransferError(f"{what} timed out after {timeout_s:.1f} s")


# ---- failure detection ---------------------------------------------------------------------
class PeerMonitor:
    """Heartbeats through a ``torch.distributed`` key-value store.

    Each rank calls ``beat()`` between steps; ``stale_peers(max_age_s)`` lists
    the ranks whose last beat is older than `max_age_s` (or that never beat),
    so a rank stops before launching work that would wait on a dead peer.
    """

    def __init__(self, store, rank: int, world: int, prefix: str = "infercache_hb"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def beat(self, step: int = 0) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", f"{time.time():.6f}:{step}")

    def last(self, rank: int) -> Optional[Tuple[float, int]]:
        key = f"{self.prefix}/{rank}"
        if not self.store.check([key]):
            return None
        t, s = self.store.get(key).decode().split(":")
        return float(t), int(s)

    def stale_peers(self, max_age_s: float) -> List[int]:
        now = time.time()
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            hb = self.last(r)
            if hb is None or now - hb[0] > max_age_s:
                out.append(r)
        return out


def rebalance_session(batch_src, session_src: int, dst: int, timeout_s: float = 30.0) -> None:
    """Sender side of moving one session to rank `dst` (the receiver calls
    ``recv_session`` + ``import_session``); the source row is then reset."""
    state = export_session(batch_src, session_src)
    if dist.get_backend() == "gloo":
        state = {k: v.cpu() for k, v in state.items()}
    send_session(state, dst, timeout_s)
    batch_src.reset([session_src], zero_kv=False)


def receive_rebalanced(batch_dst, session_dst: int, src: int, timeout_s: float = 30.0) -> None:
    dev = "cpu" if dist.get_backend() == "gloo" else batch_dst.device
    state = recv_session(session_state_like(batch_dst.cfg, dev), src, timeout_s)
    import_session(batch_dst, session_dst, state)


__all__: Sequence[str] = ("shard_sessions", "ShardMap", "max_over_ranks", "export_session", "import_session",
                          "session_state_like", "send_session", "recv_session", "SessionTransferError",
                          "PeerMonitor", "rebalance_session", "receive_rebalanced")
