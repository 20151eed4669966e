"""The reference's GPU helper API (triton_ops.py) on this library's kernels.

Same names, arguments and results as triton_ops.py:107-346 for callers that
hold plain K / V buffers and an importance vector.  Every function runs a CUDA
kernel of ``libinfercache_b200`` (``ic_index_rows``, ``ic_scatter_mass``,
``ic_argmin_range``, ``ic_compact_attention``); tensors must be on an sm_100
device — there is no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _dev(t: torch.Tensor) -> torch.device:
    if not t.is_cuda:
        raise ValueError("cache_ops run on CUDA tensors only")
    _lib.require_device(t.device)
    return t.device


def gather_cache_kv(K: torch.Tensor, slot_indices: torch.Tensor) -> torch.Tensor:
    """K [H, budget, D], slot_indices [F] -> [1, H, F, D] (triton_ops.py:107-135)."""
    dev = _dev(K)
    if K.dim() != 3 or K.stride(2) != 1:
        raise ValueError("K must be [H, budget, D] with contiguous rows")
    H, N, D = K.shape
    idx = slot_indices.to(dev, torch.int64).contiguous()
    out = torch.empty((H, idx.numel(), D), dtype=K.dtype, device=dev)
    a = _lib.ic_index_rows_args(src=K.data_ptr(), out=out.data_ptr(), idx=idx.data_ptr(), stride_h=K.stride(0),
                                stride_n=K.stride(1), H=H, N=N, F=idx.numel(), D=D, dtype=_lib.dtype_code(K.dtype))
    with torch.cuda.device(dev):
        _lib.call("ic_index_rows", a)
    return out.unsqueeze(0)


def scatter_importance(attn_weights: torch.Tensor, sorted_slots: torch.Tensor, importance: torch.Tensor) -> None:
    """importance[sorted_slots[f]] += mean over (L, H[, Q]) of attn_weights[..., f],
    for f < min(F', F), in place (triton_ops.py:148-175)."""
    dev = _dev(importance)
    if importance.dtype != torch.float32 or not importance.is_contiguous():
        raise ValueError("importance must be a contiguous float32 tensor")
    w = attn_weights.to(dev, torch.float32)
    if w.dim() not in (3, 4):
        raise ValueError("attn_weights must be [L, H, F] or [L, H, Q, F]")
    w = w.reshape(-1, w.shape[-1]).contiguous()
    slots = sorted_slots.to(dev, torch.int64).contiguous()
    a = _lib.ic_scatter_mass_args(weights=w.data_ptr(), slots=slots.data_ptr(), importance=importance.data_ptr(),
                                  rows=w.shape[0], width=w.shape[1], n_slots=slots.numel(),
                                  budget=importance.numel())
    with torch.cuda.device(dev):
        _lib.call("ic_scatter_mass", a)


def topk_min_slot(importance: torch.Tensor, l2_start: int, l2_fill: int) -> int:
    """Slot of the first minimum of importance[l2_start : l2_start + l2_fill];
    l2_start when the tier is empty (triton_ops.py:207-235)."""
    if l2_fill == 0:
        return l2_start
    dev = _dev(importance)
    x = importance.float().contiguous()
    if l2_start < 0 or l2_start + l2_fill > x.numel():
        raise ValueError("L2 range outside the importance vector")
    out = torch.empty(1, dtype=torch.int64, device=dev)
    a = _lib.ic_argmin_args(x=x.data_ptr(), start=l2_start, n=l2_fill, out_idx=out.data_ptr(), out_val=0)
    with torch.cuda.device(dev):
        _lib.call("ic_argmin_range", a)
    return int(out.item())


def compact_sdp_attention(Q: torch.Tensor, K_buf: torch.Tensor, V_buf: torch.Tensor, slots: torch.Tensor,
                          scale: Optional[float] = None) -> torch.Tensor:
    """Q [B, H, 1, D] attending over K_buf / V_buf [H, budget, D] at `slots`
    -> [B, H, 1, D] (triton_ops.py:251-287)."""
    dev = _dev(K_buf)
    B, H, one, D = Q.shape
    if one != 1 or K_buf.shape[0] != H or K_buf.shape[2] != D or V_buf.shape != K_buf.shape:
        raise ValueError("Q must be [B, H, 1, D] and K_buf / V_buf [H, budget, D]")
    if K_buf.stride(2) != 1 or V_buf.stride(2) != 1 or V_buf.dtype != K_buf.dtype:
        raise ValueError("K_buf / V_buf rows must be contiguous and share a dtype")
    q = Q.to(dev, K_buf.dtype).reshape(B, H, D).contiguous()
    sl = slots.to(dev, torch.int64).contiguous()
    out = torch.empty((B, H, D), dtype=K_buf.dtype, device=dev)
    a = _lib.ic_compact_attn_args(q=q.data_ptr(), k_buf=K_buf.data_ptr(), v_buf=V_buf.data_ptr(),
                                  slots=sl.data_ptr(), out=out.data_ptr(), k_stride_h=K_buf.stride(0),
                                  k_stride_n=K_buf.stride(1), v_stride_h=V_buf.stride(0), v_stride_n=V_buf.stride(1),
                                  B=B, H=H, F=sl.numel(), D=D, budget=K_buf.shape[1],
                                  dtype=_lib.dtype_code(K_buf.dtype), scale=float(scale or D ** -0.5))
    with torch.cuda.device(dev):
        _lib.call("ic_compact_attention", a)
    return out.unsqueeze(2)


class GPUImportanceTracker:
    """Device-resident importance vector (triton_ops.py:299-346)."""

    def __init__(self, budget: int, device: str = "cuda"):
        self.budget = budget
        self._t = torch.zeros(budget, dtype=torch.float32, device=device)
        _dev(self._t)

    def sync_from_cpu(self, cpu_tensor: torch.Tensor) -> None:
        self._t.copy_(cpu_tensor.float(), non_blocking=True)

    def sync_to_cpu(self, cpu_tensor: torch.Tensor) -> None:
        cpu_tensor.copy_(self._t.cpu())

    def scatter_add(self, sorted_slots: torch.Tensor, attn_weights: torch.Tensor) -> None:
        scatter_importance(attn_weights, sorted_slots, self._t)

    def argmin_l2(self, l2_start: int, l2_fill: int) -> int:
        return topk_min_slot(self._t, l2_start, l2_fill)

    def apply_decay(self, decay: float) -> None:
        if decay < 1.0:
            self._t.mul_(decay)

    @property
    def tensor(self) -> torch.Tensor:
        return self._t
