"""Summary-pass token scoring: received attention mass without materialising P.

Mirrors ``_attention_mass`` (two_pass.py:104-137): for a layer's causal GQA
attention, the mass key j receives is ``sum_h sum_i P[h, i, j]``; summed over
layers when ``all_layers`` is set, then normalised by its total when that
exceeds 1e-9.  The reference reads P from HF's eager ``output_attentions``
tensors ([1, H, T, T] per layer); here ``ic_summary_score`` (tcgen05 / TMEM
kernels) computes it from q and k directly, together with the attention output
and the row log-sum-exp, so a model's prefill can use it as its attention.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib


@dataclass
class SummaryScores:
    out: Optional[torch.Tensor]   # [B, Hq, T, D] or None
    lse: torch.Tensor             # [B, Hq, T] float32, natural log
    head_mass: Optional[torch.Tensor]   # [B, Hq, T] float32
    colsum: Optional[torch.Tensor]      # [B, T] float32
    importance: Optional[torch.Tensor]  # [B, T] float32, colsum / total


def _check_qkv(q: torch.Tensor, k: torch.Tensor, v: Optional[torch.Tensor]):
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError("q must be [B, Hq, T, D] and k [B, Hkv, T, D]")
    B, Hq, T, D = q.shape
    if k.shape[0] != B or k.shape[2] != T or k.shape[3] != D:
        raise ValueError(f"k shape {tuple(k.shape)} does not match q {tuple(q.shape)}")
    if v is not None and v.shape != k.shape:
        raise ValueError(f"v shape {tuple(v.shape)} != k shape {tuple(k.shape)}")
    if Hq % k.shape[1] != 0:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")
    for t in (q, k) + ((v,) if v is not None else ()):
        if t.dtype != q.dtype:
            raise ValueError("q, k and v must share a dtype")
        if not t.is_cuda:
            raise ValueError("summary_score runs on CUDA tensors only")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("summary_score needs float16 or bfloat16 inputs")
    return B, Hq, k.shape[1], T, D


def summary_score(q: torch.Tensor, k: torch.Tensor, v: Optional[torch.Tensor] = None, *,
                  scale: Optional[float] = None, with_output: bool = True,
                  colsum: Optional[torch.Tensor] = None, accumulate: bool = False,
                  normalise: bool = True, with_mass: bool = True, status: Optional[torch.Tensor] = None,
                  check_status: bool = True) -> SummaryScores:
    """One layer of the summary pass.

    q [B, Hq, T, D], k / v [B, Hkv, T, D] (fp16 / bf16, D = 128).  Returns the
    attention output (when ``with_output`` and v is given), the row
    log-sum-exp, per-head and head-summed received mass, and the normalised
    importance.  With ``accumulate`` the head-summed mass is added to
    ``colsum`` (all layers of ``_attention_mass``).  ``with_mass=False``
    computes only the output and log-sum-exp (a causal prefill attention; the
    mass fields are then None).  ``check_status`` reads
    the device status word after the launch (a synchronisation) and raises if
    a device-side wait timed out; pass False and a ``status`` tensor to keep
    the call asynchronous and check it later.
    """
    B, Hq, Hkv, T, D = _check_qkv(q, k, v)
    dev = q.device
    _lib.require_device(dev)
    q, k = q.contiguous(), k.contiguous()
    want_out = with_output and v is not None
    if not with_mass and not want_out:
        raise ValueError("nothing to compute: with_mass=False needs v and with_output")
    v = v.contiguous() if v is not None else None
    out = torch.empty_like(q) if want_out else None
    lse = torch.empty(B, Hq, T, dtype=torch.float32, device=dev)
    head_mass = torch.empty(B, Hq, T, dtype=torch.float32, device=dev) if with_mass else None
    if not with_mass:
        colsum, normalise = None, False
    elif colsum is None:
        if accumulate:
            raise ValueError("accumulate needs the colsum to add to")
        colsum = torch.empty(B, T, dtype=torch.float32, device=dev)
    elif colsum.shape != (B, T) or colsum.dtype != torch.float32 or not colsum.is_contiguous():
        raise ValueError("colsum must be a contiguous float32 [B, T] tensor")
    importance = torch.empty(B, T, dtype=torch.float32, device=dev) if normalise else None
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    a = _lib.ic_summary_args(
        q=q.data_ptr(), k=k.data_ptr(), v=_lib.ptr(v), out=_lib.ptr(out), lse=lse.data_ptr(),
        head_mass=_lib.ptr(head_mass), colsum=_lib.ptr(colsum), importance=_lib.ptr(importance),
        batch=B, num_q_heads=Hq, num_kv_heads=Hkv, seq_len=T, head_dim=D, dtype=_lib.dtype_code(q.dtype),
        accumulate=1 if accumulate else 0, scale=float(D ** -0.5 if scale is None else scale),
        dev_status=status.data_ptr())
    with torch.cuda.device(dev):
        _lib.call("ic_summary_score", a)
    if check_status:
        flags = int(status.item())
        if flags:
            raise _lib.InferCacheError(_lib.IC_ERR_DEVICE_TIMEOUT,
                                       f"summary_score: device status flags {flags:#x}")
    return SummaryScores(out, lse, head_mass, colsum, importance)


def attention_mass(layers_qk: Sequence, all_layers: bool = False, layer_idx: int = -1,
                   scale: Optional[float] = None) -> torch.Tensor:
    """``_attention_mass`` from per-layer (q, k) instead of attention tensors.

    ``layers_qk``: a sequence of (q [1, Hq, T, D], k [1, Hkv, T, D]) per layer.
    Uses every layer when ``all_layers``, else layer ``layer_idx % L``
    (two_pass.py:121).  Returns float32 [T] on the inputs' device.
    """
    layers = list(layers_qk) if all_layers else [layers_qk[layer_idx % len(layers_qk)]]
    colsum = None
    res = None
    for i, (q, k) in enumerate(layers):
        last = i == len(layers) - 1
        res = summary_score(q, k, None, scale=scale, with_output=False, colsum=colsum,
                            accumulate=colsum is not None, normalise=last)
        colsum = res.colsum
    return res.importance[0]
