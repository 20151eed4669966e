"""The received attention mass of ``_attention_mass`` (two_pass.py:104-137)
restated in torch fp32, chunked over query rows so that the config-4 size
(16 heads x 8192 tokens per sequence) needs no [H, T, T] tensor.

It is the oracle's formula (``oracle.summary.attention_mass``) on torch
tensors, so it runs on the GPU at full size; ``tests/test_oracle_golden.py``
checks it against the oracle on the CPU.  Test infrastructure only."""
from __future__ import annotations

import torch


def attention_mass_fp32(q: torch.Tensor, k: torch.Tensor, scale: float | None = None, chunk: int = 1024):
    """q [Hq, T, D], k [Hkv, T, D] (any float dtype; computed in fp32 with TF32
    off).  Returns (colsum float64 [T], importance float32 [T]) like the oracle:
    per head and query chunk the causal softmax rows, column sums accumulated
    in float64; importance = fp32(colsum) / its fp32 sum when that exceeds 1e-9."""
    Hq, T, D = q.shape
    G = Hq // k.shape[0]
    scale = D ** -0.5 if scale is None else scale
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        colsum = torch.zeros(T, dtype=torch.float64, device=q.device)
        for h in range(Hq):
            kh = k[h // G].float()
            for i0 in range(0, T, chunk):
                i1 = min(T, i0 + chunk)
                s = (q[h, i0:i1].float() @ kh[:i1].T) * scale
                rows = torch.arange(i0, i1, device=q.device)[:, None]
                cols = torch.arange(i1, device=q.device)[None, :]
                s = s.masked_fill(cols > rows, float("-inf"))
                p = torch.softmax(s, dim=1)
                colsum[:i1] += p.sum(dim=0, dtype=torch.float64)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    imp = colsum.float()
    total = imp.sum(dtype=torch.float32)
    if float(total) > 1e-9:
        imp = imp / total
    return colsum, imp
