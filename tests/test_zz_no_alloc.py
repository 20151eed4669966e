"""ic_summary_score_static: the summary scorer for callers that cannot
allocate device memory (their GPU memory belongs to another allocator, or
their language binding has no CUDA allocator).  It keeps the per-head mass
in a static device array owned by the library instead of a caller buffer.

The GPU test calls it through the C ABI twice in a row, on different inputs
and shapes, and checks every output against ic_summary_score given a
caller-allocated head_mass.  This file sorts last so that a run stopping at
its first failure has run every other test before it."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from infercache_b200 import _lib
from tolerances import elem_close

HEADER = Path(__file__).resolve().parents[1] / "include" / "infercache.h"


def test_static_limit_matches_header():
    m = re.search(r"#define IC_SUMMARY_STATIC_MASS_MAX (\d+)", HEADER.read_text())
    assert m and int(m.group(1)) == _lib.IC_SUMMARY_STATIC_MASS_MAX


def test_rejects_before_any_cuda_call():
    """Oversized shapes, a caller head_mass and missing outputs are refused on
    the host (dummy non-null pointers are never dereferenced)."""
    lib = _lib.load()
    fake = 256
    base = dict(q=fake, k=fake, v=fake, out=fake, lse=fake, head_mass=None, colsum=fake, importance=fake,
                batch=1, num_q_heads=16, num_kv_heads=2, seq_len=1024, head_dim=128, dtype=_lib.IC_BF16,
                accumulate=0, scale=1.0, dev_status=fake)
    too_big = dict(base, batch=2, seq_len=_lib.IC_SUMMARY_STATIC_MASS_MAX // 16)  # 2x the limit
    for kw in (too_big, dict(base, head_mass=fake), dict(base, colsum=None), dict(base, batch=0)):
        a = _lib.ic_summary_args(**kw)
        assert lib.ic_summary_score_static(ctypes.byref(a), None) == _lib.IC_ERR_INVALID_ARG
    assert b"static scratch" in lib.ic_last_error() or b"bad shape" in lib.ic_last_error()


def _run(name, q, k, v, with_head_mass, with_out=True, colsum0=None):
    """One call; colsum0 (if given) pre-fills colsum and sets accumulate."""
    B, Hq, T, D = q.shape
    dev = q.device
    out = torch.empty_like(q) if with_out else None
    lse = torch.empty(B, Hq, T, dtype=torch.float32, device=dev)
    hm = torch.empty(B, Hq, T, dtype=torch.float32, device=dev) if with_head_mass else None
    colsum = colsum0.clone() if colsum0 is not None else torch.empty(B, T, dtype=torch.float32, device=dev)
    imp = torch.empty(B, T, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    a = _lib.ic_summary_args(q=q.data_ptr(), k=k.data_ptr(), v=_lib.ptr(v if with_out else None),
                             out=_lib.ptr(out), lse=lse.data_ptr(), head_mass=_lib.ptr(hm), colsum=colsum.data_ptr(),
                             importance=imp.data_ptr(), batch=B, num_q_heads=Hq, num_kv_heads=k.shape[1],
                             seq_len=T, head_dim=D, dtype=_lib.dtype_code(q.dtype),
                             accumulate=1 if colsum0 is not None else 0, scale=D ** -0.5,
                             dev_status=status.data_ptr())
    _lib.call(name, a)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, lse, colsum, imp


def _compare(ref, got):
    if ref[0] is not None:
        o_ref, o_got = ref[0].float().cpu().numpy(), got[0].float().cpu().numpy()
        assert np.abs(o_got - o_ref).max() <= 1e-5 * np.abs(o_ref).max()
    for r, x in zip(ref[1:], got[1:]):
        assert elem_close(x.cpu().numpy(), r.cpu().numpy(), 1e-5)


def _inputs(seed, B, Hq, Hkv, T, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return tuple(torch.randn(B, H, T, 128, generator=g, device="cuda").to(dtype) for H in (Hq, Hkv, Hkv))


@pytest.mark.gpu
def test_static_scratch_matches_caller_buffer_twice():
    """Two calls in a row (different seeds and lengths, so the second reuses
    the array the first filled): outputs equal ic_summary_score's within the
    fp32 tolerance of the parity tests (1e-5; the kernels are the same)."""
    _lib.require_device(torch.device("cuda", 0))
    torch.cuda.set_device(0)
    for seed, B, T in ((41, 2, 1000), (42, 1, 777)):
        g = torch.Generator(device="cuda").manual_seed(seed)
        q = torch.randn(B, 16, T, 128, generator=g, device="cuda").bfloat16()
        k = torch.randn(B, 2, T, 128, generator=g, device="cuda").bfloat16()
        v = torch.randn(B, 2, T, 128, generator=g, device="cuda").bfloat16()
        ref = _run("ic_summary_score", q, k, v, True)
        got = _run("ic_summary_score_static", q, k, v, False)
        o_ref, o_got = ref[0].float().cpu().numpy(), got[0].float().cpu().numpy()
        assert np.abs(o_got - o_ref).max() <= 1e-5 * np.abs(o_ref).max()
        for r, x in zip(ref[1:], got[1:]):
            assert elem_close(x.cpu().numpy(), r.cpu().numpy(), 1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["fp16", "no_output", "accumulate", "at_limit"])
def test_static_scratch_variants(case):
    """The other argument forms against ic_summary_score with a caller
    head_mass: fp16 inputs; no attention output (out and v NULL); colsum
    accumulated onto a pre-filled buffer (the all-layers sum); and a shape
    exactly at the limit (batch * heads * seq_len == IC_SUMMARY_STATIC_MASS_MAX)."""
    _lib.require_device(torch.device("cuda", 0))
    torch.cuda.set_device(0)
    if case == "fp16":
        q, k, v = _inputs(51, 2, 16, 2, 640, torch.float16)
        ref, got = _run("ic_summary_score", q, k, v, True), _run("ic_summary_score_static", q, k, v, False)
    elif case == "no_output":
        q, k, v = _inputs(52, 1, 16, 2, 900, torch.bfloat16)
        ref = _run("ic_summary_score", q, k, v, True, with_out=False)
        got = _run("ic_summary_score_static", q, k, v, False, with_out=False)
    elif case == "accumulate":
        q, k, v = _inputs(53, 2, 8, 1, 500, torch.bfloat16)
        c0 = torch.rand(2, 500, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda")
        ref = _run("ic_summary_score", q, k, v, True, colsum0=c0)
        got = _run("ic_summary_score_static", q, k, v, False, colsum0=c0)
    else:
        T = _lib.IC_SUMMARY_STATIC_MASS_MAX // 16 // 2
        q, k, v = _inputs(54, 2, 16, 2, T, torch.bfloat16)
        assert q.shape[0] * q.shape[1] * q.shape[2] == _lib.IC_SUMMARY_STATIC_MASS_MAX
        ref = _run("ic_summary_score", q, k, v, True, with_out=False)
        got = _run("ic_summary_score_static", q, k, v, False, with_out=False)
    _compare(ref, got)
