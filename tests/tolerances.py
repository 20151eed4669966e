"""Tolerances used by every parity test.

* Attention outputs: normwise relative per output row (one query head):
  max_d |a - b| <= rtol * max_d |b|.  An elementwise relative test is
  meaningless for outputs that cancel to ~0, so the row's scale is the unit.
* Importance scores / masses: elementwise relative, |a - b| <= rtol * |b|,
  with an absolute floor of rtol * 1e-6 * max|b| for slots that hold ~0.
* rtol = 1e-5 for fp32 caches and 1e-3 for fp16 / bf16 caches.
* Index work (slot placement, positions, occupancy, eviction events,
  page tables) is compared exactly.
"""
import numpy as np

RTOL = {"float32": 1e-5, "float16": 1e-3, "bfloat16": 1e-3}


def rows_close(a, b, rtol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    err = np.abs(a - b).max(axis=-1)
    scale = np.abs(b).max(axis=-1)
    return bool(np.all(err <= rtol * scale))


def rows_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float((np.abs(a - b).max(axis=-1) / np.maximum(np.abs(b).max(axis=-1), 1e-300)).max())


def elem_close(a, b, rtol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    floor = rtol * 1e-6 * (np.abs(b).max() if b.size else 0.0)
    return bool(np.all(np.abs(a - b) <= np.maximum(rtol * np.abs(b), floor)))
