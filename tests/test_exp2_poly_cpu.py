"""The FP32-pipe 2^x of exp2_poly.cuh, emulated bit for bit in numpy (fp32
adds, the shifter reduction, Horner in fp32, the exponent-field add), against
float64 exp2: relative error within its stated 2.7e-6 bound on [-126, 1], a
result in (0, 2^-125] below the clamp, and the header's coefficients equal to
the fit script's."""
import re
import subprocess
import sys
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parents[1] / "infercache_b200" / "csrc"


def header_coeffs():
    text = (CSRC / "exp2_poly.cuh").read_text()
    vals = dict(re.findall(r"EXP2_C(\d) = 0x([0-9A-Fa-f]{8})u", text))
    return np.array([int(vals[str(k)], 16) for k in range(len(vals))], np.uint32).view(np.float32)


def fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_emulated(x, c):
    x = np.maximum(np.asarray(x, np.float32), np.float32(-126.0))
    sh = np.float32(12582912.0)
    t = (x + sh).astype(np.float32)
    f = (x - (t - sh).astype(np.float32)).astype(np.float32)
    p = np.full_like(x, c[-1])
    for ck in c[-2::-1]:
        p = fma32(p, f, np.full_like(x, ck))
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_bound():
    c = header_coeffs()
    assert len(c) == 5
    x = np.concatenate([np.linspace(-126.0, 1.0, 4_000_001, dtype=np.float32),
                        np.float32(-0.5) + np.arange(-64, 65, dtype=np.float32) * np.float32(2 ** -23),
                        np.array([0.0, -1.0, 0.5, -0.5, -125.5], np.float32)])
    y = exp2_emulated(x, c).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1)
    assert rel.max() <= 2.7e-6, rel.max()


def test_clamped_inputs_are_tiny_and_positive():
    c = header_coeffs()
    x = np.array([-126.0, -126.4, -127.0, -200.0, -1e30, -np.inf], np.float32)
    y = exp2_emulated(x, c)
    assert np.all(y > 0) and np.all(y <= np.float32(2.0 ** -125))


def test_header_matches_fit():
    out = subprocess.run([sys.executable, str(CSRC / "exp2_poly_fit.py"), "4"], capture_output=True, text=True,
                         check=True).stdout
    fit = [int(h, 16) for h in re.findall(r"c\d = 0x([0-9A-F]{8})", out)]
    assert fit == [int(v) for v in header_coeffs().view(np.uint32)]
