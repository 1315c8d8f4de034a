"""Accuracy of the exact-erf GELU polynomial the kernels evaluate
(``gelu_poly_f2`` in csrc/ptx.cuh), checked on the CPU.

The reference's baseline GELU is the exact erf form
(torch_transformer_benchmark.py:286, ``F.gelu(..., approximate="none")``). The kernels evaluate
GELU(x) = x * (1/2 + xc * Q'(t)): xc = x clamped to +-3.5 sqrt 2, t = xc^2 / 3.5^2 - 1,
and Q' = Q / (2 sqrt 2) with Q the fitted polynomial for which erf(z) = zc * Q(t). This test
reads Q' from the header, evaluates it the way the kernel does (fp32 Horner steps, each an
fma rounded to fp32) and checks the error bounds the header states against math.erf.
"""

from __future__ import annotations

import math
import pathlib
import re

import numpy as np

HEADER = (pathlib.Path(__file__).resolve().parents[1] / "gpu-kernel-for-transformer_b200" /
          "csrc" / "ptx.cuh")

ERF_BOUND = 2.6e-5   # |erf error| the header states
# |GELU error| = |x/2| * |erf error| (plus fp32 rounding): <= 1.3e-5 * |x|.
GELU_SLOPE = 0.5 * ERF_BOUND


def _coefficients() -> np.ndarray:
    text = HEADER.read_text()
    body = text[text.index("gelu_poly_f2"):]
    m = re.search(r"constexpr float kQ\[(\d+)\] = \{([^}]*)\}", body)
    assert m, "gelu_poly_f2 coefficient table not found"
    vals = [float(v.strip().rstrip("f")) for v in m.group(2).split(",") if v.strip()]
    assert len(vals) == int(m.group(1))
    return np.array(vals, dtype=np.float32)


def _fma32(a, b, c):
    # fp32 fma: the fp64 product of two fp32 values is exact; one rounding of
    # the sum to fp32 (a double rounding differs from a true fma only in rare
    # last-bit cases, far below the bounds checked here).
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


CLAMP = np.float32(4.949747562408447)   # 3.5 * sqrt 2
T_SCALE = np.float32(0.08163265138864517)  # 1 / 3.5^2


def _half_erf_term(x: np.ndarray, q: np.ndarray) -> np.ndarray:
    """xc * Q'(t) = erf(x / sqrt 2) / 2, as the kernel computes it."""
    xc = np.clip(x.astype(np.float32), -CLAMP, CLAMP)
    t = _fma32(xc, (xc * T_SCALE).astype(np.float32), np.float32(-1.0))
    p = np.full_like(t, q[-1])
    for k in range(len(q) - 2, -1, -1):
        p = _fma32(p, t, np.full_like(t, q[k]))
    return xc, p


def test_erf_polynomial_error_bound():
    q = _coefficients()
    z = np.linspace(-6.0, 6.0, 240001, dtype=np.float64)
    x = (z * math.sqrt(2.0)).astype(np.float32)
    xc, p = _half_erf_term(x, q)
    got = 2.0 * xc.astype(np.float64) * p.astype(np.float64)
    ref = np.array([math.erf(float(v) / math.sqrt(2.0)) for v in x])
    err = np.abs(got - ref)
    assert err.max() <= ERF_BOUND, err.max()


def test_gelu_error_bound():
    q = _coefficients()
    x = np.linspace(-8.0, 8.0, 160001, dtype=np.float32)
    xc, p = _half_erf_term(x, q)
    got = (x * _fma32(xc, p, np.full_like(p, np.float32(0.5)))).astype(np.float32)
    ref = np.array([0.5 * float(v) * (1.0 + math.erf(float(v) / math.sqrt(2.0))) for v in x])
    err = np.abs(got.astype(np.float64) - ref)
    bound = GELU_SLOPE * np.abs(x.astype(np.float64)) + 4e-7 * np.maximum(np.abs(ref), 1.0)
    assert np.all(err <= bound), float((err - bound).max())
