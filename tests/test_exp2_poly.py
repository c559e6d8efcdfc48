"""CPU: the FMA-pipe exponential of the window-attention softmax.

The kernel (seedvr2_ncnn_b200/csrc/attention_sm100.cu, exp2_poly2) computes
2^t for part of each score row without the MUFU: n = round(t) by adding and
subtracting 1.5 * 2^23, f = t - n, a cubic for 2^f on [-1/2, 1/2], and n
added to the result's exponent bits; t is clamped to -126 first.  This test
replays that exact float32 sequence in numpy (coefficients read from the
kernel source, so the two cannot drift apart) and bounds its error against
exact 2^t over the softmax's range, well below the 2^-9 relative rounding of
the bf16 P it feeds.
"""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "seedvr2_ncnn_b200", "csrc", "attention_sm100.cu")


def _coeffs():
    text = open(SRC).read()
    m = re.search(r"constexpr float c0 = ([0-9.eE+-]+)f, c1 = ([0-9.eE+-]+)f, c2 = ([0-9.eE+-]+)f, "
                  r"c3 = ([0-9.eE+-]+)f;", text)
    assert m, "coefficients not found in the kernel source"
    return [np.float32(float(v)) for v in m.groups()]


def exp2_poly(t: np.ndarray) -> np.ndarray:
    """The kernel's instruction sequence in float32 (round-to-nearest adds and FMAs)."""
    c0, c1, c2, c3 = _coeffs()
    t = np.maximum(t.astype(np.float32), np.float32(-126.0))
    k = np.float32(12582912.0)
    y = (t + k).astype(np.float32)
    n = (y - k).astype(np.float32)
    # f = fma(n, -1, t): exact in float32 (|t - n| <= 1/2 and both are float32)
    f = (t.astype(np.float64) - n.astype(np.float64)).astype(np.float32)

    def fma(a, b, c):  # single rounding, like fma.rn.f32x2
        return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)

    p = fma(f, np.full_like(f, c3), np.full_like(f, c2))
    p = fma(p, f, np.full_like(f, c1))
    p = fma(p, f, np.full_like(f, c0))
    bits = (p.view(np.uint32) + (y.view(np.uint32) << np.uint32(23))).astype(np.uint32)
    return bits.view(np.float32)


def test_exp2_poly_relative_error_over_softmax_range():
    # exponents of a softmax with lazy rescaling lie below 8; dense grid plus the integers and the
    # half-integers where the rounding of n changes (below -120 the results are < 1e-36 and the last
    # steps of the range leave the normal exponents: see the clamp test)
    t = np.concatenate([np.linspace(-120.0, 8.0, 2_000_001), np.arange(-120, 9, dtype=np.float64),
                        np.arange(-120, 8, dtype=np.float64) + 0.5]).astype(np.float32)
    got = exp2_poly(t).astype(np.float64)
    exact = np.exp2(t.astype(np.float64))
    rel = np.abs(got - exact) / exact
    assert rel.max() < 1.0e-4, rel.max()          # cubic fit: 7.5e-5; bf16 rounding of P: 2^-9 = 2e-3
    assert np.all(np.isfinite(got)) and np.all(got > 0)


def test_exp2_poly_clamps_far_negative_and_infinite_inputs():
    t = np.array([-1e30, -np.inf, -300.0, -127.0, -126.0], np.float32)
    got = exp2_poly(t)
    assert np.all(np.isfinite(got)) and np.all(got >= 0) and np.all(got < 2.0 ** -125)
