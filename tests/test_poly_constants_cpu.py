"""The prefill kernels' polynomial constants come from their committed fits.

csrc/prefill_common.cuh evaluates part of the softmax on the FMA pipe with two
minimax polynomials: 2^f on [-1/2, 1/2] (Exp2Poly, degrees 3 and 4) and
tanh(y)/y on |y| <= 3/4 as a polynomial in y^2 (TanhPoly, degree 4). This
re-runs the Remez fits of csrc/fit_exp2_poly.py and csrc/fit_tanh_poly.py and
checks that the float32 literals in the header are the fits' coefficients and
that their float32 evaluation keeps the stated error bounds. A float32
emulation of the softcap route (TanhPoly::fma) checks its accuracy for caps
from 1e-3 to 1e6 and that a masked score leaves it as exactly -inf. CPU only.
"""

import os
import re
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "flash-attn-mps_b200", "csrc")
sys.path.insert(0, CSRC)

import fit_exp2_poly  # noqa: E402
import fit_tanh_poly  # noqa: E402


def _header():
    with open(os.path.join(CSRC, "prefill_common.cuh")) as f:
        return f.read()


def _literals(text):
    return [np.float32(float(x)) for x in re.findall(r"([-+]?\d\.\d+e[-+]\d+)f", text)]


@pytest.mark.parametrize("deg, branch", [(3, "if constexpr (DEG3) {"), (4, "} else {")])
def test_exp2_poly_constants_match_fit(deg, branch):
    src = _header()
    body = src[src.index("struct Exp2Poly"):src.index("operator()", src.index("struct Exp2Poly"))]
    part = body[body.index(branch):]
    part = part[:part.index("}", len(branch))]
    got = _literals(part)[::2]  # each literal appears twice (f2pack of a pair)
    c, _ = fit_exp2_poly.remez(deg)
    want = [np.float32(x) for x in c[1:]]
    assert got == want, (got, want)
    f = np.linspace(-0.5, 0.5, 20001).astype(np.float32)
    rel = np.abs(fit_exp2_poly.horner32([np.float32(1)] + want, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1)
    assert rel.max() < (4.4e-4 if deg == 3 else 5.5e-6)


def test_tanh_poly_constants_match_fit():
    src = _header()
    body = src[src.index("struct TanhPoly"):src.index("fma(", src.index("struct TanhPoly"))]
    got = _literals(body)
    y0 = float(re.search(r"kSoftcapPolyY = ([0-9.]+)f", src).group(1))
    c, _ = fit_tanh_poly.remez(4, vmax=y0 * y0)
    want = [np.float32(x) for x in c[1:]]
    assert got == want, (got, want)
    y = np.linspace(-y0, y0, 40001).astype(np.float32)
    y = y[y != 0]
    t = fit_tanh_poly.tanh32([np.float32(1)] + want, y).astype(np.float64)
    ref = np.tanh(y.astype(np.float64))
    assert np.abs(t / ref - 1).max() < 8e-7 and np.abs(t - ref).max() < 5e-7


def _tanh_route(s, scale, cap, add):
    """float32 emulation of TanhPoly::fma: y = s * c, v = y * y, Horner in v
    with the score scale folded into the coefficients, then s * Q + add; each
    FMA rounds once (the exact float64 product plus the addend, rounded)."""
    f32 = np.float32
    fma = lambda a, b, c: (np.float64(a) * np.float64(b) + np.float64(c)).astype(np.float32)  # noqa: E731
    src = _header()
    body = src[src.index("struct TanhPoly"):src.index("fma(", src.index("struct TanhPoly"))]
    q = _literals(body)
    sl2 = f32(scale * 1.4426950408889634)
    c = f32(f32(scale) / f32(cap))
    k = [sl2] + [f32(sl2 * qi) for qi in q]
    s = np.asarray(s, dtype=np.float32)
    y = (s * c).astype(np.float32)
    v = (y * y).astype(np.float32)
    acc = fma(np.full_like(v, k[4]), v, k[3])
    for i in (2, 1, 0):
        acc = fma(acc, v, k[i])
    return fma(s, acc, np.full_like(s, add)), c


@pytest.mark.parametrize("cap", [1e-3, 0.25, 1.0, 6.0, 50.0, 1e3, 1e6])
@pytest.mark.parametrize("scale", [0.0884, 1.0, 3.0])
def test_softcap_route_accuracy_for_any_cap(cap, scale):
    # Over the route's whole range |s * scale / cap| <= 3/4 the capped score in
    # log2 units is within 5e-7 * cap * log2e of cap * log2e * tanh(s * scale / cap).
    lim = 0.75 * cap / scale
    s = np.linspace(-lim, lim, 20001)
    got, _ = _tanh_route(s, scale, cap, 0.0)
    ref = cap * np.log2(np.e) * np.tanh(s.astype(np.float32).astype(np.float64) * np.float32(scale) / np.float32(cap))
    assert np.abs(got.astype(np.float64) - ref).max() <= 5e-7 * cap * np.log2(np.e)


def test_softcap_route_maps_masked_scores_to_minus_infinity():
    # With scale / cap > 0, a masked score (-inf) comes out as exactly -inf for
    # any finite running max, so 2^(logit - m) is exactly 0 without a select.
    for cap, scale in [(50.0, 0.0884), (1e-3, 3.0), (1e6, 0.01)]:
        got, c = _tanh_route([-np.inf, 0.0, 1.0], scale, cap, -7.25)
        assert c > 0 and got[0] == -np.inf and np.all(np.isfinite(got[1:]))
