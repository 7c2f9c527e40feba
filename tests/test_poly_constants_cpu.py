"""The prefill kernels' polynomial constants come from their committed fits.

csrc/prefill_common.cuh evaluates part of the softmax on the FMA pipe with two
minimax polynomials: 2^f on [-1/2, 1/2] (Exp2Poly, degrees 3 and 4) and
tanh(y)/y on |y| <= 3/4 as a polynomial in y^2 (TanhPoly, degree 4). This
re-runs the Remez fits of csrc/fit_exp2_poly.py and csrc/fit_tanh_poly.py and
checks that the float32 literals in the header are the fits' coefficients and
that their float32 evaluation keeps the stated error bounds. CPU only.
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
