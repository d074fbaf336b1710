"""The polynomial 2^x of the tcgen05 prefill softmax (``tc_exp2_poly`` in
csrc/attention_tc.cu), restated in float32 numpy with the constants read from
the source: relative error against 2^x over the softmax's input range, exact
zero below -126 (masked keys)."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc", "attention_tc.cu")


def _coeffs():
    body = open(SRC).read()
    body = body[body.index("BRAID_DEVICE float tc_exp2_poly"):]
    body = body[:body.index("}\n")]
    line = next(ln for ln in body.splitlines() if "const float q =" in ln)
    c3, c2, c1, c0 = (np.float32(v) for v in re.findall(r"(\d+\.\d+)f", line))
    return c0, c1, c2, c3


def _poly(x, c):
    c0, c1, c2, c3 = c
    x = np.asarray(x, np.float32)
    xc = np.maximum(x, np.float32(-126.0))
    t = (xc + np.float32(12582912.0)).astype(np.float32)
    f = (xc - (t - np.float32(12582912.0))).astype(np.float32)
    q = ((c3 * f + c2) * f + c1) * f + c0
    n = t.view(np.int32) - np.int32(0x4B400000)
    y = (q.astype(np.float32).view(np.int32) + (n << 23)).view(np.float32)
    return np.where(x < -126.0, np.float32(0.0), y)


def test_exp2_poly_relative_error():
    c = _coeffs()
    # down to -125: at -126 the result (1.2e-38) reaches the denormal range
    x = np.linspace(-125.0, 8.0, 400001, dtype=np.float32)
    y = _poly(x, c).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y - ref) / ref
    assert rel.max() < 1e-4, rel.max()


def test_exp2_poly_masked_and_integers():
    c = _coeffs()
    assert _poly(np.array([-np.inf, -200.0, -126.5], np.float32), c).tolist() == [0.0, 0.0, 0.0]
    ints = np.arange(-20, 9, dtype=np.float32)
    np.testing.assert_allclose(_poly(ints, c), np.exp2(ints), rtol=1e-4)
