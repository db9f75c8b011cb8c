"""Host restatement (float32 numpy) of the FMA-pipe exponential of the
tcgen05 attention kernel (exp2_poly2 in csrc/attention_sm100.cu): the
polynomial coefficients are read from the kernel source, so this checks the
shipped constants and bit arithmetic: relative error against 2^x, exact zeros
for masked scores (-inf) and at the clamp, no negative or NaN results."""
import pathlib
import re

import numpy as np

SRC = pathlib.Path(__file__).resolve().parents[1] / "pytorch-parallel-compiler_b200" / "csrc" / "attention_sm100.cu"


def _coefficients():
    body = SRC.read_text()
    body = body[body.index("float2 exp2_poly2("):]
    body = body[:body.index("two_n")]
    vals = [float(v) for v in re.findall(r"make_float2\(([0-9.]+)f, \1f\)", body)]
    # Horner order in the source: c3, c2, c1, c0
    assert len(vals) == 4, vals
    return np.float32(vals[::-1])


def _poly2(x, c):
    x = np.maximum(np.float32(x), np.float32(-127))
    m = np.float32(12582912.0)
    t = (x + m).astype(np.float32)
    n = (t - m).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = np.float32(c[3])
    for ci in (c[2], c[1], c[0]):
        p = (p * f + ci).astype(np.float32)
    tb = t.view(np.int32).astype(np.int64)
    two_n = (((tb << 23) + 0x3F800000) & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return (p * two_n).astype(np.float32)


def test_exp2_polynomial_restatement():
    c = _coefficients()
    x = np.linspace(-140, 8, 400001).astype(np.float32)
    with np.errstate(all="ignore"):
        y = _poly2(x, c)
    assert not np.isnan(y).any() and (y >= 0).all()
    ok = x > -120
    rel = np.abs(y[ok] - np.exp2(x[ok].astype(np.float64))) / np.exp2(x[ok].astype(np.float64))
    assert rel.max() < 1e-4, rel.max()
    special = _poly2(np.float32([-np.inf, -127.0, -200.0]), c)
    assert (special == 0).all(), special
