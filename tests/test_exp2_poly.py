"""CPU check of the attention softmax's FMA-pipe exponential (exp2_poly2 in mfd_b200/csrc/tree_attention_tc.cu):
its coefficients are read from the source and its steps restated in float32 (each fma rounded once, as the
kernel's fma.rn.f32x2), then held to the error bound the kernel's comment states against 2^x in float64."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(__file__), "..", "mfd_b200", "csrc", "tree_attention_tc.cu")
BOUND = 1.1e-4  # relative, for x in [-126, 16]


def coefficients():
    src = open(SRC).read()
    m = re.search(r"kExpC1 = ([0-9.e+-]+)f, kExpC2 = ([0-9.e+-]+)f, kExpC3 = ([0-9.e+-]+)f;", src)
    assert m, "exp2_poly2 coefficients not found"
    return [np.float32(float(v)) for v in m.groups()]


def fma32(a, b, c):
    # a * b is exact in float64 for float32 operands; one rounding of the sum to float32 (the double rounding
    # through float64 can differ from a fused float32 fma in the last bit at most, far inside the bound)
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x):
    c1, c2, c3 = coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-127.0))  # fmaxf: NaN -> -127
    x = np.where(np.isnan(x), np.float32(-127.0), x).astype(np.float32)
    t = (x + np.float32(12582912.0)).astype(np.float32)
    f = (x - (t - np.float32(12582912.0)).astype(np.float32)).astype(np.float32)
    one = np.float32(1.0)
    q = fma32(fma32(fma32(np.full_like(f, c3), f, np.full_like(f, c2)), f, np.full_like(f, c1)), f,
              np.full_like(f, one))
    bits = q.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << np.uint64(23))
    return (bits & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)


def test_exp2_poly_relative_error_bound():
    x = np.concatenate([np.linspace(-126.0, 16.0, 400_001, dtype=np.float32),
                        np.arange(-126, 17, dtype=np.float32) + np.float32(0.5),
                        np.arange(-126, 17, dtype=np.float32)])
    y = exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() <= BOUND, (rel.max(), x[rel.argmax()])


def test_exp2_poly_masked_scores_give_zero():
    x = np.array([-np.inf, np.nan, -127.0, -200.0, -1e30], dtype=np.float32)
    y = exp2_poly(x)
    assert np.all(y == 0.0) and not np.any(np.signbit(y))


def test_exp2_poly_is_monotone_within_rounding():
    # P is rounded to bf16 next: neighbouring arguments may not swap order by more than the bound
    x = np.linspace(-20.0, 9.0, 100_001, dtype=np.float32)
    y = exp2_poly(x).astype(np.float64)
    assert np.all(np.diff(y) >= -BOUND * y[1:])

