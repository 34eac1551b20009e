"""The RGBA scorer divides by 3 with one correction step instead of an IEEE division:
q = RN(x * RN(1/3)), r = x - 3q (exact with an FMA), result RN(q + r * RN(1/3)) (Markstein's
correction).  This emulates that arithmetic on the host and checks it against IEEE f32 division
over a dense sample of [0, 4), the range of the sums of three |delta| terms it is used on (the
same check over every f32 in [0, 4) passes too, in about a minute)."""
from fractions import Fraction

import numpy as np

THIRD = np.float32(1) / np.float32(3)


def _div3_method(x: np.ndarray) -> np.ndarray:
    q = x * THIRD
    r64 = x.astype(np.float64) - q.astype(np.float64) * 3.0  # exact: the FMA residual
    r = r64.astype(np.float32)
    assert np.array_equal(r.astype(np.float64), r64), "the residual must be representable"
    s64 = q.astype(np.float64) + r.astype(np.float64) * np.float64(THIRD)
    got = s64.astype(np.float32)
    # where the f64 sum sits exactly on an f32 midpoint, round the exact value instead
    ulp = np.spacing(got).astype(np.float64)
    for i in np.flatnonzero(np.abs(s64 - got.astype(np.float64)) * 2 == ulp):
        e = Fraction(float(q[i])) + Fraction(float(r[i])) * Fraction(float(THIRD))
        g = np.float32(float(e))
        cands = [np.nextafter(g, np.float32(-np.inf)), g, np.nextafter(g, np.float32(np.inf))]
        got[i] = min(cands, key=lambda c: (abs(Fraction(float(c)) - e), int(c.view(np.uint32)) & 1))
    return got


def test_third_constant_is_rn_one_third():
    assert THIRD.view(np.uint32) == 0x3EAAAAAB  # 0x1.555556p-2


def test_div3_matches_ieee_division_on_a_dense_sample():
    top = int(np.float32(4.0).view(np.uint32))
    bits = np.arange(0, top, 97, dtype=np.uint32)
    x = bits.view(np.float32)
    assert np.array_equal(_div3_method(x).view(np.uint32), (x / np.float32(3)).view(np.uint32))


def test_div3_matches_ieee_division_on_every_value_near_the_binade_edges():
    # every f32 within 2^16 ulps of each power of two in [2^-40, 4), and the subnormals' start
    edges = [np.float32(2.0) ** e for e in range(-40, 2)]
    chunks = [np.arange(0, 1 << 16, dtype=np.uint32)]
    for v in edges:
        b = int(np.float32(v).view(np.uint32))
        chunks.append(np.arange(b - (1 << 16), b + (1 << 16), dtype=np.uint32))
    x = np.unique(np.concatenate(chunks)).view(np.float32)
    x = x[(x >= 0) & (x < 4)]
    assert np.array_equal(_div3_method(x).view(np.uint32), (x / np.float32(3)).view(np.uint32))
