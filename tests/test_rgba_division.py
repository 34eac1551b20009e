"""Host checks of the RGBA scorer's arithmetic shortcuts, on an emulation of the device's f32
operations.

It divides by 3 with one correction step instead of an IEEE division:
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


def _rn(x):
    return x.astype(np.float32)


def _luma(r, g, b):
    f = np.float32
    return _rn(_rn(_rn(r * f(0.2126)) + _rn(g * f(0.7152))) + _rn(b * f(0.0722)))


def test_pixel_score_bounds_never_drop_the_maximum():
    """The scorer skips the relative-luma and chroma quotients of a changed pixel when a
    division-free bound shows they are below max(rgb, luma) (rel_below / chroma_below).  On
    pixel pairs of several distributions the rounded score with and without the skips must be
    identical."""
    f = np.float32
    rng = np.random.default_rng(5)
    n = 2_000_000
    p = rng.integers(0, 256, size=(n, 3))
    c = p.copy()
    kind = rng.integers(0, 4, size=n)
    k = kind == 0
    c[k] = rng.integers(0, 256, size=(k.sum(), 3))
    k = kind == 1
    c[k] = np.clip(p[k] + rng.integers(-3, 4, size=(k.sum(), 3)), 0, 255)
    k = kind == 2  # dark pixels, where the chroma term is large
    p[k] = rng.integers(0, 30, size=(k.sum(), 3))
    c[k] = rng.integers(0, 30, size=(k.sum(), 3))
    k = kind == 3
    c[k] = np.clip(p[k] + rng.integers(-60, 61, size=(k.sum(), 3)), 0, 255)
    keep = ~(p == c).all(axis=1)
    inv = np.arange(256, dtype=np.float32) / f(255)
    a, b = inv[p[keep]], inv[c[keep]]
    d = [_rn(b[:, i] - a[:, i]) for i in range(3)]
    rgb = _rn(_rn(_rn(np.abs(d[0]) + np.abs(d[1])) + np.abs(d[2])) / f(3))
    pl, cl = _luma(a[:, 0], a[:, 1], a[:, 2]), _luma(b[:, 0], b[:, 1], b[:, 2])
    lum = np.abs(_rn(cl - pl))
    den = np.maximum(np.maximum(pl, cl), f(0.10))
    rel = _rn(np.minimum(_rn(lum / den), f(1)) * f(0.25))
    dp = np.maximum(_rn(_rn(a[:, 0] + a[:, 1]) + a[:, 2]), f(0.10))
    dc = np.maximum(_rn(_rn(b[:, 0] + b[:, 1]) + b[:, 2]), f(0.10))
    q = [np.abs(_rn(_rn(b[:, i] / dc) - _rn(a[:, i] / dp))) for i in range(3)]
    chroma = _rn(_rn(_rn(_rn(q[0] + q[1]) + q[2]) / f(3)) * f(0.5))
    full = np.maximum(np.maximum(np.maximum(rgb, lum), rel), chroma)

    m = np.maximum(rgb, lum)
    rel_skip = _rn(_rn(lum * f(0.25)) * f(1.00001)) <= _rn(m * den)

    def fma(x, y, z):  # exact product and sum in f64, one rounding to f32
        return _rn(x.astype(np.float64) * y.astype(np.float64) + z.astype(np.float64))

    e = [np.abs(fma(b[:, i], dp, -_rn(a[:, i] * dc))) for i in range(3)]
    w = _rn(_rn(e[0] + e[1]) + e[2])
    chroma_skip = _rn(w + f(7e-6)) < _rn(_rn(_rn(f(5.999) * m) * dc) * dp)
    fast = np.where(rel_skip, m, np.maximum(m, rel))
    fast = np.where(chroma_skip, fast, np.maximum(fast, chroma))
    assert rel_skip.mean() > 0.5 and chroma_skip.mean() > 0.5  # the skips do apply
    assert np.array_equal(fast.view(np.uint32), full.view(np.uint32))


def _div_by_rcp_method(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The device's chroma quotient: y = RN(1/b), q = RN(a y), result RN(q + (a - b q) y), with
    the FMA residual and the final FMA rounded once each (exact rationals at midpoints)."""
    y = (np.float32(1) / b).astype(np.float32)
    q = (a * y).astype(np.float32)
    r64 = a.astype(np.float64) - b.astype(np.float64) * q.astype(np.float64)  # exact in f64
    r = r64.astype(np.float32)  # the FMA's one rounding of the exact residual
    s64 = q.astype(np.float64) + r.astype(np.float64) * y.astype(np.float64)
    got = s64.astype(np.float32)
    ulp = np.spacing(got).astype(np.float64)
    exact_check = np.abs(s64 - got.astype(np.float64)) * 2 >= ulp * 0.999  # near a midpoint: redo exactly
    for i in np.flatnonzero(exact_check):
        e = Fraction(float(q[i])) + Fraction(float(r[i])) * Fraction(float(y[i]))
        g = np.float32(float(e))
        cands = [np.nextafter(g, np.float32(-np.inf)), g, np.nextafter(g, np.float32(np.inf))]
        got[i] = min(cands, key=lambda c: (abs(Fraction(float(c)) - e), int(c.view(np.uint32)) & 1))
    return got


def test_chroma_quotient_matches_ieee_division_on_every_operand_pair():
    """Every channel value i / 255 over every chroma denominator max(r + g + b, 0.10) the u8
    pixels produce (1325 values): the reciprocal-and-correction quotient equals a / b."""
    v = (np.arange(256, dtype=np.float32) / np.float32(255)).astype(np.float32)
    sums = ((v[:, None, None] + v[None, :, None]).astype(np.float32) + v[None, None, :]).astype(np.float32)
    dens = np.unique(np.maximum(sums, np.float32(0.10)))
    assert len(dens) == 1325
    a = np.repeat(v, len(dens))
    b = np.tile(dens, len(v))
    assert np.array_equal(_div_by_rcp_method(a, b).view(np.uint32), (a / b).view(np.uint32))
