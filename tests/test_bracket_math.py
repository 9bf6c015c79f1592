"""The bracket around the exact log-sum-exp, restated on the CPU.

The streaming pass's approximate part sums are emulated in numpy fp32 (the
same argument rounding, layout, addition tree, compensated accumulation and
reference moves; numpy's exp2 stands in for the hardware unit, whose own
error the GPU self-check bounds), the bracket is formed as the merge forms
it, and the oracle's exact log-sum-exp must lie inside it for rows of many
scales, shapes and part lengths.
"""

import math

import numpy as np
import pytest

import oracle as O

L2E = np.float32(1.4426950408889634)  # fl32(log2 e)
LN2 = math.log(2.0)


def _f32(v):
    return np.float32(v)


def _lane_partial(vals, aLref):
    """One tile's lane partials ([32 lanes]) as approx_lane_sum computes
    them: pairs in f32x2 halves, a four-level tree over the 16 pairs, then
    the two halves."""
    a = (vals.astype(np.float64) * np.float64(L2E) - np.float64(aLref)).astype(np.float32)
    v = np.exp2(a).astype(np.float32)
    w = v.reshape(32, 16, 2)
    h = 8
    while h >= 1:
        w = (w[:, :h, :] + w[:, h:2 * h, :]).astype(np.float32)
        h //= 2
    return (w[:, 0, 0] + w[:, 0, 1]).astype(np.float32)


def _approx_part_stats(x: np.ndarray, tiles_per_part: int):
    """(mref, eps, s) per row part, as the streaming pass computes them:
    lane L holds slots s = 0..31 of a tile at element (s // 4) * 128 + L * 4 +
    s % 4; each lane adds its tile partials by Kahan summation against the
    part's reference (the first finite tile maximum, moved up when a value
    would sit more than 2^64 above it); the part's lanes are added in fp64."""
    V = x.shape[0]
    nt = -(-V // 1024)
    pad = np.full(nt * 1024, -np.inf, np.float32)
    pad[:V] = x
    tiles = pad.reshape(nt, 1024)
    s_idx = np.arange(32)
    lane = np.arange(32)[:, None]
    elem = (s_idx // 4) * 128 + lane * 4 + s_idx % 4
    parts = []
    for t0 in range(0, nt, tiles_per_part):
        aref = aLref = -np.inf
        hi = np.zeros(32, np.float32)
        c = np.zeros(32, np.float32)
        amx = np.full(32, -np.inf, np.float32)
        nres = 0
        for t in range(t0, min(nt, t0 + tiles_per_part)):
            vals = tiles[t][elem]
            lm = vals.max(axis=1)
            if aLref == -np.inf:
                m = lm.max()
                if m == -np.inf:
                    continue
                aref, aLref = m, _f32(m * L2E)
            elif (lm.astype(np.float64) * np.float64(L2E) - np.float64(aLref) > 64).any():
                m = lm.max()
                nL = _f32(m * L2E)
                f = _f32(np.exp2(np.float64(_f32(aLref - nL))))
                hi, c = (hi * f).astype(np.float32), (c * f).astype(np.float32)
                aref, aLref, nres = m, nL, nres + 1
            tp = _lane_partial(vals, aLref)
            y = (tp - c).astype(np.float32)
            u = (hi + y).astype(np.float32)
            c = ((u - hi).astype(np.float32) - y).astype(np.float32)
            hi = u
            amx = np.maximum(amx, lm)
        mp = float(amx.max())
        atop = abs(float(_f32(mp * L2E)) - float(aLref)) if aLref > -np.inf else 0.0
        argb = 64.0 + 25.01 if nres else 25.01 + atop
        eps = float(_f32(2.0 ** -20 + 2.0 ** -24 * LN2 * argb + 1.4e-8 * (abs(mp) + 18.0) + 8 * 2.0 ** -24
                         + 1.2e-6 * nres)) if aLref > -np.inf else 0.0
        s = float(np.sum(hi.astype(np.float64) + c.astype(np.float64))) if aLref > -np.inf else 0.0
        parts.append((float(aref), eps, s))
    return parts


def _bracket(parts):
    """The merge's bracket from the parts' (mref, eps, s), in float64."""
    ml = max((float(_f32(m * L2E)) for m, _, _ in parts if m > -np.inf), default=-np.inf)
    if ml == -np.inf:
        return -np.inf, -np.inf
    z = e = 0.0
    for m, eps, s in parts:
        if m == -np.inf:
            continue
        w = s * math.exp((float(_f32(m * L2E)) - ml) * LN2)
        z += w
        e += w * eps
    lse = ml * LN2 + math.log(z)
    half = 1.0001 * e / z + 1.3e-6 + 1e-12 * abs(lse)
    down, up = np.float32(-np.inf), np.float32(np.inf)
    lo = np.float32(lse - half)
    if float(lo) > lse - half:
        lo = np.nextafter(lo, down)
    hi = np.float32(lse + half)
    if float(hi) < lse + half:
        hi = np.nextafter(hi, up)
    return float(np.nextafter(lo, down)), float(np.nextafter(hi, up))


@pytest.mark.parametrize("sigma,shift,V,tpp", [(2.5, 0.0, 262144, 110), (2.0, 0.0, 163840, 17),
                                               (0.5, 40.0, 151936, 37), (10.0, -70.0, 65536, 5),
                                               (1.0, 900.0, 40000, 40), (30.0, 0.0, 9000, 3)])
def test_bracket_holds_the_exact_lse(sigma, shift, V, tpp):
    rng = np.random.default_rng(int(sigma * 100 + V))
    for _ in range(2):
        x = (rng.standard_normal(V).astype(np.float32) * np.float32(sigma) + np.float32(shift)).astype(np.float32)
        x[rng.choice(V, 16, replace=False)] += np.float32(3 * sigma)
        c = np.float32(O.row_lse(x))
        lo, hi = _bracket(_approx_part_stats(x, tpp))
        assert lo <= c <= hi, (lo, float(c), hi)
        # the bracket stays narrow: a few parts per million of its scale
        assert hi - lo <= 2e-5 + 4e-7 * abs(float(c)), (lo, hi)


def test_bracket_when_the_reference_moves():
    """A row that climbs 400 along the vocabulary: the part's reference
    moves up several times; the bracket still holds the exact value."""
    V = 65536
    rng = np.random.default_rng(3)
    x = (np.linspace(0.0, 400.0, V) + rng.standard_normal(V) * 2.0).astype(np.float32)
    c = np.float32(O.row_lse(x))
    parts = _approx_part_stats(x, 64)
    lo, hi = _bracket(parts)
    assert lo <= c <= hi, (lo, float(c), hi)


def test_bracket_of_a_row_of_minus_infinity():
    x = np.full(3000, -np.inf, np.float32)
    assert _bracket(_approx_part_stats(x, 2)) == (-np.inf, -np.inf)
    assert O.row_lse(x) == -np.inf
