"""The bracket around the exact log-sum-exp, restated on the CPU.

The streaming pass's approximate tile sums are emulated in numpy fp32 (the
same argument rounding, layout and addition tree; numpy's exp2 stands in for
the hardware unit, whose own error the GPU self-check bounds), the bracket
is formed as the merge forms it, and the oracle's exact log-sum-exp must lie
inside it for rows of many scales and shapes.
"""

import math

import numpy as np
import pytest

import oracle as O

L2E = np.float32(1.4426950408889634)  # fl32(log2 e)
LN2 = math.log(2.0)


def _approx_tile_sums(x: np.ndarray):
    """(m_t, s_t) per 1024-token tile, as the streaming pass computes them:
    lane L holds slots s = 0..31 of the tile at element (s // 4) * 128 +
    L * 4 + s % 4; pairs of slots in f32x2 halves, a four-level tree over
    the 16 pairs, the two halves, then a five-level butterfly over lanes."""
    V = x.shape[0]
    nt = -(-V // 1024)
    pad = np.full(nt * 1024, -np.inf, np.float32)
    pad[:V] = x
    tiles = pad.reshape(nt, 1024)
    s_idx = np.arange(32)
    lane = np.arange(32)[:, None]
    elem = (s_idx // 4) * 128 + lane * 4 + s_idx % 4          # [lane, slot]
    vals = tiles[:, elem]                                       # [nt, lane, slot]
    m = tiles.max(axis=1)
    out = np.zeros(nt, np.float32)
    for t in range(nt):
        if m[t] == -np.inf:
            continue
        mL = np.float32(m[t] * L2E)
        a = (vals[t].astype(np.float64) * np.float64(L2E) - np.float64(mL)).astype(np.float32)
        v = np.exp2(a).astype(np.float32)
        w = v.reshape(32, 16, 2)                                # [lane, pair, half]
        h = 8
        while h >= 1:
            w = (w[:, :h, :] + w[:, h:2 * h, :]).astype(np.float32)
            h //= 2
        s = (w[:, 0, 0] + w[:, 0, 1]).astype(np.float32)         # [lane]
        o = 16
        while o >= 1:
            s = (s + s[np.arange(32) ^ o]).astype(np.float32)
            o //= 2
        out[t] = s[0]
    return m, out


def _bracket(m, s):
    """The merge's bracket from (m_t, s_t), in float64 as on the GPU."""
    mx = m.max()
    if mx == -np.inf:
        return -np.inf, -np.inf
    ML = float(np.float32(mx * L2E))
    z = e = 0.0
    for mt, st in zip(m, s):
        if mt == -np.inf or st <= 0:
            continue
        w = float(st) * math.exp((float(np.float32(mt * L2E)) - ML) * LN2)
        z += w
        e += w * (3e-6 + 2.1e-8 * abs(float(mt)))
    lse = ML * LN2 + math.log(z)
    half = 1.0001 * e / z + 1.3e-6 + 1e-12 * abs(lse)
    down, up = np.float32(-np.inf), np.float32(np.inf)
    lo = np.float32(lse - half)
    if float(lo) > lse - half:
        lo = np.nextafter(lo, down)
    hi = np.float32(lse + half)
    if float(hi) < lse + half:
        hi = np.nextafter(hi, up)
    return float(np.nextafter(lo, down)), float(np.nextafter(hi, up))


@pytest.mark.parametrize("sigma,shift,V", [(2.5, 0.0, 262144), (2.0, 0.0, 163840), (0.5, 40.0, 151936),
                                           (10.0, -70.0, 65536), (1.0, 900.0, 40000), (30.0, 0.0, 9000)])
def test_bracket_holds_the_exact_lse(sigma, shift, V):
    rng = np.random.default_rng(int(sigma * 100 + V))
    for _ in range(3):
        x = (rng.standard_normal(V).astype(np.float32) * np.float32(sigma) + np.float32(shift)).astype(np.float32)
        x[rng.choice(V, 16, replace=False)] += np.float32(3 * sigma)
        c = np.float32(O.row_lse(x))
        lo, hi = _bracket(*_approx_tile_sums(x))
        assert lo <= c <= hi, (lo, float(c), hi)
        # the bracket stays narrow: a few parts per million of its scale
        assert hi - lo <= 2e-5 + 4e-7 * abs(float(c)), (lo, hi)


def test_bracket_of_a_row_of_minus_infinity():
    x = np.full(3000, -np.inf, np.float32)
    assert _bracket(*_approx_tile_sums(x)) == (-np.inf, -np.inf)
    assert O.row_lse(x) == -np.inf
