"""The oracle's own building blocks: known-answer vectors and accuracy bounds."""

import math

import numpy as np
import pytest

import oracle as O


def test_philox_known_answers():
    # Random123 known-answer vectors for philox4x32-10
    assert O.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert O.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert O.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == [
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_expf_within_one_ulp():
    xs = np.linspace(-87.0, 0.0, 4001).astype(np.float32)
    worst = 0.0
    for x in xs:
        e = O.expf(float(x))
        r = math.exp(float(x))
        worst = max(worst, abs(e - r) / r)
    assert worst < 2 ** -23, worst
    assert O.expf(-88.0) == 0.0 and O.expf(float("-inf")) == 0.0 and O.expf(float("nan")) == 0.0
    assert O.expf(0.0) == 1.0


def test_exp64_log64_accuracy():
    for x in np.linspace(-700.0, 0.0, 3001):
        assert abs(O.exp64(float(x)) - math.exp(float(x))) <= 4e-16 * math.exp(float(x))
    for z in np.exp(np.linspace(-300, 300, 3001)):
        r = math.log(float(z))
        assert abs(O.log64(float(z)) - r) <= 4e-16 * max(1.0, abs(r))


def test_q52_definition():
    assert O.q52(0.0) == 1 << 52
    assert O.q52(-38.0) == 0 and O.q52(-1e30) == 0 and O.q52(float("-inf")) == 0 and O.q52(float("nan")) == 0
    # exactly floor(expf(d) * 2^52)
    for d in np.linspace(-37.0, 0.0, 513).astype(np.float32):
        e = np.float32(O.expf(float(d)))
        assert O.q52(float(d)) == int(np.float64(e) * 2.0 ** 52)


def test_gumbel_from_word_range():
    g0 = O.gumbel_from_word(0)
    g1 = O.gumbel_from_word(0xFFFFFFFF)
    assert -3.2 < g0 < -3.0 and 22.5 < g1 < 23.0
    # monotone in the word
    ws = [0, 1, 1 << 20, 1 << 31, (1 << 32) - 2, (1 << 32) - 1]
    gs = [O.gumbel_from_word(w) for w in ws]
    assert gs == sorted(gs)


def test_window_start_is_python_slicing():
    for H in range(0, 9):
        toks = list(range(H))
        for ctx in range(-10, 11):
            assert toks[O.window_start(H, ctx):] == toks[-ctx:], (H, ctx)


def test_row_lse_close_to_float64():
    rng = np.random.default_rng(0)
    for V in (1, 7, 1024, 1025, 5000, 151936):
        x = (rng.standard_normal(V) * 3).astype(np.float32)
        c = O.row_lse(x)
        ref = float(np.log(np.sum(np.exp(x.astype(np.float64) - x.max()))) + x.max())
        assert abs(c - ref) <= 2 * np.spacing(np.float32(abs(ref))) + 1e-6, (V, c, ref)
    assert O.row_lse(np.full(10, -np.inf, dtype=np.float32)) == -np.inf


def test_tile_order_is_the_definition():
    # splitting the same values into tiles differently changes only rounding
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(4096) * 2).astype(np.float32)
    m, s = O.tile_stats(x)
    assert len(m) == 4 and all(s[i] >= (1 << 52) for i in range(4))


@pytest.mark.parametrize("V", [100, 3000])
def test_full_draw_is_the_softmax(V):
    """The whole-vocabulary draw follows softmax(x / temp) (chi-square check)."""
    rng = np.random.default_rng(V)
    x = (rng.standard_normal((1, V)) * 1.5).astype(np.float32)
    x[0, 5] += 4.0
    n = 4000
    uni = rng.random((n, 2))
    toks = O.sample(np.repeat(x, n, axis=0), O.Sampler(temp=0.8), uniform=uni)["tokens"]
    p = np.exp((x[0].astype(np.float64) / 0.8) - np.max(x[0] / 0.8))
    p /= p.sum()
    top = np.argsort(-p)[:8]
    obs = np.array([(toks == t).sum() for t in top], dtype=np.float64)
    exp = n * p[top]
    chi2 = float(((obs - exp) ** 2 / exp).sum())
    assert chi2 < 40.0, (chi2, obs, exp)


def test_expf_shift_is_the_scalar_expf():
    import numpy as np
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 20, [-np.inf, 0.0]]).astype(np.float32)
    c = np.float32(1.25)
    got = O.expf_shift(x, c)
    want = np.array([O.expf(float(np.float32(v - c))) for v in x], dtype=np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
