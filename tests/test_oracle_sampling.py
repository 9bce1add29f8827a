"""The sampling restatements on the CPU.

The kernel restatement (oracle.sampling_ref.sample_like_kernel) must select
the nucleus LogitsProcessor selects (candle.rs:737-763 with
candle-transformers 0.11.0's sample_topp) and draw from the distribution it
draws from.  Seeds are fixed, so every statistic here is deterministic.
"""
import numpy as np
import pytest
from scipy.stats import chi2

from oracle.sampling_ref import candle_probs, greedy, kept_mask, sample_like_kernel


def _near_edge(x, t, p, tol=1e-6):
    """True when candle's f32 running sum passes top_p within tol of a token
    boundary: there fixed-point and f32 sums may legitimately disagree."""
    prs = candle_probs(x, t, None)
    cum = np.cumsum(np.sort(prs)[::-1].astype(np.float64))
    return bool(np.any(np.abs(cum - float(np.float32(p))) < tol))


def test_nucleus_matches_candle_on_random_rows():
    rng = np.random.default_rng(11)
    mism = 0
    for _ in range(300):
        v = int(rng.choice([7, 50, 1000, 5000]))
        x = (rng.standard_normal(v) * rng.uniform(0.5, 4)).astype(np.float32)
        t = float(rng.uniform(0.2, 2.0))
        p = float(rng.choice([0.1, 0.5, 0.8, 0.9, 0.95, 0.99]))
        a = kept_mask(x, t, p)
        b = candle_probs(x, t, p) > 0
        if not np.array_equal(a, b):
            assert _near_edge(x, t, p), (v, t, p)
            mism += 1
    assert mism <= 3


def test_ties_at_the_edge_keep_index_order():
    x = np.array([0.0, 2.0, 1.0, 1.0, 1.0, 1.0, -1.0], np.float32)
    # p(2.0) ~ 0.39, each 1.0 ~ 0.14: 0.6 needs the top token and two of the ties
    for p in (0.45, 0.6, 0.75):
        a = kept_mask(x, 1.0, p)
        b = candle_probs(x, 1.0, p) > 0
        assert np.array_equal(a, b), (p, a, b)
    a = kept_mask(x, 1.0, 0.6)
    assert a.tolist() == [False, True, True, True, False, False, False]


def test_greedy_threshold():
    assert greedy(0.0) and greedy(5e-8) and greedy(-1.0) and greedy(float("nan"))
    assert not greedy(1e-7 * 1.01) and not greedy(0.7)
    assert sample_like_kernel(np.zeros(4, np.float32), 0.0, None, 1) is None


@pytest.mark.parametrize("t,p", [(1.0, None), (0.7, 0.9), (1.5, 0.5), (0.3, 0.95)])
def test_draws_follow_candle_distribution(t, p):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(40) * 2).astype(np.float32)
    n = 20000
    counts = np.bincount([sample_like_kernel(x, t, p, s) for s in range(n)], minlength=40)
    q = candle_probs(x, t, p)
    q = q / q.sum()
    nz = q > 0
    assert counts[~nz].sum() == 0
    stat = float(((counts[nz] - n * q[nz]) ** 2 / (n * q[nz])).sum())
    assert stat < chi2.ppf(0.999, int(nz.sum()) - 1), stat
