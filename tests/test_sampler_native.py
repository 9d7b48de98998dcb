"""Sampler.sample restated in native host code vs the oracle (CPU)."""
import numpy as np
import pytest

from auratensor_b200.inference import Sampler, SamplerConfig
from oracle import ref


def test_sampler_reference_cases(kats, built_lib):
    for c in kats["sampler"]:
        t, k, p, rp, seed = c["config"]
        logits = np.array(c["logits"], dtype=np.float32)
        tok = Sampler.sample(logits, c["history"], SamplerConfig(t, k, p, rp, seed))
        assert tok in c["expect"], c["name"]
        if "first" in c:
            assert tok == c["first"]
        if c["name"] == "topPStillPicksFromAllowedSet":
            for _ in range(50):
                assert Sampler.sample(np.array(c["logits"], dtype=np.float32), None,
                                      SamplerConfig(t, k, p, rp, seed)) in c["expect"]


@pytest.mark.parametrize("seed", [1, 7, 42, 1234567])
@pytest.mark.parametrize("cfg", [(0.7, 40, 0.95, 1.0), (1.0, 5, 1.0, 1.1), (0.5, 1000, 0.9, 1.3), (1.3, 3, 0.5, 1.0)])
def test_sampler_matches_oracle(seed, cfg, built_lib):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal(2000) * 3).astype(np.float32)
    hist = rng.integers(0, 2000, size=6).tolist()
    t, k, p, rp = cfg
    a = logits.copy()
    got = Sampler.sample(a, hist, SamplerConfig(t, k, p, rp, seed))
    want = ref.sample(logits.copy(), hist, ref.SamplerConfig(t, k, p, rp, seed))
    assert got == want


def test_repetition_penalty_mutates_in_place(built_lib):
    logits = np.array([2.0, -2.0, 1.0], dtype=np.float32)
    Sampler.sample(logits, [0, 1], SamplerConfig(1.0, 1, 1.0, 2.0, 3))
    assert logits.tolist() == [1.0, -4.0, 1.0]


@pytest.mark.parametrize("seed", [3, 4, 5])
def test_sampler_special_values_match_oracle(seed, built_lib):
    """NaN (above +inf in Double.compare), infinities, signed zeros and exact
    ties, with a negative penalty flipping signs per occurrence."""
    rng = np.random.default_rng(seed)
    logits = np.round(rng.standard_normal(3000) * 2).astype(np.float32)
    idx = rng.choice(3000, size=12, replace=False)
    logits[idx[:3]] = np.nan
    logits[idx[3:5]] = np.inf
    logits[idx[5:7]] = -np.inf
    logits[idx[7:9]] = 0.0
    logits[idx[9:12]] = -0.0
    hist = rng.integers(0, 3000, size=50).tolist() + idx[7:12].tolist() * 2
    for t, k, p, rp in [(0.7, 40, 0.95, 1.0), (1.0, 1000, 1.0, -1.5), (-0.5, 7, 0.5, 1.1)]:
        a, b = logits.copy(), logits.copy()
        got = Sampler.sample(a, hist, SamplerConfig(t, k, p, rp, seed))
        want = ref.sample(b, hist, ref.SamplerConfig(t, k, p, rp, seed))
        assert got == want
        na = np.isnan(a)
        assert np.array_equal(na, np.isnan(b)) and np.array_equal(a[~na].view(np.uint32), b[~na].view(np.uint32))


def _scan_greedy(x):
    """Sampler.java's greedy loop as written: replace the best only when greater."""
    best, bs = 0, x[0]
    for i in range(1, len(x)):
        if x[i] > bs:
            bs, best = x[i], i
    return best


@pytest.mark.parametrize("n", [1, 2, 15, 16, 17, 31, 33, 64, 1000, 128256])
def test_greedy_index_matches_the_scan(n, built_lib):
    """The native greedy path (lane-wise maxima, then the first index holding
    the maximum) picks the scan's index: NaN first wins, later NaNs are
    skipped, ties and -0.0 / 0.0 keep the first index, also across the
    16-lane blocks and in the tail."""
    rng = np.random.default_rng(n)
    greedy = SamplerConfig.greedy()
    cases = [rng.standard_normal(n).astype(np.float32),
             rng.integers(-3, 3, n).astype(np.float32),          # many ties
             np.full(n, -np.inf, dtype=np.float32),
             np.zeros(n, dtype=np.float32)]
    x = rng.standard_normal(n).astype(np.float32)
    x[rng.integers(0, n, max(1, n // 7))] = np.nan               # NaNs after index 0
    cases.append(x)
    x = np.zeros(n, dtype=np.float32)
    x[::2] = -0.0                                                 # -0.0 and 0.0 are equal
    cases.append(x)
    x = rng.standard_normal(n).astype(np.float32)
    x[0] = np.nan                                                 # NaN at index 0 wins
    cases.append(x)
    x = rng.standard_normal(n).astype(np.float32)
    x[-1] = np.inf                                                # maximum in the tail
    cases.append(x)
    x = rng.standard_normal(n).astype(np.float32)
    x[rng.integers(0, n, 3)] = 50.0                               # a repeated maximum
    cases.append(x)
    for x in cases:
        want = _scan_greedy(x.tolist())
        assert Sampler.sample(x.copy(), None, greedy) == want
