"""Decoding controls (Sampler.swift) without a GPU: the CPU restatement pinned to the reference's
own known answers (SamplerTests.swift:5-49), and the library's host-side loop detector
(plamo_repetition_period) against them and against the restatement on seeded sequences."""
import numpy as np
import pytest


def test_restatement_matches_sampler_tests(oracle):
    # SamplerTests.swift:5-8 greedy picks the first maximum
    assert oracle.sampler_select([1, 2, 2, 0], [], 1, 0) == 1
    # :10-15 the repetition penalty divides positive and multiplies negative logits
    assert oracle.sampler_select([1, 5, 4], [1], 2, 0) == 2
    assert oracle.sampler_select([-1, -5, -4], [1], 2, 0) == 0
    # :17-22 the frequency penalty compounds with the count
    assert oracle.sampler_select([0, 5, 4], [1], 1, 0, frequency=0.5) == 1
    assert oracle.sampler_select([0, 5, 4], [1, 1, 1], 1, 0, frequency=0.5) == 2
    # :24-29 n-gram blocking
    assert oracle.sampler_forbidden([0, 2, 3, 5, 2, 3], 3) == {5}
    assert oracle.sampler_select([0, 0, 0, 0, 0, 9], [0, 2, 3, 5, 2, 3], 1, 3) == 0
    # :31-38 loop detection
    assert oracle.sampler_repetition_period([7] * 24, 8) == 1
    assert oracle.sampler_repetition_period([1, 2, 3, 4] * 8, 8) == 4
    assert oracle.sampler_repetition_period([1, 2, 3, 4, 5, 6, 7, 8], 8) is None
    assert oracle.sampler_repetition_period([1, 2, 3, 4], 8) is None


def test_restatement_edge_rules(oracle):
    inf, nan = np.inf, np.nan
    assert oracle.sampler_select([nan, -inf, nan], [], 1, 0) == 0          # nothing above -inf: id 0
    assert oracle.sampler_select([nan, 1, nan, 1], [], 1, 0) == 1          # NaN never wins, first max
    assert oracle.sampler_select([-0.0, 0.0], [], 1, 0) == 0               # -0 == +0: the first one
    assert oracle.sampler_select([1, inf, inf], [], 1, 0) == 1
    assert oracle.sampler_select([3, 2], [0, 0, 9999], 1, 0, presence=1.5) == 1  # out-of-range ids ignored
    assert oracle.sampler_select([0, 0, 0, 0], [1, 1], 1, 2) == 0           # [1] -> 1 blocked
    assert oracle.sampler_forbidden([4, 4], 2) == {4}


def test_library_repetition_period(pkg, oracle):
    period = pkg.runtime.repetition_period
    assert period([7] * 24, 8) == 1
    assert period([1, 2, 3, 4] * 8, 8) == 4
    assert period([1, 2, 3, 4, 5, 6, 7, 8], 8) is None
    assert period([1, 2, 3, 4], 8) is None
    assert period([5, 6] * 20, 1) is None  # repeats < 2
    rng = np.random.default_rng(3)
    for trial in range(300):
        p = int(rng.integers(1, 40))
        block = rng.integers(0, 3, size=p).tolist()
        reps = int(rng.integers(1, 30))
        tail = (block * (reps + 1))[: p * reps + int(rng.integers(0, p))]
        toks = rng.integers(0, 3, size=int(rng.integers(0, 10))).tolist() + tail
        r = int(rng.integers(2, 10))
        assert period(toks, r) == oracle.sampler_repetition_period(toks, r), (trial, p, reps, r)
