"""Next-token selection for generation on CPU.

hx_sample_next_token restates greedyArgmax / sampleTopKChecked
(nicopedia_generation.h:286-395).  It must pass the reference's own sampler
tests (host_tests/nicopedia_htp_generation_test.cpp:101-196, restated) and
pick the same token as the reference's code, compiled into oracle/_ref, on
random logit rows over temperatures, top-K sizes, seeds and steps.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx


def _greedy(row):
    return hx.sample_next_token(np.asarray(row, np.float32), greedy=True)[0]


def _sample(row, temp, k, seed, step):
    return hx.sample_next_token(np.asarray(row, np.float32), step=step, greedy=False, temperature=temp, top_k=k,
                                seed=seed)[0]


def test_greedy_known_answers():
    assert _greedy([1.0, 3.0, 3.0, 2.0, 0.5, -1.0]) == 1       # first max on ties
    assert _greedy([-2.0] * 4) == 0
    assert _greedy([0.0, 0.0, 5.0]) == 2
    bpe = np.full(1024, -1.0, np.float32)
    bpe[1023] = 9.0
    assert _greedy(bpe) == 1023                                # no uint8 truncation
    assert _sample(bpe, 1.0, 1, 1, 0) == 1023


def test_sampling_known_answers():
    logits = np.array([float(b % 7 - 3) for b in range(256)], np.float32)
    greedy = _greedy(logits)
    for seed in (0, 1, 42, 0xFFFFFFFFFFFFFFFF):
        assert _sample(logits, 0.7, 1, seed, 3) == greedy      # top-K 1 is greedy
    a1 = _sample(logits, 1.0, 8, 1234, 0)
    assert a1 == _sample(logits, 1.0, 8, 1234, 0)
    assert any(_sample(logits, 1.0, 8, 1234, s) != a1 for s in range(1, 64))
    seen = {_sample(logits, 1.0, 4, 7, s) for s in range(256)}
    assert 1 <= len(seen) <= 4 and all(logits[b] >= logits[3] for b in seen)
    distinct = np.arange(256, dtype=np.float32)
    assert _sample(distinct, 1e-4, 256, 5, 0) == 255           # cold collapses to argmax
    assert logits[_sample(logits, 1e-4, 256, 5, 0)] == logits[6]


def test_sampling_audit():
    tok, audit = hx.sample_next_token(np.array([0.0, 1.0, 2.0, -1.0], np.float32), greedy=False, temperature=0.6,
                                      top_k=3, seed=42)
    assert audit["ok"] and audit["logits_finite"] and abs(audit["probability_sum"] - 1.0) < 1e-12
    with pytest.raises(ValueError):
        hx.sample_next_token(np.array([0.0, 1.0, np.nan, -1.0], np.float32), greedy=False, temperature=0.6, top_k=3)


def test_sampler_matches_the_reference(reference):
    rng = np.random.default_rng(3)
    for vocab in (7, 256, 1024):
        for trial in range(6):
            row = (rng.standard_normal(vocab) * (0.5 + trial)).astype(np.float32)
            if trial == 5:
                row = np.round(row)                             # many ties
            for temp in (0.3, 1.0, 2.0, 0.0):
                for k in (0, 1, 4, 40):
                    for seed, step in ((0, 0), (9, 3), (2**63 + 5, 17)):
                        want, ok = reference.sample_next_token(row, step, False, temp, k, seed)
                        assert ok
                        assert _sample(row, temp, k, seed, step) == want, (vocab, trial, temp, k, seed, step)
            assert _greedy(row) == reference.sample_next_token(row, greedy=True)[0]
