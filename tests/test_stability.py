"""Momentum SGD and the training-stability modes on CPU.

The oracle's restatements and the product's host functions are held equal to
the reference's own code, compiled from its sources into oracle/_ref:
tiny_lm::momentumUpdate (tiny_language_model_cpu.cpp:123),
stabilityLearningRate / applyInitStability / validateTrainingStabilityMode
(training_stability.h:77-121) and the driver's gradientNorm
(qnn/qnn_transformer_training.cpp:920-938).  All comparisons are exact.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from hexatrain_b200 import _lib
from oracle.oracle import LmConfig as OC
from oracle.oracle import ReferenceCheckpoint, reference_checkpoint_available

DIMS = (40, 6, 8, 12, 3, 2)


def _rand(n, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


def test_momentum_oracle_equals_reference(oracle, reference):
    oc = OC.make(*DIMS)
    n = oracle.param_count(oc)
    w, g, v = _rand(n, 1), _rand(n, 2, 1e-2), _rand(n, 3, 1e-2)
    for lr, mu in ((0.01, 0.95), (0.5, 0.0), (1e-3, 0.9)):
        ow, ov = oracle.momentum(w, g, v, lr, mu)
        rw, rv = reference.momentum(oc, w, g, v, lr, mu)
        assert np.array_equal(ow, rw) and np.array_equal(ov, rv)


def test_stability_learning_rate_matches_reference(oracle, reference):
    for mode in range(7):
        for base in (1e-3, 0.003, 0.01):
            for total in (0, 100, 1000):
                for step in (1, 2, 5, 63, 64, 65, 100, 640):
                    want = reference.stability_learning_rate(mode, base, step, total)
                    assert oracle.stability_learning_rate(mode, base, step, total) == want
                    assert hx.stability_learning_rate(mode, base, step, total) == want, (mode, step, total)


def test_stability_mode_validation_matches_reference(reference):
    lib = _lib.load()
    for mode in range(10):
        got = lib.hx_stability_mode_error(mode)
        assert (got.decode() if got else "") == reference.stability_mode_error(mode), mode


@pytest.mark.parametrize("dims", [DIMS, (32, 4, 8, 16, 1, 1), (64, 8, 16, 32, 4, 2)])
def test_init_stability_matches_reference(dims, oracle, reference):
    cfg, oc = hx.LmConfig(*dims), OC.make(*dims)
    p0 = cfg.init_reference(7)
    for mode in (0, 1, 2, 3, 4, 6):
        want = reference.apply_init_stability(oc, mode, p0)
        assert np.array_equal(oracle.apply_init_stability(oc, mode, p0), want), mode
        assert np.array_equal(hx.apply_init_stability(cfg, mode, p0), want), mode
    with pytest.raises(ValueError, match="RESIDUAL_BRANCH_SCALING_UNSUPPORTED_ON_DEVICE"):
        hx.apply_init_stability(cfg, 5, p0)


@pytest.mark.skipif(not reference_checkpoint_available(), reason="reference driver codec not built")
@pytest.mark.parametrize("dims", [DIMS, (1024, 8, 16, 16, 2, 2)])
def test_gradient_norm_matches_reference(dims, oracle):
    ref = ReferenceCheckpoint()
    oc = OC.make(*dims)
    n = oracle.param_count(oc)
    for seed, scale in ((1, 1e-3), (2, 1.0), (3, 30.0)):
        g = _rand(n, seed, scale)
        norm, clip = oracle.gradient_norm(oc, g, 1.0)
        assert norm == ref.gradient_norm(oc, g)
        assert clip == np.float32(min(1.0, 1.0 / (norm + 1e-6)))
        assert oracle.gradient_norm(oc, g, 0.0)[1] == 1.0
