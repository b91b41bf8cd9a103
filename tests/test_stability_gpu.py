"""Momentum SGD and the step-side stability modes on the GPU, against the
oracle (which tests/test_stability.py holds equal to the reference).

- hx_momentum_execute: the reference's momentum graph
  (qnn/qnn_runtime_transformer.inc:799-925), elementwise, bit-exact.
- LM steps with HX_OPT_MOMENTUM: forward/backward + momentumUpdate.
- LM steps with WARMUP64 and the global-norm clip at 1 (GRADIENT_CLIP_1):
  the scheduled learning rate, gradientNorm and the clip scale applied as
  Adam's gradient-scale input (qnn_transformer_training.cpp:2432-2445).
Tolerances are those of the other LM parity tests: loss within 1e-4
relative, weights within 1e-2 max-abs after the steps.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import rel_err
from hexatrain_b200 import _lib, data
from oracle.oracle import LmConfig as OC

TOL = 1e-4
W_ABS = 1e-2


@pytest.mark.gpu
def test_momentum_optimizer_matches_oracle_bit_exact(gpu_runtime, oracle):
    rt = gpu_runtime
    n = 100003
    rng = np.random.default_rng(5)
    w, g, v = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    assert rt.prepare_momentum_optimizer(n), rt.last_error
    out = hx.MomentumOptimizerOutputs()
    for lr, mu in ((0.01, 0.95), (0.5, 0.0)):
        assert rt.execute_momentum_optimizer(w, g, v, lr, mu, out), rt.last_error
        ow, ov = oracle.momentum(w, g, v, lr, mu)
        assert np.array_equal(out.weight_next, ow) and np.array_equal(out.velocity_next, ov)
    assert not rt.execute_momentum_optimizer(w[:-1], g, v, 0.01, 0.9, out)
    assert rt.last_error == "momentum optimizer buffer size or scalar"
    assert not rt.execute_momentum_optimizer(w, g, v, float("nan"), 0.9, out)


def _lm(cfg, B, opt=None):
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    assert rt.prepare_lm(cfg, B), rt.last_error
    if opt is not None:
        assert rt.lm_set_optimizer(opt), rt.last_error
    return rt


@pytest.mark.gpu
def test_lm_momentum_steps_match_oracle(oracle):
    V, T, D, F, L, H, B = 64, 16, 32, 64, 2, 4, 4
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    oc = OC.make(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(8, 0.02)
    rt = _lm(cfg, B, hx.OptimizerConfig(kind=_lib.HX_OPT_MOMENTUM, momentum_lr=0.05, momentum=0.9))
    assert rt.lm_state_upload(p), rt.last_error
    w, vel = p.copy(), np.zeros_like(p)
    for step in (1, 2, 3):
        toks = data.lm_tokens(8, B, T, V, step=step)
        ok, loss = rt.lm_train_step(toks, step)
        assert ok, rt.last_error
        g, ref_loss = oracle.lm_batch_gradients(oc, toks, w, threads=8)
        assert abs(loss - ref_loss) <= TOL * abs(ref_loss)
        w, vel = oracle.momentum(w, g, vel, 0.05, 0.9)
    params, _, _, velocity = rt.lm_state_download()
    assert np.max(np.abs(params - w)) <= W_ABS
    assert rel_err(velocity, vel) <= 1e-3
    rt.close()


def _clip_run(oracle, cfg, oc, B, p, mode, threshold, seed):
    """Three Adam steps with the clip on the GPU and in the oracle; returns
    how many steps the clip scaled."""
    rt = _lm(cfg, B)
    assert rt.lm_set_stability(mode, 100, threshold), rt.last_error
    assert rt.lm_state_upload(p), rt.last_error
    thr = 1.0 if mode == _lib.HX_STABILITY_GRADIENT_CLIP_1 else threshold
    w, m, v = p.copy(), np.zeros_like(p), np.zeros_like(p)
    clipped = 0
    for step in (1, 2, 3):
        toks = data.lm_tokens(seed, B, cfg.tokens, cfg.vocabulary_size, step=step)
        ok, loss = rt.lm_train_step(toks, step)
        assert ok, rt.last_error
        g, ref_loss = oracle.lm_batch_gradients(oc, toks, w, threads=8)
        assert abs(loss - ref_loss) <= TOL * abs(ref_loss)
        norm, clip = oracle.gradient_norm(oc, g, thr)
        gpu_norm, gpu_clip = rt.lm_last_gradient_norm()
        assert abs(gpu_norm - norm) <= TOL * norm and abs(gpu_clip - clip) <= TOL * clip
        clipped += clip < 1.0
        c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
        m, v, _, _, w = oracle.adam(w, (g * np.float32(clip)).astype(np.float32), m, v, 1e-3, c1, c2)
    assert np.max(np.abs(rt.lm_state_download()[0] - w)) <= W_ABS
    rt.close()
    return clipped


@pytest.mark.gpu
def test_lm_warmup_and_gradient_clip_match_oracle(oracle):
    V, T, D, F, L, H, B = 64, 16, 32, 64, 2, 4, 4
    cfg = hx.LmConfig(V, T, D, F, L, H)
    oc = OC.make(V, T, D, F, L, H)
    p = cfg.init_reference(3)
    # GRADIENT_CLIP_1 (threshold fixed at 1), then a threshold at half the
    # first step's norm so that the clip certainly scales.
    _clip_run(oracle, cfg, oc, B, p, _lib.HX_STABILITY_GRADIENT_CLIP_1, 0.0, 3)
    g1, _ = oracle.lm_batch_gradients(oc, data.lm_tokens(3, B, T, V, step=1), p, threads=8)
    half = 0.5 * oracle.gradient_norm(oc, g1)[0]
    assert _clip_run(oracle, cfg, oc, B, p, _lib.HX_STABILITY_LEGACY, half, 3) >= 1

    # WARMUP64: the step's learning rate is lr * step / 64
    rt = _lm(cfg, B)
    assert rt.lm_set_stability(_lib.HX_STABILITY_WARMUP64, 100), rt.last_error
    assert rt.lm_state_upload(p), rt.last_error
    w, m, v = p.copy(), np.zeros_like(p), np.zeros_like(p)
    for step in (1, 2):
        toks = data.lm_tokens(4, B, T, V, step=step)
        assert rt.lm_train_step(toks, step)[0], rt.last_error
        g, _ = oracle.lm_batch_gradients(oc, toks, w, threads=8)
        lr = oracle.stability_learning_rate(1, 1e-3, step, 100)
        c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
        m, v, _, _, w = oracle.adam(w, g, m, v, lr, c1, c2)
    assert np.max(np.abs(rt.lm_state_download()[0] - w)) <= W_ABS
    rt.close()


@pytest.mark.gpu
def test_stability_settings_fail_closed():
    cfg = hx.LmConfig(32, 8, 16, 32, 1, 2)
    rt = _lm(cfg, 2)
    assert not rt.lm_set_stability(_lib.HX_STABILITY_RESIDUAL_BRANCH_SCALING)
    assert rt.last_error == "RESIDUAL_BRANCH_SCALING_UNSUPPORTED_ON_DEVICE"
    assert not rt.lm_set_stability(9)
    assert rt.last_error == "UNKNOWN_TRAINING_STABILITY_MODE"
    assert not rt.lm_set_stability(0, 0, -1.0)
    assert rt.lm_set_optimizer(hx.OptimizerConfig(kind=_lib.HX_OPT_MOMENTUM)), rt.last_error
    assert not rt.lm_set_stability(_lib.HX_STABILITY_GRADIENT_CLIP_1)
    assert "needs the Adam optimizer" in rt.last_error
    with pytest.raises(RuntimeError):
        rt.lm_last_gradient_norm()
    rt.close()
