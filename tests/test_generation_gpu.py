"""Forward-only LM and generation on the GPU.

- hx_lm_forward_tokens (executeTinyTransformerForwardOnly): logits of every
  row against the oracle's forward, within the LM parity tolerance (1e-4
  relative per sequence); host parameters and the device state agree bit
  for bit.
- hx_lm_generate: greedy streams against an oracle-driven loop (a token may
  differ only where the oracle's top two logits lie within 1e-4); sampled
  streams equal a replay that feeds the same windows through the
  forward-only entry point and picks tokens with the reference's own
  sampler (oracle/_ref), exactly.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import rel_err
from hexatrain_b200 import data
from oracle.oracle import LmConfig as OC

TOL = 1e-4
V, T, D, F, L, H, B = 64, 16, 32, 64, 2, 4, 2


def _setup(learned=True):
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=learned)
    oc = OC.make(V, T, D, F, L, H, learned_position=learned)
    p = cfg.init_normal(12, 0.05)
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    assert rt.prepare_lm(cfg, B), rt.last_error
    assert rt.lm_state_upload(p), rt.last_error
    return cfg, oc, p, rt


def _window(history):
    w = np.zeros(T, np.uint32)
    keep = history[-T:]
    w[T - len(keep):] = keep
    return w


@pytest.mark.gpu
def test_forward_only_logits_match_oracle(oracle):
    cfg, oc, p, rt = _setup()
    toks = data.lm_tokens(5, B, T, V)[:, :T]
    got = rt.execute_tiny_transformer_forward_only_tokens(toks, p)
    assert got is not None, rt.last_error
    state = rt.execute_tiny_transformer_forward_only_tokens(toks)
    assert np.array_equal(got, state)
    for b in range(B):
        want = oracle.lm_forward_backward(oc, toks[b], toks[b], p).logits
        assert rel_err(got[b * T:(b + 1) * T], want) <= TOL
    bad = toks.copy()
    bad[0, 3] = V
    assert rt.execute_tiny_transformer_forward_only_tokens(bad) is None
    assert rt.last_error.startswith("INVALID_TINY_LM_TOKEN")
    nan = p.copy()
    nan[5] = np.nan
    assert rt.execute_tiny_transformer_forward_only_tokens(toks, nan) is None
    rt.close()


@pytest.mark.gpu
def test_greedy_generation_matches_oracle_loop(oracle):
    cfg, oc, p, rt = _setup()
    prompts = data.lm_tokens(6, B, 5, V)[:, :5]
    steps = 12
    got = rt.lm_generate(prompts, steps)
    assert got is not None, rt.last_error
    for b in range(B):
        hist = list(prompts[b])
        for s in range(steps):
            w = _window(hist)
            row = oracle.lm_forward_backward(oc, w, w, p).logits[T - 1]
            want = int(np.argmax(row))
            if int(got[b, s]) != want:
                top2 = np.sort(row)[-2:]
                assert top2[1] - top2[0] <= 1e-4, (b, s, got[b, s], want)
                break  # the streams diverge from here on
            hist.append(want)
    rt.close()


@pytest.mark.gpu
def test_sampled_generation_equals_replay_with_reference_sampler(reference):
    cfg, oc, p, rt = _setup(learned=False)
    prompts = data.lm_tokens(7, B, 20, V)[:, :20]       # longer than T: the window slides
    steps, temp, k, seed = 10, 0.8, 8, 99
    got = rt.lm_generate(prompts, steps, greedy=False, temperature=temp, top_k=k, seed=seed)
    assert got is not None, rt.last_error
    hist = [list(prompts[b]) for b in range(B)]
    for s in range(steps):
        windows = np.stack([_window(h) for h in hist])
        logits = rt.execute_tiny_transformer_forward_only_tokens(windows)
        assert logits is not None, rt.last_error
        for b in range(B):
            tok, ok = reference.sample_next_token(logits[b * T + T - 1], s, False, temp, k, seed + b)
            assert ok and tok == int(got[b, s]), (b, s)
            hist[b].append(tok)
    assert rt.lm_generate(prompts[:, :0], 1) is None
    assert rt.last_error.startswith("PROMPT_EMPTY")
    rt.close()
