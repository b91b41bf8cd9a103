"""Canonical resume on the GPU through hx_lm_checkpoint_save / _resume.

The reference's resume contract (host_tests/nicopedia_resume_test.cpp:1-17):
a run split at step k -- train 1..k, write the checkpoint, resume in a fresh
runtime, train k+1..N with the global step driving the Adam bias
corrections and the data order -- is bit-identical to one run 1..N.  A V1
file (no Adam moments) and a step mismatch fail closed.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from hexatrain_b200 import checkpoint as ck
from hexatrain_b200 import data

HASH = "sha256:" + "89abcdef01234567" * 4


def _runtime(cfg, B):
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    assert rt.prepare_lm(cfg, B), rt.last_error
    return rt


def _train(rt, cfg, B, first, last):
    for s in range(first, last + 1):
        ok, loss = rt.lm_train_step(data.lm_tokens(31, B, cfg.tokens, cfg.vocabulary_size, step=s - 1), s)
        assert ok and np.isfinite(loss), rt.last_error


@pytest.mark.gpu
def test_split_run_resumes_bit_exact(tmp_path):
    V, T, D, F, L, H, B = 64, 16, 32, 64, 2, 4, 4
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p0 = cfg.init_normal(21, 0.02)
    path = str(tmp_path / ck.checkpoint_name(21, L, T, D, F, 3))

    straight = _runtime(cfg, B)
    assert straight.lm_state_upload(p0), straight.last_error
    _train(straight, cfg, B, 1, 6)
    want = straight.lm_state_download()[:3]
    straight.close()

    first = _runtime(cfg, B)
    assert first.lm_state_upload(p0), first.last_error
    _train(first, cfg, B, 1, 3)
    assert first.lm_checkpoint_save(path, 21, 3), first.last_error
    at3 = first.lm_state_download()[:3]
    first.close()

    info, cp, cm, cv = ck.decode(cfg, open(path, "rb").read(), 21)
    assert info.step == 3 and info.has_adam and info.finite
    assert np.array_equal(cp, at3[0]) and np.array_equal(cm, at3[1]) and np.array_equal(cv, at3[2])

    second = _runtime(cfg, B)
    got = second.lm_checkpoint_resume(path, 21, 3)
    assert got is not None and got.step == 3, second.last_error
    _train(second, cfg, B, 4, 6)
    have = second.lm_state_download()[:3]
    second.close()
    for name, a, b in zip(("params", "adam_m", "adam_v"), have, want):
        assert np.array_equal(a, b), name


@pytest.mark.gpu
def test_reference_mode_file_is_read_by_the_reference_loader(tmp_path):
    from oracle.oracle import LmConfig as OC
    from oracle.oracle import ReferenceCheckpoint, reference_checkpoint_available
    if not reference_checkpoint_available():
        pytest.skip("reference checkpoint codec not built")
    V, T, D, F, L, H, B = 1024, 16, 32, 32, 1, 2, 2
    cfg = hx.LmConfig(V, T, D, F, L, H)
    rt = _runtime(cfg, B)
    assert rt.lm_state_upload(cfg.init_reference(5)), rt.last_error
    _train(rt, cfg, B, 1, 2)
    path = str(tmp_path / "v3.ckpt")
    assert not rt.lm_checkpoint_save(path, 5, 2)            # vocabulary 1024 needs a tokenizer identity
    assert "NPRT_CKPT_WRITE_REFUSED" in rt.last_error
    assert rt.lm_checkpoint_save(path, 5, 2, "byte_bpe", HASH), rt.last_error
    p, m, v, _ = rt.lm_state_download()
    rt.close()
    ok, err, info, rp, rm, rv = ReferenceCheckpoint().load(path, OC.make(V, T, D, F, L, H), 5, p.size, HASH)
    assert ok, err
    assert info["version"] == 3 and info["step"] == 2 and info["has_adam"]
    assert np.array_equal(rp, p) and np.array_equal(rm, m) and np.array_equal(rv, v)


@pytest.mark.gpu
def test_resume_fails_closed(tmp_path):
    V, T, D, F, L, H, B = 64, 16, 32, 64, 1, 4, 2
    cfg = hx.LmConfig(V, T, D, F, L, H)
    rt = _runtime(cfg, B)
    assert rt.lm_state_upload(cfg.init_normal(2, 0.02)), rt.last_error
    _train(rt, cfg, B, 1, 2)
    path = str(tmp_path / "a.ckpt")
    assert rt.lm_checkpoint_save(path, 9, 2), rt.last_error
    assert rt.lm_checkpoint_resume(path, 9, 3) is None
    assert rt.last_error.startswith("RESUME_CHECKPOINT_IDENTITY")
    assert rt.lm_checkpoint_resume(path, 8, 2) is None
    assert rt.last_error == "RESUME_CHECKPOINT_DECODE: NPRT_CKPT_SEED_MISMATCH"
    raw = open(path, "rb").read()
    v1 = b"NPRTCKPTV1\n" + raw[11:43 + (len(raw) - 43) // 3]
    open(path, "wb").write(v1)
    assert rt.lm_checkpoint_resume(path, 9, 2) is None
    assert rt.last_error.startswith("RESUME_ADAM_STATE_MISSING")
    assert rt.lm_set_optimizer(hx.OptimizerConfig(kind=1)), rt.last_error
    assert not rt.lm_checkpoint_save(str(tmp_path / "muon.ckpt"), 9, 2)
    assert "Adam moments only" in rt.last_error
    rt.close()
