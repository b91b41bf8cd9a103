"""GPU parity of the tiny-Transformer LM step through the C ABI.

Tolerances: <= 1e-4 relative (tensor-wise, max|got-want|/max|want|) on the
per-step loss and on every gradient tensor of the registry; <= 1e-2 max-abs
on parameters after the stated number of optimizer steps.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import golden, rel_err
from hexatrain_b200 import data
from oracle.oracle import LmConfig as OC

pytestmark = pytest.mark.gpu
TOL = 1e-4
W_ABS = 1e-2

LM_FIXTURES = ["lm_V8_T3_D4_F8_L1_H1.npz", "lm_V32_T4_D8_F16_L2_H2.npz", "lm_V32_T4_D8_F16_L3_H8.npz",
               "lm_V8_T3_D8_F8_L3_H4.npz", "lm_V32_T4_D8_F16_L1_H1.npz", "lm_V32_T8_D16_F32_L1_H1.npz"]


def one_hot(ids, V):
    m = np.zeros((len(ids), V), np.float32)
    m[np.arange(len(ids)), ids] = 1.0
    return m


def check_grads(cfg: hx.LmConfig, got, want, tol=TOL):
    for name, off, shape in cfg.registry():
        n = int(np.prod(shape))
        w = want[off:off + n]
        if np.max(np.abs(w)) == 0:
            assert np.max(np.abs(got[off:off + n])) <= 1e-12, name
            continue
        assert rel_err(got[off:off + n], w) <= tol, (name, rel_err(got[off:off + n], w))


@pytest.mark.parametrize("name", LM_FIXTURES)
def test_lm_one_hot_execute_matches_golden(gpu_runtime, name):
    """The reference's execute signature: one-hot [T,V] input/target rows,
    flat registry parameters, learning rate 0, diagnostic outputs."""
    g = golden(name)
    V, T, D, F, L, H = (int(v) for v in g["cfg"])
    cfg = hx.LmConfig(V, T, D, F, L, H)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, 1, diagnostic_outputs=True), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    ok = rt.execute_tiny_transformer_training(one_hot(g["inputs"], V), one_hot(g["targets"], V), g["params"], 0.0, out)
    assert ok, rt.last_error
    assert abs(out.loss - float(g["loss"])) <= TOL * abs(float(g["loss"]))
    assert out.accuracy == float(g["accuracy"])
    check_grads(cfg, out.gradients, g["grads"])
    for a, b in (("logits", "logits"), ("probabilities", "probs"), ("d_logits", "dlogits"), ("output", "output")):
        assert rel_err(getattr(out, a), g[b]) <= TOL, a
    for l in range(L):
        assert rel_err(out.layer_input_gradients[l], g["layer_input_grads"][l]) <= TOL
    assert rel_err(out.head_probabilities.ravel(), g["head_probs"].ravel()) <= TOL


@pytest.mark.parametrize("name", ["lm_V1024_T64_D64_F64_L2_H4.npz", "lm_V1024_T64_D48_F48_L4_H4.npz"])
def test_lm_benchmark_shapes_match_golden(gpu_runtime, name):
    g = golden(name)
    V, T, D, F, L, H = (int(v) for v in g["cfg"])
    cfg = hx.LmConfig(V, T, D, F, L, H)
    p = cfg.init_reference(int(g["seed"]))
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, 1), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    assert rt.execute_tiny_transformer_training_tokens(g["ids"][:T], g["ids"][1:], p, out), rt.last_error
    assert abs(out.loss - float(g["loss"])) <= TOL * abs(float(g["loss"]))
    idx = g["grads__sample_idx"]
    scale = float(np.max(np.abs(g["grads__sample"])))
    assert np.max(np.abs(out.gradients[idx] - g["grads__sample"])) <= TOL * scale
    l2 = float(np.sqrt(np.sum(out.gradients.astype(np.float64) ** 2)))
    assert abs(l2 - float(g["grads__l2"])) <= TOL * float(g["grads__l2"])


@pytest.mark.parametrize("shape,B,learned,init", [
    ((1024, 64, 64, 64, 2, 4), 4, False, "reference"),   # T64 D64 F64 L2 H4
    ((1024, 64, 48, 48, 4, 4), 4, False, "reference"),   # T64 D48 F48 L4 H4
    ((1024, 64, 64, 64, 2, 4), 3, True, "normal"),       # T64 D64 L2 as benchmarked: learned positions, N(0, 0.02)
    ((96, 20, 24, 40, 3, 2), 5, True, "normal"),
])
def test_lm_batched_gradients_match_oracle(gpu_runtime, oracle, shape, B, learned, init):
    V, T, D, F, L, H = shape
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=learned)
    p = cfg.init_reference(3) if init == "reference" else cfg.init_normal(3, 0.02)
    toks = data.lm_tokens(11, B, T, V)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    assert rt.execute_tiny_transformer_training_tokens(toks[:, :T], toks[:, 1:], p, out), rt.last_error
    g, loss = oracle.lm_batch_gradients(OC.make(V, T, D, F, L, H, learned_position=learned), toks, p, threads=8)
    assert abs(out.loss - loss) <= TOL * abs(loss)
    check_grads(cfg, out.gradients, g)


def test_lm_largest_config_shape_matches_oracle(gpu_runtime, oracle):
    """V1024 T256 D256 F1024 L4 H8 with its own N(0, 0.02) init and learned
    positions, one sequence (the oracle needs ~3 s per sequence)."""
    V, T, D, F, L, H = 1024, 256, 256, 1024, 4, 8
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(20260710, 0.02)
    toks = data.lm_tokens(20260710, 1, T, V)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, 1), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    assert rt.execute_tiny_transformer_training_tokens(toks[:, :T], toks[:, 1:], p, out), rt.last_error
    s = oracle.lm_forward_backward(OC.make(V, T, D, F, L, H, learned_position=True), toks[0, :T], toks[0, 1:], p,
                                   want_all=False)
    assert abs(out.loss - s.loss) <= TOL * abs(s.loss)
    check_grads(cfg, out.gradients, s.grads)


def test_lm_train_steps_match_golden(gpu_runtime):
    """hx_lm_train_step = the reference driver's batched Adam loop
    (qnn/qnn_transformer_training.cpp:7281-7345) in one call per step."""
    g = golden("lm_train_3steps.npz")
    V, T, D, F, L, H, B = (int(v) for v in g["cfg"])
    cfg = hx.LmConfig(V, T, D, F, L, H)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B), rt.last_error
    assert rt.lm_state_upload(g["params0"]), rt.last_error
    for i, step in enumerate((1, 2, 3)):
        ok, loss = rt.lm_train_step(g["tokens"][i], step)
        assert ok, rt.last_error
        assert abs(loss - float(g["losses"][i])) <= TOL * abs(float(g["losses"][i]))
        params, m, v, _ = rt.lm_state_download()
        assert np.max(np.abs(params - g["params"][i])) <= W_ABS
    assert np.max(np.abs(m - g["m"])) <= 1e-6


def test_lm_data_parallel_split_equals_fused_step(gpu_runtime):
    """forward_backward_device + (all-reduce of a single rank) +
    optimizer_step_device gives the same state as train_step."""
    import torch
    V, T, D, F, L, H, B = 64, 16, 32, 64, 2, 4, 4
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p0 = cfg.init_normal(9, 0.02)
    toks = [data.lm_tokens(9, B, T, V, step=s) for s in range(3)]
    a = hx.Runtime()
    b = hx.Runtime()
    assert a.initialize(0) and b.initialize(0)
    for rt in (a, b):
        assert rt.prepare_lm(cfg, B) and rt.lm_state_upload(p0)
    for s in range(3):
        ok, _ = a.lm_train_step(toks[s], s + 1)
        assert ok, a.last_error
        t = torch.from_numpy(toks[s].astype(np.int32)).cuda()
        torch.cuda.synchronize()
        assert b.lm_forward_backward_device(t.data_ptr(), 1.0 / B), b.last_error
        assert b.lm_optimizer_step_device(s + 1), b.last_error
        assert b.synchronize()
    pa, ma, va, _ = a.lm_state_download()
    pb, mb, vb, _ = b.lm_state_download()
    assert np.array_equal(pa, pb) and np.array_equal(ma, mb) and np.array_equal(va, vb)
    gp, n = b.lm_grad_buffer()
    assert n == cfg.parameter_count() + 1
    a.close()
    b.close()


def test_lm_muon_steps_match_oracle(gpu_runtime, oracle):
    """The Muon configuration's optimizer split on a small model: Muon (momentum 0.95, Nesterov,
    5 NS steps, bf16 operands) on wq,wk,wv,wo,ffn_w1,ffn_w2; Adam elsewhere."""
    V, T, D, F, L, H, B = 64, 16, 48, 48, 2, 4, 4
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    oc = OC.make(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(4, 0.02)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B) and rt.lm_state_upload(p), rt.last_error
    opt = hx.OptimizerConfig(kind=1, muon_lr=0.02)
    assert rt.lm_set_optimizer(opt), rt.last_error
    w = p.copy()
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    buf = np.zeros_like(w)
    reg = cfg.registry()
    muon_names = ("wq", "wk", "wv", "wo", "ffn_w1", "ffn_w2")
    for step in (1, 2):
        toks = data.lm_tokens(4, B, T, V, step=step)
        ok, loss = rt.lm_train_step(toks, step)
        assert ok, rt.last_error
        g, ref_loss = oracle.lm_batch_gradients(oc, toks, w, threads=8)
        assert abs(loss - ref_loss) <= TOL * abs(ref_loss)
        c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
        nw = w.copy()
        for name, off, shape in reg:
            n = int(np.prod(shape))
            sl = slice(off, off + n)
            if name.split(".")[-1] in muon_names:
                wn, bn = oracle.muon(w[sl].reshape(shape), g[sl].reshape(shape), buf[sl].reshape(shape), 0.02)
                nw[sl], buf[sl] = wn.ravel(), bn.ravel()
            else:
                m[sl], v[sl], _, _, nw[sl] = oracle.adam(w[sl], g[sl], m[sl], v[sl], 1e-3, c1, c2)
        w = nw
        params, _, _, mbuf = rt.lm_state_download()
        assert np.max(np.abs(params - w)) <= W_ABS
        if step == 1:
            # after one step the momentum buffer is the gradient itself
            muon = np.zeros(w.size, bool)
            for name, off, shape in reg:
                if name.split(".")[-1] in muon_names:
                    muon[off:off + int(np.prod(shape))] = True
            assert rel_err(mbuf[muon], buf[muon]) <= TOL


def test_lm_errors_fail_closed():
    rt = hx.Runtime()
    assert rt.initialize(0)
    cfg = hx.LmConfig(16, 4, 8, 16, 1, 2)
    out = hx.TinyTransformerTrainingOutputs()
    p = cfg.init_reference(1)
    assert not rt.execute_tiny_transformer_training(np.zeros(64), np.zeros(64), p, 0.0, out)
    assert "not prepared" in rt.last_error
    assert rt.prepare_lm(cfg, 1)
    good = one_hot([0, 1, 2, 3], 16)
    assert not rt.execute_tiny_transformer_training(good, good, p, 0.003, out)
    assert "learningRate=0" in rt.last_error
    bad = good.copy()
    bad[1, 5] = 0.5
    assert not rt.execute_tiny_transformer_training(bad, good, p, 0.0, out)
    assert rt.last_error.startswith("INVALID_TINY_LM_ONE_HOT")
    assert not rt.execute_tiny_transformer_training_tokens(np.array([0, 1, 2, 16]), np.array([1, 2, 3, 4]), p, out)
    assert rt.last_error.startswith("INVALID_TINY_LM_TOKEN")
    assert not rt.execute_tiny_transformer_training(good, good, p[:-1], 0.0, out)
    assert "buffer schema" in rt.last_error
    assert not rt.prepare_lm(hx.LmConfig(16, 4, 10, 16, 1, 2), 1)   # head dim 5
    assert rt.last_error.startswith("UNSUPPORTED_HEAD_DIMENSION")
    assert not rt.prepare_lm(hx.LmConfig(16, 4, 9, 16, 1, 2), 1)
    assert rt.last_error.startswith("APP_CONFIGURATION_VALIDATION")
    ok, _ = rt.lm_train_step(np.zeros((1, 5), np.uint32), 1)
    assert not ok
    rt.close()


@pytest.mark.parametrize("backend", [1, 2])
def test_lm_gemm_engines_agree_with_oracle(oracle, backend):
    V, T, D, F, L, H, B = 256, 64, 128, 256, 2, 4, 3
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(8, 0.02)
    toks = data.lm_tokens(8, B, T, V)
    rt = hx.Runtime()
    assert rt.initialize(0) and rt.set_gemm_backend(backend)
    assert rt.prepare_lm(cfg, B), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    assert rt.execute_tiny_transformer_training_tokens(toks[:, :T], toks[:, 1:], p, out), rt.last_error
    g, loss = oracle.lm_batch_gradients(OC.make(V, T, D, F, L, H, learned_position=True), toks, p, threads=8)
    assert abs(out.loss - loss) <= TOL * abs(loss)
    check_grads(cfg, out.gradients, g)
    rt.close()


def test_gradient_buckets_and_their_events(gpu_runtime):
    """hx_lm_grad_buckets tiles the [P+1] buffer in completion order; with
    bucket events on, a stream that waited for every bucket sees the same
    gradients as the plain device step, also on graph replays (the events
    are external nodes of the captured backward)."""
    import torch
    V, T, D, F, L, H, B = 64, 16, 32, 64, 2, 4, 4
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p0 = cfg.init_normal(12, 0.02)
    P = cfg.parameter_count()
    ref = hx.Runtime()
    assert ref.initialize(0) and ref.prepare_lm(cfg, B) and ref.lm_state_upload(p0)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B) and rt.lm_state_upload(p0), rt.last_error
    buckets = rt.lm_grad_buckets()
    assert len(buckets) == L + 2
    reg = {n: (o, int(np.prod(sh))) for n, o, sh in cfg.registry()}
    assert buckets[0] == (reg["output_projection"][0], D * V + 1)
    assert buckets[1][0] == reg["layer_001.norm1_gamma"][0] and buckets[-1] == (0, reg["layer_000.norm1_gamma"][0])
    assert sum(n for _, n in buckets) == P + 1
    assert not rt.lm_bucket_wait(0, 0) and "not enabled" in rt.last_error
    assert rt.lm_enable_bucket_events(True), rt.last_error
    comm = torch.cuda.Stream()
    tok = torch.empty((B, T + 1), dtype=torch.int32, device="cuda")
    for step in range(3):
        toks = data.lm_tokens(12, B, T, V, step=step)
        tok.copy_(torch.from_numpy(toks.astype(np.int32)))
        torch.cuda.synchronize()
        for r in (rt, ref):
            assert r.lm_forward_backward_device(tok.data_ptr(), 1.0 / B), r.last_error
        gp, n = rt.lm_grad_buffer()
        for i in range(len(buckets)):
            assert rt.lm_bucket_wait(i, comm.cuda_stream), rt.last_error
        comm.synchronize()  # returns once every bucket's event has fired
        assert rt.synchronize() and ref.synchronize()
        from hexatrain_b200.parallel import _device_view
        got = _device_view(gp, n).cpu().numpy()
        rp, rn = ref.lm_grad_buffer()
        want = _device_view(rp, rn).cpu().numpy()
        assert np.array_equal(got, want), step
        for r in (rt, ref):
            assert r.lm_optimizer_step_device(step + 1), r.last_error
    assert rt.lm_enable_bucket_events(False)
    ref.close()
