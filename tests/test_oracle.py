"""Pins the oracle (oracle/hx_oracle.c) before any parity test trusts it.

1. The reference's own known-answer tests
   (host_tests/cpu_reference_training_test.cpp:18-61) on the oracle.
2. Value-for-value equality with the committed golden fixtures, which
   tests/golden/make_golden.py produced from the reference's compiled CPU code.
3. Value-for-value equality with the live reference build (oracle/_ref), when
   present, on fresh random cases.
4. Finite-difference gradient checks as the reference runs them
   (:63-70, :82-88, :265-310), including the learned-position extension.
5. Properties of the Muon restatement (no reference counterpart).
"""
import numpy as np
import pytest

from conftest import golden, rel_err
from oracle.oracle import LmConfig


# -- 1. reference KATs -------------------------------------------------------------

def test_matmul_kat(oracle):
    # cpu_reference_training_test.cpp:18-31
    x = np.array([[1, 2], [3, 4]], np.float32)
    w = np.array([[0.5, -1.0], [2.0, 0.25]], np.float32)
    np.testing.assert_allclose(oracle.matmul(x, w), [[4.5, -0.5], [9.5, -2.0]], atol=1e-5)


def test_loss_gradients_sgd_kat(oracle):
    # cpu_reference_training_test.cpp:33-61
    x = np.array([[1, 2], [3, 4]], np.float32)
    w = np.array([[0.5, -1.0], [2.0, 0.25]], np.float32)
    t = np.array([[4.0, 0.0], [10.0, -1.0]], np.float32)
    loss, pred, err, dp, dw, dx = oracle.linear_forward_backward(x, t, w)
    assert abs(loss - 0.4375) <= 1e-5
    assert abs(dp[0, 0] - 0.25) <= 1e-5 and abs(dp[1, 1] + 0.5) <= 1e-5
    np.testing.assert_allclose(dw, [[-0.5, -1.75], [-0.5, -2.5]], atol=1e-5)
    np.testing.assert_allclose(dx, [[0.375, 0.4375], [0.375, -0.625]], atol=1e-5)
    np.testing.assert_allclose(oracle.sgd(w, dw, 0.1), [[0.55, -0.825], [2.05, 0.5]], atol=1e-5)


def test_mlp_micro_vectors(oracle):
    # MSE / dP / SGD micro check of the reference driver (qnn/qnn_mlp_training.cpp:547-598)
    p = np.array([0.25, -0.5, 0.75, 1.0, -1.25, 1.5], np.float32)
    y = np.array([-0.1, -0.2, 0.3, 0.4, -0.5, 0.6], np.float32)
    w = np.array([0.2, -0.3, 0.4, -0.5, 0.6, -0.7], np.float32)
    dw = np.array([-0.11, 0.12, -0.13, 0.14, -0.15, 0.16], np.float32)
    e = (p - y).astype(np.float64)
    assert abs(oracle.mse(p, y) - float(np.mean(e * e))) < 1e-7
    np.testing.assert_allclose(oracle.sgd(w, dw, 0.125), w - np.float32(0.125) * dw, atol=0)


# -- 2. golden fixtures ------------------------------------------------------------

MLP_FIXTURES = ["mlp_2x4x5x3.npz", "mlp_5x7x3x2.npz", "mlp_8x128x128x64.npz"]
LM_FIXTURES = ["lm_V8_T3_D4_F8_L1_H1.npz", "lm_V32_T4_D8_F16_L2_H2.npz", "lm_V32_T4_D8_F16_L3_H8.npz",
               "lm_V8_T3_D8_F8_L3_H4.npz", "lm_V32_T4_D8_F16_L1_H1.npz", "lm_V32_T8_D16_F32_L1_H1.npz"]


@pytest.mark.parametrize("name", MLP_FIXTURES)
def test_oracle_mlp_equals_golden(oracle, name):
    g = golden(name)
    s = oracle.mlp_step(g["x"], g["y"], g["w1"], g["w2"], float(g["lr"]))
    assert s.loss == g["loss"]
    for k in ("w1_next", "w2_next", "z1", "h", "p", "e", "dp", "dw2", "dh", "mask", "dz1", "dw1"):
        assert np.array_equal(getattr(s, k), g[k]), k


def test_oracle_mlp_trajectory_equals_golden(oracle):
    g = golden("mlp_trajectory_8x128x128x64.npz")
    X, Y, w1, w2, lr, B = g["X"], g["Y"], g["w1_init"], g["w2_init"], float(g["lr"]), int(g["batch"])
    for st, want in enumerate(g["losses"]):
        rows = (st * B + np.arange(B)) % X.shape[0]
        s = oracle.mlp_step(X[rows], Y[rows], w1, w2, lr)
        assert s.loss == want
        w1, w2 = s.w1_next, s.w2_next
    assert np.array_equal(w1, g["w1_final"]) and np.array_equal(w2, g["w2_final"])


@pytest.mark.parametrize("name", LM_FIXTURES)
def test_oracle_lm_equals_golden(oracle, name):
    g = golden(name)
    cfg = LmConfig.make(*[int(v) for v in g["cfg"]])
    s = oracle.lm_forward_backward(cfg, g["inputs"], g["targets"], g["params"])
    assert s.loss == g["loss"] and s.accuracy == g["accuracy"]
    for k in ("grads", "logits", "probs", "dlogits", "output", "layer_input_grads"):
        assert np.array_equal(getattr(s, k), g[k]), k
    assert np.array_equal(s.head_probs.ravel(), g["head_probs"].ravel())


@pytest.mark.parametrize("name", ["lm_V1024_T64_D64_F64_L2_H4.npz", "lm_V1024_T64_D48_F48_L4_H4.npz"])
def test_oracle_lm_benchmark_shapes_equal_golden(oracle, name):
    import hexatrain_b200 as hx
    g = golden(name)
    V, T, D, F, L, H = (int(v) for v in g["cfg"])
    params = hx.LmConfig(V, T, D, F, L, H).init_reference(int(g["seed"]))
    assert params[g["params__sample_idx"]].tolist() == g["params__sample"].tolist()
    s = oracle.lm_forward_backward(LmConfig.make(V, T, D, F, L, H), g["ids"][:T], g["ids"][1:], params)
    assert s.loss == g["loss"]
    assert np.array_equal(s.grads[g["grads__sample_idx"]], g["grads__sample"])
    assert float(s.grads.astype(np.float64).sum()) == float(g["grads__sum"])


def test_oracle_adam_equals_golden(oracle):
    g = golden("adam_n208.npz")
    mn, vn, mh, vh, wn = oracle.adam(g["w"], g["g"], g["m"], g["v"], float(g["lr"]), float(g["c1"]), float(g["c2"]))
    for k, a in (("m_next", mn), ("v_next", vn), ("m_hat", mh), ("v_hat", vh), ("w_next", wn)):
        assert np.array_equal(a, g[k]), k


def test_oracle_batched_train_steps_equal_golden(oracle):
    """Driver loop of qnn/qnn_transformer_training.cpp:7295-7345 restated:
    batch gradients (grad*(1/B) accumulated in order) + Adam."""
    g = golden("lm_train_3steps.npz")
    V, T, D, F, L, H, B = (int(v) for v in g["cfg"])
    cfg = LmConfig.make(V, T, D, F, L, H)
    p = g["params0"].copy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    for i, step in enumerate((1, 2, 3)):
        grads, loss = oracle.lm_batch_gradients(cfg, g["tokens"][i], p)
        assert loss == g["losses"][i]
        c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
        m, v, _, _, p = oracle.adam(p, grads, m, v, 1e-3, c1, c2)
        assert np.array_equal(p, g["params"][i])
    assert np.array_equal(m, g["m"]) and np.array_equal(v, g["v"])


# -- 3. live reference --------------------------------------------------------------

@pytest.mark.parametrize("shape", [(3, 9, 4, 6), (16, 64, 32, 8)])
def test_oracle_mlp_equals_live_reference(oracle, reference, shape):
    B, I, H, O = shape
    rng = np.random.default_rng(B * 1000 + I)
    x, y = rng.uniform(-1, 1, (B, I)).astype(np.float32), rng.uniform(-1, 1, (B, O)).astype(np.float32)
    w1, w2 = rng.normal(0, 0.3, (I, H)).astype(np.float32), rng.normal(0, 0.3, (H, O)).astype(np.float32)
    a, b = oracle.mlp_step(x, y, w1, w2, 0.05), reference.mlp_step(x, y, w1, w2, 0.05)
    assert a.loss == b.loss
    for k in ("w1_next", "w2_next", "dw1", "dw2", "dh", "dz1", "mask"):
        assert np.array_equal(getattr(a, k), getattr(b, k)), k


@pytest.mark.parametrize("cfg", [(16, 5, 12, 20, 2, 3), (50, 7, 16, 8, 2, 1), (64, 12, 24, 40, 3, 6)])
def test_oracle_lm_equals_live_reference(oracle, reference, cfg):
    V, T, D, F, L, H = cfg
    c = LmConfig.make(V, T, D, F, L, H)
    p = reference.initial_parameters(c, 11)
    rng = np.random.default_rng(V)
    ids = rng.integers(0, V, T + 1).astype(np.uint32)
    a = oracle.lm_forward_backward(c, ids[:T], ids[1:], p)
    b = reference.lm_forward_backward(c, ids[:T], ids[1:], p)
    assert a.loss == b.loss and a.accuracy == b.accuracy
    for k in ("grads", "logits", "probs", "dlogits", "output", "layer_input_grads", "head_probs"):
        assert np.array_equal(getattr(a, k), getattr(b, k)), k


def test_reference_own_gradient_check_passes(reference):
    ok, max_abs, _ = reference.gradient_check()
    assert ok and max_abs <= 2e-3


# -- 4. finite differences ------------------------------------------------------------

def _fd(loss_fn, params, idx, eps=1e-3):
    p = params.copy()
    p[idx] += eps
    plus = loss_fn(p)
    p[idx] -= 2 * eps
    minus = loss_fn(p)
    return (plus - minus) / (2 * eps)


@pytest.mark.parametrize("learned", [False, True])
def test_oracle_lm_finite_differences(oracle, learned):
    # host_tests/cpu_reference_training_test.cpp:265-310: V8 T3 D8 F8 L3 H4,
    # |analytic - numeric| <= 3e-3 (float losses, eps 1e-3)
    import hexatrain_b200 as hx
    V, T, D, F, L, H = 8, 3, 8, 8, 3, 4
    c = LmConfig.make(V, T, D, F, L, H, learned_position=learned)
    p = hx.LmConfig(V, T, D, F, L, H, learned_position=learned).init_reference(20260731)
    a, b = np.array([0, 1, 2], np.uint32), np.array([1, 2, 3], np.uint32)
    g = oracle.lm_forward_backward(c, a, b, p).grads
    loss = lambda q: oracle.lm_forward_backward(c, a, b, q, want_all=False).loss
    reg = hx.LmConfig(V, T, D, F, L, H, learned_position=learned).registry()
    checked = 0
    for name, off, shape in reg:
        n = int(np.prod(shape))
        for k in sorted({0, n // 2, n - 1}):
            if name == "token_embedding" and (k // D) not in (0, 1, 2):
                continue  # rows of unused tokens have zero gradient and zero FD
            assert abs(g[off + k] - _fd(loss, p, off + k)) <= 3e-3, (name, k)
            checked += 1
    assert checked > 30


def test_oracle_mlp_finite_differences(oracle):
    # qnn/qnn_mlp_training.cpp:105-150 gradient check (2/4/5/3, eps 1e-3, abs < 2e-4)
    rng = np.random.default_rng(20260710)
    x, y = rng.uniform(-0.5, 0.5, (2, 4)).astype(np.float32), rng.uniform(-1, 1, (2, 3)).astype(np.float32)
    w1, w2 = rng.normal(0, 0.6, (4, 5)).astype(np.float32), rng.normal(0, 0.5, (5, 3)).astype(np.float32)
    s = oracle.mlp_step(x, y, w1, w2, 0.1)
    for (w, dw, which) in ((w1, s.dw1, 0), (w2, s.dw2, 1)):
        for i in range(w.size):
            def loss(q, which=which):
                qq = q.reshape(w.shape)
                return oracle.mlp_step(x, y, qq if which == 0 else w1, qq if which == 1 else w2, 0.1).loss
            num = _fd(loss, w.ravel().copy(), i)
            assert abs(num - dw.ravel()[i]) < 2e-4


# -- 5. Muon properties ------------------------------------------------------------------

def test_oracle_muon_orthogonalises(oracle):
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (48, 48)).astype(np.float32)
    g = rng.normal(0, 1e-3, (48, 48)).astype(np.float32)
    buf = np.zeros_like(w)
    lr = 1.0
    wn, bn = oracle.muon(w, g, buf, lr, bf16_inputs=False)
    np.testing.assert_array_equal(bn, g)  # buf' = 0.95*0 + g
    upd = (w - wn) / lr
    sv = np.linalg.svd(upd.astype(np.float64), compute_uv=False)
    # five quintic NS steps drive the bulk of the spectrum into roughly
    # [0.68, 1.13]; the smallest singular values of a random square matrix
    # are only partly lifted (expected behaviour of the quintic iteration)
    assert np.percentile(sv, 10) > 0.6 and sv.max() < 1.25, (np.percentile(sv, 10), sv.max())
    wn16, _ = oracle.muon(w, g, buf, lr, bf16_inputs=True)
    assert rel_err(wn16 - w, wn - w) < 5e-2


def test_oracle_muon_rectangular_scale(oracle):
    rng = np.random.default_rng(4)
    w = np.zeros((64, 16), np.float32)
    g = rng.normal(0, 1, (64, 16)).astype(np.float32)
    wn, _ = oracle.muon(w, g, np.zeros_like(w), 1.0, bf16_inputs=False)
    sv = np.linalg.svd(-wn.astype(np.float64), compute_uv=False)
    # update scaled by sqrt(max(1, rows/cols)) = 2
    assert 0.7 < sv.mean() / 2.0 < 1.25


def test_round_bf16(oracle):
    assert oracle.round_bf16(1.0) == 1.0
    assert oracle.round_bf16(1.0 + 2 ** -9) == 1.0          # tie -> even
    assert oracle.round_bf16(1.0 + 3 * 2 ** -9) == 1.0 + 2 ** -7
