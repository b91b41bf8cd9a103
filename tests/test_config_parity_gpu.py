"""Parity at the five configurations as stated, the benchmarked shape included.

Each case runs the product through the C ABI on the default engines and
compares it with the reference's own CPU code (oracle/_ref, built from the
reference's sources) or with the oracle pinned to it:

* the benchmarked LM shape (V1024 T256 D256 F1024 L4 H8) at 16 sequences,
  where every GEMM runs on the tcgen05 kernel and the weight gradients split
  K = 4096;
* a weight-gradient GEMM at K = 131072 rows, the split-K depth of the
  benchmark's 512-sequence step, against fp64;
* the small LM configurations at their batch sizes over 8 optimizer steps
  with the reference driver's anchors at steps 2, 4 and 8
  (qnn/qnn_transformer_training.cpp:7222-7233), Adam and Muon;
* the MLP trajectories over the full step counts: 640 steps at B8 I128 H128
  O64 and 1000 ping-pong steps at B32 I256 H256 O128, gated like the
  reference driver (qnn/qnn_mlp_training.cpp:783-787).

Tolerances: per-step loss and every gradient tensor within 1e-4
relative (max|got-want| / max|want|), weights within 1e-2 max-abs after the
stated steps.  The tests also record tighter figures in their messages.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import rel_err
from hexatrain_b200 import data
from oracle.oracle import LmConfig as OC

pytestmark = pytest.mark.gpu
TOL = 1e-4
W_ABS = 1e-2


def _grads_per_tensor(cfg, got, want, tol=TOL):
    worst = 0.0
    for name, off, shape in cfg.registry():
        n = int(np.prod(shape))
        w = want[off:off + n]
        if np.max(np.abs(w)) == 0:
            assert np.max(np.abs(got[off:off + n])) <= 1e-12, name
            continue
        e = rel_err(got[off:off + n], w)
        worst = max(worst, e)
        assert e <= tol, (name, e)
    return worst


def test_benchmark_shape_16_sequences_matches_reference(gpu_runtime, reference):
    """One Adam step of V1024 T256 D256 F1024 L4 H8 on 16 sequences, the
    reference model (fixed positions), against the reference's own batched
    train step on the host threads.  After one step Adam's first moment is
    0.1 * gradient, so m checks every gradient element."""
    V, T, D, F, L, H, B = 1024, 256, 256, 1024, 4, 8, 16
    cfg = hx.LmConfig(V, T, D, F, L, H)
    oc = OC.make(V, T, D, F, L, H)
    p0 = cfg.init_normal(20260710, 0.02)
    toks = data.lm_tokens(20260710, B, T, V)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B), rt.last_error
    assert rt.lm_state_upload(p0), rt.last_error
    ok, loss = rt.lm_train_step(toks, 1)
    assert ok, rt.last_error
    params, m, v, _ = rt.lm_state_download()
    rp, rm, rv = p0.copy(), np.zeros_like(p0), np.zeros_like(p0)
    rloss = reference.lm_train_step(oc, toks, rp, rm, rv, 1e-3, 1, threads=16)
    assert abs(loss - rloss) <= TOL * abs(rloss), (loss, rloss)
    worst = _grads_per_tensor(cfg, m, rm)
    assert np.max(np.abs(params - rp)) <= W_ABS
    assert rel_err(v, rv) <= 2 * TOL, rel_err(v, rv)
    print(f"T256 D256 F1024 L4 H8, B16: loss {loss} ref {rloss}; worst gradient tensor {worst:.2e}")


def test_benchmark_shape_learned_positions_matches_oracle(gpu_runtime, oracle):
    """The benchmark's own model (learned positions, N(0, 0.02)) at 16
    sequences: every gradient tensor against the oracle."""
    V, T, D, F, L, H, B = 1024, 256, 256, 1024, 4, 8, 16
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(20260711, 0.02)
    toks = data.lm_tokens(20260711, B, T, V)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    assert rt.execute_tiny_transformer_training_tokens(toks[:, :T], toks[:, 1:], p, out), rt.last_error
    g, loss = oracle.lm_batch_gradients(OC.make(V, T, D, F, L, H, learned_position=True), toks, p, threads=16)
    assert abs(out.loss - loss) <= TOL * abs(loss)
    _grads_per_tensor(cfg, out.gradients, g)


def test_weight_gradient_split_k_131072_rows_against_fp64(gpu_runtime):
    """dW1 = X^T dZ1 and dW2 = H^T dP with K = 131072 rows (I256 H1024 O256):
    the 1024-wide and 256-wide weight-gradient GEMMs of the benchmark at its
    split-K depth, through the public MLP step, against fp64 sums over the
    GPU's own ReLU mask."""
    B, I, H, O = 131072, 256, 1024, 256
    x, y, w1, w2 = data.mlp_data(20260712, B, I, H, O)
    rt = gpu_runtime
    assert rt.prepare_mlp_full_step(B, I, H, O, True), rt.last_error
    out = hx.MlpFullStepOutputs()
    assert rt.execute_mlp_full_step(x, y, w1, w2, 0.05, out), rt.last_error
    x64, w1_64, w2_64 = x.astype(np.float64), w1.astype(np.float64), w2.astype(np.float64)
    z1 = x64 @ w1_64
    h_gpu = out.hidden.reshape(B, H)
    assert rel_err(h_gpu, np.maximum(z1, 0)) <= 1e-5
    mask = out.mask.reshape(B, H) != 0
    h64 = h_gpu.astype(np.float64)
    e = h64 @ w2_64 - y
    dp = e * (2.0 / (B * O))
    dw2 = h64.T @ dp
    dz1 = np.where(mask, dp @ w2_64.T, 0.0)
    dw1 = x64.T @ dz1
    e1, e2 = rel_err(out.d_w1, dw1), rel_err(out.d_w2, dw2)
    assert e1 <= TOL and e2 <= TOL, (e1, e2)
    assert abs(out.loss - np.mean(e * e)) <= TOL * np.mean(e * e)
    print(f"K=131072 split-K: dW1 {e1:.2e}, dW2 {e2:.2e} of max|ref|")


ANCHORS = (2, 4, 8)


def test_lm_t64_d64_reference_model_8_steps_matches_reference(gpu_runtime, reference):
    """The T64 D64 L2 shape and batch (V1024 T64 D64 F64 L2 H4, 16 sequences) on the
    reference model, 8 Adam steps of hx_lm_train_step against the
    reference's own batched train step, loss every step, weights at the
    anchors."""
    V, T, D, F, L, H, B = 1024, 64, 64, 64, 2, 4, 16
    cfg = hx.LmConfig(V, T, D, F, L, H)
    oc = OC.make(V, T, D, F, L, H)
    p0 = cfg.init_normal(20260713, 0.02)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B), rt.last_error
    assert rt.lm_state_upload(p0), rt.last_error
    rp, rm, rv = p0.copy(), np.zeros_like(p0), np.zeros_like(p0)
    worst_w = 0.0
    for step in range(1, 9):
        toks = data.lm_tokens(20260713, B, T, V, step=step)
        ok, loss = rt.lm_train_step(toks, step)
        assert ok, rt.last_error
        rloss = reference.lm_train_step(oc, toks, rp, rm, rv, 1e-3, step, threads=8)
        assert abs(loss - rloss) <= TOL * abs(rloss), (step, loss, rloss)
        if step in ANCHORS:
            params, m, _, _ = rt.lm_state_download()
            worst_w = max(worst_w, float(np.max(np.abs(params - rp))))
            assert np.max(np.abs(params - rp)) <= W_ABS, step
            if step == 2:
                assert rel_err(m, rm) <= TOL, rel_err(m, rm)
    print(f"T64 D64 L2 reference model: worst weight difference at anchors {worst_w:.2e}")


def _oracle_trajectory(oracle, oc, cfg, p0, B, T, V, seed, steps, muon):
    """The oracle's step-by-step trajectory: batch gradients at its own
    weights, then Adam (and Muon on the hidden 2-D weights when asked)."""
    w = p0.copy()
    m, v, buf = np.zeros_like(w), np.zeros_like(w), np.zeros_like(w)
    muon_names = ("wq", "wk", "wv", "wo", "ffn_w1", "ffn_w2")
    reg = cfg.registry()
    for step in range(1, steps + 1):
        toks = data.lm_tokens(seed, B, T, V, step=step)
        g, loss = oracle.lm_batch_gradients(oc, toks, w, threads=8)
        c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
        nw = w.copy()
        if muon:
            for name, off, shape in reg:
                n = int(np.prod(shape))
                sl = slice(off, off + n)
                if name.split(".")[-1] in muon_names:
                    wn, bn = oracle.muon(w[sl].reshape(shape), g[sl].reshape(shape), buf[sl].reshape(shape), 0.02)
                    nw[sl], buf[sl] = wn.ravel(), bn.ravel()
                else:
                    m[sl], v[sl], _, _, nw[sl] = oracle.adam(w[sl], g[sl], m[sl], v[sl], 1e-3, c1, c2)
        else:
            m, v, _, _, nw = oracle.adam(w, g, m, v, 1e-3, c1, c2)
        w = nw
        yield step, toks, loss, w


@pytest.mark.parametrize("name,shape,B,muon", [
    ("t64-d64-l2-adam", (1024, 64, 64, 64, 2, 4), 16, False),
    ("t64-d48-l4-muon", (1024, 64, 48, 48, 4, 4), 32, True),
])
def test_small_lm_configs_as_specified_8_steps_match_oracle(gpu_runtime, oracle, name, shape, B, muon):
    """T64 D64 L2 H4 (Adam) and T64 D48 L4 H4 (Muon momentum 0.95 Nesterov, NS5 on bf16
    operands, Adam elsewhere) as specified: learned positions, N(0, 0.02),
    Zipf ids, their batch sizes, 8 steps; loss every step, weights at the
    anchors."""
    V, T, D, F, L, H = shape
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    oc = OC.make(V, T, D, F, L, H, learned_position=True)
    p0 = cfg.init_normal(20260714, 0.02)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, B), rt.last_error
    if muon:
        assert rt.lm_set_optimizer(hx.OptimizerConfig(kind=1, muon_lr=0.02)), rt.last_error
    assert rt.lm_state_upload(p0), rt.last_error
    worst = 0.0
    for step, toks, rloss, rw in _oracle_trajectory(oracle, oc, cfg, p0, B, T, V, 20260714, 8, muon):
        ok, loss = rt.lm_train_step(toks, step)
        assert ok, rt.last_error
        assert abs(loss - rloss) <= TOL * abs(rloss), (name, step, loss, rloss)
        if step in ANCHORS:
            params, _, _, _ = rt.lm_state_download()
            d = float(np.max(np.abs(params - rw)))
            worst = max(worst, d)
            assert d <= W_ABS, (name, step, d)
    print(f"{name}: worst weight difference at anchors {worst:.2e}")


def _mlp_gates(x, y, w1, w2, B, lr, steps, reference, step_fn):
    """Runs `steps` cyclic-batch steps of both sides; checks the loss every
    step and the weights at the end (the reference driver's trajectory)."""
    S = x.shape[0]
    cw1, cw2 = w1.copy(), w2.copy()
    worst_loss = 0.0
    for st in range(steps):
        xb, yb = data.batch(x, (st * B) % S, B), data.batch(y, (st * B) % S, B)
        loss, g1, g2 = step_fn(st, xb, yb)
        ref = reference.mlp_step(xb, yb, cw1, cw2, lr)
        worst_loss = max(worst_loss, abs(loss - ref.loss) / abs(ref.loss))
        assert abs(loss - ref.loss) <= TOL * abs(ref.loss), (st, loss, ref.loss)
        cw1, cw2 = ref.w1_next.reshape(cw1.shape), ref.w2_next.reshape(cw2.shape)
    return cw1, cw2, worst_loss


def test_mlp_8x128x128x64_640_steps_matches_reference(gpu_runtime, reference):
    """MLP B8 I128 H128 O64, lr 0.5, 512 samples, 10 epochs = 640 steps of
    the host-vector execute, ping-pong on the host."""
    B, I, H, O, S, lr = 8, 128, 128, 64, 512, 0.5
    x, y, w1, w2 = data.mlp_data(20260710, S, I, H, O)
    rt = gpu_runtime
    assert rt.prepare_mlp_full_step(B, I, H, O, False), rt.last_error
    cur = [w1.ravel().copy(), w2.ravel().copy()]
    out = hx.MlpFullStepOutputs()

    def step(st, xb, yb):
        assert rt.execute_mlp_full_step(xb, yb, cur[0], cur[1], lr, out), rt.last_error
        cur[0], cur[1] = out.w1_next.copy(), out.w2_next.copy()
        return out.loss, cur[0], cur[1]

    rw1, rw2, wl = _mlp_gates(x, y, w1, w2, B, lr, 640, reference, step)
    d = max(float(np.max(np.abs(cur[0] - rw1.ravel()))), float(np.max(np.abs(cur[1] - rw2.ravel()))))
    assert d <= W_ABS, d
    print(f"MLP 8x128x128x64, 640 steps: worst loss {wl:.2e} relative, final weights {d:.2e} max-abs")


def test_mlp_32x256x256x128_1000_ping_pong_steps_matches_reference(gpu_runtime, reference):
    """MLP B32 I256 H256 O128, lr 0.05, 1000 steps of the device step with
    the two weight buffers swapped every step (no weight copies)."""
    import torch
    B, I, H, O, lr = 32, 256, 256, 128, 0.05
    S = 4 * B
    x, y, w1, w2 = data.mlp_data(20260715, S, I, H, O)
    rt = gpu_runtime
    assert rt.prepare_mlp_full_step(B, I, H, O, False), rt.last_error
    xd, yd = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    a = [torch.from_numpy(w1.ravel().copy()).cuda(), torch.from_numpy(w2.ravel().copy()).cuda()]
    b = [torch.empty_like(t) for t in a]
    loss = torch.zeros(1, device="cuda")
    bufs = [a, b]

    def step(st, xb, yb):
        cur, nxt = bufs[st % 2], bufs[(st + 1) % 2]
        off = (st * B) % S
        assert rt.execute_mlp_full_step_device(xd[off:off + B].data_ptr(), yd[off:off + B].data_ptr(),
                                               cur[0].data_ptr(), cur[1].data_ptr(), lr, loss.data_ptr(),
                                               nxt[0].data_ptr(), nxt[1].data_ptr()), rt.last_error
        assert rt.synchronize(), rt.last_error
        return float(loss.item()), None, None

    torch.cuda.synchronize()
    rw1, rw2, wl = _mlp_gates(x, y, w1, w2, B, lr, 1000, reference, step)
    fin = bufs[1000 % 2]
    d = max(float(np.max(np.abs(fin[0].cpu().numpy() - rw1.ravel()))),
            float(np.max(np.abs(fin[1].cpu().numpy() - rw2.ravel()))))
    assert d <= W_ABS, d
    print(f"MLP 32x256x256x128, 1000 steps: worst loss {wl:.2e} relative, final weights {d:.2e} max-abs")
