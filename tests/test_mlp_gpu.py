"""GPU parity of phonelm_mlp_training_step through the C ABI.

Tolerances are the stated ones: <= 1e-4 relative on the per-step loss and
every gradient tensor (tensor-wise: max|got-want| / max|want|), <= 1e-2
max-abs on weights after the stated number of steps.  The ReLU mask must
match except where the oracle's Z1 is within 1e-3 of zero, the reference's
own gate (qnn/qnn_mlp_training.cpp:783-787).
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import golden, rel_err
from hexatrain_b200 import data

pytestmark = pytest.mark.gpu
TOL = 1e-4
W_ABS = 1e-2


def run(rt, x, y, w1, w2, lr, diag=True):
    B, I = x.shape
    H, O = w2.shape
    assert rt.prepare_mlp_full_step(B, I, H, O, diag), rt.last_error
    out = hx.MlpFullStepOutputs()
    assert rt.execute_mlp_full_step(x, y, w1, w2, lr, out), rt.last_error
    return out


def check_step(out, want, B, I, H, O, x=None, lr=None):
    """Tolerance checks of one step.  Where the GPU's ReLU mask differs from
    the reference's (allowed only where the reference's Z1 is within 1e-3 of
    zero), the mask-dependent tensors dZ1, dW1 and W1_next are compared with
    their fp64 values under the GPU's own mask: the step is piecewise linear
    and a kink flip moves a whole dW1 row by one term."""
    assert abs(out.loss - float(want["loss"])) <= TOL * abs(float(want["loss"]))
    mism = out.mask != np.asarray(want["mask"]).ravel()
    assert np.all(np.abs(np.asarray(want["z1"]).ravel()[mism]) < 1e-3)
    want = dict(want)
    if mism.any():
        assert x is not None and lr is not None
        dh = np.asarray(want["dh"], np.float64).reshape(B, H)
        dz1 = np.where(out.mask.reshape(B, H) > 0, dh, 0.0)
        dw1 = np.asarray(x, np.float64).T @ dz1
        want["dz1"], want["dw1"] = dz1, dw1
        w1 = np.asarray(want["w1_next"], np.float64).reshape(I, H) + lr * np.asarray(want["dw1_orig"], np.float64)
        want["w1_next"] = w1 - lr * dw1
    pairs = [("d_w1", "dw1"), ("d_w2", "dw2"), ("d_hidden", "dh"), ("d_z1", "dz1"), ("d_prediction", "dp"),
             ("prediction", "p"), ("error", "e"), ("hidden", "h")]
    for a, b in pairs:
        assert rel_err(getattr(out, a), want[b]) <= TOL, (a, rel_err(getattr(out, a), want[b]))
    for a, b in (("w1_next", "w1_next"), ("w2_next", "w2_next")):
        got = getattr(out, a)
        assert np.max(np.abs(got - np.asarray(want[b]).ravel())) <= W_ABS
        assert rel_err(got, want[b]) <= TOL
    # internal consistency: mask == (hidden > 0), dZ1 = mask ? dH : 0
    assert np.array_equal(out.mask.astype(bool), out.hidden > 0)
    assert np.array_equal(out.d_z1, np.where(out.hidden > 0, out.d_hidden, 0).astype(np.float32))


def expected(ref_obj_or_dict):
    keys = ("loss", "dw1", "dw2", "dh", "dz1", "dp", "p", "e", "h", "w1_next", "w2_next", "mask", "z1")
    if isinstance(ref_obj_or_dict, dict):
        d = {k: ref_obj_or_dict[k] for k in keys}
    else:
        d = {k: getattr(ref_obj_or_dict, k) for k in keys}
    d["dw1_orig"] = d["dw1"]
    return d


@pytest.mark.parametrize("name", ["mlp_2x4x5x3.npz", "mlp_5x7x3x2.npz", "mlp_8x128x128x64.npz"])
def test_mlp_matches_golden(gpu_runtime, name):
    g = golden(name)
    B, I = g["x"].shape
    H, O = g["w2"].shape
    out = run(gpu_runtime, g["x"], g["y"], g["w1"], g["w2"], float(g["lr"]))
    check_step(out, expected(g), B, I, H, O, g["x"], float(g["lr"]))


@pytest.mark.parametrize("shape,lr", [((8, 128, 128, 64), 0.5), ((32, 256, 256, 128), 0.05), ((37, 129, 65, 33), 0.05),
                                      ((1, 1, 1, 1), 0.1), ((300, 40, 520, 7), 0.05)])
def test_mlp_matches_oracle(gpu_runtime, oracle, shape, lr):
    B, I, H, O = shape
    x, y, w1, w2 = data.mlp_data(20260710, B, I, H, O)
    out = run(gpu_runtime, x, y, w1, w2, lr)
    ref = oracle.mlp_step(x, y, w1, w2, lr)
    check_step(out, expected(ref), B, I, H, O, x, lr)


def mlp_fp64(x, y, w1, w2, lr):
    """float64 restatement used at sizes the scalar oracle cannot finish quickly."""
    x, y, w1, w2 = (a.astype(np.float64) for a in (x, y, w1, w2))
    z1 = x @ w1
    h = np.maximum(z1, 0)
    p = h @ w2
    e = p - y
    dp = e * (2.0 / e.size)
    dw2 = h.T @ dp
    dh = dp @ w2.T
    dz1 = np.where(h > 0, dh, 0)
    dw1 = x.T @ dz1
    return dict(loss=np.mean(e * e), dw1=dw1, dw2=dw2, dh=dh, dz1=dz1, dp=dp, p=p, e=e, h=h, z1=z1,
                w1_next=w1 - lr * dw1, w2_next=w2 - lr * dw2, mask=(h > 0).astype(np.uint8))


def test_mlp_largest_config_against_fp64(gpu_runtime):
    # B/I/H/O = 4096/1024/1024/512, lr 0.05
    B, I, H, O = 4096, 1024, 1024, 512
    x, y, w1, w2 = data.mlp_data(20260711, B, I, H, O)
    out = run(gpu_runtime, x, y, w1, w2, 0.05)
    check_step(out, expected(mlp_fp64(x, y, w1, w2, 0.05)), B, I, H, O, x, 0.05)


def test_mlp_trajectory_matches_golden(gpu_runtime):
    """16 cyclic-batch steps with ping-pong weights through the host API
    (trainFullStep, qnn/qnn_mlp_training.cpp:674-770)."""
    g = golden("mlp_trajectory_8x128x128x64.npz")
    X, Y, B = g["X"], g["Y"], int(g["batch"])
    I, H = g["w1_init"].shape
    O = g["w2_init"].shape[1]
    rt = gpu_runtime
    assert rt.prepare_mlp_full_step(B, I, H, O, False), rt.last_error
    w1, w2 = g["w1_init"].ravel().copy(), g["w2_init"].ravel().copy()
    out = hx.MlpFullStepOutputs()
    for st, want in enumerate(g["losses"]):
        xb, yb = data.batch(X, st * B, B), data.batch(Y, st * B, B)
        assert rt.execute_mlp_full_step(xb, yb, w1, w2, float(g["lr"]), out), rt.last_error
        assert abs(out.loss - want) <= TOL * abs(want)
        w1, out.w1_next = out.w1_next, w1   # ping-pong: swap owners, no copy
        w2, out.w2_next = out.w2_next, w2
    assert np.max(np.abs(w1 - g["w1_final"].ravel())) <= W_ABS
    assert np.max(np.abs(w2 - g["w2_final"].ravel())) <= W_ABS
    assert rel_err(w1, g["w1_final"]) <= 1e-5


def test_mlp_device_ping_pong_uses_two_graphs(gpu_runtime):
    import torch
    B, I, H, O, lr, steps = 8, 128, 128, 64, 0.5, 10
    X, Y, w1, w2 = data.mlp_data(5, 64, I, H, O)
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    assert rt.prepare_mlp_full_step(B, I, H, O, False), rt.last_error
    dev = "cuda:0"
    bufs1 = [torch.from_numpy(w1.copy()).to(dev), torch.empty(I * H, device=dev)]
    bufs2 = [torch.from_numpy(w2.copy()).to(dev), torch.empty(H * O, device=dev)]
    xd = torch.from_numpy(X).to(dev)
    yd = torch.from_numpy(Y).to(dev)
    loss = torch.zeros(1, device=dev)
    torch.cuda.synchronize()
    host = hx.Runtime()
    assert host.initialize(0) and host.prepare_mlp_full_step(B, I, H, O, False)
    hw1, hw2 = w1.ravel().copy(), w2.ravel().copy()
    hout = hx.MlpFullStepOutputs()
    for st in range(steps):
        rows = (st * B) % 64
        cur, nxt = st % 2, (st + 1) % 2
        ok = rt.execute_mlp_full_step_device(xd[rows:rows + B].data_ptr(), yd[rows:rows + B].data_ptr(), bufs1[cur].data_ptr(),
                                             bufs2[cur].data_ptr(), lr, loss.data_ptr(), bufs1[nxt].data_ptr(),
                                             bufs2[nxt].data_ptr())
        assert ok, rt.last_error
        assert host.execute_mlp_full_step(data.batch(X, rows, B), data.batch(Y, rows, B), hw1, hw2, lr, hout)
        hw1, hw2 = hout.w1_next.copy(), hout.w2_next.copy()
        assert rt.synchronize()
        assert abs(float(loss.item()) - hout.loss) <= 1e-6 * abs(hout.loss)
    np.testing.assert_array_equal(bufs1[steps % 2].cpu().numpy().ravel(), hw1)
    m = rt.metrics()
    # eight distinct batches x two ping-pong phases; graphs are cached per binding
    assert m.graph_execute_count == steps and m.execute_failure_count == 0
    assert m.graph_finalize_count <= steps
    rt.close()
    host.close()


def test_mlp_errors_fail_closed():
    rt = hx.Runtime()
    assert rt.initialize(0)
    out = hx.MlpFullStepOutputs()
    z = np.zeros(10, np.float32)
    assert not rt.execute_mlp_full_step(z, z, z, z, 0.1, out)
    assert rt.last_error == "full step graph not prepared"
    assert not rt.prepare_mlp_full_step(0, 4, 5, 3, True)
    assert rt.last_error == "full step invalid runtime or shape"
    assert rt.prepare_mlp_full_step(2, 4, 5, 3, True)
    assert not rt.execute_mlp_full_step(np.zeros(7), np.zeros(6), np.zeros(20), np.zeros(15), 0.1, out)
    assert rt.last_error == "full step buffer size mismatch"
    assert not rt.execute_mlp_full_step(np.zeros(8), np.zeros(6), np.zeros(20), np.zeros(15), float("nan"), out)
    assert "learning rate" in rt.last_error
    rt.close()


def test_mlp_host_failure_injection():
    """failGraphExecuteAt (qnn/qnn_runtime_full_step.inc:383-397): the chosen
    execute reports failure after its device work; later calls succeed."""
    rt = hx.Runtime()
    rt.set_options(hx.RuntimeOptions(fail_graph_execute_at=2))
    assert rt.initialize(0) and rt.prepare_mlp_full_step(2, 4, 5, 3, False)
    x, y, w1, w2 = data.mlp_data(1, 2, 4, 5, 3)
    out = hx.MlpFullStepOutputs()
    results = [rt.execute_mlp_full_step(x, y, w1, w2, 0.1, out) for _ in range(4)]
    assert results == [True, True, False, True]
    m = rt.metrics()
    assert m.execute_attempt_count == 4 and m.execute_failure_count == 1 and m.first_failure_call == 2
    rt.close()


@pytest.mark.parametrize("shape", [(300, 160, 520, 12), (1000, 256, 384, 128), (128, 128, 128, 128), (4096, 512, 256, 64)])
def test_mlp_gemm_engines_agree_with_oracle(oracle, shape):
    """The same step on the CUDA-core FP32 GEMM and on the tcgen05 3xTF32
    GEMM (forced), both within tolerance of the oracle: covers the three
    operand layouts of the step (K x MN, MN x MN, K x K majors), M/N/K tails
    and the split-K path of the weight-gradient GEMMs."""
    B, I, H, O = shape
    x, y, w1, w2 = data.mlp_data(77, B, I, H, O)
    ref = oracle.mlp_step(x, y, w1, w2, 0.05)
    for backend in (1, 2):
        rt = hx.Runtime()
        assert rt.initialize(0) and rt.set_gemm_backend(backend)
        out = run(rt, x, y, w1, w2, 0.05)
        check_step(out, expected(ref), B, I, H, O, x, 0.05)
        rt.close()
