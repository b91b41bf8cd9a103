"""Writes the committed golden fixtures from the reference's own CPU code.

Run from the repository root after `make -C oracle` has built
oracle/_ref/libhexaref.so from the HexaTrain sources:

    python tests/golden/make_golden.py

Every array below is produced by the reference's compiled
cpu_reference_training.cpp / tiny_language_model_cpu.cpp through
oracle/ref_adapter.cpp.  Inputs come from numpy's seeded generator, so the
fixtures do not depend on this repository's product code.  Large results are
stored as summaries (sums, weighted checksum, a strided sample) to keep the
files small.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.oracle import LmConfig, Reference  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def summary(a: np.ndarray, n_sample: int = 256) -> dict:
    a = np.asarray(a, np.float32).ravel()
    k = np.arange(a.size)
    idx = np.linspace(0, a.size - 1, min(n_sample, a.size)).astype(np.int64)
    return {
        "sum": np.float64(a.astype(np.float64).sum()),
        "abs_sum": np.float64(np.abs(a.astype(np.float64)).sum()),
        "l2": np.float64(np.sqrt((a.astype(np.float64) ** 2).sum())),
        # the reference driver's trajectory checksum (qnn/qnn_mlp_training.cpp:600-605)
        "checksum": np.float64((a.astype(np.float64) * ((k % 997) + 1)).sum()),
        "sample_idx": idx,
        "sample": a[idx],
    }


def save(name: str, **arrays):
    flat = {}
    for k, v in arrays.items():
        if isinstance(v, dict):
            for kk, vv in v.items():
                flat[f"{k}__{kk}"] = vv
        else:
            flat[k] = v
    np.savez_compressed(os.path.join(OUT, name), **flat)
    print("wrote", name, sum(np.asarray(v).nbytes for v in flat.values()), "bytes raw")


def mlp_cases(ref: Reference):
    rng = np.random.default_rng(20260710)
    for (B, I, H, O, lr) in [(2, 4, 5, 3, 0.5), (8, 128, 128, 64, 0.5), (5, 7, 3, 2, 0.125)]:
        x = rng.uniform(-1, 1, (B, I)).astype(np.float32)
        y = rng.uniform(-1, 1, (B, O)).astype(np.float32)
        w1 = (rng.uniform(-1, 1, (I, H)) / np.sqrt(I)).astype(np.float32)
        w2 = (rng.uniform(-1, 1, (H, O)) / np.sqrt(H)).astype(np.float32)
        s = ref.mlp_step(x, y, w1, w2, lr)
        save(f"mlp_{B}x{I}x{H}x{O}.npz", x=x, y=y, w1=w1, w2=w2, lr=np.float32(lr), loss=np.float32(s.loss),
             w1_next=s.w1_next, w2_next=s.w2_next, z1=s.z1, h=s.h, p=s.p, e=s.e, dp=s.dp, dw2=s.dw2, dh=s.dh,
             mask=s.mask, dz1=s.dz1, dw1=s.dw1)


def mlp_trajectory(ref: Reference):
    """Trajectory of the 8/128/128/64 MLP: 64 samples, cyclic batches of 8, 16 steps."""
    rng = np.random.default_rng(7)
    B, I, H, O, lr, samples, steps = 8, 128, 128, 64, 0.5, 64, 16
    X = rng.uniform(-1, 1, (samples, I)).astype(np.float32)
    Y = rng.uniform(-1, 1, (samples, O)).astype(np.float32)
    w1 = (rng.uniform(-1, 1, (I, H)) / np.sqrt(I)).astype(np.float32)
    w2 = (rng.uniform(-1, 1, (H, O)) / np.sqrt(H)).astype(np.float32)
    w1_0, w2_0 = w1.copy(), w2.copy()
    losses, c1, c2 = [], [], []
    for st in range(steps):
        rows = (st * B + np.arange(B)) % samples
        s = ref.mlp_step(np.ascontiguousarray(X[rows]), np.ascontiguousarray(Y[rows]), w1, w2, lr)
        losses.append(s.loss)
        w1, w2 = s.w1_next, s.w2_next
        c1.append(summary(w1)["checksum"])
        c2.append(summary(w2)["checksum"])
    save("mlp_trajectory_8x128x128x64.npz", X=X, Y=Y, w1_init=w1_0, w2_init=w2_0, lr=np.float32(lr),
         batch=np.int64(B), losses=np.array(losses, np.float32), w1_checksums=np.array(c1),
         w2_checksums=np.array(c2), w1_final=w1, w2_final=w2)


# (V, T, D, F, L, H, init seed, input ids, target ids): the reference's own
# host-test cases (host_tests/cpu_reference_training_test.cpp:82-88 via
# tiny_lm::gradientCheck, :117-144, :146-178, :265-310, :312-334).
LM_SMALL = [
    (8, 3, 4, 8, 1, 1, 20260725, [0, 1, 2], [1, 2, 3]),
    (32, 4, 8, 16, 2, 2, 7, [0, 1, 2, 3], [1, 2, 3, 4]),
    (32, 4, 8, 16, 3, 8, 13, [0, 1, 2, 3], [1, 2, 3, 4]),
    (8, 3, 8, 8, 3, 4, 20260731, [0, 1, 2], [1, 2, 3]),
    (32, 4, 8, 16, 1, 1, 19, [0, 1, 2, 3], [1, 2, 3, 4]),
    (32, 8, 16, 32, 1, 1, 1, [0, 1, 2, 3, 0, 1, 2, 3], [1, 2, 3, 0, 1, 2, 3, 0]),
]


def lm_small(ref: Reference):
    for (V, T, D, F, L, H, seed, a, b) in LM_SMALL:
        cfg = LmConfig.make(V, T, D, F, L, H)
        p = ref.initial_parameters(cfg, seed)
        s = ref.lm_forward_backward(cfg, np.array(a, np.uint32), np.array(b, np.uint32), p)
        save(f"lm_V{V}_T{T}_D{D}_F{F}_L{L}_H{H}.npz", cfg=np.array([V, T, D, F, L, H], np.int64), seed=np.int64(seed),
             inputs=np.array(a, np.uint32), targets=np.array(b, np.uint32), params=p, loss=np.float32(s.loss),
             accuracy=np.float32(s.accuracy), grads=s.grads, logits=s.logits, probs=s.probs, dlogits=s.dlogits,
             output=s.output, layer_input_grads=s.layer_input_grads, head_probs=s.head_probs)


def lm_large(ref: Reference):
    """Single sequences of the benchmarked LM shapes (T64 D64 F64 L2 H4 and T64 D48 F48 L4 H4), summarised."""
    rng = np.random.default_rng(1234)
    for (V, T, D, F, L, H) in [(1024, 64, 64, 64, 2, 4), (1024, 64, 48, 48, 4, 4)]:
        cfg = LmConfig.make(V, T, D, F, L, H)
        p = ref.initial_parameters(cfg, 7)
        ids = rng.integers(0, V, T + 1).astype(np.uint32)
        s = ref.lm_forward_backward(cfg, ids[:T], ids[1:], p)
        save(f"lm_V{V}_T{T}_D{D}_F{F}_L{L}_H{H}.npz", cfg=np.array([V, T, D, F, L, H], np.int64), seed=np.int64(7),
             ids=ids, loss=np.float32(s.loss), accuracy=np.float32(s.accuracy), params=summary(p),
             grads=summary(s.grads), logits=summary(s.logits), dlogits=summary(s.dlogits))


def adam_case(ref: Reference):
    cfg = LmConfig.make(8, 3, 4, 8, 1, 1)
    n = ref.param_count(cfg)
    rng = np.random.default_rng(99)
    w = rng.normal(0, 0.1, n).astype(np.float32)
    g = rng.normal(0, 0.01, n).astype(np.float32)
    g[:5] = 0.0
    m = rng.normal(0, 0.001, n).astype(np.float32)
    v = np.abs(rng.normal(0, 1e-5, n)).astype(np.float32)
    m[:5] = 0.0
    v[:5] = 0.0
    step = 3
    c1 = np.float32(1.0 / (1.0 - 0.9 ** step))
    c2 = np.float32(1.0 / (1.0 - 0.999 ** step))
    mn, vn, mh, vh, wn = ref.adam(cfg, w, g, m, v, 1e-3, float(c1), float(c2))
    save("adam_n208.npz", w=w, g=g, m=m, v=v, lr=np.float32(1e-3), c1=c1, c2=c2, m_next=mn, v_next=vn, m_hat=mh,
         v_hat=vh, w_next=wn)


def lm_train_steps(ref: Reference):
    """Three batched Adam steps of the reference driver loop on a small model."""
    V, T, D, F, L, H, B = 32, 8, 16, 32, 2, 2, 4
    cfg = LmConfig.make(V, T, D, F, L, H)
    p = ref.initial_parameters(cfg, 5)
    p0 = p.copy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    rng = np.random.default_rng(5)
    toks, losses, snaps = [], [], []
    for step in (1, 2, 3):
        t = rng.integers(0, V, (B, T + 1)).astype(np.uint32)
        toks.append(t)
        losses.append(ref.lm_train_step(cfg, t, p, m, v, 1e-3, step, threads=1))
        snaps.append(p.copy())
    save("lm_train_3steps.npz", cfg=np.array([V, T, D, F, L, H, B], np.int64), params0=p0, tokens=np.stack(toks),
         losses=np.array(losses, np.float32), params=np.stack(snaps), m=m, v=v)


def main():
    ref = Reference()
    mlp_cases(ref)
    mlp_trajectory(ref)
    lm_small(ref)
    lm_large(ref)
    adam_case(ref)
    lm_train_steps(ref)


if __name__ == "__main__":
    main()
