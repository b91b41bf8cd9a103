"""GPU parity of the tensor-core attention (head dimension 32, T <= 256).

These shapes take the tcgen05 kernels under the default attention engine.
Each case is checked against the oracle (per-step loss and every gradient
tensor, <= 1e-4 relative, tensor-wise) and against the FP32 CUDA-core
attention kernels selected with HX_ATTN_CUDA_CORES.  Ragged T (not a
multiple of the 128-row query tile) covers the tile tails.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import rel_err
from hexatrain_b200 import _lib, data
from oracle.oracle import LmConfig as OC

pytestmark = pytest.mark.gpu
TOL = 1e-4


def run(cfg, B, p, toks, backend=_lib.HX_ATTN_AUTO):
    rt = hx.Runtime()
    assert rt.initialize(0) and rt.set_attention_backend(backend)
    assert rt.prepare_lm(cfg, B), rt.last_error
    out = hx.TinyTransformerTrainingOutputs()
    assert rt.execute_tiny_transformer_training_tokens(toks[:, :cfg.tokens], toks[:, 1:], p, out), rt.last_error
    rt.close()
    return out


def check(cfg, got, want):
    # A tensor whose exact gradient is zero (wq, wk at T = 1: one visible key
    # gives dS = P (dP - dO.O) = 0) is held to TOL of the largest gradient.
    scale = float(np.max(np.abs(want)))
    for name, off, shape in cfg.registry():
        n = int(np.prod(shape))
        w, g = want[off:off + n], got[off:off + n]
        if np.max(np.abs(w)) == 0:
            assert np.max(np.abs(g)) <= TOL * scale, name
            continue
        assert rel_err(g, w) <= TOL, (name, rel_err(g, w))


@pytest.mark.parametrize("T", [256, 200, 129, 128, 100, 37, 1])
def test_head_dim_32_matches_oracle(oracle, T):
    # std 0.3 makes the attention rows peaked rather than near-uniform
    V, D, F, L, H, B = 64, 64, 64, 2, 2, 3
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(T, 0.3)
    toks = data.lm_tokens(100 + T, B, T, V)
    out = run(cfg, B, p, toks)
    g, loss = oracle.lm_batch_gradients(OC.make(V, T, D, F, L, H, learned_position=True), toks, p, threads=8)
    assert abs(out.loss - loss) <= TOL * abs(loss)
    check(cfg, out.gradients, g)


def test_tensor_core_and_cuda_core_attention_agree_at_model_width():
    """The benchmark's layer shape (D256, H8, T256) on a few sequences."""
    V, T, D, F, L, H, B = 1024, 256, 256, 1024, 2, 8, 6
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    p = cfg.init_normal(9, 0.05)
    toks = data.lm_tokens(9, B, T, V)
    tc = run(cfg, B, p, toks)
    cc = run(cfg, B, p, toks, _lib.HX_ATTN_CUDA_CORES)
    assert abs(tc.loss - cc.loss) <= TOL * abs(cc.loss)
    check(cfg, tc.gradients, cc.gradients)
