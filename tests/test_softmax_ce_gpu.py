"""The softmax/cross-entropy kernels against IEEE float32 arithmetic, bit for
bit.  The LM step's diagnostic outputs give the logits, the probabilities and
dlogits that the kernel wrote; the test recomputes them with torch on the same
GPU from the same logits:
  m = max_j l_j;  e_j = exp(l_j - m) (float32, the device expf);
  s = the double sum of e in the kernel's order (lane k adds columns
      k, k + 32, ... in order, then a butterfly over lanes 16, 8, 4, 2, 1);
  p_j = e_j / float(s);  dlogits_j = (p_j - [j == target]) / T
with IEEE division.  V = 1024 runs the vectorised kernel (the row held in
registers), V = 1000 the general one, so both are checked for the same
results."""
import numpy as np
import pytest

import hexatrain_b200 as hx
from hexatrain_b200 import data

pytestmark = pytest.mark.gpu


def kernel_order_sum(e):
    """Row sums of e [rows, V] in double, in the order the kernels add them."""
    rows, V = e.shape
    ed = e.astype(np.float64)
    lanes = np.zeros((rows, 32))
    for j0 in range(0, V, 32):
        n = min(32, V - j0)
        lanes[:, :n] += ed[:, j0:j0 + n]
    for o in (16, 8, 4, 2, 1):
        lanes = lanes + lanes[:, np.arange(32) ^ o]
    return lanes[:, 0]


@pytest.mark.parametrize("V", [1024, 1000])
def test_softmax_ce_matches_ieee_division(gpu_runtime, V):
    import torch

    T = 64
    cfg = hx.LmConfig(V, T, 32, 64, 1, 1)
    rt = gpu_runtime
    assert rt.prepare_lm(cfg, 1, diagnostic_outputs=True), rt.last_error
    for seed, std in ((20260710, 0.5), (20260711, 2.0)):
        params = cfg.init_normal(seed, std)
        ids = data.lm_tokens(seed, 1, T, V)[0]
        out = hx.TinyTransformerTrainingOutputs()
        assert rt.execute_tiny_transformer_training_tokens(ids[:T], ids[1:], params, out), rt.last_error
        logits = out.logits.reshape(T, V)
        dev = torch.device("cuda", 0)
        l = torch.from_numpy(logits).to(dev)
        m = l.max(dim=1, keepdim=True).values
        e = torch.exp(l - m)
        s = kernel_order_sum(e.cpu().numpy())
        sf = torch.from_numpy(s.astype(np.float32)).to(dev).unsqueeze(1)
        p = e / sf
        onehot = torch.zeros_like(p)
        onehot[torch.arange(T, device=dev), torch.from_numpy(ids[1:].astype(np.int64)).to(dev)] = 1.0
        d = (p - onehot) / torch.tensor(float(T), device=dev)
        p_want, d_want = p.cpu().numpy(), d.cpu().numpy()
        assert np.array_equal(out.probabilities.reshape(T, V).view(np.uint32), p_want.view(np.uint32)), \
            int(np.sum(out.probabilities.reshape(T, V) != p_want))
        assert np.array_equal(out.d_logits.reshape(T, V).view(np.uint32), d_want.view(np.uint32)), \
            int(np.sum(out.d_logits.reshape(T, V) != d_want))
        assert float(np.min(p_want)) < 1e-3  # the spread of the logits reaches small probabilities
