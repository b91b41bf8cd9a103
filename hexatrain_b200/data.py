"""Seeded synthetic inputs for the training-step workloads.

The reference's generators use std::mt19937_64 with libc++/libstdc++
distributions, whose outputs differ between standard libraries, so its
published trajectories cannot be regenerated bit-for-bit; parity is checked
in-process instead (the same arrays go to the oracle and to the GPU).  These
generators are counter-based (splitmix64 of seed and index), identical on
every platform:

* MLP: X ~ U(-1,1), Y ~ U(-1,1), W1 ~ U(+-1/sqrt(I)), W2 ~ U(+-1/sqrt(H)).
* LM: token ids ~ Zipf(s) over the vocabulary (id 0 most frequent).
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.uint64)
    with np.errstate(over="ignore"):
        z = x + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _stream(seed: int, tag: int, n: int) -> np.ndarray:
    key = splitmix64(np.uint64(seed & 0xFFFFFFFFFFFFFFFF) ^ splitmix64(np.uint64(tag)))
    with np.errstate(over="ignore"):
        return splitmix64(key + np.arange(n, dtype=np.uint64) * _GOLDEN)


def uniform(seed: int, tag: int, shape, lo: float, hi: float) -> np.ndarray:
    """float32 uniform in [lo, hi) from the top 24 bits of each word."""
    n = int(np.prod(shape))
    u = (_stream(seed, tag, n) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def mlp_data(seed: int, samples: int, I: int, H: int, O: int):
    """(X [samples,I], Y [samples,O], W1 [I,H], W2 [H,O])."""
    x = uniform(seed, 1, (samples, I), -1.0, 1.0)
    y = uniform(seed, 2, (samples, O), -1.0, 1.0)
    a1, a2 = 1.0 / np.sqrt(I), 1.0 / np.sqrt(H)
    w1 = uniform(seed, 3, (I, H), -a1, a1)
    w2 = uniform(seed, 4, (H, O), -a2, a2)
    return x, y, w1, w2


def batch(m: np.ndarray, start: int, count: int) -> np.ndarray:
    """Cyclic batch slice (qnn/qnn_mlp_training.cpp:98-104 batch())."""
    rows = (start + np.arange(count)) % m.shape[0]
    return np.ascontiguousarray(m[rows])


def zipf_tokens(seed: int, shape, vocab: int, s: float = 1.1) -> np.ndarray:
    """uint32 ids with P(id = k) proportional to (k+1)^-s, by inverse CDF."""
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    cdf = np.cumsum(ranks ** -s)
    cdf /= cdf[-1]
    n = int(np.prod(shape))
    u = (_stream(seed, 7, n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    ids = np.searchsorted(cdf, u, side="right")
    return np.minimum(ids, vocab - 1).astype(np.uint32).reshape(shape)


def lm_tokens(seed: int, batch_size: int, tokens: int, vocab: int, step: int = 0, s: float = 1.1) -> np.ndarray:
    """[batch, T+1] ids for training step `step` (input ids[:, :T], targets ids[:, 1:])."""
    return zipf_tokens(seed * 1000003 + step, (batch_size, tokens + 1), vocab, s)
