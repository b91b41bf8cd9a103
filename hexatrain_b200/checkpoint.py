"""NPRTCKPTV2 / V3 checkpoints of the LM training state (host side).

Thin wrappers over the C codec in libhexatrain_b200.so (hx_nprt_*), which
restates the reference's nprtSaveCheckpointV2 / nprtLoadCheckpointForGeneration
(qnn/qnn_transformer_training.cpp:5164-5252, :5390-5522).  The flat float32
buffers are in registry order, the order hx_lm_state_download returns.
Errors raise ``CheckpointError`` carrying the reference's NPRT_CKPT_* code.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib


class CheckpointError(RuntimeError):
    pass


@dataclass
class CheckpointInfo:
    version: int
    seed: int
    step: int
    finite: bool
    has_adam: bool
    parameter_count: int
    parameter_hash: str
    tokenizer_hash: str


def _info(c: _lib.NprtInfoC) -> CheckpointInfo:
    return CheckpointInfo(int(c.version), int(c.seed), int(c.step), bool(c.finite), bool(c.has_adam),
                          int(c.parameter_count), c.parameter_hash.decode(), c.tokenizer_hash.decode())


def _b(s):
    return None if s is None else s.encode()


def _f32(a, n):
    a = np.ascontiguousarray(a, dtype=np.float32).ravel()
    if a.size != n:
        raise CheckpointError(f"NPRT_CKPT_ELEMENT_COUNT_MISMATCH: expected {n} floats, got {a.size}")
    return a


def encode(config, seed: int, step: int, params, adam_m, adam_v, tokenizer_kind: str | None = None,
           tokenizer_hash: str | None = None) -> bytes:
    """nprtSaveCheckpointV2 into bytes (V3 at vocabulary 1024)."""
    lib = _lib.load()
    cfg = config.to_c()
    n = config.parameter_count()
    p, m, v = _f32(params, n), _f32(adam_m, n), _f32(adam_v, n)
    cap = lib.hx_nprt_encoded_bytes(C.byref(cfg), _b(tokenizer_kind), _b(tokenizer_hash))
    out = (C.c_uint8 * cap)()
    written = C.c_size_t(0)
    err = C.create_string_buffer(256)
    rc = lib.hx_nprt_encode(C.byref(cfg), seed, step, _b(tokenizer_kind), _b(tokenizer_hash), p.ctypes.data,
                            m.ctypes.data, v.ctypes.data, out, cap, C.byref(written), err, 256)
    if rc != _lib.HX_OK:
        raise CheckpointError(err.value.decode())
    return bytes(out[:written.value])


def decode(config, data: bytes, expected_seed: int, tokenizer_hash: str | None = None):
    """Validates and decodes; returns (info, params, adam_m, adam_v) with the
    moments None for a V1 file."""
    lib = _lib.load()
    cfg = config.to_c()
    n = config.parameter_count()
    p, m, v = (np.zeros(n, np.float32) for _ in range(3))
    info = _lib.NprtInfoC()
    err = C.create_string_buffer(256)
    buf = (C.c_uint8 * len(data)).from_buffer_copy(data) if data else (C.c_uint8 * 1)()
    rc = lib.hx_nprt_decode(C.byref(cfg), expected_seed, _b(tokenizer_hash), buf, len(data), C.byref(info),
                            p.ctypes.data, m.ctypes.data, v.ctypes.data, err, 256)
    if rc != _lib.HX_OK:
        raise CheckpointError(err.value.decode())
    out = _info(info)
    return out, p, (m if out.has_adam else None), (v if out.has_adam else None)


def checkpoint_name(seed: int, layers: int, tokens: int, dimension: int, feed_forward_dimension: int,
                    step: int) -> str:
    """nicopedia_checkpoint::checkpointName."""
    buf = C.create_string_buffer(128)
    rc = _lib.load().hx_nprt_checkpoint_name(seed, layers, tokens, dimension, feed_forward_dimension, step, buf, 128)
    if rc != _lib.HX_OK:
        raise CheckpointError("checkpoint name does not fit")
    return buf.value.decode()


def training_order(record_count: int, steps: int, batch: int) -> np.ndarray:
    """nprtTrainingOrder: record index per (step, slot), flat [steps*batch]."""
    out = np.zeros(steps * batch, np.uint64)
    rc = _lib.load().hx_nprt_training_order(record_count, steps, batch, out.ctypes.data)
    if rc != _lib.HX_OK:
        raise CheckpointError("NPRT_TRAIN_CACHE_EMPTY")
    return out
