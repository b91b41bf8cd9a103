"""ctypes bindings for the checker libraries.

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke entry and bench.py's
cpu_baseline / reference legs.  The product package never imports this.

  * ``Oracle`` wraps ``oracle/_build/libhxoracle.so``: the C restatement of the
    reference's CPU arithmetic (oracle/hx_oracle.c).
  * ``Reference`` wraps ``oracle/_ref/libhexaref.so``: the reference's own CPU
    sources compiled by oracle/Makefile (present only where the HexaTrain tree
    was available at build time; the built file travels with the repository
    snapshot).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Optional
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libhxoracle.so")
REF_SO = os.path.join(HERE, "_ref", "libhexaref.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


class LmConfig(C.Structure):
    """Mirror of hxo_lm_config (oracle/hx_oracle.h)."""

    _fields_ = [
        ("vocab", C.c_uint32),
        ("tokens", C.c_uint32),
        ("dim", C.c_uint32),
        ("ffn", C.c_uint32),
        ("layers", C.c_uint32),
        ("heads", C.c_uint32),
        ("eps", C.c_float),
        ("learned_position", C.c_int),
    ]

    @staticmethod
    def make(V, T, D, F, L, H, eps=1e-5, learned_position=False):
        return LmConfig(V, T, D, F, L, H, eps, int(bool(learned_position)))


def build(quiet: bool = True, reference_tree: Optional[str] = None) -> None:
    """Build the checker libraries with oracle/Makefile (the reference part
    only when the HexaTrain tree is given, here or by the environment
    variable HEXATRAIN_REFERENCE)."""
    ref = reference_tree or os.environ.get("HEXATRAIN_REFERENCE", "")
    out = subprocess.run(["make", "-s", "-C", HERE, "all", f"REF={ref}"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def param_count(cfg: LmConfig) -> int:
    V, T, D, F, L = cfg.vocab, cfg.tokens, cfg.dim, cfg.ffn, cfg.layers
    return 2 * V * D + (T * D if cfg.learned_position else 0) + L * (4 * D * D + 4 * D + 2 * D * F)


@dataclass
class MlpStep:
    loss: float
    w1_next: np.ndarray
    w2_next: np.ndarray
    z1: np.ndarray
    h: np.ndarray
    p: np.ndarray
    e: np.ndarray
    dp: np.ndarray
    dw2: np.ndarray
    dh: np.ndarray
    mask: np.ndarray
    dz1: np.ndarray
    dw1: np.ndarray


@dataclass
class LmStep:
    loss: float
    accuracy: float
    grads: np.ndarray
    logits: np.ndarray
    probs: np.ndarray
    dlogits: np.ndarray
    output: np.ndarray
    layer_input_grads: np.ndarray
    head_probs: np.ndarray


def _mlp_call(fn, B, I, H, O, x, y, w1, w2, lr):
    f = lambda *s: np.zeros(s, np.float32)
    out = MlpStep(0.0, f(I, H), f(H, O), f(B, H), f(B, H), f(B, O), f(B, O), f(B, O),
                  f(H, O), f(B, H), np.zeros((B, H), np.uint8), f(B, H), f(I, H))
    loss = C.c_float()
    rc = fn(B, I, H, O, *[np.ascontiguousarray(a, np.float32) for a in (x, y, w1, w2)], C.c_float(lr),
            C.byref(loss), out.w1_next, out.w2_next, out.z1, out.h, out.p, out.e, out.dp, out.dw2,
            out.dh, out.mask, out.dz1, out.dw1)
    if rc != 0:
        raise ValueError("mlp step rejected its arguments")
    out.loss = loss.value
    return out


class Oracle:
    """The C restatement (oracle/hx_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        self.lib = L = C.CDLL(path)
        L.hxo_mlp_step.restype = C.c_int
        L.hxo_mlp_step.argtypes = [C.c_int] * 4 + [_f32p] * 4 + [C.c_float, C.POINTER(C.c_float)] + \
            [_f32p] * 9 + [_u8p, _f32p, _f32p]
        L.hxo_matmul.argtypes = [C.c_int] * 3 + [_f32p] * 3
        L.hxo_mse.restype = C.c_float
        L.hxo_mse.argtypes = [C.c_size_t, _f32p, _f32p]
        L.hxo_linear_forward_backward.restype = C.c_float
        L.hxo_linear_forward_backward.argtypes = [C.c_int, C.c_int] + [_f32p] * 8
        L.hxo_sgd.argtypes = [C.c_size_t, _f32p, _f32p, C.c_float]
        L.hxo_lm_param_count.restype = C.c_size_t
        L.hxo_lm_param_count.argtypes = [C.POINTER(LmConfig)]
        L.hxo_lm_fixed_position.argtypes = [C.POINTER(LmConfig), _f32p]
        L.hxo_lm_forward_backward.restype = C.c_int
        L.hxo_lm_forward_backward.argtypes = [C.POINTER(LmConfig), _u32p, _u32p, _f32p,
                                              C.POINTER(C.c_float), C.POINTER(C.c_float), _f32p] + [C.c_void_p] * 7
        L.hxo_lm_batch_gradients.restype = C.c_int
        L.hxo_lm_batch_gradients.argtypes = [C.POINTER(LmConfig), C.c_int, _u32p, _f32p, _f32p,
                                             C.POINTER(C.c_float), C.c_int]
        L.hxo_adam.argtypes = [C.c_size_t] + [_f32p] * 4 + [C.c_float] * 6 + [C.c_void_p] * 5
        L.hxo_adam_correction.restype = C.c_float
        L.hxo_adam_correction.argtypes = [C.c_double, C.c_int]
        L.hxo_muon.argtypes = [C.c_int, C.c_int] + [_f32p] * 3 + [C.c_float, C.c_float, C.c_int, C.c_int,
                                                                   C.c_float, C.c_float, C.c_float, C.c_int,
                                                                   _f32p, _f32p]
        L.hxo_round_bf16.restype = C.c_float
        L.hxo_round_bf16.argtypes = [C.c_float]

    # -- MLP -------------------------------------------------------------
    def mlp_step(self, x, y, w1, w2, lr) -> MlpStep:
        B, I = x.shape
        H, O = w2.shape
        return _mlp_call(self.lib.hxo_mlp_step, B, I, H, O, x, y, w1, w2, lr)

    def matmul(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.zeros((a.shape[0], b.shape[1]), np.float32)
        self.lib.hxo_matmul(a.shape[0], b.shape[1], a.shape[1], a, b, out)
        return out

    def mse(self, p, y):
        p = np.ascontiguousarray(p, np.float32).ravel()
        y = np.ascontiguousarray(y, np.float32).ravel()
        return self.lib.hxo_mse(p.size, p, y)

    def linear_forward_backward(self, x, target, w):
        B, D = x.shape
        f = lambda *s: np.zeros(s, np.float32)
        pred, err, dp, dw, dx = f(B, D), f(B, D), f(B, D), f(D, D), f(B, D)
        loss = self.lib.hxo_linear_forward_backward(B, D, *[np.ascontiguousarray(a, np.float32) for a in (x, target, w)],
                                                    pred, err, dp, dw, dx)
        return loss, pred, err, dp, dw, dx

    def sgd(self, w, dw, lr):
        w = np.array(w, np.float32, copy=True)
        self.lib.hxo_sgd(w.size, w.ravel(), np.ascontiguousarray(dw, np.float32).ravel(), lr)
        return w

    # -- LM ----------------------------------------------------------------
    def param_count(self, cfg: LmConfig) -> int:
        return int(self.lib.hxo_lm_param_count(C.byref(cfg)))

    def fixed_position(self, cfg: LmConfig):
        out = np.zeros((cfg.tokens, cfg.dim), np.float32)
        self.lib.hxo_lm_fixed_position(C.byref(cfg), out)
        return out

    def lm_forward_backward(self, cfg: LmConfig, inputs, targets, params, want_all=True) -> LmStep:
        T, V, D, L, H = cfg.tokens, cfg.vocab, cfg.dim, cfg.layers, cfg.heads
        inputs = np.ascontiguousarray(inputs, np.uint32)
        targets = np.ascontiguousarray(targets, np.uint32)
        params = np.ascontiguousarray(params, np.float32)
        grads = np.zeros(self.param_count(cfg), np.float32)
        z = lambda *s: np.zeros(s, np.float32) if want_all else None
        logits, probs, dlogits = z(T, V), z(T, V), z(T, V)
        output, dout, lig, hp = z(T, D), z(T, D), z(L, T, D), z(L, H, T, T)
        loss, acc = C.c_float(), C.c_float()
        rc = self.lib.hxo_lm_forward_backward(C.byref(cfg), inputs, targets, params, C.byref(loss), C.byref(acc),
                                              grads, _ptr(logits), _ptr(probs), _ptr(dlogits), _ptr(output),
                                              _ptr(dout), _ptr(lig), _ptr(hp))
        if rc != 0:
            raise ValueError("invalid LM configuration or tokens")
        return LmStep(loss.value, acc.value, grads, logits, probs, dlogits, output, lig, hp)

    def lm_batch_gradients(self, cfg: LmConfig, tokens, params, threads=1):
        tokens = np.ascontiguousarray(tokens, np.uint32)
        B = tokens.shape[0]
        grads = np.zeros(self.param_count(cfg), np.float32)
        loss = C.c_float()
        rc = self.lib.hxo_lm_batch_gradients(C.byref(cfg), B, tokens, np.ascontiguousarray(params, np.float32),
                                             grads, C.byref(loss), threads)
        if rc != 0:
            raise ValueError("invalid LM configuration or tokens")
        return grads, loss.value

    def adam(self, w, g, m, v, lr, c1, c2, beta1=0.9, beta2=0.999, eps=1e-8):
        w, g, m, v = [np.ascontiguousarray(a, np.float32).ravel() for a in (w, g, m, v)]
        outs = [np.zeros_like(w) for _ in range(5)]
        self.lib.hxo_adam(w.size, w, g, m, v, lr, beta1, beta2, eps, c1, c2, *[_ptr(o) for o in outs])
        return tuple(outs)  # m_next, v_next, m_hat, v_hat, w_next

    def adam_correction(self, beta: float, step: int) -> float:
        return float(self.lib.hxo_adam_correction(beta, step))

    def muon(self, w, g, buf, lr, momentum=0.95, nesterov=True, ns_steps=5,
             abc=(3.4445, -4.7750, 2.0315), bf16_inputs=True):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        w_next = np.zeros_like(w)
        buf_next = np.zeros_like(w)
        self.lib.hxo_muon(rows, cols, w, np.ascontiguousarray(g, np.float32), np.ascontiguousarray(buf, np.float32),
                          lr, momentum, int(nesterov), ns_steps, abc[0], abc[1], abc[2], int(bf16_inputs),
                          w_next, buf_next)
        return w_next, buf_next

    def round_bf16(self, x: float) -> float:
        return float(self.lib.hxo_round_bf16(x))

    def nprt_encode(self, cfg: LmConfig, seed, step, params, m, v, kind=None, hash=None) -> bytes:
        """hxo_nprt_encode; raises ValueError when the writer refuses."""
        L = self.lib
        L.hxo_nprt_encode.restype = C.c_size_t
        L.hxo_nprt_encode.argtypes = [C.POINTER(LmConfig), C.c_uint32, C.c_uint32, C.c_char_p, C.c_char_p,
                                      _f32p, _f32p, _f32p, C.c_void_p, C.c_size_t]
        args = [C.byref(cfg), seed, step, None if kind is None else kind.encode(),
                None if hash is None else hash.encode()] + [np.ascontiguousarray(a, np.float32) for a in (params, m, v)]
        need = L.hxo_nprt_encode(*args, None, 0)
        if need == 0:
            raise ValueError("oracle writer refused")
        out = np.zeros(need, np.uint8)
        L.hxo_nprt_encode(*args, out.ctypes.data, need)
        return out.tobytes()

    def nprt_parameter_hash(self, cfg: LmConfig, params) -> str:
        self.lib.hxo_nprt_parameter_hash.argtypes = [C.POINTER(LmConfig), _f32p, C.c_char_p]
        out = C.create_string_buffer(32)
        self.lib.hxo_nprt_parameter_hash(C.byref(cfg), np.ascontiguousarray(params, np.float32), out)
        return out.value.decode()

    def momentum(self, w, g, v, lr, momentum):
        L = self.lib
        L.hxo_momentum.argtypes = [C.c_size_t, _f32p, _f32p, _f32p, C.c_float, C.c_float, _f32p, _f32p]
        w, g, v = (np.ascontiguousarray(a, np.float32).ravel() for a in (w, g, v))
        wn, vn = np.empty_like(w), np.empty_like(w)
        L.hxo_momentum(w.size, w, g, v, lr, momentum, wn, vn)
        return wn, vn

    def stability_learning_rate(self, mode, base, step, total):
        self.lib.hxo_stability_learning_rate.restype = C.c_float
        self.lib.hxo_stability_learning_rate.argtypes = [C.c_uint32, C.c_float, C.c_uint32, C.c_uint32]
        return self.lib.hxo_stability_learning_rate(mode, base, step, total)

    def apply_init_stability(self, cfg: LmConfig, mode, params):
        self.lib.hxo_apply_init_stability.argtypes = [C.POINTER(LmConfig), C.c_uint32, _f32p]
        out = np.array(params, np.float32, copy=True).ravel()
        self.lib.hxo_apply_init_stability(C.byref(cfg), mode, out)
        return out

    def gradient_norm(self, cfg: LmConfig, grads, threshold=0.0):
        """(norm, clip scale)."""
        self.lib.hxo_gradient_norm.restype = C.c_double
        self.lib.hxo_gradient_norm.argtypes = [C.POINTER(LmConfig), _f32p, C.c_float, C.POINTER(C.c_float)]
        clip = C.c_float()
        n = self.lib.hxo_gradient_norm(C.byref(cfg), np.ascontiguousarray(grads, np.float32).ravel(), threshold,
                                       C.byref(clip))
        return n, clip.value

    def nprt_training_order(self, records, steps, batch):
        self.lib.hxo_nprt_training_order.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p]
        out = np.zeros(steps * batch, np.uint64)
        self.lib.hxo_nprt_training_order(records, steps, batch, out.ctypes.data)
        return out


class Reference:
    """The reference's own CPU code (oracle/_ref/libhexaref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = L = C.CDLL(path)
        L.hxr_last_error.restype = C.c_char_p
        L.hxr_param_count.restype = C.c_int
        L.hxr_param_count.argtypes = [C.POINTER(LmConfig)]
        L.hxr_matmul.argtypes = [C.c_int] * 3 + [_f32p] * 3
        L.hxr_linear_forward_backward.restype = C.c_float
        L.hxr_linear_forward_backward.argtypes = [C.c_int, C.c_int] + [_f32p] * 3 + [C.c_float] + [_f32p] * 6
        L.hxr_mlp_step.restype = C.c_int
        L.hxr_mlp_step.argtypes = [C.c_int] * 4 + [_f32p] * 4 + [C.c_float, C.POINTER(C.c_float)] + \
            [_f32p] * 9 + [_u8p, _f32p, _f32p]
        L.hxr_lm_fixed_position.argtypes = [C.POINTER(LmConfig), _f32p]
        L.hxr_lm_initial_parameters.restype = C.c_int
        L.hxr_lm_initial_parameters.argtypes = [C.POINTER(LmConfig), C.c_uint32, _f32p]
        L.hxr_lm_validate.restype = C.c_int
        L.hxr_lm_validate.argtypes = [C.POINTER(LmConfig)]
        L.hxr_lm_forward_backward.restype = C.c_int
        L.hxr_lm_forward_backward.argtypes = [C.POINTER(LmConfig), _u32p, _u32p, _f32p, C.c_float,
                                              C.POINTER(C.c_float), C.POINTER(C.c_float), _f32p] + [C.c_void_p] * 7
        L.hxr_lm_adam.restype = C.c_int
        L.hxr_lm_adam.argtypes = [C.POINTER(LmConfig)] + [_f32p] * 4 + [C.c_float] * 6 + [C.c_void_p] * 5
        L.hxr_lm_train_step.restype = C.c_int
        L.hxr_lm_train_step.argtypes = [C.POINTER(LmConfig), C.c_int, _u32p, _f32p, _f32p, _f32p, C.c_float,
                                        C.c_int, C.c_int, C.POINTER(C.c_float)]
        L.hxr_lm_gradient_check.restype = C.c_int
        L.hxr_lm_gradient_check.argtypes = [C.c_uint32, C.c_float, C.POINTER(C.c_float), C.POINTER(C.c_float)]

    def last_error(self) -> str:
        return self.lib.hxr_last_error().decode()

    def mlp_step(self, x, y, w1, w2, lr) -> MlpStep:
        B, I = x.shape
        H, O = w2.shape
        return _mlp_call(self.lib.hxr_mlp_step, B, I, H, O, x, y, w1, w2, lr)

    def matmul(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.zeros((a.shape[0], b.shape[1]), np.float32)
        self.lib.hxr_matmul(a.shape[0], b.shape[1], a.shape[1], a, b, out)
        return out

    def linear_forward_backward(self, x, target, w, lr=0.0):
        B, D = x.shape
        f = lambda *s: np.zeros(s, np.float32)
        pred, err, dp, dw, dx, wn = f(B, D), f(B, D), f(B, D), f(D, D), f(B, D), f(D, D)
        loss = self.lib.hxr_linear_forward_backward(B, D, *[np.ascontiguousarray(a, np.float32) for a in (x, target, w)],
                                                    lr, pred, err, dp, dw, dx, wn)
        return loss, pred, err, dp, dw, dx, wn

    def param_count(self, cfg):
        return int(self.lib.hxr_param_count(C.byref(cfg)))

    def validate(self, cfg) -> bool:
        return self.lib.hxr_lm_validate(C.byref(cfg)) == 0

    def fixed_position(self, cfg):
        out = np.zeros((cfg.tokens, cfg.dim), np.float32)
        self.lib.hxr_lm_fixed_position(C.byref(cfg), out)
        return out

    def initial_parameters(self, cfg, seed):
        out = np.zeros(self.param_count(cfg), np.float32)
        if self.lib.hxr_lm_initial_parameters(C.byref(cfg), seed, out) != 0:
            raise ValueError(self.last_error())
        return out

    def lm_forward_backward(self, cfg, inputs, targets, params, lr=0.0) -> LmStep:
        T, V, D, L, H = cfg.tokens, cfg.vocab, cfg.dim, cfg.layers, cfg.heads
        z = lambda *s: np.zeros(s, np.float32)
        grads = z(self.param_count(cfg))
        logits, probs, dlogits, output, lig, hp = z(T, V), z(T, V), z(T, V), z(T, D), z(L, T, D), z(L, H, T, T)
        nxt = z(self.param_count(cfg))
        loss, acc = C.c_float(), C.c_float()
        rc = self.lib.hxr_lm_forward_backward(C.byref(cfg), np.ascontiguousarray(inputs, np.uint32),
                                              np.ascontiguousarray(targets, np.uint32),
                                              np.ascontiguousarray(params, np.float32), lr, C.byref(loss),
                                              C.byref(acc), grads, _ptr(nxt), _ptr(logits), _ptr(probs),
                                              _ptr(dlogits), _ptr(output), _ptr(lig), _ptr(hp))
        if rc != 0:
            raise ValueError(self.last_error())
        step = LmStep(loss.value, acc.value, grads, logits, probs, dlogits, output, lig, hp)
        step.next = nxt
        return step

    def adam(self, cfg, w, g, m, v, lr, c1, c2, beta1=0.9, beta2=0.999, eps=1e-8):
        outs = [np.zeros_like(w) for _ in range(5)]
        rc = self.lib.hxr_lm_adam(C.byref(cfg), *[np.ascontiguousarray(a, np.float32) for a in (w, g, m, v)],
                                  lr, beta1, beta2, eps, c1, c2, *[_ptr(o) for o in outs])
        if rc != 0:
            raise ValueError(self.last_error())
        return tuple(outs)

    def lm_train_step(self, cfg, tokens, params, m, v, lr, step, threads=1):
        """In-place batched Adam step; returns the mean loss."""
        loss = C.c_float()
        tokens = np.ascontiguousarray(tokens, np.uint32)
        rc = self.lib.hxr_lm_train_step(C.byref(cfg), tokens.shape[0], tokens, params, m, v, lr, step, threads,
                                        C.byref(loss))
        if rc != 0:
            raise ValueError(self.last_error())
        return loss.value

    def momentum(self, cfg, w, g, v, lr, momentum):
        L = self.lib
        L.hxr_lm_momentum.restype = C.c_int
        L.hxr_lm_momentum.argtypes = [C.POINTER(LmConfig), _f32p, _f32p, _f32p, C.c_float, C.c_float, _f32p, _f32p]
        w, g, v = (np.ascontiguousarray(a, np.float32).ravel() for a in (w, g, v))
        wn, vn = np.empty_like(w), np.empty_like(w)
        if L.hxr_lm_momentum(C.byref(cfg), w, g, v, lr, momentum, wn, vn) != 0:
            raise RuntimeError(self.last_error())
        return wn, vn

    def stability_learning_rate(self, mode, base, step, total):
        self.lib.hxr_stability_learning_rate.restype = C.c_float
        self.lib.hxr_stability_learning_rate.argtypes = [C.c_uint32, C.c_float, C.c_uint32, C.c_uint32]
        return self.lib.hxr_stability_learning_rate(mode, base, step, total)

    def apply_init_stability(self, cfg, mode, params):
        self.lib.hxr_apply_init_stability.restype = C.c_int
        self.lib.hxr_apply_init_stability.argtypes = [C.POINTER(LmConfig), C.c_uint32, _f32p]
        out = np.array(params, np.float32, copy=True).ravel()
        if self.lib.hxr_apply_init_stability(C.byref(cfg), mode, out) != 0:
            raise RuntimeError(self.last_error())
        return out

    def sample_next_token(self, logits, step=0, greedy=False, temperature=1.0, top_k=0, seed=0):
        """(token, ok) from the reference's greedyArgmax / sampleTopKChecked."""
        L = self.lib
        L.hxr_sample_next_token.restype = C.c_uint32
        L.hxr_sample_next_token.argtypes = [_f32p, C.c_uint32, C.c_int, C.c_float, C.c_uint32, C.c_uint64,
                                            C.c_uint64, C.POINTER(C.c_int)]
        row = np.ascontiguousarray(logits, np.float32).ravel()
        ok = C.c_int()
        tok = L.hxr_sample_next_token(row, row.size, int(greedy), temperature, top_k, seed, step, C.byref(ok))
        return int(tok), bool(ok.value)

    def stability_mode_error(self, mode) -> str:
        self.lib.hxr_stability_mode_error.restype = C.c_char_p
        self.lib.hxr_stability_mode_error.argtypes = [C.c_uint32]
        return self.lib.hxr_stability_mode_error(mode).decode()

    def gradient_check(self, seed=20260725, eps=1e-3):
        a, r = C.c_float(), C.c_float()
        ok = self.lib.hxr_lm_gradient_check(seed, eps, C.byref(a), C.byref(r))
        return bool(ok), a.value, r.value


REF_CKPT_SO = os.path.join(HERE, "_ref", "libhexaref_ckpt.so")


class ReferenceCheckpoint:
    """The reference's own NPRTCKPT codec (oracle/_ref/libhexaref_ckpt.so):
    nprtSaveCheckpointV2 / nprtLoadCheckpointForGeneration / nprtParameterHash
    / nprtTrainingOrder / nprtCheckpointName from
    qnn/qnn_transformer_training.cpp, compiled by oracle/Makefile."""

    def __init__(self, path: str = REF_CKPT_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = L = C.CDLL(path)
        u = C.c_uint32
        L.hxr_nprt_save.restype = C.c_int
        L.hxr_nprt_save.argtypes = [C.c_char_p] + [u] * 8 + [_f32p] * 3 + [C.c_char_p, C.c_char_p]
        L.hxr_nprt_load.restype = C.c_int
        L.hxr_nprt_load.argtypes = [C.c_char_p] + [u] * 7 + [C.c_char_p, C.POINTER(u), C.POINTER(u),
                                                             C.POINTER(C.c_int), C.POINTER(C.c_int)] + \
            [C.c_void_p] * 3 + [C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t]
        L.hxr_nprt_parameter_hash.argtypes = [u] * 6 + [_f32p, C.c_char_p, C.c_size_t]
        L.hxr_nprt_training_order.argtypes = [C.c_uint64, u, u, C.c_void_p]
        L.hxr_nprt_checkpoint_name.argtypes = [u] * 6 + [C.c_char_p, C.c_size_t]

    @staticmethod
    def _dims(cfg):
        return [cfg.vocab, cfg.tokens, cfg.dim, cfg.ffn, cfg.layers, cfg.heads]

    def save(self, path, cfg, seed, step, params, m, v, kind=None, hash=None) -> bool:
        f = [np.ascontiguousarray(a, np.float32) for a in (params, m, v)]
        return self.lib.hxr_nprt_save(path.encode(), *self._dims(cfg), seed, step, *f,
                                      None if kind is None else kind.encode(),
                                      None if hash is None else hash.encode()) == 1

    def load(self, path, cfg, seed, n, tokenizer_hash=None):
        """Returns (ok, error, info dict, params, m, v)."""
        step, version = C.c_uint32(), C.c_uint32()
        finite, has_adam = C.c_int(), C.c_int()
        p, m, v = (np.zeros(n, np.float32) for _ in range(3))
        ph, err = C.create_string_buffer(64), C.create_string_buffer(256)
        ok = self.lib.hxr_nprt_load(path.encode(), *self._dims(cfg), seed,
                                    None if tokenizer_hash is None else tokenizer_hash.encode(),
                                    C.byref(step), C.byref(version), C.byref(finite), C.byref(has_adam),
                                    p.ctypes.data, m.ctypes.data, v.ctypes.data, ph, 64, err, 256) == 1
        info = dict(step=step.value, version=version.value, finite=bool(finite.value),
                    has_adam=bool(has_adam.value), parameter_hash=ph.value.decode())
        return ok, err.value.decode(), info, p, m, v

    def parameter_hash(self, cfg, params) -> str:
        out = C.create_string_buffer(64)
        self.lib.hxr_nprt_parameter_hash(*self._dims(cfg), np.ascontiguousarray(params, np.float32), out, 64)
        return out.value.decode()

    def gradient_norm(self, cfg, grads) -> float:
        self.lib.hxr_gradient_norm.restype = C.c_double
        self.lib.hxr_gradient_norm.argtypes = [C.c_uint32] * 6 + [_f32p]
        return self.lib.hxr_gradient_norm(*self._dims(cfg), np.ascontiguousarray(grads, np.float32).ravel())

    def training_order(self, records, steps, batch):
        out = np.zeros(steps * batch, np.uint64)
        self.lib.hxr_nprt_training_order(records, steps, batch, out.ctypes.data)
        return out

    def checkpoint_name(self, seed, layers, T, D, F, step) -> str:
        out = C.create_string_buffer(128)
        self.lib.hxr_nprt_checkpoint_name(seed, layers, T, D, F, step, out, 128)
        return out.value.decode()


def reference_checkpoint_available() -> bool:
    return os.path.exists(REF_CKPT_SO)


def reference_available() -> bool:
    return os.path.exists(REF_SO)


REF_DRIVER_SO = os.path.join(HERE, "_ref", "libhexaref_driver.so")


class ReferenceDriver:
    """The reference's own experiment drivers (trainFullStep for the MLP
    modes, languageModelAdam for the LM modes), compiled with the product's
    Runtime adapter in place of the stub/QAIRT runtime
    (oracle/_ref/libhexaref_driver.so).  run_mode returns the driver's
    KEY=VALUE report as a dict plus the raw text."""

    def __init__(self, path: str = REF_DRIVER_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        self.lib.hxd_run_mode.restype = C.c_long
        self.lib.hxd_run_mode.argtypes = [C.c_int] * 10 + [C.c_float, C.c_ulonglong, C.c_int, C.c_int,
                                                           C.c_char_p, C.c_size_t]

    def run_mode(self, mode, batch=8, dimension=128, hidden=128, output=64, steps=100, epochs=0,
                 sample_count=512, measured_steps=0, correctness_interval=0, learning_rate=0.1,
                 seed=20260710, benchmark=False, feed_forward=32):
        cap = 1 << 16
        while True:
            buf = C.create_string_buffer(cap)
            n = self.lib.hxd_run_mode(mode, batch, dimension, hidden, output, steps, epochs, sample_count,
                                      measured_steps, correctness_interval, learning_rate, seed, int(benchmark),
                                      feed_forward, buf, cap)
            if n < cap:
                break
            cap = int(n) + 1
        text = buf.value.decode(errors="replace")
        kv = {}
        for line in text.splitlines():
            if "=" in line:
                k, v = line.split("=", 1)
                kv.setdefault(k, v)
        return kv, text


def reference_driver_available() -> bool:
    return os.path.exists(REF_DRIVER_SO)
