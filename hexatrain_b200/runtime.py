"""Python host surface mirroring the reference's runtime seam.

``Runtime`` has the method names, argument meaning and error behaviour of
``phonelm::qnn::Runtime`` (app/src/main/cpp/qnn/qnn_runtime.h:250-451) for the
training-step path: every call returns ``True``/``False`` and leaves a
human-readable message in ``last_error`` (the reference's ``std::string&
error`` out-parameter); output objects are resized by the callee.  All work
runs in libhexatrain_b200.so through the C ABI of include/hexatrain.h.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _lib
from ._lib import fptr, ptr


@dataclass
class RuntimeOptions:
    """Subset of RuntimeOptions (qnn/qnn_runtime.h:133-171) that applies here.

    ``fail_graph_execute_at`` makes the execute call with that attempt index
    report failure after its device work completed (host-side injection; no
    device fault)."""

    fail_graph_execute_at: int = -1


@dataclass
class RuntimeMetrics:
    graph_create_count: int = 0
    graph_finalize_count: int = 0
    graph_execute_count: int = 0
    execute_attempt_count: int = 0
    execute_failure_count: int = 0
    first_failure_call: int = -1
    last_execute_us: float = 0.0
    total_execute_us: float = 0.0
    last_input_bind_us: float = 0.0
    last_output_bind_us: float = 0.0
    kernel_launches: int = 0
    device_bytes: int = 0


@dataclass
class MlpFullStepOutputs:
    """MlpFullStepOutputs (qnn/qnn_runtime.h:236-249)."""

    loss: float = 0.0
    w1_next: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    w2_next: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    prediction: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    hidden: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    error: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    d_prediction: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    d_w2: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    d_hidden: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    mask: np.ndarray = field(default_factory=lambda: np.zeros(0, np.uint8))
    d_z1: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    d_w1: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))


@dataclass
class TinyTransformerTrainingOutputs:
    """TinyTransformerTrainingOutputs (qnn/qnn_runtime.h:209-222), with the
    gradients as one flat registry-ordered array."""

    loss: float = 0.0
    accuracy: float = 0.0
    gradients: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    logits: Optional[np.ndarray] = None
    probabilities: Optional[np.ndarray] = None
    d_logits: Optional[np.ndarray] = None
    output: Optional[np.ndarray] = None
    d_output: Optional[np.ndarray] = None
    layer_input_gradients: Optional[np.ndarray] = None
    head_probabilities: Optional[np.ndarray] = None


@dataclass
class AdamOptimizerOutputs:
    """AdamOptimizerOutputs (qnn/qnn_runtime.h:230-235)."""

    first_moment_next: np.ndarray = None
    second_moment_next: np.ndarray = None
    first_moment_hat: np.ndarray = None
    second_moment_hat: np.ndarray = None
    second_root: np.ndarray = None
    denominator: np.ndarray = None
    divided_update: np.ndarray = None
    normalized_update: np.ndarray = None
    scaled_update: np.ndarray = None
    weight_next: np.ndarray = None


@dataclass
class MomentumOptimizerOutputs:
    """MomentumOptimizerOutputs (qnn/qnn_runtime.h:227-229)."""

    velocity_next: np.ndarray = None
    weight_next: np.ndarray = None


def sample_next_token(logits, step: int = 0, greedy: bool = True, temperature: float = 0.0, top_k: int = 0,
                      seed: int = 0):
    """greedyArgmax / sampleTopKChecked (nicopedia_generation.h:286-395).
    Returns (token, audit dict); raises ValueError on non-finite input."""
    row = np.ascontiguousarray(logits, np.float32).ravel()
    tok, audit = C.c_uint32(), _lib.SamplingAuditC()
    s = _lib.SamplingC(int(greedy), temperature, top_k, seed)
    rc = _lib.load().hx_sample_next_token(row.ctypes.data, row.size, C.byref(s), step, C.byref(tok), C.byref(audit))
    info = dict(ok=bool(audit.ok), logits_finite=bool(audit.logits_finite), weight_sum=audit.weight_sum,
                probability_sum=audit.probability_sum)
    if rc != 0:
        raise ValueError(f"sampling failed ({rc}): {info}")
    return int(tok.value), info


def stability_learning_rate(mode: int, base: float, step: int, total_steps: int) -> float:
    """stabilityLearningRate (training_stability.h:88-99)."""
    return float(_lib.load().hx_stability_learning_rate(mode, base, step, total_steps))


def apply_init_stability(cfg: "LmConfig", mode: int, params: np.ndarray) -> np.ndarray:
    """applyInitStability (training_stability.h:104-121) on a copy of a flat
    registry-ordered parameter array."""
    out = np.array(params, dtype=np.float32, copy=True).ravel()
    rc = _lib.load().hx_lm_apply_init_stability(C.byref(cfg.to_c()), mode, out.ctypes.data)
    if rc != 0:
        msg = _lib.load().hx_stability_mode_error(mode)
        raise ValueError(msg.decode() if msg else "invalid arguments")
    return out


@dataclass
class OptimizerConfig:
    """hx_optimizer_config.  Defaults: Adam 1e-3/0.9/0.999/1e-8; Muon lr
    0.02, momentum 0.95 with Nesterov, 5 quintic Newton-Schulz steps
    (3.4445, -4.7750, 2.0315) on bf16-rounded operands."""

    kind: int = _lib.HX_OPT_ADAM
    adam_lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    adam_eps: float = 1e-8
    muon_lr: float = 0.02
    muon_momentum: float = 0.95
    muon_nesterov: bool = True
    muon_ns_steps: int = 5
    ns_a: float = 3.4445
    ns_b: float = -4.7750
    ns_c: float = 2.0315
    muon_bf16_inputs: bool = True
    momentum_lr: float = 0.01
    momentum: float = 0.95

    def to_c(self) -> _lib.OptimizerConfigC:
        return _lib.OptimizerConfigC(self.kind, self.adam_lr, self.beta1, self.beta2, self.adam_eps, self.muon_lr,
                                     self.muon_momentum, int(self.muon_nesterov), self.muon_ns_steps, self.ns_a,
                                     self.ns_b, self.ns_c, int(self.muon_bf16_inputs), self.momentum_lr,
                                     self.momentum)


@dataclass(frozen=True)
class LmConfig:
    """tiny_lm::Config (tiny_language_model_cpu.h:10-14) plus the
    learned-position switch."""

    vocabulary_size: int = 32
    tokens: int = 8
    dimension: int = 16
    feed_forward_dimension: int = 32
    num_layers: int = 1
    num_heads: int = 1
    epsilon: float = 1e-5
    learned_position: bool = False

    def to_c(self) -> _lib.LmConfigC:
        return _lib.LmConfigC(self.vocabulary_size, self.tokens, self.dimension, self.feed_forward_dimension,
                              self.num_layers, self.num_heads, self.epsilon,
                              _lib.HX_LM_LEARNED_POSITION if self.learned_position else 0)

    @property
    def head_dim(self) -> int:
        return self.dimension // self.num_heads

    def parameter_count(self) -> int:
        return int(_lib.load().hx_lm_param_count(C.byref(self.to_c())))

    def registry(self):
        """[(name, offset, shape)] in registry order
        (tiny_language_model_cpu.cpp parameterRegistry)."""
        V, T, D, F = self.vocabulary_size, self.tokens, self.dimension, self.feed_forward_dimension
        out, off = [], 0

        def add(name, shape):
            nonlocal off
            out.append((name, off, shape))
            off += int(np.prod(shape))

        add("token_embedding", (V, D))
        if self.learned_position:
            add("position_embedding", (T, D))
        for i in range(self.num_layers):
            p = f"layer_{i:03d}."
            for n, s in (("norm1_gamma", (D,)), ("norm1_beta", (D,)), ("wq", (D, D)), ("wk", (D, D)),
                         ("wv", (D, D)), ("wo", (D, D)), ("norm2_gamma", (D,)), ("norm2_beta", (D,)),
                         ("ffn_w1", (D, F)), ("ffn_w2", (F, D))):
                add(p + n, s)
        add("output_projection", (D, V))
        return out

    def validate(self) -> tuple[bool, str]:
        buf = C.create_string_buffer(512)
        rc = _lib.load().hx_lm_validate(C.byref(self.to_c()), buf, 512)
        return rc == 0, buf.value.decode()

    def init_reference(self, seed: int) -> np.ndarray:
        """tiny_lm::initialParameters (tiny_language_model_cpu.cpp:69-70)."""
        p = np.zeros(self.parameter_count(), np.float32)
        rc = _lib.load().hx_lm_init_reference(C.byref(self.to_c()), seed, ptr(p))
        if rc != 0:
            raise ValueError("invalid LM configuration")
        return p

    def init_normal(self, seed: int, std: float = 0.02) -> np.ndarray:
        p = np.zeros(self.parameter_count(), np.float32)
        rc = _lib.load().hx_lm_init_normal(C.byref(self.to_c()), seed, std, ptr(p))
        if rc != 0:
            raise ValueError("invalid LM configuration")
        return p


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Runtime:
    """CUDA runtime seam: one device, one stream, prepared plans."""

    def __init__(self):
        self._rt = None
        self.last_error = ""
        self._options = RuntimeOptions()
        self._mlp_shape = None
        self._mlp_diag = False
        self._lm_cfg: Optional[LmConfig] = None
        self._lm_batch = 0
        self._lm_diag = False
        self._adam_n = 0
        self._lib = _lib.load()

    # -- lifecycle --------------------------------------------------------
    def initialize(self, device: int = 0) -> bool:
        """Runtime::initialize (qnn/qnn_runtime.h:266)."""
        if self._rt is not None:
            return True
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        rc = self._lib.hx_runtime_create(device, C.byref(h), err, 512)
        if rc != 0:
            self.last_error = err.value.decode()
            return False
        self._rt = h
        self._apply_options()
        return True

    def close(self):
        if self._rt is not None:
            self._lib.hx_runtime_destroy(self._rt)
            self._rt = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _ok(self, rc: int) -> bool:
        if rc == 0:
            self.last_error = ""
            return True
        msg = self._lib.hx_runtime_last_error(self._rt) if self._rt is not None else b"runtime not initialized"
        self.last_error = (msg or b"").decode()
        return False

    def _need(self) -> bool:
        if self._rt is None:
            self.last_error = "runtime not initialized"
            return False
        return True

    def set_options(self, options: RuntimeOptions) -> None:
        self._options = options
        if self._rt is not None:
            self._apply_options()

    def _apply_options(self):
        self._lib.hx_runtime_inject_execute_failure(self._rt, int(self._options.fail_graph_execute_at))

    def set_stream(self, stream_handle: int) -> bool:
        """Run on an external cudaStream_t (e.g. torch.cuda.current_stream().cuda_stream)."""
        return self._need() and self._ok(self._lib.hx_runtime_set_stream(self._rt, C.c_void_p(stream_handle or None)))

    def synchronize(self) -> bool:
        return self._need() and self._ok(self._lib.hx_runtime_synchronize(self._rt))

    def metrics(self) -> RuntimeMetrics:
        m = _lib.Metrics()
        if self._rt is not None:
            self._lib.hx_runtime_metrics(self._rt, C.byref(m))
        return RuntimeMetrics(**{f: getattr(m, f) for f, _ in _lib.Metrics._fields_})

    def check_wait_timeout(self, cycles: int) -> bool:
        """Failure-path self-test of the kernels' bounded waits: one thread
        waits `cycles` clock cycles on an mbarrier nothing arrives at.  Returns
        False with a DEVICE_WAIT_TIMEOUT message in last_error (expected)."""
        return self._need() and self._ok(self._lib.hx_runtime_check_wait_timeout(self._rt, int(cycles)))

    def set_gemm_backend(self, backend: int) -> bool:
        """0 = auto (tensor cores for large aligned GEMMs), 1 = CUDA cores, 2 = tensor cores when aligned."""
        return self._need() and self._ok(self._lib.hx_runtime_set_gemm_backend(self._rt, int(backend)))

    def set_attention_backend(self, backend: int) -> bool:
        """0 = auto (tensor cores for head dimension 32, T <= 256), 1 = CUDA cores everywhere."""
        return self._need() and self._ok(self._lib.hx_runtime_set_attention_backend(self._rt, int(backend)))

    def profile(self, enable: bool) -> bool:
        """Start/stop per-kernel-class CUDA-event timing (hx_runtime_profile)."""
        return self._need() and self._ok(self._lib.hx_runtime_profile(self._rt, int(bool(enable))))

    def profile_read(self) -> dict:
        """{kernel class: dict(launches, total_ms, flops, bytes)}; clears the records."""
        arr = (_lib.ProfileEntry * 16)()
        n = C.c_int(0)
        if not (self._need() and self._ok(self._lib.hx_runtime_profile_read(self._rt, arr, 16, C.byref(n)))):
            raise RuntimeError(self.last_error)
        return {arr[i].name.decode(): dict(launches=int(arr[i].launches), total_ms=float(arr[i].total_ms),
                                           flops=float(arr[i].flops), bytes=float(arr[i].bytes))
                for i in range(n.value)}

    def api_trace_summary(self) -> str:
        """KEY=VALUE counters in the style of Runtime::apiTraceSummary."""
        m = self.metrics()
        return "".join(f"api_trace_{k}={v}\n" for k, v in m.__dict__.items())

    # -- MLP full step ------------------------------------------------------
    def prepare_mlp_full_step(self, batch_size: int, input_dimension: int, hidden_dimension: int,
                              output_dimension: int, diagnostic_outputs: bool) -> bool:
        """Runtime::prepareMlpFullStep (qnn/qnn_runtime.h:422-424)."""
        if not self._need():
            return False
        ok = self._ok(self._lib.hx_mlp_prepare(self._rt, batch_size, input_dimension, hidden_dimension,
                                               output_dimension, int(bool(diagnostic_outputs))))
        if ok:
            self._mlp_shape = (batch_size, input_dimension, hidden_dimension, output_dimension)
            self._mlp_diag = bool(diagnostic_outputs)
        return ok

    def execute_mlp_full_step(self, input, target, w1_current, w2_current, learning_rate: float,
                              outputs: MlpFullStepOutputs) -> bool:
        """Runtime::executeMlpFullStep (qnn/qnn_runtime.h:425-430)."""
        if not self._need():
            return False
        if self._mlp_shape is None:
            self.last_error = "full step graph not prepared"
            return False
        B, I, H, O = self._mlp_shape
        x, y, w1, w2 = (_f32(a).ravel() for a in (input, target, w1_current, w2_current))
        loss = np.zeros(1, np.float32)
        outputs.w1_next = np.empty(I * H, np.float32)
        outputs.w2_next = np.empty(H * O, np.float32)
        o = _lib.MlpOutputsC()
        o.loss, o.w1_next, o.w2_next = fptr(loss), fptr(outputs.w1_next), fptr(outputs.w2_next)
        if self._mlp_diag:
            outputs.prediction = np.empty(B * O, np.float32)
            outputs.error = np.empty(B * O, np.float32)
            outputs.d_prediction = np.empty(B * O, np.float32)
            outputs.d_w2 = np.empty(H * O, np.float32)
            outputs.d_hidden = np.empty(B * H, np.float32)
            outputs.mask = np.empty(B * H, np.uint8)
            outputs.d_z1 = np.empty(B * H, np.float32)
            outputs.d_w1 = np.empty(I * H, np.float32)
            outputs.hidden = np.empty(B * H, np.float32)
            o.prediction, o.error, o.d_prediction = fptr(outputs.prediction), fptr(outputs.error), fptr(outputs.d_prediction)
            o.d_w2, o.d_hidden, o.d_z1, o.d_w1 = fptr(outputs.d_w2), fptr(outputs.d_hidden), fptr(outputs.d_z1), fptr(outputs.d_w1)
            o.mask = outputs.mask.ctypes.data_as(C.POINTER(C.c_uint8))
            o.hidden = fptr(outputs.hidden)
        else:
            for n in ("prediction", "hidden", "error", "d_prediction", "d_w2", "d_hidden", "d_z1", "d_w1"):
                setattr(outputs, n, np.zeros(0, np.float32))
            outputs.mask = np.zeros(0, np.uint8)
        rc = self._lib.hx_mlp_execute(self._rt, ptr(x), x.size, ptr(y), y.size, ptr(w1), w1.size, ptr(w2), w2.size,
                                      learning_rate, C.byref(o))
        outputs.loss = float(loss[0])
        return self._ok(rc)

    def execute_mlp_full_step_device(self, x: int, y: int, w1: int, w2: int, learning_rate: float, loss: int,
                                     w1_next: int, w2_next: int, **diag) -> bool:
        """Device-pointer form (ping-pong weights, no per-step weight copies).
        Pointers are integers (e.g. torch.Tensor.data_ptr())."""
        if not self._need():
            return False
        o = _lib.MlpOutputsC()
        o.loss = C.cast(C.c_void_p(loss), _lib._fp)
        o.w1_next = C.cast(C.c_void_p(w1_next), _lib._fp)
        o.w2_next = C.cast(C.c_void_p(w2_next), _lib._fp)
        for k, v in diag.items():
            if v:
                setattr(o, k, C.cast(C.c_void_p(v), _lib._u8p if k == "mask" else _lib._fp))
        return self._ok(self._lib.hx_mlp_execute_device(self._rt, C.c_void_p(x), C.c_void_p(y), C.c_void_p(w1),
                                                        C.c_void_p(w2), learning_rate, C.byref(o)))

    def execute_mlp_full_step_device_noalloc(self, batch_size: int, input_dimension: int, hidden_dimension: int,
                                             output_dimension: int, x: int, y: int, w1: int, w2: int,
                                             learning_rate: float, loss: int, w1_next: int, w2_next: int) -> bool:
        """The device-pointer step for callers that cannot let the library
        allocate device memory (their allocator owns the GPU's memory, or
        cudaMalloc is not allowed on their step path).  Needs no prepare; the
        intermediates use a fixed 4 MiB device array shared by every call on
        the device, so calls overlapping on the GPU race.  Not part of the
        reference's Runtime."""
        if not self._need():
            return False
        return self._ok(self._lib.hx_mlp_execute_device_noalloc(
            self._rt, batch_size, input_dimension, hidden_dimension, output_dimension, C.c_void_p(x), C.c_void_p(y),
            C.c_void_p(w1), C.c_void_p(w2), learning_rate, C.c_void_p(loss), C.c_void_p(w1_next),
            C.c_void_p(w2_next)))

    # -- tiny Transformer LM -------------------------------------------------
    def prepare_tiny_transformer_training(self, tokens: int, dimension: int, feed_forward_dimension: int,
                                          epsilon: float, diagnostic_outputs: bool, vocabulary_size: int,
                                          num_layers: int = 1, num_heads: int = 1, batch: int = 1,
                                          learned_position: bool = False) -> bool:
        """Runtime::prepareTinyTransformerTraining (qnn/qnn_runtime.h:398-408),
        generalized builder; ``batch`` sequences per execute."""
        if not self._need():
            return False
        cfg = LmConfig(vocabulary_size, tokens, dimension, feed_forward_dimension, num_layers, num_heads, epsilon,
                       learned_position)
        ok = self._ok(self._lib.hx_lm_prepare(self._rt, C.byref(cfg.to_c()), batch, int(bool(diagnostic_outputs))))
        if ok:
            self._lm_cfg, self._lm_batch, self._lm_diag = cfg, batch, bool(diagnostic_outputs)
        return ok

    def prepare_lm(self, cfg: LmConfig, batch: int, diagnostic_outputs: bool = False) -> bool:
        return self.prepare_tiny_transformer_training(cfg.tokens, cfg.dimension, cfg.feed_forward_dimension,
                                                      cfg.epsilon, diagnostic_outputs, cfg.vocabulary_size,
                                                      cfg.num_layers, cfg.num_heads, batch, cfg.learned_position)

    def _lm_outputs(self, outputs: TinyTransformerTrainingOutputs):
        cfg, B = self._lm_cfg, self._lm_batch
        V, T, D, L, H = cfg.vocabulary_size, cfg.tokens, cfg.dimension, cfg.num_layers, cfg.num_heads
        loss, acc = np.zeros(1, np.float32), np.zeros(1, np.float32)
        outputs.gradients = np.empty(cfg.parameter_count(), np.float32)
        o = _lib.LmOutputsC()
        o.loss, o.accuracy, o.grads = fptr(loss), fptr(acc), fptr(outputs.gradients)
        if self._lm_diag:
            outputs.logits = np.empty((B * T, V), np.float32)
            outputs.probabilities = np.empty((B * T, V), np.float32)
            outputs.d_logits = np.empty((B * T, V), np.float32)
            outputs.output = np.empty((B * T, D), np.float32)
            outputs.d_output = np.empty((B * T, D), np.float32)
            outputs.layer_input_gradients = np.empty((L, B * T, D), np.float32)
            outputs.head_probabilities = np.empty((L, B, H, T, T), np.float32)
            o.logits, o.probabilities, o.d_logits = fptr(outputs.logits), fptr(outputs.probabilities), fptr(outputs.d_logits)
            o.output, o.d_output = fptr(outputs.output), fptr(outputs.d_output)
            o.layer_input_grads, o.head_probabilities = fptr(outputs.layer_input_gradients), fptr(outputs.head_probabilities)
        return o, loss, acc

    def execute_tiny_transformer_training(self, input, target, current, learning_rate: float,
                                          outputs: TinyTransformerTrainingOutputs) -> bool:
        """Runtime::executeTinyTransformerTraining (qnn/qnn_runtime.h:409-412):
        one-hot [batch*T, V] input/target rows, flat registry-ordered
        parameters, learning_rate must be 0."""
        if not self._need():
            return False
        if self._lm_cfg is None:
            self.last_error = "generalized tiny training graph not prepared"
            return False
        x, y, p = _f32(input).ravel(), _f32(target).ravel(), _f32(current).ravel()
        n = self._lm_batch * self._lm_cfg.tokens * self._lm_cfg.vocabulary_size
        if x.size != n or y.size != n:
            self.last_error = "generalized tiny training buffer schema"
            return False
        o, loss, acc = self._lm_outputs(outputs)
        rc = self._lib.hx_lm_execute(self._rt, ptr(x), ptr(y), ptr(p), p.size, learning_rate, C.byref(o))
        outputs.loss, outputs.accuracy = float(loss[0]), float(acc[0])
        return self._ok(rc)

    def execute_tiny_transformer_training_tokens(self, input_tokens, target_tokens, current,
                                                 outputs: TinyTransformerTrainingOutputs) -> bool:
        if not self._need():
            return False
        if self._lm_cfg is None:
            self.last_error = "generalized tiny training graph not prepared"
            return False
        a = np.ascontiguousarray(input_tokens, np.uint32).ravel()
        b = np.ascontiguousarray(target_tokens, np.uint32).ravel()
        n = self._lm_batch * self._lm_cfg.tokens
        if a.size != n or b.size != n:
            self.last_error = "generalized tiny training buffer schema"
            return False
        p = _f32(current).ravel()
        o, loss, acc = self._lm_outputs(outputs)
        rc = self._lib.hx_lm_execute_tokens(self._rt, ptr(a), ptr(b), ptr(p), p.size, C.byref(o))
        outputs.loss, outputs.accuracy = float(loss[0]), float(acc[0])
        return self._ok(rc)

    # device-resident training state
    def lm_state_upload(self, params, adam_m=None, adam_v=None, muon_buffer=None) -> bool:
        if not self._need():
            return False
        p = _f32(params).ravel()
        arrs = [None if a is None else _f32(a).ravel() for a in (adam_m, adam_v, muon_buffer)]
        return self._ok(self._lib.hx_lm_state_upload(self._rt, ptr(p), *[ptr(a) for a in arrs], p.size))

    def lm_state_download(self):
        n = self._lm_cfg.parameter_count()
        outs = [np.empty(n, np.float32) for _ in range(4)]
        if not self._ok(self._lib.hx_lm_state_download(self._rt, *[ptr(a) for a in outs], n)):
            raise RuntimeError(self.last_error)
        return tuple(outs)  # params, adam_m, adam_v, muon_buffer

    def execute_tiny_transformer_forward_only_tokens(self, tokens, params=None):
        """executeTinyTransformerForwardOnly (qnn/qnn_runtime.h:418-421) on
        token ids [batch, T]; params None uses the device state.  Returns
        logits [batch*T, V] or None (last_error set)."""
        if not self._need():
            return None
        cfg = self._lm_cfg
        t = np.ascontiguousarray(tokens, np.uint32).ravel()
        logits = np.empty((t.size, cfg.vocabulary_size), np.float32)
        p = None if params is None else _f32(params).ravel()
        ok = self._ok(self._lib.hx_lm_forward_tokens(self._rt, ptr(t), None if p is None else ptr(p),
                                                     0 if p is None else p.size, ptr(logits)))
        return logits if ok else None

    def lm_generate(self, prompts, max_new: int, greedy: bool = True, temperature: float = 0.0, top_k: int = 0,
                    seed: int = 0):
        """The prepared generation loop on the device state: prompts [batch,
        prompt_len] ids -> generated ids [batch, max_new] (None on failure)."""
        if not self._need():
            return None
        pr = np.ascontiguousarray(prompts, np.uint32)
        if pr.ndim == 1:
            pr = pr[None, :]
        out = np.zeros((pr.shape[0], max_new), np.uint32)
        s = _lib.SamplingC(int(greedy), temperature, top_k, seed)
        ok = self._ok(self._lib.hx_lm_generate(self._rt, ptr(pr), pr.shape[1], max_new, C.byref(s), ptr(out)))
        return out if ok else None

    def lm_checkpoint_save(self, path: str, seed: int, step: int, tokenizer_kind: str | None = None,
                           tokenizer_hash: str | None = None) -> bool:
        """nprtSaveCheckpointV2 of the device state (qnn_transformer_training.cpp:5171-5252):
        parameters and Adam moments, written to path.tmp and renamed."""
        enc = (lambda s: None if s is None else s.encode())
        return self._need() and self._ok(self._lib.hx_lm_checkpoint_save(
            self._rt, path.encode(), seed, step, enc(tokenizer_kind), enc(tokenizer_hash)))

    def lm_checkpoint_resume(self, path: str, seed: int, step: int = 0, tokenizer_hash: str | None = None):
        """Canonical resume (qnn_transformer_training.cpp:7068-7109).  Returns
        the CheckpointInfo, or None with last_error set (RESUME_* codes)."""
        from .checkpoint import _info
        info = _lib.NprtInfoC()
        ok = self._need() and self._ok(self._lib.hx_lm_checkpoint_resume(
            self._rt, path.encode(), seed, step, None if tokenizer_hash is None else tokenizer_hash.encode(),
            C.byref(info)))
        return _info(info) if ok else None

    def lm_set_stability(self, mode: int, total_steps: int = 0, clip_threshold: float = 0.0) -> bool:
        """Step-side training-stability mode (training_stability.h) and the
        global-norm gradient clip threshold (0 = off)."""
        return self._need() and self._ok(self._lib.hx_lm_set_stability(self._rt, mode, total_steps, clip_threshold))

    def lm_last_gradient_norm(self):
        """(pre-clip global gradient norm, clip scale) of the last optimizer step."""
        n, s = C.c_double(), C.c_float()
        if not (self._need() and self._ok(self._lib.hx_lm_last_gradient_norm(self._rt, C.byref(n), C.byref(s)))):
            raise RuntimeError(self.last_error)
        return n.value, s.value

    def lm_set_optimizer(self, opt: OptimizerConfig) -> bool:
        return self._need() and self._ok(self._lib.hx_lm_set_optimizer(self._rt, C.byref(opt.to_c())))

    def lm_train_step(self, tokens, step: int):
        """One batched step: tokens [batch, T+1] ids.  Returns (ok, mean loss)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        loss = C.c_float(0.0)
        ok = self._need() and self._ok(self._lib.hx_lm_train_step(self._rt, ptr(t), step, C.byref(loss)))
        return ok, float(loss.value)

    def lm_forward_backward_device(self, tokens_ptr: int, grad_scale: float) -> bool:
        return self._need() and self._ok(
            self._lib.hx_lm_forward_backward_device(self._rt, C.c_void_p(tokens_ptr), grad_scale))

    def lm_grad_buffer(self):
        p, n = C.c_void_p(), C.c_size_t()
        if not self._ok(self._lib.hx_lm_grad_buffer(self._rt, C.byref(p), C.byref(n))):
            raise RuntimeError(self.last_error)
        return int(p.value), int(n.value)

    def lm_grad_buckets(self):
        """[(offset, count)] of the gradient buffer's buckets, in the order
        the backward finishes them (hx_lm_grad_buckets)."""
        n = C.c_int()
        if not self._ok(self._lib.hx_lm_grad_buckets(self._rt, None, None, 0, C.byref(n))):
            raise RuntimeError(self.last_error)
        off = (C.c_size_t * n.value)()
        cnt = (C.c_size_t * n.value)()
        if not self._ok(self._lib.hx_lm_grad_buckets(self._rt, off, cnt, n.value, C.byref(n))):
            raise RuntimeError(self.last_error)
        return [(int(off[i]), int(cnt[i])) for i in range(n.value)]

    def lm_enable_bucket_events(self, enable: bool) -> bool:
        return self._need() and self._ok(self._lib.hx_lm_enable_bucket_events(self._rt, int(bool(enable))))

    def lm_bucket_wait(self, bucket: int, stream_handle: int) -> bool:
        """Make cudaStream_t `stream_handle` wait for bucket `bucket` of the
        most recent forward_backward (hx_lm_bucket_wait)."""
        return self._need() and self._ok(self._lib.hx_lm_bucket_wait(self._rt, int(bucket),
                                                                     C.c_void_p(stream_handle or None)))

    def lm_optimizer_step_device(self, step: int) -> bool:
        return self._need() and self._ok(self._lib.hx_lm_optimizer_step_device(self._rt, step))

    def lm_loss_device(self) -> int:
        p = C.c_void_p()
        if not self._ok(self._lib.hx_lm_loss_device(self._rt, C.byref(p))):
            raise RuntimeError(self.last_error)
        return int(p.value)

    # -- Adam ------------------------------------------------------------------
    def prepare_adam_optimizer(self, elements: int) -> bool:
        """Runtime::prepareAdamOptimizer (qnn/qnn_runtime.h:360)."""
        if not self._need():
            return False
        ok = self._ok(self._lib.hx_adam_prepare(self._rt, elements))
        if ok:
            self._adam_n = elements
        return ok

    def execute_adam_optimizer(self, current, gradient, first_moment, second_moment, learning_rate: float,
                               gradient_scale: float, first_correction: float, second_correction: float,
                               outputs: AdamOptimizerOutputs) -> bool:
        """Runtime::executeAdamOptimizer (qnn/qnn_runtime.h:361-369)."""
        if not self._need():
            return False
        arrs = [_f32(a).ravel() for a in (current, gradient, first_moment, second_moment)]
        if self._adam_n == 0 or any(a.size != self._adam_n for a in arrs):
            self.last_error = "Adam optimizer buffer size or scalar"
            return False
        names = ("first_moment_next", "second_moment_next", "first_moment_hat", "second_moment_hat", "second_root",
                 "denominator", "divided_update", "normalized_update", "scaled_update", "weight_next")
        o = _lib.AdamOutputsC()
        for cname, pname in zip([f for f, _ in _lib.AdamOutputsC._fields_], names):
            arr = np.empty(self._adam_n, np.float32)
            setattr(outputs, pname, arr)
            setattr(o, cname, fptr(arr))
        rc = self._lib.hx_adam_execute(self._rt, *[ptr(a) for a in arrs], learning_rate, gradient_scale,
                                       first_correction, second_correction, C.byref(o))
        return self._ok(rc)

    # -- momentum SGD --------------------------------------------------------------
    def prepare_momentum_optimizer(self, elements: int) -> bool:
        """Runtime::prepareMomentumOptimizer (qnn/qnn_runtime.h:353)."""
        if not self._need():
            return False
        ok = self._ok(self._lib.hx_momentum_prepare(self._rt, elements))
        if ok:
            self._momentum_n = elements
        return ok

    def execute_momentum_optimizer(self, current, gradient, velocity, learning_rate: float, momentum: float,
                                   outputs: "MomentumOptimizerOutputs") -> bool:
        """Runtime::executeMomentumOptimizer (qnn/qnn_runtime.h:354-359)."""
        if not self._need():
            return False
        arrs = [_f32(a).ravel() for a in (current, gradient, velocity)]
        n = getattr(self, "_momentum_n", 0)
        if n == 0 or any(a.size != n for a in arrs):
            self.last_error = "momentum optimizer buffer size or scalar"
            return False
        outputs.velocity_next = np.empty(n, np.float32)
        outputs.weight_next = np.empty(n, np.float32)
        return self._ok(self._lib.hx_momentum_execute(self._rt, *[ptr(a) for a in arrs], learning_rate, momentum,
                                                      ptr(outputs.velocity_next), ptr(outputs.weight_next)))

    # -- Muon --------------------------------------------------------------------
    def execute_muon(self, weight, gradient, momentum_buffer, learning_rate: float, momentum: float = 0.95,
                     nesterov: bool = True, ns_steps: int = 5, abc=(3.4445, -4.7750, 2.0315),
                     bf16_inputs: bool = True):
        """Returns (ok, weight_next, momentum_buffer_next)."""
        w = _f32(weight)
        rows, cols = w.shape
        wn, bn = np.empty_like(w), np.empty_like(w)
        ok = self._need() and self._ok(self._lib.hx_muon_execute(
            self._rt, rows, cols, ptr(w), ptr(_f32(gradient)), ptr(_f32(momentum_buffer)), learning_rate, momentum,
            int(nesterov), ns_steps, abc[0], abc[1], abc[2], int(bf16_inputs), ptr(wn), ptr(bn)))
        return ok, wn, bn
