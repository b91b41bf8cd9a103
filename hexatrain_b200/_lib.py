"""ctypes binding of libhexatrain_b200.so (the C ABI in include/hexatrain.h).

The library is built in-tree by ``hexatrain_b200/build.py``.  There is no
fallback: if the shared object is missing or fails to load, importing any
runtime entry point raises ``NativeLibraryError``.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhexatrain_b200.so")

HX_OK = 0
HX_ERR_ARGUMENT = 1
HX_ERR_STATE = 2
HX_ERR_CUDA = 3
HX_ERR_NONFINITE = 4
HX_ERR_MEMORY = 5
HX_ERR_UNSUPPORTED = 6

HX_LM_LEARNED_POSITION = 1
HX_GEMM_AUTO = 0
HX_GEMM_CUDA_CORES = 1
HX_GEMM_TENSOR_CORES = 2
HX_ATTN_AUTO = 0
HX_ATTN_CUDA_CORES = 1
HX_OPT_ADAM = 0
HX_OPT_MUON = 1
HX_OPT_MOMENTUM = 2
HX_STABILITY_LEGACY = 0
HX_STABILITY_WARMUP64 = 1
HX_STABILITY_DECAY_LINEAR = 2
HX_STABILITY_ZERO_OUTPUT_PROJ_BRANCH_INIT = 3
HX_STABILITY_DEPTH_SCALED_BRANCH_INIT = 4
HX_STABILITY_RESIDUAL_BRANCH_SCALING = 5
HX_STABILITY_GRADIENT_CLIP_1 = 6

_fp = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)


class NativeLibraryError(RuntimeError):
    pass


class Metrics(C.Structure):
    _fields_ = [
        ("graph_create_count", C.c_uint64),
        ("graph_finalize_count", C.c_uint64),
        ("graph_execute_count", C.c_uint64),
        ("execute_attempt_count", C.c_uint64),
        ("execute_failure_count", C.c_uint64),
        ("first_failure_call", C.c_int64),
        ("last_execute_us", C.c_double),
        ("total_execute_us", C.c_double),
        ("last_input_bind_us", C.c_double),
        ("last_output_bind_us", C.c_double),
        ("kernel_launches", C.c_uint64),
        ("device_bytes", C.c_uint64),
    ]


class ProfileEntry(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_uint64), ("total_ms", C.c_double), ("flops", C.c_double),
                ("bytes", C.c_double)]


class MlpOutputsC(C.Structure):
    _fields_ = [(n, _fp) for n in ("loss", "w1_next", "w2_next", "prediction", "error", "d_prediction",
                                   "d_w2", "d_hidden")] + [("mask", _u8p)] + \
               [(n, _fp) for n in ("d_z1", "d_w1", "hidden")]


class LmConfigC(C.Structure):
    _fields_ = [("vocab", C.c_uint32), ("tokens", C.c_uint32), ("dim", C.c_uint32), ("ffn", C.c_uint32),
                ("layers", C.c_uint32), ("heads", C.c_uint32), ("eps", C.c_float), ("flags", C.c_uint32)]


class LmOutputsC(C.Structure):
    _fields_ = [(n, _fp) for n in ("loss", "accuracy", "grads", "logits", "probabilities", "d_logits", "output",
                                   "d_output", "layer_input_grads", "head_probabilities")]


class OptimizerConfigC(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("adam_lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("adam_eps", C.c_float), ("muon_lr", C.c_float), ("muon_momentum", C.c_float),
                ("muon_nesterov", C.c_uint32), ("muon_ns_steps", C.c_uint32), ("ns_a", C.c_float),
                ("ns_b", C.c_float), ("ns_c", C.c_float), ("muon_bf16_inputs", C.c_uint32),
                ("momentum_lr", C.c_float), ("momentum", C.c_float)]


class AdamOutputsC(C.Structure):
    _fields_ = [(n, _fp) for n in ("m_next", "v_next", "m_hat", "v_hat", "sqrt_v_hat", "denominator", "divided",
                                   "normalized", "scaled_update", "w_next")]


class NprtInfoC(C.Structure):
    _fields_ = [("version", C.c_uint32), ("seed", C.c_uint32), ("step", C.c_uint32), ("finite", C.c_uint32),
                ("has_adam", C.c_uint32), ("parameter_count", C.c_uint64), ("parameter_hash", C.c_char * 32),
                ("tokenizer_hash", C.c_char * 80)]


class SamplingC(C.Structure):
    _fields_ = [("greedy", C.c_uint32), ("temperature", C.c_float), ("top_k", C.c_uint32), ("seed", C.c_uint64)]


class SamplingAuditC(C.Structure):
    _fields_ = [("ok", C.c_uint32), ("logits_finite", C.c_uint32), ("weight_sum", C.c_double),
                ("probability_sum", C.c_double)]


# name -> (restype, argtypes).  Must match include/hexatrain.h.
SIGNATURES = {
    "hx_runtime_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]),
    "hx_runtime_destroy": (None, [C.c_void_p]),
    "hx_runtime_last_error": (C.c_char_p, [C.c_void_p]),
    "hx_runtime_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "hx_runtime_stream": (C.c_void_p, [C.c_void_p]),
    "hx_runtime_synchronize": (C.c_int, [C.c_void_p]),
    "hx_runtime_metrics": (C.c_int, [C.c_void_p, C.POINTER(Metrics)]),
    "hx_runtime_inject_execute_failure": (C.c_int, [C.c_void_p, C.c_int64]),
    "hx_runtime_check_wait_timeout": (C.c_int, [C.c_void_p, C.c_longlong]),
    "hx_runtime_set_gemm_backend": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_runtime_set_attention_backend": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_runtime_profile": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_runtime_profile_read": (C.c_int, [C.c_void_p, C.POINTER(ProfileEntry), C.c_int, C.POINTER(C.c_int)]),
    "hx_mlp_prepare": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int]),
    "hx_mlp_execute": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p,
                                 C.c_size_t, C.c_void_p, C.c_size_t, C.c_float, C.POINTER(MlpOutputsC)]),
    "hx_mlp_execute_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                        C.POINTER(MlpOutputsC)]),
    "hx_mlp_execute_device_noalloc": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                                C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                                C.c_void_p, C.c_void_p, C.c_void_p]),
    "hx_lm_param_count": (C.c_size_t, [C.POINTER(LmConfigC)]),
    "hx_lm_validate": (C.c_int, [C.POINTER(LmConfigC), C.c_char_p, C.c_size_t]),
    "hx_lm_init_reference": (C.c_int, [C.POINTER(LmConfigC), C.c_uint32, C.c_void_p]),
    "hx_lm_init_normal": (C.c_int, [C.POINTER(LmConfigC), C.c_uint64, C.c_float, C.c_void_p]),
    "hx_lm_prepare": (C.c_int, [C.c_void_p, C.POINTER(LmConfigC), C.c_uint32, C.c_int]),
    "hx_lm_execute": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_float,
                                C.POINTER(LmOutputsC)]),
    "hx_lm_execute_tokens": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                       C.POINTER(LmOutputsC)]),
    "hx_lm_state_upload": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "hx_lm_state_download": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "hx_lm_set_optimizer": (C.c_int, [C.c_void_p, C.POINTER(OptimizerConfigC)]),
    "hx_lm_train_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, _fp]),
    "hx_lm_forward_backward_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_float]),
    "hx_lm_grad_buffer": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]),
    "hx_lm_optimizer_step_device": (C.c_int, [C.c_void_p, C.c_uint32]),
    "hx_lm_loss_device": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "hx_lm_grad_buckets": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.c_int,
                                     C.POINTER(C.c_int)]),
    "hx_lm_enable_bucket_events": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_lm_bucket_wait": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "hx_adam_prepare": (C.c_int, [C.c_void_p, C.c_uint32]),
    "hx_adam_execute": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                  C.c_float, C.c_float, C.c_float, C.POINTER(AdamOutputsC)]),
    "hx_adam_execute_device": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_float, C.c_float, C.c_float, C.c_float, C.POINTER(AdamOutputsC)]),
    "hx_muon_execute": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_float, C.c_float, C.c_int, C.c_uint32, C.c_float, C.c_float, C.c_float,
                                  C.c_int, C.c_void_p, C.c_void_p]),
    "hx_lm_forward_tokens": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "hx_sample_next_token": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(SamplingC), C.c_uint64,
                                       C.POINTER(C.c_uint32), C.POINTER(SamplingAuditC)]),
    "hx_lm_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(SamplingC), C.c_void_p]),
    "hx_bridge_environment_report": (C.c_char_p, []),
    "hx_bridge_status_report": (C.c_char_p, []),
    "hx_bridge_run_execution_mode": (C.c_char_p, [C.c_void_p]),
    "hx_bridge_request_stop": (None, []),
    "hx_bridge_clear_stop": (None, []),
    "hx_momentum_prepare": (C.c_int, [C.c_void_p, C.c_uint32]),
    "hx_momentum_execute": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_float,
                                      C.c_void_p, C.c_void_p]),
    "hx_momentum_execute_device": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                             C.c_float, C.c_void_p, C.c_void_p]),
    "hx_stability_mode_error": (C.c_char_p, [C.c_uint32]),
    "hx_stability_learning_rate": (C.c_float, [C.c_uint32, C.c_float, C.c_uint32, C.c_uint32]),
    "hx_lm_apply_init_stability": (C.c_int, [C.POINTER(LmConfigC), C.c_uint32, C.c_void_p]),
    "hx_lm_set_stability": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_float]),
    "hx_lm_last_gradient_norm": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_float)]),
    "hx_nprt_encoded_bytes": (C.c_size_t, [C.c_void_p, C.c_char_p, C.c_char_p]),
    "hx_nprt_encode": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_char_p, C.c_char_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t]),
    "hx_nprt_decode": (C.c_int, [C.c_void_p, C.c_uint32, C.c_char_p, C.c_void_p, C.c_size_t, C.POINTER(NprtInfoC),
                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]),
    "hx_nprt_checkpoint_name": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                          C.c_char_p, C.c_size_t]),
    "hx_nprt_training_order": (C.c_int, [C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p]),
    "hx_lm_checkpoint_save": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint32, C.c_uint32, C.c_char_p, C.c_char_p]),
    "hx_lm_checkpoint_resume": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint32, C.c_uint32, C.c_char_p,
                                          C.POINTER(NprtInfoC)]),
}

_LIB = None


def load(path: str = LIB_PATH):
    """Load the native library once and bind every declared entry point."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise NativeLibraryError(
            f"{path} is missing: build it with `python hexatrain_b200/build.py` (there is no CPU fallback)")
    try:
        lib = C.CDLL(path)
    except OSError as e:  # pragma: no cover - environment problem
        raise NativeLibraryError(f"cannot load {path}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def ptr(a):
    """Data pointer of a numpy array (or None)."""
    if a is None:
        return None
    return C.c_void_p(a.ctypes.data)


def fptr(a):
    return None if a is None else a.ctypes.data_as(_fp)
