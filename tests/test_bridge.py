"""The host-app bridge (include/hexatrain_bridge.h) and its JNI wrapper.

The core restates the reference's NativeBridge entry points
(app/src/main/cpp/native_bridge.cpp) over this library and returns KEY=VALUE
reports.  The JNI wrapper (hexatrain_b200/jni/native_bridge_b200.cpp) is
compiled here against tests/jni_double/jni.h -- no JDK is installed -- and
driven through a ctypes JNIEnv whose function table records strings and
progress calls.  GPU runs are checked against replays through the Python
runtime on the same seeded data.
"""
import ctypes as C
import os

import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import HAS_GPU, ROOT
from hexatrain_b200 import _lib, build, data

JNI_PREFIX = "Java_com_yuubinnkyoku_phonelm_NativeBridge_"
# The Kotlin declarations these symbols bind (NativeBridge.kt:15-59).
JNI_NAMES = ["nativeGetEnvironmentInfo", "nativeGetQnnStatus", "nativeRunExecutionMode", "nativeRequestStop",
             "nativeClearStop"]


def parse(report: str) -> dict:
    out = {}
    for line in report.splitlines():
        if "=" in line:
            k, v = line.split("=", 1)
            out[k] = v
    return out


class Run(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("execution_mode", "batch_size", "dimension", "hidden_dimension",
                                         "output_dimension", "steps", "warmup_steps")] + \
               [("learning_rate", C.c_float), ("seed", C.c_int64)] + \
               [(n, C.c_int32) for n in ("sample_count", "epochs", "measured_steps", "correctness_interval",
                                         "benchmark_mode", "seed_selection_mode", "training_stability_mode",
                                         "depth_pair_init_mode", "checkpoint_selection_mode",
                                         "diagnostic_trajectory")] + \
               [("diagnostic_checkpoint_dir", C.c_char_p), ("diagnostic_resume_step", C.c_int32),
                ("diagnostic_checkpoint_interval", C.c_int32),
                ("progress", C.CFUNCTYPE(None, C.c_void_p, C.c_char_p)), ("progress_context", C.c_void_p)]


def run_core(**kw) -> dict:
    lines = []
    cb = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p)(lambda ctx, line: lines.append(line.decode()))
    r = Run(**{k: (v.encode() if isinstance(v, str) else v) for k, v in kw.items()})
    r.progress = cb
    rep = parse(_lib.load().hx_bridge_run_execution_mode(C.byref(r)).decode())
    rep["_progress"] = lines
    return rep


# ---- a JNIEnv for the wrapper ----------------------------------------------
_F = C.CFUNCTYPE


class _Table(C.Structure):
    _fields_ = [("NewStringUTF", _F(C.c_void_p, C.c_void_p, C.c_char_p)),
                ("GetStringUTFChars", _F(C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p)),
                ("ReleaseStringUTFChars", _F(None, C.c_void_p, C.c_void_p, C.c_void_p)),
                ("GetObjectClass", _F(C.c_void_p, C.c_void_p, C.c_void_p)),
                ("GetMethodID", _F(C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_char_p)),
                ("CallVoidMethodOneArg", _F(None, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p)),
                ("ExceptionCheck", _F(C.c_uint8, C.c_void_p)),
                ("ExceptionClear", _F(None, C.c_void_p)),
                ("DeleteLocalRef", _F(None, C.c_void_p, C.c_void_p))]


class _Env(C.Structure):
    _fields_ = [("functions", C.POINTER(_Table))]


class FakeJni:
    """Strings are integer handles; the method signature asked for is kept."""

    def __init__(self):
        self.strings, self.buffers, self.progress, self.method_sig = {}, {}, [], None

        def new_string(env, s):
            h = len(self.strings) + 1
            self.strings[h] = s.decode()
            return h

        def get_chars(env, h, copy):
            buf = C.create_string_buffer(self.strings[h].encode())
            self.buffers[h] = buf
            return C.addressof(buf)

        def get_method(env, cls, name, sig):
            self.method_sig = (name.decode(), sig.decode())
            return 77

        funcs = [new_string, get_chars, lambda env, h, p: None, lambda env, o: 55, get_method,
                 lambda env, o, m, arg: self.progress.append(self.strings[arg]), lambda env: 0,
                 lambda env: None, lambda env, o: None]
        self._callbacks = [t(f) for (_, t), f in zip(_Table._fields_, funcs)]  # kept alive with the table
        self.table = _Table(*self._callbacks)
        self.env = _Env(C.pointer(self.table))

    def text(self, handle) -> str:
        return self.strings[handle]


@pytest.fixture(scope="module")
def jni(tmp_path_factory):
    _lib.load()  # the wrapper's DT_NEEDED resolves to the loaded library by soname
    out = str(tmp_path_factory.mktemp("jni") / "libhexatrain_b200_jni_test.so")
    assert build.build_jni(include_dirs=[os.path.join(ROOT, "tests", "jni_double")], out=out) == out
    lib = C.CDLL(out)
    for n in ("nativeGetEnvironmentInfo", "nativeGetQnnStatus"):
        getattr(lib, JNI_PREFIX + n).restype = C.c_void_p
    f = getattr(lib, JNI_PREFIX + "nativeRunExecutionMode")
    f.restype = C.c_void_p
    f.argtypes = [C.c_void_p, C.c_void_p] + [C.c_int32] * 7 + [C.c_float, C.c_int64] + [C.c_int32] * 4 + \
        [C.c_uint8] + [C.c_int32] * 4 + [C.c_uint8, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]
    return lib


def test_wrapper_exports_the_reference_jni_symbols(jni):
    for n in JNI_NAMES:
        assert hasattr(jni, JNI_PREFIX + n), n
    assert hasattr(jni, "JNI_OnLoad")


def test_reports_on_the_host(jni):
    env = parse(_lib.load().hx_bridge_environment_report().decode())
    assert env["backend"] == "CUDA_B200" and int(env["cuda_device_count"]) >= (1 if HAS_GPU else 0)
    status = parse(_lib.load().hx_bridge_status_report().decode())
    assert status["status"] == ("AVAILABLE" if HAS_GPU else "UNAVAILABLE") and status["cpu_fallback"] == "false"
    fake = FakeJni()
    h = getattr(jni, JNI_PREFIX + "nativeGetEnvironmentInfo")(C.byref(fake.env), None)
    assert fake.text(h).startswith("ENVIRONMENT\n")


def test_unsupported_modes_fail_closed(jni):
    for mode in (0, 9, 47, 100, 1000):
        rep = run_core(execution_mode=mode)
        assert rep["status"] == "FAILED" and rep["failure_classification"] == "UNSUPPORTED_EXECUTION_MODE"
    fake = FakeJni()
    h = getattr(jni, JNI_PREFIX + "nativeRunExecutionMode")(C.byref(fake.env), None, 47, *([0] * 6), 0.0, 0,
                                                            *([0] * 4), 0, *([0] * 4), 0, None, 0, 0, None)
    assert parse(fake.text(h))["failure_classification"] == "UNSUPPORTED_EXECUTION_MODE"
    # a stop requested outside a run is cleared by nativeClearStop
    lib = _lib.load()
    lib.hx_bridge_request_stop()
    lib.hx_bridge_clear_stop()


def _mlp_replay(seed, N, B, I, H, O, steps, lr):
    x, y, w1, w2 = data.mlp_data(seed, N, I, H, O)
    rt, ev = hx.Runtime(), hx.Runtime()
    assert rt.initialize(0) and ev.initialize(0)
    assert rt.prepare_mlp_full_step(B, I, H, O, False) and ev.prepare_mlp_full_step(N, I, H, O, False)

    def loss(a, b):
        o = hx.MlpFullStepOutputs()
        assert ev.execute_mlp_full_step(x, y, a, b, 0.0, o), ev.last_error
        return o.loss

    first = loss(w1, w2)
    for s in range(steps):
        o = hx.MlpFullStepOutputs()
        assert rt.execute_mlp_full_step(data.batch(x, s * B, B), data.batch(y, s * B, B), w1, w2, lr, o)
        w1, w2 = o.w1_next.reshape(w1.shape), o.w2_next.reshape(w2.shape)
    last = loss(w1, w2)
    rt.close()
    ev.close()
    return first, last


def _mlp_oracle_replay(oracle, seed, N, B, I, H, O, steps, lr):
    """The same run on the oracle (the reference's pass() + sgdUpdate)."""
    x, y, w1, w2 = data.mlp_data(seed, N, I, H, O)
    first = oracle.mlp_step(x, y, w1, w2, 0.0).loss
    for s in range(steps):
        r = oracle.mlp_step(data.batch(x, s * B, B), data.batch(y, s * B, B), w1, w2, lr)
        w1, w2 = r.w1_next.reshape(w1.shape), r.w2_next.reshape(w2.shape)
    return first, oracle.mlp_step(x, y, w1, w2, 0.0).loss


@pytest.mark.gpu
def test_mlp_full_step_mode_matches_runtime_replay(jni, oracle):
    N, B, I, H, O, seed, lr = 64, 8, 128, 128, 64, 20260710, 0.5
    fake = FakeJni()
    h = getattr(jni, JNI_PREFIX + "nativeRunExecutionMode")(C.byref(fake.env), None, 32, B, I, H, O, 0, 0, lr, seed,
                                                            N, 2, 0, 0, 0, 0, 0, 0, 0, 0, None, 0, 0, 55)
    rep = parse(fake.text(h))
    assert rep["status"] == "SUCCESS", rep
    assert rep["steps"] == "16" and rep["training_graph_execute_count"] == "16"
    assert fake.method_sig == ("onNativeProgress", "(Ljava/lang/String;)V") and fake.progress
    first, last = _mlp_replay(seed, N, B, I, H, O, 16, lr)
    assert float(rep["initial_loss"]) == pytest.approx(first, rel=1e-6)
    assert float(rep["final_loss"]) == pytest.approx(last, rel=1e-6)
    # and the oracle's run of the same 16 steps
    ofirst, olast = _mlp_oracle_replay(oracle, seed, N, B, I, H, O, 16, lr)
    assert float(rep["initial_loss"]) == pytest.approx(ofirst, rel=1e-4)
    assert float(rep["final_loss"]) == pytest.approx(olast, rel=1e-4)


@pytest.mark.gpu
def test_mlp_fail_execute_mode_reports_the_injected_failure():
    rep = run_core(execution_mode=35, batch_size=8, dimension=16, hidden_dimension=16, output_dimension=8,
                   learning_rate=0.1, seed=3, sample_count=64, epochs=5)
    assert rep["status"] == "FAILED" and rep["failed_api"] == "full_step_execute"
    assert "injected execute failure" in rep["error"]


@pytest.mark.gpu
def test_generic_lm_mode_trains_checkpoints_and_resumes(tmp_path, oracle):
    V, T, D, F, L, H, B, seed = 64, 16, 32, 64, 2, 4, 4, 5
    common = dict(execution_mode=99, batch_size=B, dimension=D, hidden_dimension=F, output_dimension=V,
                  learning_rate=1e-3, seed=seed, sample_count=T, epochs=L, measured_steps=H,
                  diagnostic_checkpoint_dir=str(tmp_path))
    straight = run_core(steps=5, **{**common, "diagnostic_checkpoint_dir": ""})
    assert straight["status"] == "SUCCESS", straight
    first = run_core(steps=3, **common)
    assert first["status"] == "SUCCESS" and first["checkpoint_written"].endswith("-step3.ckpt"), first
    resumed = run_core(steps=5, diagnostic_resume_step=3, **common)
    assert resumed["status"] == "SUCCESS" and resumed["first_step"] == "4", resumed
    assert resumed["final_loss"] == straight["final_loss"]
    # the straight run equals the runtime driven from Python on the same data
    cfg = hx.LmConfig(V, T, D, F, L, H)
    rt = hx.Runtime()
    assert rt.initialize(0) and rt.prepare_lm(cfg, B) and rt.lm_state_upload(cfg.init_reference(seed))
    losses = [rt.lm_train_step(data.lm_tokens(seed, B, T, V, step=s - 1), s)[1] for s in range(1, 6)]
    rt.close()
    assert float(straight["first_loss"]) == pytest.approx(losses[0], rel=1e-7)
    assert float(straight["final_loss"]) == pytest.approx(losses[-1], rel=1e-7)
    assert len(straight["_progress"]) == 5
    # and the oracle's trajectory: batch gradients at its own weights, then Adam
    from oracle.oracle import LmConfig as OC
    oc = OC.make(V, T, D, F, L, H)
    w = cfg.init_reference(seed)
    m, v = np.zeros_like(w), np.zeros_like(w)
    olosses = []
    for step in range(1, 6):
        g, lo = oracle.lm_batch_gradients(oc, data.lm_tokens(seed, B, T, V, step=step - 1), w, threads=4)
        olosses.append(lo)
        c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
        m, v, _, _, w = oracle.adam(w, g, m, v, 1e-3, c1, c2)
    assert float(straight["first_loss"]) == pytest.approx(olosses[0], rel=1e-4)
    assert float(straight["final_loss"]) == pytest.approx(olosses[-1], rel=1e-4)
