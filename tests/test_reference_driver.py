"""The reference's own experiment drivers on this repository's Runtime.

hexatrain_b200/runtime_adapter/qnn_runtime_hexatrain.cpp implements the
reference's phonelm::qnn::Runtime (qnn/qnn_runtime.h:250-451) over the C ABI.
oracle/_ref/libhexaref_driver.so is the reference's driver code compiled
with that adapter in place of its stub/QAIRT runtime.  The drivers gate the
GPU's results against their own CPU code and say so in their report:
trainFullStep's correctness gates (qnn/qnn_mlp_training.cpp:783-787) and
status, its failure-injection modes, and the LM Adam driver
(languageModelAdam, qnn/qnn_transformer_training.cpp) in its generic mode.
"""
import pytest

from conftest import HAS_GPU


@pytest.fixture(scope="module")
def driver():
    from oracle.oracle import ReferenceDriver, reference_driver_available
    if not reference_driver_available():
        pytest.skip("reference driver build (oracle/_ref/libhexaref_driver.so) not present")
    return ReferenceDriver()


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device path")
def test_driver_fails_closed_without_a_device(driver):
    kv, text = driver.run_mode(32, 8, 128, 128, 64, epochs=10, sample_count=512, learning_rate=0.5)
    assert kv["status"] == "FAILED" and kv["failed_api"] == "HTP_prepare"
    assert kv["error"].startswith("CUDA_DEVICE_NOT_FOUND") and kv["cpu_fallback"] == "false"
    assert kv["api_trace_backend_library"] == "libhexatrain_b200.so"


@pytest.mark.gpu
def test_mlp_full_step_mode_32_passes_the_reference_gates(driver):
    """The 8/128/128/64 MLP through the reference driver: 8/128/128/64, lr 0.5, 512 samples,
    10 epochs (640 steps) of executeMlpFullStep with all diagnostic outputs,
    each step compared with the driver's own pass()."""
    kv, text = driver.run_mode(32, 8, 128, 128, 64, epochs=10, sample_count=512, learning_rate=0.5)
    assert kv.get("status") == "SUCCESS", text[:3000]
    assert int(kv["steps"]) == 640
    assert kv["cpu_fallback"] == "false"
    for k in ("hidden_max_abs_error", "prediction_max_abs_difference", "loss_abs_error", "dp_max_abs_error"):
        assert float(kv[k]) < 1e-3, (k, kv[k])
    for k in ("dw2_max_abs_error", "dh_max_abs_error"):
        assert float(kv[k]) < 1e-2, (k, kv[k])
    assert float(kv["final_loss"]) < float(kv["initial_loss"])
    print({k: kv[k] for k in ("initial_loss", "final_loss", "loss_abs_error", "dw2_max_abs_error")})


@pytest.mark.gpu
def test_mlp_full_step_failure_injection_modes(driver):
    kv, text = driver.run_mode(35, 8, 128, 128, 64, epochs=10, sample_count=512, learning_rate=0.5)
    assert kv["status"] == "FAILED", text[:2000]
    assert "injected graphExecute failure" in text
    assert kv["api_trace_failure_injection_call"] == "37"
    kv, text = driver.run_mode(36, 8, 128, 128, 64, epochs=10, sample_count=512, learning_rate=0.5)
    assert kv["status"] == "FAILED" and kv["failed_api"] == "HTP_prepare", text[:2000]
    assert "injected graphFinalize failure" in text


@pytest.mark.gpu
def test_generic_lm_mode_99_passes_the_reference_gates(driver):
    """The LM Adam driver in its generic mode: B=1, T=8, V=16, D=16, FFN 16,
    2 layers, 2 heads, 8 Adam steps, one seed -- executeTinyTransformerTraining
    (one-hot rows, diagnostic outputs and per-head probability taps) and the
    chunked executeAdamOptimizer on the GPU, compared with the driver's CPU
    model at its checkpoints."""
    kv, text = driver.run_mode(99, batch=1, dimension=16, hidden=16, output=16, steps=8, epochs=2,
                               sample_count=8, measured_steps=2, correctness_interval=1, learning_rate=1e-3,
                               seed=1)
    assert kv.get("status") == "SUCCESS", text[:4000]
