"""CPU checks of the C-ABI library and the host-side logic (no kernels run)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import hexatrain_b200 as hx
from conftest import HAS_GPU, ROOT, golden
from hexatrain_b200 import _lib, data

HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def declared_symbols():
    names = set()
    for path in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
        names.update(re.findall(r"\b(hx_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares exactly the header's entry points
    assert sorted(_lib.SIGNATURES) == names


def test_library_has_no_torch_dependency():
    import subprocess
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "libcudart.so" not in out  # static cudart, no torch


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device failure path")
def test_runtime_fails_closed_without_device():
    rt = hx.Runtime()
    assert not rt.initialize(0)
    assert rt.last_error.startswith("CUDA_DEVICE_NOT_FOUND")
    # every call on an uninitialised runtime fails closed
    assert not rt.prepare_mlp_full_step(2, 4, 5, 3, True)
    assert rt.last_error == "runtime not initialized"
    out = hx.MlpFullStepOutputs()
    assert not rt.execute_mlp_full_step(np.zeros(8), np.zeros(6), np.zeros(20), np.zeros(15), 0.1, out)


def test_null_runtime_is_rejected():
    lib = _lib.load()
    assert lib.hx_mlp_prepare(None, 2, 4, 5, 3, 1) == _lib.HX_ERR_ARGUMENT
    assert lib.hx_runtime_synchronize(None) == _lib.HX_ERR_ARGUMENT
    assert lib.hx_runtime_last_error(None) == b"null runtime"


@pytest.mark.parametrize("cfg", [(1024, 64, 64, 64, 2, 4), (1024, 64, 48, 48, 4, 4), (1024, 256, 256, 1024, 4, 8),
                                 (8, 3, 4, 8, 1, 1)])
def test_parameter_count_matches_registry(cfg, oracle):
    from oracle.oracle import LmConfig as OC
    c = hx.LmConfig(*cfg)
    assert c.parameter_count() == oracle.param_count(OC.make(*cfg))
    reg = c.registry()
    assert reg[0][0] == "token_embedding" and reg[-1][0] == "output_projection"
    assert reg[1][0] == "layer_000.norm1_gamma" and reg[3][0] == "layer_000.wq"
    last = reg[-1]
    assert last[1] + int(np.prod(last[2])) == c.parameter_count()


def test_lm_parameter_counts():
    # per-sequence parameter counts of the three LM configurations (V1024: T64 D64 F64 L2 H4, T64 D48 F48 L4 H4, T256 D256 F1024 L4 H8)
    assert hx.LmConfig(1024, 64, 64, 64, 2, 4).parameter_count() == 180736
    assert hx.LmConfig(1024, 64, 48, 48, 4, 4).parameter_count() == 154368
    assert hx.LmConfig(1024, 256, 256, 1024, 4, 8).parameter_count() == 3674112
    assert hx.LmConfig(1024, 256, 256, 1024, 4, 8, learned_position=True).parameter_count() == 3674112 + 256 * 256


@pytest.mark.parametrize("bad,msg", [
    (dict(num_layers=0), "APP_CONFIGURATION_VALIDATION"),
    (dict(num_heads=0), "APP_CONFIGURATION_VALIDATION"),
    (dict(dimension=17, num_heads=2), "divisible by numHeads"),
    (dict(dimension=2 ** 20, feed_forward_dimension=2 ** 20), "APP_RESOURCE_ESTIMATOR"),
])
def test_validate_fails_closed(bad, msg):
    # host_tests/cpu_reference_training_test.cpp:238-244 invalid configurations
    ok, err = hx.LmConfig(**bad).validate()
    assert not ok and msg in err


def test_init_reference_matches_golden():
    for name in ("lm_V32_T4_D8_F16_L2_H2.npz", "lm_V8_T3_D8_F8_L3_H4.npz", "lm_V32_T4_D8_F16_L3_H8.npz"):
        g = golden(name)
        V, T, D, F, L, H = (int(v) for v in g["cfg"])
        p = hx.LmConfig(V, T, D, F, L, H).init_reference(int(g["seed"]))
        assert np.array_equal(p, g["params"]), name


def test_init_reference_matches_live_reference(reference):
    from oracle.oracle import LmConfig as OC
    for cfg, seed in (((1024, 64, 64, 64, 2, 4), 7), ((50, 9, 12, 20, 3, 3), 123456789)):
        assert np.array_equal(hx.LmConfig(*cfg).init_reference(seed), reference.initial_parameters(OC.make(*cfg), seed))


def test_init_learned_position_starts_at_fixed_table(oracle):
    from oracle.oracle import LmConfig as OC
    c = hx.LmConfig(32, 8, 16, 32, 2, 2, learned_position=True)
    p = c.init_reference(3)
    pos = p[32 * 16: 32 * 16 + 8 * 16].reshape(8, 16)
    assert np.array_equal(pos, oracle.fixed_position(OC.make(32, 8, 16, 32, 2, 2)))


def test_init_normal_statistics():
    c = hx.LmConfig(1024, 256, 256, 1024, 4, 8)
    p = c.init_normal(20260710, 0.02)
    assert np.array_equal(p, c.init_normal(20260710, 0.02))
    assert not np.array_equal(p, c.init_normal(20260711, 0.02))
    reg = {n: (o, s) for n, o, s in c.registry()}
    o, s = reg["token_embedding"]
    e = p[o:o + int(np.prod(s))]
    assert abs(e.std() - 0.02) < 5e-4 and abs(e.mean()) < 5e-4
    o, s = reg["layer_002.norm1_gamma"]
    assert np.all(p[o:o + s[0]] == 1.0)


def test_data_generators_are_deterministic():
    a = data.mlp_data(20260710, 512, 128, 128, 64)
    b = data.mlp_data(20260710, 512, 128, 128, 64)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    x, y, w1, w2 = a
    assert x.min() >= -1 and x.max() < 1 and abs(x.mean()) < 0.02
    assert np.abs(w1).max() <= 1 / np.sqrt(128)
    np.testing.assert_array_equal(data.batch(x, 510, 4), x[[510, 511, 0, 1]])


def test_zipf_tokens_follow_power_law():
    t = data.zipf_tokens(3, (200000,), 1024, 1.1)
    assert t.dtype == np.uint32 and t.max() < 1024
    counts = np.bincount(t, minlength=1024).astype(np.float64)
    ranks = np.arange(1, 1025, dtype=np.float64)
    expect = ranks ** -1.1 / np.sum(ranks ** -1.1) * t.size
    assert abs(counts[0] / expect[0] - 1) < 0.02
    assert abs(counts[9] / expect[9] - 1) < 0.06
    toks = data.lm_tokens(5, 16, 64, 1024, step=3)
    assert toks.shape == (16, 65) and np.array_equal(toks, data.lm_tokens(5, 16, 64, 1024, step=3))
