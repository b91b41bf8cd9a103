"""The device-side failure path of the tensor-core kernels, without a fault.

Every pipeline wait of the tensor-core GEMM and attention kernels is bounded:
when it gives up, the kernel records a code in the runtime's error word,
tears down and returns, and the next synchronising call reports
DEVICE_WAIT_TIMEOUT.  hx_runtime_check_wait_timeout runs that path with the
same bounded wait on an mbarrier that nothing arrives at (no TMA copy, MMA or
TMEM in flight), with a short limit, so the wait runs out in well under a
millisecond and the context stays usable.
"""
import numpy as np
import pytest

import hexatrain_b200 as hx
from hexatrain_b200 import data

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_runtime_recovers(oracle):
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    try:
        assert not rt.check_wait_timeout(100000)
        assert rt.last_error.startswith("DEVICE_WAIT_TIMEOUT"), rt.last_error
        assert "wait self-test" in rt.last_error and "role 21" in rt.last_error
        # the error word was cleared: synchronising again succeeds
        assert rt.synchronize(), rt.last_error
        # and the next normal call on the same runtime runs and is correct
        B, I, H, O = 8, 128, 128, 64
        x, y, w1, w2 = data.mlp_data(20260710, B, I, H, O)
        assert rt.prepare_mlp_full_step(B, I, H, O, False), rt.last_error
        out = hx.MlpFullStepOutputs()
        assert rt.execute_mlp_full_step(x, y, w1, w2, 0.5, out), rt.last_error
        ref = oracle.mlp_step(x, y, w1, w2, 0.5)
        assert abs(out.loss - ref.loss) <= 1e-4 * abs(ref.loss)
        assert np.max(np.abs(out.w1_next - ref.w1_next.ravel())) <= 1e-4
        # a second timeout on the same runtime is reported again
        assert not rt.check_wait_timeout(1000)
        assert rt.last_error.startswith("DEVICE_WAIT_TIMEOUT")
        assert rt.synchronize(), rt.last_error
    finally:
        rt.close()


def test_wait_self_test_rejects_bad_limits():
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    try:
        assert not rt.check_wait_timeout(0)
        assert "cycles" in rt.last_error
        assert not rt.check_wait_timeout(10 ** 10)
    finally:
        rt.close()
