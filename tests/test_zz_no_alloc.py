"""hx_mlp_execute_device_noalloc against hx_mlp_execute_device.

The no-alloc entry point is for callers that cannot let this library
allocate device memory: a process whose GPU memory already belongs to its
own allocator, or a step path where cudaMalloc/cudaFree would synchronise
the device.  It keeps the step's intermediates in a fixed 4 MiB device array
instead.  These tests call both entry points through the C ABI on the same
device inputs, two steps in a row, and hold the no-alloc results to the
tolerance the other MLP parity tests use.

This file is named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

TOL = 1e-5  # relative, per tensor; the shapes that split K in the allocating step reorder their sums


def _runtime():
    import hexatrain_b200 as hx
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    return rt


def _data(seed, B, I, H, O):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (2, B, I)).astype(np.float32)   # two batches, one per step
    y = rng.uniform(-1, 1, (2, B, O)).astype(np.float32)
    w1 = rng.uniform(-1, 1, (I, H)).astype(np.float32) / np.float32(np.sqrt(I))
    w2 = rng.uniform(-1, 1, (H, O)).astype(np.float32) / np.float32(np.sqrt(H))
    return x, y, w1, w2


def _two_steps(shape, gemm_backend=0, lr=0.05, seed=None):
    """Runs both entry points for two ping-ponged steps on the same device
    inputs; returns per step (loss, w1_next, w2_next) of each, as numpy."""
    import torch
    from hexatrain_b200 import _lib

    B, I, H, O = shape
    dev = torch.device("cuda", 0)
    x, y, w1, w2 = _data(20260710 + B if seed is None else seed, B, I, H, O)
    xd, yd = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
    rt = _runtime()
    steps = []
    try:
        lib = _lib.load()
        assert rt.set_gemm_backend(gemm_backend), rt.last_error
        assert rt.prepare_mlp_full_step(B, I, H, O, diagnostic_outputs=False), rt.last_error
        # two independent weight trajectories, one per entry point
        ref_w = [torch.from_numpy(w1.ravel().copy()).to(dev), torch.from_numpy(w2.ravel().copy()).to(dev)]
        na_w = [t.clone() for t in ref_w]
        ref_next = [torch.empty_like(t) for t in ref_w]
        na_next = [torch.empty_like(t) for t in ref_w]
        ref_loss = torch.zeros(1, device=dev)
        na_loss = torch.full((1,), float("nan"), device=dev)
        torch.cuda.synchronize()
        for step in range(2):
            ok = rt.execute_mlp_full_step_device(xd[step].data_ptr(), yd[step].data_ptr(), ref_w[0].data_ptr(),
                                                 ref_w[1].data_ptr(), lr, ref_loss.data_ptr(),
                                                 ref_next[0].data_ptr(), ref_next[1].data_ptr())
            assert ok, rt.last_error
            assert rt.synchronize(), rt.last_error
            rc = lib.hx_mlp_execute_device_noalloc(rt._rt, B, I, H, O, C.c_void_p(xd[step].data_ptr()),
                                                   C.c_void_p(yd[step].data_ptr()), C.c_void_p(na_w[0].data_ptr()),
                                                   C.c_void_p(na_w[1].data_ptr()), C.c_float(lr),
                                                   C.c_void_p(na_loss.data_ptr()), C.c_void_p(na_next[0].data_ptr()),
                                                   C.c_void_p(na_next[1].data_ptr()))
            assert rc == _lib.HX_OK, (rc, lib.hx_runtime_last_error(rt._rt))
            torch.cuda.synchronize()
            steps.append({"inputs": (x[step], y[step], ref_w[0].cpu().numpy(), ref_w[1].cpu().numpy()),
                          "ref": (ref_loss.cpu().numpy(), ref_next[0].cpu().numpy(), ref_next[1].cpu().numpy()),
                          "noalloc": (na_loss.cpu().numpy(), na_next[0].cpu().numpy(), na_next[1].cpu().numpy())})
            # ping-pong both trajectories into the second step
            ref_w, ref_next = ref_next, ref_w
            na_w, na_next = na_next, na_w
            na_loss.fill_(float("nan"))
    finally:
        rt.close()
    return steps


def _check_steps(steps):
    for i, st in enumerate(steps):
        (gl, g1, g2), (wl, w1, w2) = st["noalloc"], st["ref"]
        assert np.isfinite(gl).all()
        assert rel_err(gl, wl) < TOL, (i, gl, wl)
        for name, g, w in (("w1_next", g1, w1), ("w2_next", g2, w2)):
            e = rel_err(g, w)
            assert e < TOL, (i, name, e)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(8, 128, 128, 64), (32, 256, 256, 128), (256, 512, 512, 128)],
                         ids=["B8_I128_H128_O64", "B32_I256_H256_O128", "B256_I512_H512_O128_tensor_cores"])
def test_noalloc_step_matches_allocating_step_two_calls(shape):
    _check_steps(_two_steps(shape))


@pytest.mark.gpu
def test_noalloc_step_all_gemms_on_tensor_cores():
    """HX_GEMM_TENSOR_CORES sends all five GEMMs of both entry points to the
    tcgen05 kernel (the automatic choice keeps the small ones on CUDA cores)."""
    _check_steps(_two_steps((256, 512, 512, 128), gemm_backend=2))


@pytest.mark.gpu
def test_noalloc_step_matches_oracle(oracle):
    """The no-alloc step against the CPU oracle (the reference's pass() and
    sgdUpdate), one step at the 32/256/256/128 shape, on the same inputs."""
    st = _two_steps((32, 256, 256, 128), lr=0.05)
    for s in st:
        x, y, w1, w2 = s["inputs"]
        B, I, H, O = 32, 256, 256, 128
        ref = oracle.mlp_step(x, y, w1.reshape(I, H), w2.reshape(H, O), 0.05)
        gl, g1, g2 = s["noalloc"]
        assert abs(float(gl[0]) - ref.loss) <= 1e-4 * abs(ref.loss)
        assert np.max(np.abs(g1 - ref.w1_next.ravel())) <= 1e-4
        assert np.max(np.abs(g2 - ref.w2_next.ravel())) <= 1e-4


# Largest admissible shape: 4352 + 2*B*H*4 + 2*B*O*4 bytes = 4194048, the
# largest multiple of 512 bytes (the size granularity at B = 64) that fits the
# 4194304-byte array; one more output column needs 4194560 bytes.
LIMIT_SHAPE = (64, 32, 4096, 4087)
OVER_SHAPE = (64, 32, 4096, 4088)


def _need(B, H, O):
    r = lambda b: (b + 255) // 256 * 256
    return 4352 + 2 * r(4 * B * H) + 2 * r(4 * B * O)


def test_limit_shapes_bracket_the_array():
    assert _need(*LIMIT_SHAPE[:1], *LIMIT_SHAPE[2:]) == 4194048 <= 4 << 20
    assert _need(*OVER_SHAPE[:1], *OVER_SHAPE[2:]) == 4194560 > 4 << 20


@pytest.mark.gpu
def test_noalloc_step_at_the_array_limit():
    """The largest shape the array holds runs and matches the allocating step;
    the next size up is rejected before any launch."""
    import torch
    from hexatrain_b200 import _lib

    _check_steps(_two_steps(LIMIT_SHAPE, lr=0.01, seed=5))
    rt = _runtime()
    try:
        lib = _lib.load()
        bufs = [torch.zeros(16, device="cuda") for _ in range(7)]
        p = [C.c_void_p(t.data_ptr()) for t in bufs]
        B, I, H, O = OVER_SHAPE
        rc = lib.hx_mlp_execute_device_noalloc(rt._rt, B, I, H, O, p[0], p[1], p[2], p[3], C.c_float(0.01), p[4],
                                               p[5], p[6])
        assert rc == _lib.HX_ERR_UNSUPPORTED
        assert "4194560" in lib.hx_runtime_last_error(rt._rt).decode()
    finally:
        rt.close()


@pytest.mark.gpu
def test_noalloc_step_rejects_shapes_beyond_its_array():
    import torch
    from hexatrain_b200 import _lib

    rt = _runtime()
    try:
        lib = _lib.load()
        # 2*B*H + 2*B*O floats = 2*4096*1024 + 2*4096*512 floats = 48 MiB > 4 MiB.
        # The size check comes before any launch, so small real buffers stand in.
        bufs = [torch.zeros(16, device="cuda") for _ in range(7)]
        p = [C.c_void_p(t.data_ptr()) for t in bufs]
        rc = lib.hx_mlp_execute_device_noalloc(rt._rt, 4096, 1024, 1024, 512, p[0], p[1], p[2], p[3],
                                               C.c_float(0.05), p[4], p[5], p[6])
        assert rc == _lib.HX_ERR_UNSUPPORTED
        msg = lib.hx_runtime_last_error(rt._rt).decode()
        assert "scratch" in msg and "4194304" in msg, msg
    finally:
        rt.close()
