"""Data-parallel host logic on CPU: two gloo ranks, oracle-backed backend.

The trainer in hexatrain_b200/parallel.py is the code bench.py runs over
NCCL on GPUs; here its sharding, gradient scaling, loss slot, all-reduce and
lock-step optimizer are checked against a single-process full-batch run.
Failure detection is exercised on the host: a rank that dies before the
all-reduce makes the survivor's collective fail within the group timeout.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from hexatrain_b200 import data
from hexatrain_b200.parallel import DataParallelLmTrainer, replica_seeds, shard_bounds

V, T, D, F, L, H = 40, 6, 8, 12, 2, 2
GLOBAL_B = 4
LR = 1e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleBackend:
    """CPU stand-in for GpuLmBackend built on the oracle."""

    def __init__(self, params):
        from oracle.oracle import LmConfig, Oracle
        self.o = Oracle()
        self.cfg = LmConfig.make(V, T, D, F, L, H, learned_position=True)
        self.params = params.astype(np.float32).copy()
        self.m = np.zeros_like(self.params)
        self.v = np.zeros_like(self.params)
        self.P = self.params.size
        self.grads = torch.zeros(self.P + 1, dtype=torch.float32)

    def forward_backward(self, tokens, grad_scale):
        g, loss = self.o.lm_batch_gradients(self.cfg, tokens, self.params)
        b = tokens.shape[0]
        self.grads[:self.P] = torch.from_numpy(g * np.float32(b * grad_scale))
        self.grads[self.P] = float(loss) * b * grad_scale

    def grad_buffer(self):
        return self.grads

    def optimizer_step(self, step):
        c1, c2 = self.o.adam_correction(0.9, step), self.o.adam_correction(0.999, step)
        g = self.grads[:self.P].numpy().copy()
        self.m, self.v, _, _, self.params = self.o.adam(self.params, g, self.m, self.v, LR, c1, c2)


class BucketedOracleBackend(OracleBackend):
    """The same, exposing the gradient buckets the GPU backend reduces one by
    one (output projection + loss slot, layers from the last, embeddings);
    on CPU the communication stream is the current thread."""

    def buckets(self):
        import hexatrain_b200 as hx
        reg = {n: (o, int(np.prod(sh))) for n, o, sh in
               hx.LmConfig(V, T, D, F, L, H, learned_position=True).registry()}
        out_off = reg["output_projection"][0]
        b = [(out_off, self.P + 1 - out_off)]
        for l in reversed(range(L)):
            first = reg[f"layer_{l:03d}.norm1_gamma"][0]
            last_off, last_n = reg[f"layer_{l:03d}.ffn_w2"]
            b.append((first, last_off + last_n - first))
        b.append((0, reg["layer_000.norm1_gamma"][0]))
        return b

    def comm(self, i):
        import contextlib
        return contextlib.nullcontext()

    def join_comm(self):
        pass


def _params0():
    import hexatrain_b200 as hx
    return hx.LmConfig(V, T, D, F, L, H, learned_position=True).init_normal(3, 0.02)


def _run(rank, world, port, out, steps=2, die_before_step=None, bucketed=False):
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    be = (BucketedOracleBackend if bucketed else OracleBackend)(_params0())
    tr = DataParallelLmTrainer(be, GLOBAL_B, rank, world)
    assert tr.overlap == (bucketed and world > 1)
    losses = []
    try:
        for s in range(steps):
            if die_before_step is not None and rank == 1 and s == die_before_step:
                os._exit(3)  # a rank that leaves between steps, with no collective in flight
            toks = data.lm_tokens(7, GLOBAL_B, T, V, step=s)
            g = tr.step(tr.shard(toks))
            losses.append(float(g[-1]))
        out.put((rank, "ok", be.params, losses))
    except Exception as e:  # noqa: BLE001 -- report the failure to the parent
        out.put((rank, "error", repr(e), losses))
    finally:
        if world > 1 and dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_shard_bounds():
    assert shard_bounds(512, 0, 8) == (0, 64) and shard_bounds(512, 7, 8) == (448, 512)
    with pytest.raises(ValueError):
        shard_bounds(510, 0, 4)
    assert replica_seeds(20260710, 8) == list(range(20260710, 20260718))


def test_two_rank_data_parallel_equals_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, status, params, losses = q.get(timeout=120)
        assert status == "ok", params
        res[rank] = (params, losses)
    for p in procs:
        p.join(timeout=30)
    # replicas stay identical
    assert np.array_equal(res[0][0], res[1][0])
    assert res[0][1] == res[1][1]
    # and equal the single-process full-batch run up to summation order
    q1 = ctx.Queue()
    _run(0, 1, 0, q1)
    _, status, p_full, l_full = q1.get(timeout=60)
    assert status == "ok"
    rel = np.max(np.abs(res[0][0] - p_full)) / np.max(np.abs(p_full))
    assert rel < 1e-5, rel
    np.testing.assert_allclose(res[0][1], l_full, rtol=1e-6)


def test_rank_failure_is_detected_by_the_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, q, 3, 1)) for r in range(2)]
    for p in procs:
        p.start()
    rank, status, detail, losses = q.get(timeout=120)
    assert rank == 0 and status == "error" and len(losses) == 1, (rank, status, detail)
    for p in procs:
        p.join(timeout=30)
    assert procs[1].exitcode == 3


def test_bucketed_all_reduce_equals_single_all_reduce():
    """The per-bucket all-reduces cover the whole [P+1] buffer exactly once,
    in the same order on every rank: the bucketed run equals the unbucketed
    one bit for bit (two gloo ranks sum exactly in any grouping)."""
    ctx = mp.get_context("spawn")
    results = {}
    for bucketed in (False, True):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_run, args=(r, 2, port, q, 2, None, bucketed)) for r in range(2)]
        for p in procs:
            p.start()
        res = {}
        for _ in range(2):
            rank, status, params, losses = q.get(timeout=120)
            assert status == "ok", params
            res[rank] = (params, losses)
        for p in procs:
            p.join(timeout=30)
        assert np.array_equal(res[0][0], res[1][0])
        results[bucketed] = res[0]
    assert np.array_equal(results[False][0], results[True][0])
    assert results[False][1] == results[True][1]
    b = BucketedOracleBackend(_params0()).buckets()
    covered = sorted((o, o + n) for o, n in b)
    assert covered[0][0] == 0 and all(x[1] == y[0] for x, y in zip(covered, covered[1:]))
    assert covered[-1][1] == _params0().size + 1
