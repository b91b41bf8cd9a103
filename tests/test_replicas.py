"""The independent-seed replica sweep (hexatrain_b200/replicas.py).

CPU: two gloo ranks with a CPU stand-in for the GPU trainer check the seed
assignment (first_seed + rank), that nothing is exchanged before training
ends, and the gathered summary rank 0 writes.  GPU: two seeds trained on one
GPU through the C ABI, each against the oracle's trajectory.
"""
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from hexatrain_b200 import replicas


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def fake_train(config, seed, steps, device=0, batch=None):
    """Seed-dependent losses, no GPU: a stand-in with the trainer's signature."""
    rng = np.random.default_rng(seed)
    start = 7.0 + rng.uniform(0, 0.1)
    return {"config": config, "seed": seed, "batch": batch or 4, "steps": steps,
            "losses": [start * (0.9 ** s) for s in range(steps)], "ms_per_step": 1.0,
            "final_param_l2": float(seed), "final_param_checksum": 0.0}


def _rank(rank, world, port, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    replicas.run("lm-t64-d64-f64-l2-h4", 5, out if rank == 0 else None, train=fake_train)


def test_two_gloo_ranks_train_their_own_seeds(tmp_path):
    out = str(tmp_path / "sweep.json")
    mp.start_processes(_rank, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    s = json.load(open(out))
    assert s["seeds"] == [20260710, 20260711] and s["world"] == 2
    assert [r["rank"] for r in s["replicas"]] == [0, 1]
    assert s["initial_loss"][0] != s["initial_loss"][1]
    assert len(s["final_loss"]) == 2 and s["final_loss_stdev"] > 0
    assert abs(s["loss_reduction_ratio_mean"] - 0.9 ** 4) < 1e-12


def test_single_process_runs_the_first_seed(tmp_path, monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    s = replicas.run("lm-t64-d48-f48-l4-h4-muon", 3, None, first_seed=11, train=fake_train)
    assert s["seeds"] == [11] and s["final_loss_stdev"] == 0.0


@pytest.mark.gpu
def test_two_seeds_on_one_gpu_match_the_oracle(oracle):
    """Two replicas of the T64 D64 L2 model (V1024 T64 D64 F64 L2 H4, learned
    positions, N(0, 0.02), Adam) at 8 sequences, 4 steps each, each against
    the oracle's own trajectory for the same seed."""
    import hexatrain_b200 as hx
    from hexatrain_b200 import data
    from oracle.oracle import LmConfig as OC
    V, T, D, F, L, H = 1024, 64, 64, 64, 2, 4
    B, steps = 8, 4
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    oc = OC.make(V, T, D, F, L, H, learned_position=True)
    finals = []
    for seed in (20260710, 20260711):
        rec = replicas.train_replica_gpu("lm-t64-d64-f64-l2-h4", seed, steps, batch=B)
        w = cfg.init_normal(seed, 0.02)
        m, v = np.zeros_like(w), np.zeros_like(w)
        for step in range(1, steps + 1):
            toks = data.lm_tokens(seed, B, T, V, step=step)
            g, loss = oracle.lm_batch_gradients(oc, toks, w, threads=8)
            assert abs(rec["losses"][step - 1] - loss) <= 1e-4 * abs(loss), (seed, step)
            c1, c2 = oracle.adam_correction(0.9, step), oracle.adam_correction(0.999, step)
            m, v, _, _, w = oracle.adam(w, g, m, v, 1e-3, c1, c2)
        assert abs(rec["final_param_l2"] - float(np.sqrt(np.sum(w.astype(np.float64) ** 2)))) <= 1e-4 * rec["final_param_l2"]
        finals.append(rec["losses"][-1])
    assert finals[0] != finals[1]
