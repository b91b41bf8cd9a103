"""Independent-seed replica sweep: one process per GPU, no communication.

Rank r of an N-process launch trains its own model with seed
first_seed + r (20260710 .. 20260717 on 8 GPUs): its own N(0, 0.02)
initialisation and its own seeded Zipf token stream, on its own GPU, with
nothing exchanged between ranks while training.  Each replica records its
loss trajectory, the per-step device time, and a checksum of its final
parameters.  When every rank has finished, the records are gathered once
over a host (gloo) group and rank 0 writes one JSON document: the counterpart
of the reference's multi-seed table (README.md:159-180,
docs/results/qnn-htp-full-training-step-2026-07/seeds.csv), which reports
initial and final loss per seed and their spread.

  python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
      -m hexatrain_b200.replicas --config lm-t256-d256-f1024-l4-h8 --steps 50 --out sweep.json

The training function is injectable so that the host logic (seed
assignment, gather, summary) is tested with CPU stand-ins.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
from typing import Callable, Optional

import numpy as np

FIRST_SEED = 20260710

# (V, T, D, F, L, H), batch, optimizer: the LM configurations.
LM_CONFIGS = {
    "lm-t64-d64-f64-l2-h4": ((1024, 64, 64, 64, 2, 4), 16, "adam"),
    "lm-t64-d48-f48-l4-h4-muon": ((1024, 64, 48, 48, 4, 4), 32, "muon"),
    "lm-t256-d256-f1024-l4-h8": ((1024, 256, 256, 1024, 4, 8), 512, "adam"),
}


def seed_of(rank: int, first_seed: int = FIRST_SEED) -> int:
    return first_seed + rank


def train_replica_gpu(config: str, seed: int, steps: int, device: int = 0, batch: Optional[int] = None) -> dict:
    """Trains one replica on one GPU through the C ABI: learned positions,
    N(0, 0.02) init from `seed`, token ids lm_tokens(seed, ..., step=s).
    Returns the per-step losses, device ms per step and a final-parameter
    checksum."""
    import torch

    import hexatrain_b200 as hx
    from hexatrain_b200 import data

    shape, B0, opt = LM_CONFIGS[config]
    B = batch or B0
    V, T, D, F, L, H = shape
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    rt = hx.Runtime()
    if not rt.initialize(device):
        raise RuntimeError(rt.last_error)
    try:
        if not rt.prepare_lm(cfg, B):
            raise RuntimeError(rt.last_error)
        if opt == "muon" and not rt.lm_set_optimizer(hx.OptimizerConfig(kind=1, muon_lr=0.02)):
            raise RuntimeError(rt.last_error)
        p0 = cfg.init_normal(seed, 0.02)
        if not rt.lm_state_upload(p0):
            raise RuntimeError(rt.last_error)
        losses, ms = [], []
        for step in range(1, steps + 1):
            toks = data.lm_tokens(seed, B, T, V, step=step)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ok, loss = rt.lm_train_step(toks, step)
            e1.record()
            if not ok:
                raise RuntimeError(rt.last_error)
            torch.cuda.synchronize()
            losses.append(float(loss))
            ms.append(e0.elapsed_time(e1))
        params, _, _, _ = rt.lm_state_download()
    finally:
        rt.close()
    return {"config": config, "seed": seed, "batch": B, "steps": steps, "losses": losses,
            "ms_per_step": statistics.median(ms) if ms else None,
            "final_param_l2": float(np.sqrt(np.sum(params.astype(np.float64) ** 2))),
            "final_param_checksum": float(np.sum(params.astype(np.float64)))}


def summarize(records: list) -> dict:
    """The sweep's table: per seed initial/final loss, and their spread."""
    records = sorted(records, key=lambda r: r["seed"])
    first = [r["losses"][0] for r in records]
    last = [r["losses"][-1] for r in records]
    return {"seeds": [r["seed"] for r in records],
            "initial_loss": first, "final_loss": last,
            "final_loss_mean": statistics.fmean(last),
            "final_loss_stdev": statistics.stdev(last) if len(last) > 1 else 0.0,
            "loss_reduction_ratio_mean": statistics.fmean(b / a for a, b in zip(first, last)),
            "replicas": records}


def run(config: str, steps: int, out: Optional[str], first_seed: int = FIRST_SEED,
        train: Callable[..., dict] = train_replica_gpu, batch: Optional[int] = None) -> Optional[dict]:
    """Runs this process's replica (rank from the environment) and, on rank
    0, returns and writes the gathered summary."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    rec = train(config, seed_of(rank, first_seed), steps, device=local, batch=batch)
    rec["rank"] = rank
    records = [rec]
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        if not dist.is_initialized():
            dist.init_process_group("gloo", timeout=timedelta(seconds=600))
        gathered = [None] * world
        dist.all_gather_object(gathered, rec)  # once, after training: host gloo only
        records = gathered
        dist.destroy_process_group()
    if rank != 0:
        return None
    summary = summarize(records)
    summary["config"] = config
    summary["world"] = world
    if out:
        with open(out, "w") as f:
            json.dump(summary, f, indent=1)
    return summary


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=sorted(LM_CONFIGS), default="lm-t256-d256-f1024-l4-h8")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--first-seed", type=int, default=FIRST_SEED)
    ap.add_argument("--batch", type=int, default=None, help="sequences per replica step (default: the config's)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    s = run(args.config, args.steps, args.out, args.first_seed, batch=args.batch)
    if s is not None:
        brief = {k: v for k, v in s.items() if k != "replicas"}
        print(json.dumps(brief), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
