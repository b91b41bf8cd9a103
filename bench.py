#!/usr/bin/env python
"""Training-step throughput of the HexaTrain hot paths on B200.

Default workload (the data-parallel configuration quoted at 1/2/4/8 GPUs):
the tiny-Transformer LM step, vocab 1024, T=256, d_model 256, FFN 1024, 4
layers, 8 heads, learned positions, N(0, 0.02) init, FP32 master weights and
arithmetic, Adam (1e-3, 0.9, 0.999, 1e-8), global batch 512 sequences of
seeded Zipf(1.1) token ids split evenly over ranks; per-step gradient
all-reduce (NCCL) for N > 1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config lm-t256-d256-f1024-l4-h8|lm-t64-d64-f64-l2-h4|lm-t64-d48-f48-l4-h4-muon|mlp-8x128x128x64|mlp-32x256x256x128|mlp-4096x1024x1024x512]

Prints one JSON line (rank 0).  `value` is device-timed whole-job tokens/s
with the step's inputs already in HBM (steps replay captured CUDA graphs);
`e2e` is the same metric through the public API with host buffers (host
inputs copied in and the loss read back every step).  `kernels` and
`roofline` come from a separate pass with the per-launch event profiler on
(steps then run eagerly), right after the timed region.  At N = 1 the
default line also carries `small_configs`: steps/s, tokens/s, us/step and
launches/step of the four small configurations, each next to the
reference's own single-thread CPU step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED = 20260710
FP32_CUDA_CORE_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal, at max SM clock

# The five configurations.  LM: (V, T, D, F, L, H), batch, optimizer.  MLP:
# B/I/H/O, SGD learning rate, sample-set size (cyclic batches) and steps.
CONFIGS = {
    "lm-t256-d256-f1024-l4-h8": dict(kind="lm", shape=(1024, 256, 256, 1024, 4, 8), batch=512, opt="adam"),
    "lm-t64-d64-f64-l2-h4": dict(kind="lm", shape=(1024, 64, 64, 64, 2, 4), batch=16, opt="adam"),
    "lm-t64-d48-f48-l4-h4-muon": dict(kind="lm", shape=(1024, 64, 48, 48, 4, 4), batch=32, opt="muon"),
    "mlp-8x128x128x64": dict(kind="mlp", dims=(8, 128, 128, 64), lr=0.5, samples=512, steps=640),
    "mlp-32x256x256x128": dict(kind="mlp", dims=(32, 256, 256, 128), lr=0.05, samples=4 * 32, steps=1000),
    "mlp-4096x1024x1024x512": dict(kind="mlp", dims=(4096, 1024, 1024, 512), lr=0.05, samples=4 * 4096, steps=1000),
}
SMALL = ["mlp-8x128x128x64", "mlp-32x256x256x128", "mlp-4096x1024x1024x512", "lm-t64-d64-f64-l2-h4", "lm-t64-d48-f48-l4-h4-muon"]


def lm_workload(name, global_batch=None):
    """Workload and metric names; the metric keeps the configuration's own
    global batch, the workload names the batch actually run."""
    c = CONFIGS[name]
    V, T, D, F, L, H = c["shape"]
    opt = "Muon (hidden 2-D weights) + Adam" if c["opt"] == "muon" else "Adam"
    gb = global_batch or c["batch"]
    return (f"tiny_lm_train_step V{V} T{T} D{D} F{F} L{L} H{H} {opt} learned-pos global_batch={gb}",
            f"train-step tokens/s (LM V{V} T{T} D{D} F{F} L{L} H{H}, global batch {c['batch']})")


def mlp_workload(name):
    c = CONFIGS[name]
    B, I, H, O = c["dims"]
    return (f"phonelm_mlp_training_step B{B} I{I} H{H} O{O} SGD lr={c['lr']} samples={c['samples']} "
            f"ping-pong weights", f"train-step samples/s (MLP B{B} I{I} H{H} O{O})")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="lm-t256-d256-f1024-l4-h8")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-small-configs", action="store_true")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="sequences per step (default: the configuration's; smaller only for profiling captures)")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    read every 10 ms from a host thread (read-only queries), or nvidia-smi at
    200 ms where NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        import threading

        self.gpu, self.p, self.thread = gpu_index, None, None
        self.mhz, self.mx, self.reasons = [], [], set()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self.done = threading.Event()

            def loop():
                while not self.done.wait(period_s):
                    self.sample()

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-i", str(gpu_index), "-lms", "200"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def sample(self):
        try:
            mhz = float(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
            mask = int(self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
        except Exception:
            return
        self.mhz.append(mhz)
        self.mx.append(self.max_mhz)
        for n, bit in self.REASONS:
            if mask & bit:
                self.reasons.add(n)

    def stop(self):
        if self.thread is not None:
            self.done.set()
            self.thread.join(timeout=5)
            if not self.mhz:
                self.sample()  # a region shorter than the period: one sample at its end
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
            return self.summary("nvml, 10 ms")
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out = self.p.communicate(timeout=10)[0]
        except subprocess.TimeoutExpired:
            self.p.kill()
            out = self.p.communicate()[0]
        names = [n for n, _ in self.REASONS]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.mhz.append(float(parts[1]))
                self.mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    self.reasons.add(n)
        return self.summary("nvidia-smi, 200 ms")

    def summary(self, source):
        if not self.mhz:
            return None
        return {"sm_mhz": statistics.median(self.mhz), "sm_max_mhz": max(self.mx), "reasons": sorted(self.reasons),
                "samples": len(self.mhz), "source": source}


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x for x in vis.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


def cpu_threads() -> int:
    try:
        return max(1, min(len(os.sched_getaffinity(0)), 64))
    except AttributeError:
        return max(1, min(os.cpu_count() or 1, 64))


# ---- CPU baselines: the reference's own CPU code (oracle/_ref) -------------

def _lm_cpu_runner(shape):
    """A batched train step of the reference's CPU code (oracle/_ref, built
    from its sources), else the oracle's port.  Both run the reference model,
    which has a fixed positional sinusoid (same FLOPs as the learned table).
    Parameters come from numpy's N(0, 0.02): no product code is involved."""
    from oracle.oracle import LmConfig as OC, Oracle, Reference, reference_available
    cfg = OC.make(*shape)
    if reference_available():
        ref = Reference()

        def step(tokens, params, m, v, step_no, threads):
            return ref.lm_train_step(cfg, tokens, params, m, v, 1e-3, step_no, threads)
        return step, "reference", ref.param_count(cfg)
    port = Oracle()

    def step(tokens, params, m, v, step_no, threads):
        g, loss = port.lm_batch_gradients(cfg, tokens, params, threads)
        c1, c2 = port.adam_correction(0.9, step_no), port.adam_correction(0.999, step_no)
        m[:], v[:], _, _, params[:] = port.adam(params, g, m, v, 1e-3, c1, c2)
        return loss
    return step, "port", port.param_count(cfg)


def cpu_lm_sample(name, seqs, threads, steps=2, warmup=1, note=""):
    """Times the reference's CPU train step on `seqs` sequences per step with
    `threads` host threads: `warmup` untimed steps, then `steps` timed ones."""
    from hexatrain_b200 import data
    c = CONFIGS[name]
    V, T = c["shape"][0], c["shape"][1]
    step_fn, kind, P = _lm_cpu_runner(c["shape"])
    params = (np.random.default_rng(SEED).standard_normal(P) * 0.02).astype(np.float32)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    times = []
    for s in range(warmup + steps):
        toks = data.lm_tokens(SEED, seqs, T, V, step=s)
        t0 = time.perf_counter()
        step_fn(toks, params, m, v, s + 1, threads)
        if s >= warmup:
            times.append(time.perf_counter() - t0)
    tokens = seqs * T * len(times)
    sample = (f"{seqs} of the {c['batch']} sequences of T={T} per step, forward+backward+Adam over all {P} "
              f"parameters of the reference model, {len(times)} timed steps after {warmup} warm-up")
    return {"value": tokens / sum(times), "unit": "tokens/s", "cores": threads, "kind": kind,
            "ms_per_step_of_sample": 1e3 * sum(times) / len(times), "sample": sample + note}


def cpu_mlp_sample(name, steps=3, warmup=1, rows=None):
    """Times the reference's scalar MLP step (pass() + sgdUpdate, oracle/_ref)
    on one thread; `rows` < B times a row slice of the batch (FLOPs scale
    with the rows; the SGD update is a small fixed cost)."""
    from oracle.oracle import Oracle, Reference, reference_available
    from hexatrain_b200 import data
    c = CONFIGS[name]
    B, I, H, O = c["dims"]
    r = min(B, rows or B)
    x, y, w1, w2 = data.mlp_data(SEED, max(r, 1), I, H, O)
    impl = Reference() if reference_available() else Oracle()
    kind = "reference" if reference_available() else "port"
    times = []
    for s in range(warmup + steps):
        t0 = time.perf_counter()
        out = impl.mlp_step(x[:r], y[:r], w1, w2, c["lr"])
        if s >= warmup:
            times.append(time.perf_counter() - t0)
        w1, w2 = out.w1_next.reshape(I, H), out.w2_next.reshape(H, O)
    sample = (f"{'all' if r == B else r} of the {B} rows per step, scalar pass()+sgdUpdate, "
              f"{len(times)} timed steps after {warmup} warm-up")
    return {"value": r * len(times) / sum(times), "unit": "samples/s", "cores": 1, "kind": kind,
            "ms_per_step_of_sample": 1e3 * sum(times) / len(times), "sample": sample}


def run_reference_arm(args):
    """The reference's own CPU implementation of the configuration's step on
    the host cores (all threads it can use), in this arm's metric and unit.
    Under torchrun only rank 0 runs it; other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    name = args.config
    c = CONFIGS[name]
    steps, warmup = max(1, min(args.steps, 20)), min(max(0, args.warmup), 2)
    threads = cpu_threads()
    if c["kind"] == "lm":
        workload, metric = lm_workload(name)
        seqs = min(c["batch"], threads) if c["batch"] > 64 else c["batch"]
        note = "; Adam in place of Muon (the reference has no Muon)" if c["opt"] == "muon" else ""
        cb = cpu_lm_sample(name, seqs, threads, steps, warmup, note)
        unit, T = "tokens/s", c["shape"][1]
        cfg = {"workload": workload, "global_batch": c["batch"], "seq_len": T, "parallelism": "host threads",
               "sample": cb["sample"]}
    else:
        workload, metric = mlp_workload(name)
        B = c["dims"][0]
        cb = cpu_mlp_sample(name, steps, warmup, rows=64 if B > 64 else None)
        unit = "samples/s"
        cfg = {"workload": workload, "global_batch": B, "parallelism": "one host thread (scalar reference)",
               "sample": cb["sample"]}
    line = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": unit, "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "config": cfg, "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU arm -----------------------------------------------------------------

def roofline_of(prof, K, t_ms):
    """The dominant kernel class of a profiled pass of K steps against the
    measured peaks: tensor-bound when its algorithmic FLOP/byte ratio > 50."""
    if not prof:
        return None
    peaks, peak_kind = measured_peaks()
    name, d = max(prof.items(), key=lambda kv: kv[1]["total_ms"])
    common = {"kernel": name, "launches_per_step": d["launches"] / K, "share_of_step": d["total_ms"] / t_ms,
              "measured_in": f"profiled pass of {K} steps after the timed region (CUDA events around every "
                             f"launch on the launching stream; steps run eagerly)",
              "traffic": traffic_from_profiles(name), "traffic_source": "profiles/dram_traffic.json (ncu capture)"}
    if d["flops"] / max(d["bytes"], 1.0) > 50:
        achieved = d["flops"] / (d["total_ms"] / 1e3) / 1e12
        peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
        return {**common, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": f"{peak_kind} bf16 dense, sustained",
                "frac_of_3xtf32_ceiling": achieved / (peak / 6.0),
                "frac_of_fp32_cuda_core_nominal": achieved / FP32_CUDA_CORE_PEAK_TFLOPS}
    achieved = d["bytes"] / (d["total_ms"] / 1e3) / 1e9
    peak = float(peaks["hbm_gbs"])
    return {**common, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": f"{peak_kind} HBM copy"}


def kernel_table(prof, K):
    return {k: {"ms_per_step": v["total_ms"] / K, "launches_per_step": v["launches"] / K,
                "tflops": v["flops"] / max(v["total_ms"], 1e-9) / 1e9,
                "gbs": v["bytes"] / max(v["total_ms"], 1e-9) / 1e6} for k, v in prof.items()}


def run_lm(name, K, W, world=1, rank=0, local=0, global_batch=None, profile_steps=3, clocks=False, dist=None):
    """Device-timed and end-to-end LM steps of one configuration; returns the
    measured numbers (rank 0 gets the max over ranks)."""
    import torch

    import hexatrain_b200 as hx
    from hexatrain_b200 import data
    from hexatrain_b200.parallel import DataParallelLmTrainer, GpuLmBackend

    c = CONFIGS[name]
    V, T, D, F, L, H = c["shape"]
    GB = global_batch or c["batch"]
    if GB % world:
        raise SystemExit("global batch must divide evenly over ranks")
    B = GB // world
    cfg = hx.LmConfig(V, T, D, F, L, H, learned_position=True)
    rt = hx.Runtime()
    if not rt.initialize(local):
        raise SystemExit(rt.last_error)
    # A dedicated stream (torch's default stream has handle 0, which the C ABI
    # reads as "the runtime's own stream"): kernels, NCCL and timing events
    # all go to this one stream.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0
    assert rt.set_stream(stream.cuda_stream), rt.last_error
    assert rt.prepare_lm(cfg, B), rt.last_error
    if c["opt"] == "muon":
        assert rt.lm_set_optimizer(hx.OptimizerConfig(kind=1, muon_lr=0.02)), rt.last_error
    assert rt.lm_state_upload(cfg.init_normal(SEED, 0.02)), rt.last_error
    backend = GpuLmBackend(rt)
    trainer = DataParallelLmTrainer(backend, GB, rank, world)
    loss_t = backend.local_mean_loss()
    grads = backend.grad_buffer()

    def ids(step):
        return trainer.shard(data.lm_tokens(SEED, GB, T, V, step=step))

    # Each step's ids are staged (device to device) into one static buffer
    # that the captured step graph reads, as a graph-replaying training loop
    # does.
    dev_tokens = [torch.from_numpy(ids(s).astype(np.int32)).cuda() for s in range(W + K)]
    tok_static = torch.empty_like(dev_tokens[0])
    torch.cuda.synchronize()

    def device_step(i):
        tok_static.copy_(dev_tokens[i], non_blocking=True)
        return trainer.step(tok_static)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def tmax(ms):
        t = torch.tensor([ms], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for s in range(W):
        device_step(s)
    barrier()
    sampler = ClockSampler(physical_gpu(local)) if (clocks and rank == 0) else None
    launches0 = rt.metrics().kernel_launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for s in range(K):
        device_step(W + s)
    e1.record(stream)
    barrier()
    t_ms = tmax(e0.elapsed_time(e1))
    launches = rt.metrics().kernel_launches - launches0
    clk = sampler.stop() if sampler else None
    final_loss = float(grads[-1].item()) if world > 1 else float(loss_t.item())

    # per-kernel-class timing: a separate profiled pass (eager launches)
    prof, p_ms = {}, 0.0
    if profile_steps:
        assert rt.profile(True), rt.last_error
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        for s in range(profile_steps):
            device_step(s % (W + K))
        p1.record(stream)
        barrier()
        p_ms = p0.elapsed_time(p1)
        prof = rt.profile_read()
        rt.profile(False)

    # ---- end to end through the public API with host buffers ----
    pinned = [torch.from_numpy(ids(1000 + s).astype(np.int32)).pin_memory() for s in range(W + K)]
    tok_buf = torch.empty((B, T + 1), dtype=torch.int32, device="cuda")
    host_loss = np.zeros(1, np.float32)

    def e2e_step(i):
        if world == 1:
            trainer.step_count += 1
            ok, lv = rt.lm_train_step(pinned[i].numpy().view(np.uint32), trainer.step_count)
            assert ok, rt.last_error
            return lv
        tok_buf.copy_(pinned[i], non_blocking=True)
        g = trainer.step(tok_buf)
        return float(g[-1].item())

    for i in range(W):
        e2e_step(i)
    barrier()
    t0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(K):
        host_loss[0] = e2e_step(W + i)
    e3.record(stream)
    barrier()
    te_ms = tmax(max(e2.elapsed_time(e3), (time.perf_counter() - t0) * 1e3))
    rt.close()
    return {"t_ms": t_ms, "te_ms": te_ms, "launches": launches, "clocks": clk, "final_loss": final_loss,
            "prof": prof, "prof_ms": p_ms, "profile_steps": profile_steps, "B": B, "GB": GB, "T": T,
            "h2d": B * (T + 1) * 4, "d2h": 4}


def run_mlp(name, local=0, K=None, profile_steps=3):
    """Device-timed and end-to-end MLP full steps of one configuration: the
    reference driver's loop (qnn/qnn_mlp_training.cpp:674-770) with cyclic
    batches over the sample set and ping-pong weight buffers."""
    import torch

    import hexatrain_b200 as hx
    from hexatrain_b200 import data

    c = CONFIGS[name]
    B, I, H, O = c["dims"]
    lr, S = c["lr"], c["samples"]
    K = K or c["steps"]
    assert S % B == 0
    nb = S // B
    x, y, w1, w2 = data.mlp_data(SEED, S, I, H, O)
    rt = hx.Runtime()
    if not rt.initialize(local):
        raise SystemExit(rt.last_error)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    assert rt.set_stream(stream.cuda_stream), rt.last_error
    assert rt.prepare_mlp_full_step(B, I, H, O, False), rt.last_error
    xd, yd = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    w0 = [torch.from_numpy(w1.ravel().copy()).cuda(), torch.from_numpy(w2.ravel().copy()).cuda()]
    wa = [t.clone() for t in w0]
    wb = [torch.empty_like(t) for t in w0]
    loss = torch.zeros(1, device="cuda")
    torch.cuda.synchronize()

    # The C entry point's arguments for every (batch, buffer) binding, built
    # once, so that the host issues a step in a few microseconds.
    import ctypes as C
    from hexatrain_b200 import _lib
    lib = _lib.load()
    f32 = 4

    def outs(nxt):
        o = _lib.MlpOutputsC()
        o.loss = C.cast(C.c_void_p(loss.data_ptr()), _lib._fp)
        o.w1_next = C.cast(C.c_void_p(nxt[0].data_ptr()), _lib._fp)
        o.w2_next = C.cast(C.c_void_p(nxt[1].data_ptr()), _lib._fp)
        return o

    o_ab, o_ba = outs(wb), outs(wa)
    args = []
    for st in range(2 * nb):
        cur, o = (wa, o_ab) if st % 2 == 0 else (wb, o_ba)
        off = (st * B) % S
        args.append((rt._rt, C.c_void_p(xd.data_ptr() + off * I * f32), C.c_void_p(yd.data_ptr() + off * O * f32),
                     C.c_void_p(cur[0].data_ptr()), C.c_void_p(cur[1].data_ptr()), C.c_float(lr), C.byref(o)))
    run = lib.hx_mlp_execute_device

    def step(st):
        rc = run(*args[st % (2 * nb)])
        assert rc == 0, lib.hx_runtime_last_error(rt._rt)

    def reset():
        for a, b in zip(wa, w0):
            a.copy_(b)

    W = max(3, 2 * nb)  # every (batch, buffer) binding is captured before timing
    for st in range(W):
        step(st)
    reset()
    torch.cuda.synchronize()
    launches0 = rt.metrics().kernel_launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for st in range(K):
        step(st)
    e1.record(stream)
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    launches = rt.metrics().kernel_launches - launches0
    final_loss = float(loss.item())

    prof, p_ms = {}, 0.0
    if profile_steps:
        assert rt.profile(True), rt.last_error
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        for st in range(profile_steps):
            step(st)
        p1.record(stream)
        torch.cuda.synchronize()
        p_ms = p0.elapsed_time(p1)
        prof = rt.profile_read()
        rt.profile(False)

    # end to end: the reference's host-vector execute (inputs copied in,
    # loss and both next weights copied out every step), ping-pong on host
    Ke = min(K, 200)
    out = hx.MlpFullStepOutputs()
    hw1, hw2 = w1.ravel().copy(), w2.ravel().copy()
    batches = [(data.batch(x, (st * B) % S, B), data.batch(y, (st * B) % S, B)) for st in range(nb)]
    for st in range(3):
        assert rt.execute_mlp_full_step(*batches[st % nb], hw1, hw2, lr, out), rt.last_error
    hw1, hw2 = w1.ravel().copy(), w2.ravel().copy()
    t0 = time.perf_counter()
    for st in range(Ke):
        assert rt.execute_mlp_full_step(*batches[st % nb], hw1, hw2, lr, out), rt.last_error
        hw1, out.w1_next = out.w1_next, hw1
        hw2, out.w2_next = out.w2_next, hw2
    te_ms = (time.perf_counter() - t0) * 1e3
    rt.close()
    return {"t_ms": t_ms, "K": K, "te_ms": te_ms, "Ke": Ke, "launches": launches, "final_loss": final_loss,
            "prof": prof, "prof_ms": p_ms, "profile_steps": profile_steps, "B": B,
            "h2d": 4 * (B * I + B * O + I * H + H * O), "d2h": 4 * (1 + I * H + H * O)}


def small_config_entry(name, cpu=True):
    """One small configuration on this GPU, with the reference's single-thread
    CPU step beside it."""
    c = CONFIGS[name]
    if c["kind"] == "lm":
        r = run_lm(name, K=200, W=20, profile_steps=2)
        T = r["T"]
        tok = r["GB"] * T
        K, unit = 200, "tokens/s"
        workload, metric = lm_workload(name)
        e2e = {"value": tok * K / (r["te_ms"] / 1e3), "unit": unit, "h2d_bytes_per_step": r["h2d"],
               "d2h_bytes_per_step": r["d2h"]}
    else:
        r = run_mlp(name, profile_steps=2)
        tok, K, unit = r["B"], r["K"], "samples/s"
        workload, metric = mlp_workload(name)
        e2e = {"value": tok * r["Ke"] / (r["te_ms"] / 1e3), "unit": unit, "h2d_bytes_per_step": r["h2d"],
               "d2h_bytes_per_step": r["d2h"]}
    us = 1e3 * r["t_ms"] / K
    busy = sum(v["total_ms"] for v in r["prof"].values())
    entry = {"workload": workload, "metric": metric, "value": tok * K / (r["t_ms"] / 1e3), "unit": unit,
             "steps": K, "steps_per_s": 1e6 / us, "us_per_step": us, "launches_per_step": r["launches"] / K,
             "us_per_launch": us / max(r["launches"] / K, 1e-9), "e2e": e2e,
             "kernel_busy_frac_eager": busy / max(r["prof_ms"], 1e-9), "kernels": kernel_table(r["prof"],
                                                                                             r["profile_steps"]),
             "final_loss": r["final_loss"]}
    if cpu:
        if c["kind"] == "lm":
            note = "; Adam in place of Muon (the reference has no Muon)" if c["opt"] == "muon" else ""
            cb = cpu_lm_sample(name, c["batch"], 1, steps=2, warmup=1, note=note)
        else:
            B = c["dims"][0]
            cb = cpu_mlp_sample(name, steps=3, warmup=1, rows=64 if B > 64 else None)
        entry["cpu_single_thread"] = cb
        entry["vs_cpu_single_thread"] = entry["value"] / cb["value"]
    return entry


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    name = args.config
    c = CONFIGS[name]
    K, W = args.steps, max(3, args.warmup)
    if c["kind"] == "lm":
        r = run_lm(name, K, W, world, rank, local, args.global_batch, profile_steps=3, clocks=True, dist=dist)
        workload, metric = lm_workload(name, r["GB"])
        GB, T, B = r["GB"], r["T"], r["B"]
        tokens_per_step, unit = GB * T, "tokens/s"
        t_ms = r["t_ms"]
        config = {"workload": workload, "global_batch": GB, "seq_len": T, "parallelism": f"dp{world}",
                  "per_rank_batch": B, "l2": "no flush: the per-step working set (activations of every layer) "
                                            "exceeds the 126 MB L2" if GB * T >= 16384 else
                  "no flush: steps run back to back on resident inputs (latency-bound shape)"}
        e2e = {"value": tokens_per_step * K / (r["te_ms"] / 1e3), "unit": unit, "h2d_bytes_per_step": r["h2d"],
               "d2h_bytes_per_step": r["d2h"]}
        scaling = "strong"
    else:
        # The MLP configurations do not shard: N > 1 runs N independent replicas.
        r = run_mlp(name, local, K=None)
        K = r["K"]
        workload, metric = mlp_workload(name)
        tokens_per_step, unit = r["B"] * world, "samples/s"
        t_ms = r["t_ms"]
        if world > 1:
            tt = torch.tensor([t_ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_ms = float(tt.item())
        config = {"workload": workload, "global_batch": r["B"], "parallelism": f"replicas{world}",
                  "l2": "no flush: steps run back to back on resident inputs (latency-bound shape)"}
        e2e = {"value": r["B"] * world * r["Ke"] / (r["te_ms"] / 1e3), "unit": unit, "h2d_bytes_per_step": r["h2d"],
               "d2h_bytes_per_step": r["d2h"]}
        scaling = "weak"
        W = max(3, 2 * (c["samples"] // r["B"]))
    if rank == 0:
        prof, ps = r["prof"], r["profile_steps"]
        roof = roofline_of(prof, ps, r["prof_ms"]) if prof else None
        line = {"metric": metric, "value": tokens_per_step * K / (t_ms / 1e3), "unit": unit, "n_gpus": world,
                "steps": K, "warmup": W, "ms_per_step": t_ms / K, "steps_per_s": 1e3 * K / t_ms,
                "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded; Zipf(1.1) token ids and N(0,0.02) init for the LM)",
                "config": config, "e2e": e2e, "roofline": roof, "kernels": kernel_table(prof, ps) if prof else {},
                "profiled_pass": {"steps": ps, "ms_per_step": r["prof_ms"] / max(ps, 1)},
                "gpu_launches": int(r["launches"]), "launches_per_step": r["launches"] / K,
                "clocks": r.get("clocks"), "final_loss": r["final_loss"]}
        if world == 1 and not args.no_cpu_baseline:
            threads = cpu_threads()
            if c["kind"] == "lm":
                note = "; Adam in place of Muon (the reference has no Muon)" if c["opt"] == "muon" else ""
                seqs = min(GB, threads) if GB > 64 else GB
                cb = cpu_lm_sample(name, seqs, threads, steps=2, warmup=1, note=note)
                cb["single_thread"] = cpu_lm_sample(name, 1 if GB > 64 else GB, 1, steps=2, warmup=1, note=note)
            else:
                B = c["dims"][0]
                cb = cpu_mlp_sample(name, steps=3, warmup=1, rows=64 if B > 64 else None)
            line["cpu_baseline"] = cb
        if world == 1 and name == "lm-t256-d256-f1024-l4-h8" and not args.no_small_configs:
            line["small_configs"] = {n: small_config_entry(n, cpu=not args.no_cpu_baseline) for n in SMALL}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def traffic_from_profiles(kernel: str):
    """DRAM bytes per launch of a kernel class at the default workload, from
    the committed ncu summary (not measured in this run)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        t = json.load(f)
    e = t.get("tiny_lm_train_step V1024 T256 D256 F1024 L4 H8 Adam learned-pos global_batch=512", {}).get(kernel)
    return e.get("dram_bytes_per_launch") if e else None


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
