"""Batch-sharded data parallelism for the LM training step.

One process per GPU.  The global batch of B sequences is split evenly over
the ranks (rank r takes sequences [r*B/N, (r+1)*B/N)); every rank runs the
forward and backward pass on its shard with gradients scaled by 1/B, so the
all-reduce SUM of the flat gradient buffer yields exactly the reference's
sum_b grad_b * (1/B) (qnn/qnn_transformer_training.cpp:7322-7330) up to
summation order.  The buffer carries one extra element, the loss sum scaled
the same way, so the same all-reduce also produces the global mean loss.
Every rank then applies the identical optimizer update and the replicas stay
bit-identical.

The backend is injectable: ``GpuLmBackend`` drives libhexatrain_b200.so on
one device (torch tensors are only views of its buffers, so NCCL reduces
them in place); tests use a CPU stand-in with the same methods.

Overlap: a backend that exposes gradient buckets (``buckets()``, the
[P+1] buffer's contiguous pieces in the order the backward finishes them)
has each bucket all-reduced as soon as it is final, on a communication
stream that waits for that bucket's event (``comm(i)``), while the backward
continues on the compute streams; ``join_comm()`` then makes the compute
stream wait for every reduction before the optimizer step.  The buckets'
all-reduces run in the same order on every rank.
"""
from __future__ import annotations

import contextlib
from typing import Optional, Protocol

import numpy as np


class LmBackend(Protocol):
    def forward_backward(self, tokens, grad_scale: float) -> None: ...
    def grad_buffer(self):  # torch tensor [P+1] (last element: scaled loss sum)
        ...
    def optimizer_step(self, step: int) -> None: ...


def shard_bounds(global_batch: int, rank: int, world: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not divide over {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


class DataParallelLmTrainer:
    def __init__(self, backend: LmBackend, global_batch: int, rank: int = 0, world: int = 1, group=None,
                 overlap: bool = True):
        self.backend = backend
        self.global_batch = global_batch
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = shard_bounds(global_batch, rank, world)
        self.step_count = 0
        # bucketed all-reduce overlapped with the backward, when the backend can
        self.overlap = bool(overlap and world > 1 and hasattr(backend, "buckets"))
        if self.overlap and hasattr(backend, "enable_buckets"):
            backend.enable_buckets()

    def shard(self, global_tokens: np.ndarray) -> np.ndarray:
        """This rank's rows of a [global_batch, T+1] token array."""
        if global_tokens.shape[0] != self.global_batch:
            raise ValueError("token batch does not match the global batch")
        return np.ascontiguousarray(global_tokens[self.lo:self.hi])

    def step(self, local_tokens) -> "object":
        """One optimizer step on this rank's shard; returns the grad buffer
        (after the all-reduce) whose last element is the global mean loss."""
        self.step_count += 1
        self.backend.forward_backward(local_tokens, 1.0 / self.global_batch)
        grads = self.backend.grad_buffer()
        if self.world > 1:
            import torch.distributed as dist
            if self.overlap:
                for i, (off, cnt) in enumerate(self.backend.buckets()):
                    with self.backend.comm(i):
                        dist.all_reduce(grads[off:off + cnt], op=dist.ReduceOp.SUM, group=self.group)
                self.backend.join_comm()
            else:
                dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=self.group)
        self.backend.optimizer_step(self.step_count)
        return grads


class GpuLmBackend:
    """LmBackend over a prepared hexatrain_b200 Runtime (device-resident state)."""

    def __init__(self, runtime, torch_stream=None):
        import torch
        self.rt = runtime
        if torch_stream is not None:
            if not runtime.set_stream(torch_stream.cuda_stream):
                raise RuntimeError(runtime.last_error)
        ptr, n = runtime.lm_grad_buffer()
        self._grads = _device_view(ptr, n)
        self._loss = _device_view(runtime.lm_loss_device(), 1)
        self._tok = None
        self._torch = torch

    def forward_backward(self, tokens, grad_scale: float) -> None:
        torch = self._torch
        if isinstance(tokens, np.ndarray):  # host ids: stage them on the device
            t = torch.from_numpy(np.ascontiguousarray(tokens).astype(np.int32))
            if self._tok is None or self._tok.shape != t.shape:
                self._tok = torch.empty(t.shape, dtype=torch.int32, device="cuda")
            self._tok.copy_(t, non_blocking=False)
            tokens = self._tok
        if not self.rt.lm_forward_backward_device(tokens.data_ptr(), grad_scale):
            raise RuntimeError(self.rt.last_error)

    def grad_buffer(self):
        return self._grads

    def optimizer_step(self, step: int) -> None:
        if not self.rt.lm_optimizer_step_device(step):
            raise RuntimeError(self.rt.last_error)

    def local_mean_loss(self):
        return self._loss

    # ---- gradient buckets (overlapped all-reduce) ----
    def enable_buckets(self) -> None:
        if not self.rt.lm_enable_bucket_events(True):
            raise RuntimeError(self.rt.last_error)
        self._buckets = self.rt.lm_grad_buckets()
        self._comm = self._torch.cuda.Stream()

    def buckets(self):
        return self._buckets

    @contextlib.contextmanager
    def comm(self, i: int):
        """The communication stream, after bucket i's gradients are final."""
        if not self.rt.lm_bucket_wait(i, self._comm.cuda_stream):
            raise RuntimeError(self.rt.last_error)
        with self._torch.cuda.stream(self._comm):
            yield

    def join_comm(self) -> None:
        self._torch.cuda.current_stream().wait_stream(self._comm)


def _device_view(ptr: int, count: int):
    """Zero-copy float32 torch tensor over a device pointer owned by the runtime."""
    import torch

    class _View:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4", "data": (ptr, False),
                                             "version": 3, "strides": None}
    return torch.as_tensor(_View(), device="cuda")


def replica_seeds(first_seed: int, world: int) -> list[int]:
    """Independent-seed replica sweep: rank r trains its own model with seed
    first_seed + r and never communicates (seeds 20260710..20260717 at 8
    GPUs); hexatrain_b200/replicas.py runs the sweep."""
    return [first_seed + r for r in range(world)]
