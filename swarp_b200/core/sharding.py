"""Env-sharded data parallelism: one process per GPU, each stepping its own slice of envs.

Environments never interact (every kernel reads only its own env's agents), so a batch of
``n_envs`` splits into contiguous per-rank slices with no exchange during the forward or
the adjoint rollout. The only collective is one all-reduce (sum) of two scalars after the
backward pass: the BPTT loss and the squared norm of the action gradient. The reference
steps one device only (``swarp/core/world.py:35-41``); this is the multi-GPU layer the
build adds around it.
"""

from __future__ import annotations

import torch


def env_shard(n_envs: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous ``[start, stop)`` env range of ``rank``; sizes differ by at most one."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world size {world_size}")
    if n_envs < world_size:
        raise ValueError(f"{n_envs} envs cannot be sharded over {world_size} ranks")
    base, extra = divmod(n_envs, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_loss_and_grad_norm(loss: torch.Tensor, grads, group=None) -> torch.Tensor:
    """Sum ``(loss, sum ||g||^2 over grads)`` across ranks in ONE all-reduce.

    Returns a 2-element float64 tensor on the loss's device: ``[global loss, global
    squared gradient norm]``. Without an initialized process group it is the local pair.
    """
    if torch.is_tensor(grads):
        grads = (grads,)
    pair = torch.zeros(2, dtype=torch.float64, device=loss.device)
    pair[0] = loss.detach().to(torch.float64)
    for g in grads:
        if g is not None:
            v = g.detach().reshape(-1)
            pair[1] += torch.dot(v, v).to(torch.float64)  # one read of g, no temporary
    dist = torch.distributed
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(pair, op=dist.ReduceOp.SUM, group=group)
    return pair


class PairReducer:
    """Asynchronous per-step all-reduce of a small ``[loss, ||g||^2]`` pair.

    Each call copies the pair into one of ``depth`` ring buffers and starts its all-reduce
    on the collective's own stream without making the compute stream wait, so the next
    rollout overlaps the reduction. The compute stream waits for a reduction only when its
    buffer comes round again (``depth`` steps later). ``result(i)`` is the reduced pair of
    the ``i``-th call from the end (0 = latest), valid after :meth:`drain`.
    """

    def __init__(self, like: torch.Tensor, depth: int = 3, group=None) -> None:
        self.bufs = [torch.zeros(2, dtype=like.dtype, device=like.device) for _ in range(depth)]
        self.works: list = [None] * depth
        self.group = group
        self.n = 0

    def __call__(self, pair: torch.Tensor) -> None:
        i = self.n % len(self.bufs)
        if self.works[i] is not None:
            self.works[i].wait()  # stream-ordered: the buffer's previous reduction is done
        self.bufs[i].copy_(pair)
        dist = torch.distributed
        if dist.is_available() and dist.is_initialized():
            self.works[i] = dist.all_reduce(self.bufs[i], group=self.group, async_op=True)
        self.n += 1

    def drain(self) -> None:
        for i, w in enumerate(self.works):
            if w is not None:
                w.wait()
                self.works[i] = None

    def result(self, back: int = 0) -> torch.Tensor:
        return self.bufs[(self.n - 1 - back) % len(self.bufs)]
