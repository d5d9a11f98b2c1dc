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
