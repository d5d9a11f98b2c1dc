"""Multi-rank host logic on CPU (gloo, world size 2): env partition and the single
(loss, ||grad||^2) all-reduce that is the only collective of the env-sharded rollout."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from swarp_b200.core.sharding import PairReducer, env_shard, reduce_loss_and_grad_norm


@pytest.mark.parametrize("n,w", [(16000, 1), (16000, 2), (16001, 4), (7, 7), (1025, 8)])
def test_env_shard_partitions_contiguously(n, w):
    ranges = [env_shard(n, r, w) for r in range(w)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1


def test_env_shard_rejects_bad_ranks():
    with pytest.raises(ValueError):
        env_shard(10, 2, 2)
    with pytest.raises(ValueError):
        env_shard(3, 0, 4)


def test_local_pair_without_process_group():
    g = torch.tensor([[3.0, 4.0]])
    pair = reduce_loss_and_grad_norm(torch.tensor(2.0), g)
    assert pair.tolist() == [2.0, 25.0]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_envs, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        grads_all = torch.randn(n_envs, 3, 2, generator=g, dtype=torch.float64)
        loss_all = torch.rand(n_envs, generator=g, dtype=torch.float64)
        a, b = env_shard(n_envs, rank, world)
        pair = reduce_loss_and_grad_norm(loss_all[a:b].sum(), grads_all[a:b])
        red = PairReducer(pair, depth=2)
        for k in range(5):  # ring reuse: each step's pair is reduced on its own
            red(torch.tensor([float(k), float(rank)], dtype=torch.float64))
        red.drain()
        out[rank] = pair.tolist() + red.result(0).tolist() + red.result(1).tolist()
    finally:
        dist.destroy_process_group()


def test_two_rank_allreduce_equals_whole_batch():
    n_envs, world = 11, 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_worker, args=(world, port, n_envs, out), nprocs=world,
                           start_method="spawn")
        results = dict(out)
    g = torch.Generator().manual_seed(0)
    grads_all = torch.randn(n_envs, 3, 2, generator=g, dtype=torch.float64)
    loss_all = torch.rand(n_envs, generator=g, dtype=torch.float64)
    expect = [float(loss_all.sum()), float(grads_all.square().sum())]
    ranks_sum = float(sum(range(world)))
    for r in range(world):
        assert results[r][:2] == pytest.approx(expect, rel=1e-12)
        assert results[r][2:] == [4.0 * world, ranks_sum, 3.0 * world, ranks_sum]
