"""Environment / World / make on the CUDA path (GPU): the reference's environment
contract (shape/dtype errors, reset, truncation, auto-reset), determinism
(reference tests/unit/test_determinism.py:27-33) and grad-mode stepping."""

import pytest
import torch

import swarp_b200 as swarp

pytestmark = pytest.mark.gpu


def test_step_contract_and_shapes():
    env = swarp.make("navigation", n_envs=64, n_agents=6, device="cuda:0", dt=0.05, max_steps=5)
    obs = env.reset(seed=3)
    assert obs.shape == (64, 6, env.scenario.obs_dim)
    act = torch.zeros(64, 6, 2, device="cuda:0")
    with pytest.raises(ValueError, match="shape"):
        env.step(torch.zeros(64, 5, 2, device="cuda:0"))
    with pytest.raises(TypeError, match="dtype"):
        env.step(act.double())
    for i in range(5):
        obs, rew, term, trunc, info = env.step(act)
        assert rew.shape == (64, 6) and term.shape == (64,) and trunc.shape == (64,)
    assert bool(trunc.all())
    assert set(info) >= {"dist_to_goal", "on_goal", "collisions", "neighbor_overflow"}


def _trajectory(seed, T=20):
    env = swarp.make("navigation", n_envs=32, n_agents=8, device="cuda:0", dt=0.05)
    env.reset(seed=seed)
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(T):
        a = torch.randn(32, 8, 2, generator=g).to("cuda:0")
        obs, rew, *_ = env.step(a)
        out.append((obs.clone(), rew.clone(), env.world.state.pos.clone()))
    return out


def test_same_seed_bit_identical_different_seed_differs():
    a, b = _trajectory(1234), _trajectory(1234)
    for x, y in zip(a, b, strict=True):
        for u, v in zip(x, y, strict=True):
            assert torch.equal(u, v)
    c = _trajectory(4321, T=5)
    assert not torch.equal(a[4][2], c[4][2])


def test_auto_reset_restarts_finished_envs():
    env = swarp.make("navigation", n_envs=16, n_agents=4, device="cuda:0", dt=0.05, max_steps=3,
                     auto_reset=True)
    env.reset(seed=0)
    act = torch.zeros(16, 4, 2, device="cuda:0")
    for _ in range(3):
        env.step(act)
    assert int(env._step_count.max()) == 0  # every env truncated at 3 and was reset


def test_grad_mode_env_step_differentiates_to_actions():
    env = swarp.make("navigation", n_envs=8, n_agents=4, device="cuda:0", dt=0.05)
    env.reset(seed=1)
    act = (0.5 * torch.randn(8, 4, 2, device="cuda:0")).requires_grad_(True)
    obs, rew, *_ = env.step(act)
    rew.sum().backward()
    assert act.grad is not None and torch.isfinite(act.grad).all() and act.grad.abs().sum() > 0


def test_neighbor_views_and_radius_graph():
    env = swarp.make("navigation", n_envs=4, n_agents=12, device="cuda:0", dt=0.05,
                     neighbor_radius=0.6)
    env.reset(seed=2)
    idx, cnt = env.world.neighbors()
    assert idx.shape == (4, 12, 12) and cnt.shape == (4, 12)
    ei = env.radius_graph()
    assert ei.shape[0] == 2 and ei.shape[1] == int(cnt.sum())
    assert env.world.neighbor_overflow().dtype == torch.bool
