"""Per-env agent parameters ``[n_envs, n_agents, NUM_PARAMS]`` on the CUDA path (GPU),
restating the reference's tests/unit/test_per_env_params.py cases (analytic contacts,
broadcast = shared bit for bit, gradients, validation) plus a multi-step oracle check."""

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import (
    NUM_PARAMS,
    P_MASS,
    P_MAX_SPEED,
    P_RADIUS,
    AgentConfig,
    ControlMode,
    DynamicsModel,
    per_env_float_template,
)
from swarp_b200.interop.autograd import TorchState, rollout, warp_step

from ref_bridge import ref_obstacles, ref_world

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = torch.float64


def holo(n, radius=0.1, mode=ControlMode.VELOCITY):
    return [AgentConfig(radius=radius, ctrl_mode=mode, max_speed=10.0, max_accel=10.0)
            for _ in range(n)]


def state_of(pos, n_envs, vel=None):
    pos = torch.as_tensor(pos, dtype=D)
    pos = pos.unsqueeze(0).expand(n_envs, *pos.shape).contiguous().to(DEV)
    v = torch.zeros_like(pos) if vel is None else torch.as_tensor(vel, dtype=D).unsqueeze(0).expand_as(pos).contiguous().to(DEV)
    z = torch.zeros(pos.shape[:2], dtype=D, device=DEV)
    return TorchState(pos, z.clone(), v, z.clone(), z.clone())


def test_mass_divergence_analytic():
    """reference test_per_env_params.py:56-82: same contact, mass 1 vs 2 -> dv = F/m dt."""
    world = WorldConfig(collision_k=100.0, collision_c=0.0, collision_margin=0.02)
    cfgs = holo(1, radius=0.1)
    st = Stepper(cfgs, dt=0.1, device=DEV, dtype=D, world=world)
    st.set_obstacles(Obstacles(pos=torch.tensor([[[0.3, 0.0]], [[0.3, 0.0]]], dtype=D),
                               radius=torch.tensor([0.15], dtype=D)))
    f = per_env_float_template(cfgs, n_envs=2)
    f[0, 0, P_MASS], f[1, 0, P_MASS] = 1.0, 2.0
    st.set_agent_params_per_env(f)
    with torch.no_grad():
        out = warp_step(st, state_of([[0.1, 0.0]], 2), torch.zeros(2, 1, 2, dtype=D, device=DEV))
    np.testing.assert_allclose(out.pos[0, 0].cpu(), [0.1 - 0.07, 0.0], atol=1e-12)
    np.testing.assert_allclose(out.pos[1, 0].cpu(), [0.1 - 0.035, 0.0], atol=1e-12)


def test_radius_changes_contact_analytic():
    """reference test_per_env_params.py:85-124."""
    world = WorldConfig(collision_k=100.0, collision_c=0.0, collision_margin=0.02)
    cfgs = holo(2, radius=0.15)
    st = Stepper(cfgs, dt=0.1, device=DEV, dtype=D, world=world)
    f = per_env_float_template(cfgs, n_envs=2)
    f[0, :, P_RADIUS], f[1, :, P_RADIUS] = 0.1, 0.15
    st.set_agent_params_per_env(f)
    with torch.no_grad():
        out = warp_step(st, state_of([[0.0, 0.0], [0.25, 0.0]], 2),
                        torch.zeros(2, 2, 2, dtype=D, device=DEV))
    np.testing.assert_allclose(out.pos[0].cpu(), [[0.0, 0.0], [0.25, 0.0]], atol=1e-12)
    np.testing.assert_allclose(out.pos[1].cpu(), [[-0.07, 0.0], [0.32, 0.0]], atol=1e-12)


def mixed(world, substeps=1):
    return [AgentConfig(model=DynamicsModel.HOLONOMIC, radius=0.1, max_speed=2.0, max_accel=2.0),
            AgentConfig(model=DynamicsModel.DIFF_DRIVE, radius=0.1, max_speed=2.0, max_ang_vel=2.0),
            AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, radius=0.1, max_speed=2.0,
                        max_accel=2.0, max_steer=0.6, l_f=0.16, l_r=0.14)]


def test_broadcast_matches_shared_bit_exact():
    """reference test_per_env_params.py:127-155, over a 6-step rollout with grads."""
    world = WorldConfig(collision_k=30.0, collision_c=1.0, collision_margin=0.05,
                        bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft")
    cfgs = mixed(world)
    outs = []
    for per_env in (False, True):
        st = Stepper(cfgs, dt=0.05, substeps=3, device=DEV, dtype=D, world=world)
        st.set_obstacles(Obstacles(pos=torch.tensor([[[0.4, 0.4]]] * 4, dtype=D),
                                   radius=torch.tensor([0.12], dtype=D)))
        if per_env:
            st.set_agent_params_per_env(per_env_float_template(cfgs, n_envs=4))
        rng = np.random.default_rng(0)
        s = state_of(rng.random((3, 2)) * 0.3 - 0.15, 4)
        s = TorchState(*(t.requires_grad_(True) for t in s[:5]))
        a = torch.as_tensor(0.4 * rng.standard_normal((6, 4, 3, 2)), dtype=D,
                            device=DEV).requires_grad_(True)
        fin, _ = rollout(st, s, a)
        g = torch.autograd.grad((fin.pos ** 2).sum() + fin.theta.sum(), [a, *s[:5]])
        outs.append((*fin[:5], *g))
    for x, y in zip(*outs, strict=True):
        assert torch.equal(x, y)


def test_randomized_per_env_rollout_matches_oracle():
    """Per-env mass, radius and speed limit drawn per env; 8-step rollout vs the f64
    oracle with [E, A, 22] parameters (states 1e-12, gradients 1e-10)."""
    world = WorldConfig(collision_k=60.0, collision_c=1.0, collision_margin=0.03,
                        bounds=(-0.5, 0.5, -0.5, 0.5), bounds_mode="soft", neighbor_radius=0.35)
    cfgs = [AgentConfig(radius=0.12, ctrl_mode=ControlMode.ACCELERATION, max_accel=3.0),
            AgentConfig(model=DynamicsModel.DIFF_DRIVE, radius=0.12)] * 3
    E, T = 5, 8
    st = Stepper(cfgs, dt=0.05, substeps=2, device=DEV, dtype=D, world=world)
    f = per_env_float_template(cfgs, n_envs=E)
    rng = np.random.default_rng(4)
    f[..., P_MASS] = rng.uniform(0.5, 2.0, (E, len(cfgs)))
    f[..., P_RADIUS] = rng.uniform(0.06, 0.12, (E, len(cfgs)))
    f[..., P_MAX_SPEED] = rng.uniform(0.5, 1.5, (E, len(cfgs)))
    st.set_agent_params_per_env(f)
    g = torch.Generator().manual_seed(5)
    init = [(torch.rand(E, 6, 2, generator=g, dtype=D) - 0.5) * 0.6, torch.rand(E, 6, generator=g, dtype=D),
            torch.randn(E, 6, 2, generator=g, dtype=D) * 0.2, torch.zeros(E, 6, dtype=D),
            torch.zeros(E, 6, dtype=D)]
    acts = torch.randn(T, E, 6, 2, generator=g, dtype=D)
    w = torch.randn(E, 6, 2, generator=g, dtype=D)
    s_r = [x.clone().requires_grad_(True) for x in init]
    a_r = acts.clone().requires_grad_(True)
    fin_r, _, _ = R.rollout(tuple(s_r), a_r, ref_world(st), ref_obstacles(st))
    (fin_r[0] * w).sum().backward()
    s = [x.to(DEV).requires_grad_(True) for x in init]
    a = acts.to(DEV).requires_grad_(True)
    fin, _ = rollout(st, TorchState(*s), a)
    (fin.pos * w.to(DEV)).sum().backward()
    torch.testing.assert_close(fin.pos.detach().cpu(), fin_r[0].detach(), rtol=1e-12, atol=1e-13)
    torch.testing.assert_close(a.grad.cpu(), a_r.grad, rtol=1e-10, atol=1e-12)
    for x, y in zip(s, s_r):
        torch.testing.assert_close(x.grad.cpu(), y.grad, rtol=1e-10, atol=1e-12)


def test_validation():
    """reference test_per_env_params.py:206-230."""
    world = WorldConfig(collision_k=10.0, collision_margin=0.02)
    st = Stepper(holo(2, radius=0.1), dt=0.1, device=DEV, dtype=D, world=world)
    with pytest.raises(ValueError, match="n_agents|NUM_PARAMS|shape"):
        st.set_agent_params_per_env(torch.zeros(4, 3, NUM_PARAMS, dtype=D))
    with pytest.raises(ValueError, match="n_agents|NUM_PARAMS|shape"):
        st.set_agent_params_per_env(torch.zeros(4, 2, NUM_PARAMS + 1, dtype=D))
    f = per_env_float_template(holo(2, radius=0.1), n_envs=2)
    f[1, :, P_RADIUS] = 0.5
    with pytest.raises(ValueError, match="neighbor_radius"):
        st.set_agent_params_per_env(f)
