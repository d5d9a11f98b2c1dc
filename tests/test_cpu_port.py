"""The C restatement (the timed CPU baseline) against the torch oracle, float64 (CPU only).

Two independent restatements of the reference: the C port with a hand-written adjoint,
and the torch one with autograd. They must agree on trajectories and on the gradient of
<w, final pos> w.r.t. actions and the initial state.
"""

import numpy as np
import pytest
import torch

from oracle import cpu_port
from oracle import torch_ref as R
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, param_rows

D = torch.float64


def _case(cfgs, E, T, seed, *, dt=0.05, substeps=1, k=40.0, c=1.0, margin=0.03, R_=0.3, K=32,
          bounds=(-0.6, 0.6, -0.6, 0.6), mode=1, obstacles=None, spread=0.4):
    A = len(cfgs)
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1) * spread
    th = torch.rand(E, A, generator=g, dtype=D) * 3
    vel = torch.randn(E, A, 2, generator=g, dtype=D) * 0.3
    sp = torch.randn(E, A, generator=g, dtype=D) * 0.3
    om = torch.randn(E, A, generator=g, dtype=D) * 0.3
    acts = (torch.rand(T, E, A, 2, generator=g, dtype=D) * 2 - 1) * 1.5
    gf = torch.randn(E, A, 2, generator=g, dtype=D)
    params = param_rows(cfgs)
    tags = [int(c_.model) for c_ in cfgs]
    modes = [int(c_.ctrl_mode) for c_ in cfgs]
    w = R.RefWorld(params=torch.tensor(params), model_tag=tags, ctrl_mode=modes, dt=dt,
                   substeps=substeps, k=k, c=c, margin=margin, neighbor_radius=R_,
                   max_neighbors=K, bounds=bounds, soft_walls=mode == 1, clamp_bounds=mode == 2)
    ob = None
    if obstacles is not None:
        ob = R.RefObstacles(pos=torch.tensor(obstacles["pos"]), angle=torch.tensor(obstacles["angle"]),
                            vel=torch.tensor(obstacles["vel"]), ang_vel=torch.tensor(obstacles["ang_vel"]),
                            radius=torch.tensor(obstacles["radius"]), half=torch.tensor(obstacles["half"]),
                            shape=list(obstacles["shape"]), kind=[0] * len(obstacles["shape"]))
    st = [x.clone().requires_grad_(True) for x in (pos, th, vel, sp, om)]
    a = acts.clone().requires_grad_(True)
    fin, traj, _ = R.rollout(tuple(st), a, w, ob)
    (fin[0] * gf).sum().backward()
    traj_c, ga_c, gi_c = cpu_port.rollout(
        params=params, model_tag=tags, ctrl_mode=modes, dt=dt, substeps=substeps, collisions=True,
        k=k, c=c, margin=margin, max_overlap=0.0, neighbor_radius=R_, max_neighbors=K,
        bounds_mode=mode, bounds=bounds, init=[x.numpy() for x in (pos, th, vel, sp, om)],
        actions=acts.numpy(), grad_final_pos=gf.numpy(), obstacles=obstacles, threads=2,
        dtype=np.float64)
    for f in range(5):
        ref = torch.stack([traj[t][f] for t in range(T)]).detach().numpy()
        np.testing.assert_allclose(traj_c[f], ref, rtol=1e-10, atol=1e-12)
    scale = lambda x: 1e-9 * max(np.abs(x).max(), 1e-30)  # noqa: E731
    np.testing.assert_allclose(ga_c, a.grad.numpy(), rtol=1e-9, atol=scale(a.grad.numpy()))
    for f in range(5):
        ref = st[f].grad.numpy()
        np.testing.assert_allclose(gi_c[f], ref, rtol=1e-9, atol=scale(ref))


def test_cpu_port_holonomic_contacts_walls():
    cfgs = [AgentConfig(radius=0.08, max_speed=1.0, max_accel=2.0) for _ in range(8)]
    _case(cfgs, E=4, T=10, seed=0)


def test_cpu_port_mixed_models_substeps_truncation():
    cfgs = ([AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.ACCELERATION,
                         radius=0.07, max_speed=1.5, max_accel=2.0) for _ in range(3)]
            + [AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=m, radius=0.07)
               for m in (ControlMode.VELOCITY, ControlMode.ACCELERATION, ControlMode.SERVO)]
            + [AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, radius=0.07, max_speed=1.0,
                           max_accel=1.0, max_steer=0.5, l_f=0.16, l_r=0.14) for _ in range(3)])
    _case(cfgs, E=3, T=6, seed=1, substeps=2, K=3, spread=0.25)


def test_cpu_port_obstacles_and_clamp():
    cfgs = [AgentConfig(radius=0.06, max_speed=1.2, max_accel=2.0) for _ in range(6)]
    rng = np.random.default_rng(3)
    E, N = 3, 5
    obstacles = dict(pos=(rng.random((E, N, 2)) * 2 - 1) * 0.4, angle=rng.random((E, N)) * 3,
                     vel=rng.standard_normal((E, N, 2)) * 0.2, ang_vel=rng.standard_normal((E, N)) * 0.3,
                     radius=np.array([0.1, 0.0, 0.03, 0.08, 0.0]),
                     half=np.array([[0, 0], [0.1, 0.05], [0.2, 0], [0, 0], [0.05, 0.12]]),
                     shape=np.array([0, 1, 2, 0, 1], dtype=np.int32))
    _case(cfgs, E=E, T=8, seed=2, mode=2, obstacles=obstacles)
