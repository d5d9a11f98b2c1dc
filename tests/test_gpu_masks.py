"""Checkpointed contact masks for envs of 33-256 agents (with and without list truncation).

The forward kernel stores, per agent and substep, the mask of every in-radius agent it is
in contact with (ceil(A/32) words, listed or not); the adjoint gathers its pair VJPs from
those bits instead of rescanning the env, and with list truncation gates the own and cross
terms by the stored cutoffs. The pairs it visits with a nonzero term are exactly those the
rescan visits, in the same ascending order, so trajectories, gradients and uncapped counts
must be bitwise those of the rescan path (forced with SWARP_CONTACT_MASKS=0). Parity of
these worlds with the oracle is covered by the > 32-agent and truncation cases of
test_gpu_parity.py and the config-5 cases of test_gpu_parity_f32.py, which take this path.
"""

from __future__ import annotations

import contextlib
import os

import numpy as np
import pytest
import torch

from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel
from swarp_b200.interop.autograd import TorchState, rollout

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@contextlib.contextmanager
def rescan_path():
    old = os.environ.get("SWARP_CONTACT_MASKS")
    os.environ["SWARP_CONTACT_MASKS"] = "0"
    try:
        yield
    finally:
        if old is None:
            os.environ.pop("SWARP_CONTACT_MASKS", None)
        else:
            os.environ["SWARP_CONTACT_MASKS"] = old


def _run(cfgs, world, dtype, E, T, seed, substeps, obstacles):
    A = len(cfgs)
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=torch.float64) * 2 - 1) * 0.5
    th = (torch.rand(E, A, generator=g, dtype=torch.float64) * 2 - 1) * 3.0
    vel = torch.randn(E, A, 2, generator=g, dtype=torch.float64) * 0.3
    sp = torch.randn(E, A, generator=g, dtype=torch.float64) * 0.3
    om = torch.randn(E, A, generator=g, dtype=torch.float64) * 0.3
    acts = (torch.rand(T, E, A, 2, generator=g, dtype=torch.float64) * 2 - 1) * 1.5
    st = Stepper(cfgs, dt=0.05, substeps=substeps, device=DEV, dtype=dtype, world=world)
    if obstacles is not None:
        st.set_obstacles(obstacles)
    st.track_neighbor_overflow = True
    st.track_grad_norm = True
    s = [x.to(DEV, dtype).requires_grad_(True) for x in (pos, th, vel, sp, om)]
    a = acts.to(DEV, dtype).requires_grad_(True)
    fin, traj = rollout(st, TorchState(*s), a)
    loss = sum((x * (i + 1)).sum() for i, x in enumerate(traj.stacked))
    loss = loss + fin.pos.square().sum()
    loss.backward()
    return ([x.detach().clone() for x in traj.stacked] + [a.grad, *[x.grad for x in s]]
            + [st.last_true_count_max, st.last_grad_sqnorm])


def _obstacles(E, seed):
    rng = np.random.default_rng(seed)
    return Obstacles(pos=torch.from_numpy(rng.uniform(-0.5, 0.5, (E, 3, 2))),
                     radius=torch.tensor([0.06, 0.0, 0.02]), shape=torch.tensor([0, 1, 2]),
                     angle=torch.from_numpy(rng.uniform(-3, 3, (E, 3))),
                     half_extents=torch.tensor([[0.0, 0.0], [0.08, 0.05], [0.12, 0.0]]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("A,K,substeps,obs", [(40, 64, 1, False), (40, 3, 1, True),
                                              (96, 8, 2, False), (256, 10, 1, False),
                                              (256, 12, 2, True)])
def test_masks_bitwise_rescan(dtype, A, K, substeps, obs):
    models = [DynamicsModel.HOLONOMIC, DynamicsModel.DIFF_DRIVE, DynamicsModel.KINEMATIC_BICYCLE]
    cfgs = [AgentConfig(model=models[i % 3], ctrl_mode=ControlMode.ACCELERATION
                        if i % 3 < 2 else ControlMode.VELOCITY, radius=0.03, max_speed=1.5,
                        max_accel=3.0, max_ang_vel=4.0, max_ang_accel=8.0, max_steer=0.6,
                        l_f=0.1, l_r=0.1) for i in range(A)]
    world = WorldConfig(collision_k=80.0, collision_c=1.0, bounds=(-0.6, 0.6, -0.6, 0.6),
                        neighbor_radius=0.1, max_neighbors=K)
    E, T = 6, 5
    ob = _obstacles(E, A) if obs else None
    got = _run(cfgs, world, dtype, E, T, A + K, substeps, ob)
    with rescan_path():
        ref = _run(cfgs, world, dtype, E, T, A + K, substeps, ob)
    assert int(got[11].max()) > 0, "the case has contacts"
    if K < A - 1:
        assert int(got[11].max()) > K, "the truncating case truncates"
    for i, (x, y) in enumerate(zip(got, ref)):
        assert torch.equal(x, y), f"output {i} differs"


def test_masks_bitwise_rescan_holonomic_velocity_f32():
    """The config-5 kernel instance (holonomic velocity fleet, truncating lists)."""
    A = 256
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.15, max_neighbors=32)
    got = _run(cfgs, world, torch.float32, 8, 6, 5, 1, None)
    with rescan_path():
        ref = _run(cfgs, world, torch.float32, 8, 6, 5, 1, None)
    for i, (x, y) in enumerate(zip(got, ref)):
        assert torch.equal(x, y), f"output {i} differs"
