"""The RK4 integrator (WorldConfig.integrator = Integrator.RK4) on the CUDA path (GPU):
forward and hand-derived adjoint against the float64 oracle for every 2-D model and
control mode, with contacts, walls, substeps and clamped bounds, plus the reference's
RK4 known answers (tests/unit/test_dynamics.py:261-298, 484-560)."""

import numpy as np
import pytest
import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, Integrator
from swarp_b200.interop.autograd import TorchState, rollout

from test_gpu_parity import MODEL_CASES, cfgs_of, check, rand_actions, rand_state

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = torch.float64
CASES = MODEL_CASES + [("bicycle-vel", DynamicsModel.KINEMATIC_BICYCLE, ControlMode.VELOCITY)]


@pytest.mark.parametrize("name,model,mode", CASES, ids=[c[0] for c in CASES])
def test_rk4_models_contacts_walls_substeps_f64(name, model, mode):
    world = WorldConfig(collision_k=30.0, collision_c=1.0, collision_margin=0.05,
                        bounds=(-0.4, 0.4, -0.4, 0.4), bounds_mode="soft",
                        integrator=Integrator.RK4)
    st = Stepper(cfgs_of(model, mode, 5, max_speed=1.5, max_accel=2.0, max_ang_vel=2.0,
                         max_ang_accel=4.0), dt=0.05, substeps=2, device=DEV, dtype=D, world=world)
    check(st, rand_state(3, 5, 31), rand_actions(6, 3, 5, 32, scale=2.0), seed=33, final=True)


def test_rk4_saturating_limits_and_clamp_bounds_f64():
    cfgs = [AgentConfig(model=DynamicsModel.HOLONOMIC, radius=0.08, max_speed=1.0),
            AgentConfig(model=DynamicsModel.DIFF_DRIVE, radius=0.08, max_speed=1.0, max_ang_vel=1.0),
            AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, radius=0.08, max_speed=1.0,
                        max_accel=1.0, max_steer=0.5, min_speed=0.0)]
    world = WorldConfig(collision_k=50.0, collision_c=2.0, collision_margin=0.02,
                        bounds=(-0.3, 0.3, -0.3, 0.3), bounds_mode="clamp",
                        integrator=Integrator.RK4)
    st = Stepper(cfgs, dt=0.1, device=DEV, dtype=D, world=world)
    check(st, rand_state(4, 3, 35, spread=0.25), rand_actions(8, 4, 3, 36, scale=3.0), seed=37)


def test_rk4_holonomic_fleet_f32():
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft",
                        neighbor_radius=0.125, max_neighbors=16, integrator=Integrator.RK4)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0)] * 16, dt=0.05,
                 device=DEV, dtype=torch.float32, world=world)
    check(st, rand_state(40, 16, 41, spread=0.9), rand_actions(10, 40, 16, 42, scale=1.0),
          seed=43, dtype=torch.float32, rtol_f=1e-5, rtol_g=1e-4)


def _final_pos(cfg, init, acts, dt, integrator):
    st = Stepper([cfg], dt=dt, device=DEV, dtype=D,
                 world=WorldConfig(collisions=False, integrator=integrator))
    s = TorchState(*(torch.tensor(x, dtype=D, device=DEV).reshape(shape) for x, shape in
                     zip(init, [(1, 1, 2), (1, 1), (1, 1, 2), (1, 1), (1, 1)])))
    a = torch.tensor(acts, dtype=D, device=DEV).reshape(len(acts), 1, 1, 2)
    with torch.no_grad():
        fin, traj = rollout(st, s, a)
    return fin, traj


def test_rk4_convergence_order_circle():
    cfg = AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=ControlMode.VELOCITY,
                      max_speed=5.0, max_ang_vel=5.0)
    s, w = 1.3, 0.9
    init = ([0.2, -0.1], [0.3], [0.0, 0.0], [0.0], [0.0])
    th = 0.3 + w * 2.0
    exact = np.array([0.2 + (s / w) * (np.sin(th) - np.sin(0.3)),
                      -0.1 - (s / w) * (np.cos(th) - np.cos(0.3))])

    def err(integ, N):
        fin, _ = _final_pos(cfg, init, [[s, w]] * N, 2.0 / N, integ)
        return np.linalg.norm(fin.pos[0, 0].cpu().numpy() - exact)

    e1, e2 = err(Integrator.RK4, 100), err(Integrator.RK4, 200)
    u1, u2 = err(Integrator.EULER, 100), err(Integrator.EULER, 200)
    assert np.log2(e1 / e2) > 3.5
    assert 0.8 < np.log2(u1 / u2) < 1.3
    assert e1 < u1 * 1e-3


def test_rk4_matches_euler_on_straight_line():
    cfg = AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.VELOCITY, max_speed=2.0)
    init = ([0.0, 0.0], [0.0], [0.0, 0.0], [0.0], [0.0])
    fe, _ = _final_pos(cfg, init, [[0.7, -0.4]] * 20, 0.05, Integrator.EULER)
    fr, _ = _final_pos(cfg, init, [[0.7, -0.4]] * 20, 0.05, Integrator.RK4)
    torch.testing.assert_close(fr.pos, fe.pos, rtol=0, atol=1e-12)


def test_rk4_bicycle_min_speed_brakes_to_a_stop():
    cfg = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=5.0, max_accel=1.0,
                      l_f=1.25, l_r=1.25, max_steer=0.6, min_speed=0.0)
    init = ([0.0, 0.0], [0.0], [0.5, 0.0], [0.5], [0.0])
    _, traj = _final_pos(cfg, init, [[-1.0, 0.3]] * 30, 0.1, Integrator.RK4)
    speeds = traj.stacked[3][:, 0, 0].cpu().numpy()
    assert speeds.min() == 0.0 and speeds[-1] == 0.0
    rev = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=5.0, max_accel=1.0,
                      l_f=1.25, l_r=1.25, max_steer=0.6)
    fin, _ = _final_pos(rev, init, [[-1.0, 0.3]] * 30, 0.1, Integrator.RK4)
    assert float(fin.speed[0, 0]) < 0.0
