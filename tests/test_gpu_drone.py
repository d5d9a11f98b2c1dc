"""The 6-DOF quadrotor drone (DynamicsModel.DRONE) on the CUDA path (GPU): the reference's
drone known answers (tests/unit/test_drone.py:120-234: hover, closed-form climb, pure yaw,
agreement with a numpy restatement) through the public API, and forward plus
hand-derived adjoint against the float64 oracle (autograd) for mixed drone / 2-D fleets
with contacts, walls, obstacles, clamped bounds, substeps and both integrators."""

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, Integrator
from swarp_b200.interop.autograd import TorchState, rollout, warp_step

from ref_bridge import ref_obstacles, ref_world
from test_gpu_boxes import obstacle_mix
from test_gpu_parity import close
from test_oracle_drone_kats import (ARM, G, HOVER, IXX, IYY, IZZ, KAPPA, MASS, TMAX, fields,
                                    np_euler)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = torch.float64
NAMES = ["pos", "theta", "vel", "speed", "ang_vel", "z", "vz", "attitude", "body_rates"]


def drone(**kw):
    base = dict(model=DynamicsModel.DRONE, mass=MASS, arm_length=ARM, inertia_xx=IXX,
                inertia_yy=IYY, inertia_zz=IZZ, torque_coeff=KAPPA, gravity=G, thrust_max=TMAX)
    base.update(kw)
    return AgentConfig(**base)


def state9(E, A, seed, spread=0.3, tilt=0.2):
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1) * spread
    th = (torch.rand(E, A, generator=g, dtype=D) * 2 - 1) * 3.0
    v = torch.randn(E, A, 2, generator=g, dtype=D) * 0.4
    s = torch.randn(E, A, generator=g, dtype=D) * 0.4
    w = torch.randn(E, A, generator=g, dtype=D) * 0.4
    z = torch.rand(E, A, generator=g, dtype=D) + 0.5
    vz = torch.randn(E, A, generator=g, dtype=D) * 0.2
    q = torch.cat([torch.randn(E, A, 3, generator=g, dtype=D) * tilt, torch.ones(E, A, 1, dtype=D)], -1)
    q = q / q.norm(dim=-1, keepdim=True)
    br = torch.randn(E, A, 3, generator=g, dtype=D) * 0.3
    return (pos, th, v, s, w, z, vz, q, br)


def thrusts(T, E, A, seed, spread=1.5, D_=4):
    g = torch.Generator().manual_seed(seed)
    return HOVER + (torch.rand(T, E, A, D_, generator=g, dtype=D) * 2 - 1) * spread


def weights(T, E, A, seed):
    g = torch.Generator().manual_seed(seed)
    shp = [(T, E, A, 2), (T, E, A), (T, E, A, 2), (T, E, A), (T, E, A), (T, E, A), (T, E, A),
           (T, E, A, 4), (T, E, A, 3)]
    return [torch.randn(*s, generator=g, dtype=D) for s in shp]


def check9(st, s9, acts, seed, dtype=D, rtol_f=1e-10, rtol_g=1e-10):
    T, E, A, _ = acts.shape
    wts = weights(T, E, A, seed)
    # oracle
    ro = [t.clone().requires_grad_(True) for t in s9]
    ra = acts.clone().requires_grad_(True)
    _, traj, _ = R.rollout(tuple(ro), ra, ref_world(st), ref_obstacles(st))
    loss = sum((wf[t] * traj[t][f]).sum() for t in range(T) for f, wf in enumerate(wts))
    gref = torch.autograd.grad(loss, [ra, *ro])
    tref = [torch.stack([traj[t][f] for t in range(T)]).detach() for f in range(9)]
    # CUDA
    co = [t.to(DEV, dtype).clone().requires_grad_(True) for t in s9]
    ca = acts.to(DEV, dtype).clone().requires_grad_(True)
    _, tr = rollout(st, TorchState(*co), ca)
    loss = sum((wf.to(DEV, dtype)[t] * tr[t][f]).sum() for t in range(T) for f, wf in enumerate(wts))
    gcuda = torch.autograd.grad(loss, [ca, *co])
    tcuda = [torch.stack([tr[t][f] for t in range(T)]).detach().cpu().double() for f in range(9)]
    for f in range(9):
        close(tcuda[f], tref[f], rtol_f, f"traj {NAMES[f]}")
    for i, n in enumerate(["actions", *NAMES]):
        close(gcuda[i].cpu().double(), gref[i], rtol_g, f"grad {n}")


# ------------------------------------------------------------ known answers
def run_one(init, thrust_seq, dt):
    st = Stepper([drone()], dt=dt, device=DEV, dtype=D, world=WorldConfig(collisions=False))
    s = TorchState(*(t.to(DEV) for t in init))
    acts = torch.as_tensor(np.asarray(thrust_seq, dtype=np.float64)).reshape(-1, 1, 1, 4).to(DEV)
    with torch.no_grad():
        fin, _ = rollout(st, s, acts)
    return tuple(t.cpu() for t in fin)


def init_state(p=(0.3, -0.2), z=1.0, v=(0.0, 0.0), vz=0.0, q=(0, 0, 0, 1.0), br=(0, 0, 0.0)):
    t = lambda x, shp: torch.tensor(np.asarray(x, dtype=np.float64)).reshape(shp)  # noqa: E731
    zero = torch.zeros(1, 1, dtype=D)
    return (t(p, (1, 1, 2)), zero, t(v, (1, 1, 2)), zero, zero, t(z, (1, 1)), t(vz, (1, 1)),
            t(q, (1, 1, 4)), t(br, (1, 1, 3)))


def test_hover_equilibrium():
    last = fields(run_one(init_state(), np.full((50, 4), HOVER), 0.02))
    np.testing.assert_allclose(last[0], [0.3, -0.2], atol=1e-10)
    np.testing.assert_allclose(last[1], 1.0, atol=1e-10)
    np.testing.assert_allclose(last[4], [0.0, 0.0, 0.0, 1.0], atol=1e-10)
    np.testing.assert_allclose(last[5], [0.0, 0.0, 0.0], atol=1e-12)


def test_vertical_climb_closed_form():
    dt, T, f = 0.02, 40, HOVER + 0.5
    last = fields(run_one(init_state(), np.full((T, 4), f), dt))
    az = 4.0 * f / MASS - G
    np.testing.assert_allclose(last[1], 1.0 + az * dt * dt * T * (T + 1) / 2.0, atol=1e-9)
    np.testing.assert_allclose(last[3], az * dt * T, atol=1e-10)
    np.testing.assert_allclose(last[4], [0.0, 0.0, 0.0, 1.0], atol=1e-12)


def test_pure_yaw_and_numpy_restatement():
    dt, T, d = 0.01, 30, 0.5
    seq = np.tile([HOVER + d, HOVER - d, HOVER + d, HOVER - d], (T, 1))
    last = fields(run_one(init_state(), seq, dt))
    np.testing.assert_allclose(last[1], 1.0, atol=1e-9)
    assert last[5][2] > 1e-3 and abs(last[4][2]) > 1e-3
    ref = np_euler([0.3, -0.2], 1.0, [0.0, 0.0], 0.0, [0, 0, 0, 1.0], [0, 0, 0], seq, dt)
    np.testing.assert_allclose(last[4], ref[4], atol=1e-9)
    rng = np.random.default_rng(0)
    seq = HOVER + 0.4 * rng.standard_normal((60, 4))
    init = dict(p=(0.0, 0.0), z=0.5, v=(0.1, -0.05), vz=0.2, q=(0, 0, 0, 1.0), br=(0.05, -0.03, 0.1))
    last = fields(run_one(init_state(**init), seq, 0.01))
    ref = np_euler(init["p"], init["z"], init["v"], init["vz"], init["q"], init["br"], seq, 0.01)
    for got, want in zip(last, ref):
        np.testing.assert_allclose(got, want, atol=1e-9)


# ------------------------------------------------------------ oracle parity
def fleet(n):
    kinds = [drone(), AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.ACCELERATION,
                                  max_speed=2.0, max_accel=3.0),
             drone(mass=0.8, thrust_max=8.0),
             AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=ControlMode.VELOCITY, max_speed=1.5,
                         max_ang_vel=2.0),
             AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=ControlMode.SERVO, max_speed=1.5,
                         max_ang_vel=2.0, max_accel=2.0, max_ang_accel=4.0)]
    return [kinds[i % len(kinds)] for i in range(n)]


@pytest.mark.parametrize("rk4", [False, True], ids=["euler", "rk4"])
@pytest.mark.parametrize("walls", ["soft", "clamp"])
def test_mixed_fleet_contacts_obstacles_f64(rk4, walls):
    world = WorldConfig(collision_k=40.0, collision_c=1.0, collision_margin=0.02,
                        bounds=(-0.5, 0.5, -0.5, 0.5), bounds_mode=walls,
                        integrator=Integrator.RK4 if rk4 else Integrator.EULER)
    st = Stepper(fleet(7), dt=0.02, substeps=2, device=DEV, dtype=D, world=world)
    E = 4
    st.set_obstacles(obstacle_mix(E, 5))
    check9(st, state9(E, 7, 6, spread=0.45), thrusts(6, E, 7, 7), seed=8)


def test_truncated_lists_and_action_slots_f64():
    """More in-radius neighbors than max_neighbors, and 3 action slots (the fourth rotor
    reads zero)."""
    world = WorldConfig(collision_k=20.0, collision_c=0.5, collision_margin=0.02,
                        neighbor_radius=0.3, max_neighbors=3)
    st = Stepper(fleet(10), dt=0.02, device=DEV, dtype=D, world=world)
    check9(st, state9(3, 10, 11, spread=0.2), thrusts(5, 3, 10, 12, D_=3), seed=13)


def test_sixteen_agent_fleet_f32():
    world = WorldConfig(collision_k=40.0, collision_c=1.0, collision_margin=0.02,
                        bounds=(-1.0, 1.0, -1.0, 1.0))
    st = Stepper(fleet(16), dt=0.02, device=DEV, dtype=torch.float32, world=world)
    check9(st, state9(16, 16, 21, spread=0.9), thrusts(4, 16, 16, 22, spread=0.5), seed=23,
           dtype=torch.float32, rtol_f=1e-5, rtol_g=1e-4)


def test_warp_step_and_default_drone_fields():
    """warp_step on a drone fleet steps all nine fields; a TorchState without drone fields
    starts level at z = 0 (identity attitude)."""
    st = Stepper(fleet(3), dt=0.02, device=DEV, dtype=D, world=WorldConfig(collisions=False))
    s5 = TorchState(*(t.to(DEV) for t in state9(2, 3, 31)[:5]))
    acts = torch.full((2, 3, 4), HOVER, dtype=D, device=DEV)
    out = warp_step(st, s5, acts)
    assert out.z.shape == (2, 3) and out.attitude.shape == (2, 3, 4)
    ref = R.step(tuple(t.cpu() for t in (*tuple(s5)[:5], torch.zeros(2, 3, device=DEV, dtype=D),
                                         torch.zeros(2, 3, device=DEV, dtype=D),
                                         torch.tensor([0, 0, 0, 1.0], dtype=D, device=DEV).expand(2, 3, 4),
                                         torch.zeros(2, 3, 3, device=DEV, dtype=D))),
                 acts.cpu(), ref_world(st))[0]
    for f in range(9):
        close(out[f].cpu(), ref[f], 1e-10, NAMES[f])


@pytest.mark.parametrize("substeps", [1, 2])
def test_drones_push_movable_body_f64(substeps):
    """A mixed fleet with drones around a movable three-circle body: the drones push it as
    discs (their 2-D position, velocity and radius), the body moves on grad rollouts
    (bodies_in_grad), and trajectories (all nine fields), the final body state and the
    gradients of a loss on both match the oracle at the float64 bars."""
    from swarp_b200.interop.autograd import rollout_bodies

    from test_gpu_bodies import compound_body, transport_world

    E, A, T = 4, 6, 12
    st = Stepper(fleet(A), dt=0.02, substeps=substeps, device=DEV, dtype=D,
                 world=transport_world())
    obs = compound_body(E, 31)
    st.set_obstacles(obs)
    st.bodies_in_grad = True
    s9 = list(state9(E, A, 32, spread=0.25))
    s9[0] = obs.pos[:, 1:2, :] + (s9[0] - s9[0].mean(1, keepdim=True)) * 0.9
    acts = thrusts(T, E, A, 33, spread=1.0)
    goal = torch.tensor([0.3, -0.1], dtype=D)

    w = ref_world(st)
    ob = ref_obstacles(st)
    ro = [t.clone().requires_grad_(True) for t in s9]
    ra = acts.clone().requires_grad_(True)
    fin_r, traj_r, body_r = R.rollout(tuple(ro), ra, w, ob)
    loss_r = ((body_r[-1].body_pos[:, 0] - goal) ** 2).sum() + (fin_r[0] ** 2).sum() \
        + 0.1 * fin_r[5].sum()
    gref = torch.autograd.grad(loss_r, [ra, *ro])

    co = [t.to(DEV).clone().requires_grad_(True) for t in s9]
    ca = acts.to(DEV).clone().requires_grad_(True)
    fin, traj, body = rollout_bodies(st, TorchState(*co), ca)
    loss = ((body.pos[:, 0] - goal.to(DEV)) ** 2).sum() + (fin.pos ** 2).sum() + 0.1 * fin.z.sum()
    gcuda = torch.autograd.grad(loss, [ca, *co])
    for f in range(9):
        close(traj.stacked[f].detach().cpu(), torch.stack([t[f] for t in traj_r]).detach(), 1e-10,
              f"traj {NAMES[f]}")
    close(body.pos[:, 0].detach().cpu(), body_r[-1].body_pos[:, 0].detach(), 1e-10, "body pos")
    close(body.angle[:, 0].detach().cpu(), body_r[-1].body_angle[:, 0].detach(), 1e-10,
          "body angle")
    moved = (body.pos[:, 0].detach().cpu() - ob.body_pos[:, 0]).norm(dim=-1).max()
    assert float(moved) > 1e-3, "the body was pushed"
    for i, n in enumerate(["actions", *NAMES]):
        close(gcuda[i].cpu(), gref[i], 1e-9, f"grad {n}")
