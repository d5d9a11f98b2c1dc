"""Pin the CPU oracle against the reference's known-answer tests (CPU only).

Each case restates a known answer from the reference test-suite (ddebenedittis/swarp):
numpy recurrences (``tests/unit/test_dynamics.py:28-93,137-381``), hand-computed
contacts (``tests/unit/test_collisions.py:24-138``), analytic BPTT gradients
(``tests/unit/test_gradients.py:174-221``) and the neighbor overflow flag
(``tests/unit/test_neighbors.py:229-264``). The reference has no stored golden
arrays; these in-test answers are what pins its behaviour.
"""

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, param_rows

D = torch.float64
BIG = 100.0


def world(cfgs, dt, **kw):
    return R.RefWorld(
        params=torch.tensor(param_rows(cfgs), dtype=D),
        model_tag=[int(c.model) for c in cfgs],
        ctrl_mode=[int(c.ctrl_mode) for c in cfgs],
        dt=dt,
        **kw,
    )


def state_of(pos, theta=None, vel=None, speed=None, ang_vel=None):
    pos = torch.as_tensor(np.asarray(pos, dtype=np.float64)).reshape(1, -1, 2)
    n = pos.shape[1]

    def s(x):
        return torch.zeros(1, n, dtype=D) if x is None else torch.as_tensor(
            np.asarray(x, dtype=np.float64)).reshape(1, n)

    v = torch.zeros(1, n, 2, dtype=D) if vel is None else torch.as_tensor(
        np.asarray(vel, dtype=np.float64)).reshape(1, n, 2)
    return (pos, s(theta), v, s(speed), s(ang_vel))


def run(w, st, actions):
    traj = []
    for a in actions:
        st, _, _ = R.step(st, torch.as_tensor(a, dtype=D).reshape(1, -1, 2), w)
        traj.append(st)
    return traj


def _clamp_norm(v, limit):
    n = np.linalg.norm(v)
    return v * (limit / max(n, limit))


@pytest.mark.parametrize("mode", [ControlMode.VELOCITY, ControlMode.ACCELERATION])
def test_holonomic_recurrence(mode):
    cfg = AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=mode, max_speed=1.3, max_accel=2.0)
    rng = np.random.default_rng(0)
    T, dt = 100, 0.05
    acts = 2.0 * rng.standard_normal((T, 1, 2))
    traj = run(world([cfg], dt, collisions=False), state_of([[0.3, -0.2]], vel=[[0.1, 0.2]]), acts)
    p, v = np.array([0.3, -0.2]), np.array([0.1, 0.2])
    for t in range(T):
        if mode == ControlMode.VELOCITY:
            v = _clamp_norm(acts[t, 0], cfg.max_speed)
        else:
            v = _clamp_norm(v + _clamp_norm(acts[t, 0], cfg.max_accel) * dt, cfg.max_speed)
        p = p + v * dt
        np.testing.assert_allclose(traj[t][0][0, 0].numpy(), p, atol=1e-12)
        np.testing.assert_allclose(traj[t][2][0, 0].numpy(), v, atol=1e-12)
    assert traj[-1][1][0, 0].item() == 0.0
    np.testing.assert_allclose(traj[-1][3][0, 0].item(), np.linalg.norm(v), atol=1e-12)


@pytest.mark.parametrize("mode", list(ControlMode))
def test_diff_drive_recurrence(mode):
    cfg = AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=mode, max_speed=1.0,
                      max_accel=1.5, max_ang_vel=2.0, max_ang_accel=4.0, cmd_gain_v=1.1,
                      cmd_gain_w=0.8)
    rng = np.random.default_rng(1)
    T, dt = 100, 0.05
    acts = 2.0 * rng.standard_normal((T, 1, 2))
    st = state_of([[0.0, 0.0]], theta=[0.7], speed=[0.2], ang_vel=[-0.3])
    traj = run(world([cfg], dt, collisions=False), st, acts)
    p, th, s, w = np.zeros(2), 0.7, 0.2, -0.3
    for t in range(T):
        a = acts[t, 0]
        if mode == ControlMode.VELOCITY:
            s_n = np.clip(a[0], -cfg.max_speed, cfg.max_speed)
            w_n = np.clip(a[1], -cfg.max_ang_vel, cfg.max_ang_vel)
        elif mode == ControlMode.SERVO:
            tv = np.clip(a[0], -cfg.max_speed, cfg.max_speed) * cfg.cmd_gain_v
            tw = np.clip(a[1], -cfg.max_ang_vel, cfg.max_ang_vel) * cfg.cmd_gain_w
            dv, dw = cfg.max_accel * dt, cfg.max_ang_accel * dt
            s_n = np.clip(s + np.clip(tv - s, -dv, dv), -cfg.max_speed, cfg.max_speed)
            w_n = np.clip(w + np.clip(tw - w, -dw, dw), -cfg.max_ang_vel, cfg.max_ang_vel)
        else:
            s_n = np.clip(s + np.clip(a[0], -cfg.max_accel, cfg.max_accel) * dt,
                          -cfg.max_speed, cfg.max_speed)
            w_n = np.clip(w + np.clip(a[1], -cfg.max_ang_accel, cfg.max_ang_accel) * dt,
                          -cfg.max_ang_vel, cfg.max_ang_vel)
        vt = s_n * np.array([np.cos(th), np.sin(th)])
        p = p + vt * dt
        th = th + w_n * dt
        s, w = s_n, w_n
        got = traj[t]
        np.testing.assert_allclose(got[0][0, 0].numpy(), p, atol=1e-12)
        np.testing.assert_allclose(got[1][0, 0].item(), th, atol=1e-12)
        np.testing.assert_allclose(got[2][0, 0].numpy(), vt, atol=1e-12)
        np.testing.assert_allclose(got[3][0, 0].item(), s, atol=1e-12)
        np.testing.assert_allclose(got[4][0, 0].item(), w, atol=1e-12)


def _bicycle_ref(p, th, s, acts, cfg, dt):
    wb = cfg.l_f + cfg.l_r
    out = []
    lo = -cfg.max_speed if cfg.min_speed is None else cfg.min_speed
    for a in acts:
        acc = np.clip(a[0], -cfg.max_accel, cfg.max_accel)
        delta = np.clip(a[1], -cfg.max_steer, cfg.max_steer)
        s = np.clip(s + acc * dt, lo, cfg.max_speed)
        beta = np.arctan2(np.tan(delta) * cfg.l_r / wb, 1.0)
        vt = s * np.array([np.cos(th + beta), np.sin(th + beta)])
        w = s / wb * np.cos(beta) * np.tan(delta)
        p = p + vt * dt
        th = th + w * dt
        out.append((p.copy(), th, vt, s, w))
    return out


def test_bicycle_recurrence():
    cfg = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, ctrl_mode=ControlMode.ACCELERATION,
                      max_speed=2.0, max_accel=1.0, l_f=0.16, l_r=0.14, max_steer=0.6)
    rng = np.random.default_rng(2)
    T, dt = 100, 0.05
    acts = 2.0 * rng.standard_normal((T, 1, 2))
    traj = run(world([cfg], dt, collisions=False),
               state_of([[1.0, -1.0]], theta=[-0.5], speed=[0.5]), acts)
    ref = _bicycle_ref(np.array([1.0, -1.0]), -0.5, 0.5, acts[:, 0], cfg, dt)
    for t in range(T):
        np.testing.assert_allclose(traj[t][0][0, 0].numpy(), ref[t][0], atol=1e-12)
        np.testing.assert_allclose(traj[t][1][0, 0].item(), ref[t][1], atol=1e-12)
        np.testing.assert_allclose(traj[t][3][0, 0].item(), ref[t][3], atol=1e-12)
        np.testing.assert_allclose(traj[t][4][0, 0].item(), ref[t][4], atol=1e-12)


def test_bicycle_straight_line_analytic():
    cfg = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=10.0, max_accel=1.0,
                      l_f=0.15, l_r=0.15, max_steer=0.6)
    T, dt, acc = 20, 0.1, 0.8
    traj = run(world([cfg], dt, collisions=False), state_of([[0.0, 0.0]]),
               np.tile(np.array([acc, 0.0]), (T, 1, 1)))
    np.testing.assert_allclose(traj[-1][0][0, 0].numpy(),
                               [acc * dt * dt * T * (T + 1) / 2, 0.0], atol=1e-12)
    np.testing.assert_allclose(traj[-1][3][0, 0].item(), acc * dt * T, atol=1e-12)


def test_bicycle_min_speed_brakes_to_a_stop():
    cfg = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=5.0, max_accel=1.0,
                      l_f=1.25, l_r=1.25, max_steer=0.6, min_speed=0.0)
    traj = run(world([cfg], 0.1, collisions=False),
               state_of([[0.0, 0.0]], vel=[[0.5, 0.0]], speed=[0.5]),
               np.tile(np.array([-1.0, 0.3]), (30, 1, 1)))
    speeds = np.array([s[3][0, 0].item() for s in traj])
    assert speeds.min() == 0.0 and speeds[-1] == 0.0
    stopped = int(np.argmax(speeds == 0.0))
    assert torch.equal(traj[stopped][0], traj[-1][0])


def test_clamping_saturates():
    dt = 0.1
    big = np.array([[[100.0, 100.0]]])
    h = AgentConfig(model=DynamicsModel.HOLONOMIC, max_speed=1.0)
    out = run(world([h], dt, collisions=False), state_of([[0.0, 0.0]]), big)
    np.testing.assert_allclose(np.linalg.norm(out[0][2][0, 0].numpy()), 1.0, atol=1e-12)
    b = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=1.0, max_accel=0.5,
                    max_steer=0.3, l_f=0.1, l_r=0.1)
    out = run(world([b], dt, collisions=False), state_of([[0.0, 0.0]]), big)
    np.testing.assert_allclose(out[0][3][0, 0].item(), 0.5 * dt, atol=1e-12)
    ref = _bicycle_ref(np.zeros(2), 0.0, 0.0, np.array([[100.0, 100.0]]), b, dt)
    np.testing.assert_allclose(out[0][1][0, 0].item(), ref[0][1], atol=1e-12)


def holo(n, radius=0.1, mode=ControlMode.VELOCITY):
    return [AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=mode, radius=radius,
                        max_speed=BIG, max_accel=BIG) for _ in range(n)]


def test_two_agent_spring_analytic():
    w = world(holo(2), 0.1, k=100.0, c=0.0, margin=0.02, neighbor_radius=0.22)
    st, _, _ = R.step(state_of([[0.0, 0.0], [0.15, 0.0]]), torch.zeros(1, 2, 2, dtype=D), w)
    np.testing.assert_allclose(st[0][0, 0].numpy(), [-0.07, 0.0], atol=1e-12)
    np.testing.assert_allclose(st[0][0, 1].numpy(), [0.22, 0.0], atol=1e-12)
    np.testing.assert_allclose(st[2][0, 0].numpy(), [-0.7, 0.0], atol=1e-12)


def test_two_agent_spring_damper_analytic():
    w = world(holo(2, mode=ControlMode.ACCELERATION), 0.1, k=100.0, c=2.0, margin=0.02,
              neighbor_radius=0.22)
    st, _, _ = R.step(state_of([[0.0, 0.0], [0.15, 0.0]], vel=[[0.5, 0.0], [-0.5, 0.0]]),
                      torch.zeros(1, 2, 2, dtype=D), w)
    # coeff = (100*0.07 + 2*1) / (1 + 2*0.1/1) = 7.5 -> v0 = 0.5 - 0.75
    np.testing.assert_allclose(st[2][0, 0].numpy(), [-0.25, 0.0], atol=1e-12)
    np.testing.assert_allclose(st[0][0, 0].numpy(), [-0.025, 0.0], atol=1e-12)
    np.testing.assert_allclose(st[2][0, 1].numpy(), [0.25, 0.0], atol=1e-12)


def test_momentum_symmetry():
    w = world(holo(4, mode=ControlMode.ACCELERATION), 0.05, substeps=2, k=50.0, c=0.5,
              margin=0.05, neighbor_radius=0.25)
    rng = np.random.default_rng(0)
    pos0 = rng.random((4, 2)) * 0.2
    st = state_of(pos0)
    com0 = st[0].mean(1)
    for _ in range(20):
        st, _, _ = R.step(st, torch.zeros(1, 4, 2, dtype=D), w)
    torch.testing.assert_close(st[0].mean(1), com0, atol=1e-10, rtol=0)
    assert (st[0][0, 0] - st[0][0, 1]).norm() > np.linalg.norm(pos0[0] - pos0[1])


def _circle_obstacles(pos, radius):
    pos = torch.tensor(pos, dtype=D)
    E, N = pos.shape[0], pos.shape[1]
    return R.RefObstacles(pos=pos, angle=torch.zeros(E, N, dtype=D),
                          vel=torch.zeros(E, N, 2, dtype=D), ang_vel=torch.zeros(E, N, dtype=D),
                          radius=torch.tensor(radius, dtype=D), half=torch.zeros(N, 2, dtype=D),
                          shape=[0] * N, kind=[0] * N)


def test_obstacle_repulsion_analytic():
    w = world(holo(1), 0.1, k=100.0, c=0.0, margin=0.02, neighbor_radius=0.22)
    st, _, _ = R.step(state_of([[0.1, 0.0]]), torch.zeros(1, 1, 2, dtype=D), w,
                      _circle_obstacles([[[0.3, 0.0]]], [0.15]))
    np.testing.assert_allclose(st[0][0, 0].numpy(), [0.1 - 0.07, 0.0], atol=1e-12)


def test_soft_wall_analytic():
    w = world(holo(1, radius=0.05), 0.1, k=100.0, c=0.0, margin=0.02, neighbor_radius=0.12,
              bounds=(-1.0, 1.0, -1.0, 1.0), soft_walls=True)
    st, _, _ = R.step(state_of([[0.95, 0.0]]), torch.zeros(1, 1, 2, dtype=D), w)
    np.testing.assert_allclose(st[0][0, 0].numpy(), [0.95 - 0.02, 0.0], atol=1e-12)


def test_clamp_bounds():
    w = world(holo(1, radius=0.05), 0.1, collisions=False, bounds=(-1.0, 1.0, -1.0, 1.0),
              clamp_bounds=True)
    st, _, _ = R.step(state_of([[0.98, 0.0]]), torch.tensor([[[5.0, 0.0]]], dtype=D), w)
    np.testing.assert_allclose(st[0][0, 0].numpy(), [0.95, 0.0], atol=1e-12)


def _grad_state(seed, n=1):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(*s, generator=g, dtype=D) * 0.5
                 for s in ((1, n, 2), (1, n), (1, n, 2), (1, n), (1, n)))


def test_bptt_analytic_holonomic():
    T, dt = 6, 0.1
    w = world([AgentConfig(model=DynamicsModel.HOLONOMIC, max_speed=BIG)], dt, collisions=False)
    acts = (0.2 * torch.randn(T, 1, 1, 2, dtype=D)).requires_grad_(True)
    final, _, _ = R.rollout(_grad_state(4), acts, w)
    final[0][0, 0, 0].backward()
    expected = torch.zeros_like(acts)
    expected[:, 0, 0, 0] = dt
    torch.testing.assert_close(acts.grad, expected)


def test_bptt_analytic_holonomic_accel():
    dt = 0.1
    w = world([AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.ACCELERATION,
                           max_speed=BIG, max_accel=BIG)], dt, collisions=False)
    acts = (0.2 * torch.randn(2, 1, 1, 2, dtype=D)).requires_grad_(True)
    final, _, _ = R.rollout(_grad_state(5), acts, w)
    final[0][0, 0, 0].backward()
    torch.testing.assert_close(acts.grad[0, 0, 0, 0], torch.tensor(2 * dt * dt, dtype=D))


def test_grads_zero_when_saturated():
    w = world([AgentConfig(model=DynamicsModel.DIFF_DRIVE, max_speed=1.0, max_ang_vel=1.0)], 0.1,
              collisions=False)
    acts = torch.full((1, 1, 2), 50.0, dtype=D, requires_grad=True)
    st, _, _ = R.step(_grad_state(6), acts, w)
    st[0].sum().backward()
    assert torch.isfinite(acts.grad).all() and acts.grad.abs().sum() == 0.0


def test_neighbor_overflow_flag():
    pos = torch.zeros(1, 5, 2, dtype=D)
    pos[0, :, 0] = torch.linspace(0.0, 0.04, 5, dtype=D)
    in_list, idx, cnt, true = R.brute_neighbors(pos, 0.5, 2)
    assert torch.equal(true, torch.full((1, 5), 4))
    assert torch.equal(cnt, torch.full((1, 5), 2))
    for a in range(5):
        picked = set(idx[0, a, :2].tolist())
        assert len(picked) == 2 and a not in picked
        # first two by index
        assert sorted(picked) == [b for b in range(5) if b != a][:2]
    _, _, cnt8, _ = R.brute_neighbors(pos, 0.5, 8)
    assert torch.equal(cnt8, true)


def test_gradcheck_oracle_with_collisions_and_walls():
    w = world(holo(2, mode=ControlMode.ACCELERATION), 0.1, substeps=2, k=10.0, c=1.0,
              margin=0.02, neighbor_radius=0.22, bounds=(-1.0, 1.0, -1.0, 1.0), soft_walls=True)
    st = state_of([[0.0, 0.0], [0.18, 0.02]], vel=[[0.1, 0.0], [-0.1, 0.05]])
    acts = 0.1 * torch.randn(1, 2, 2, dtype=D, generator=torch.Generator().manual_seed(0))

    def fn(pos, th, vel, sp, om, act):
        out, _, _ = R.step((pos, th, vel, sp, om), act, w)
        return out

    inputs = tuple(t.clone().requires_grad_(True) for t in (*st, acts))
    assert torch.autograd.gradcheck(fn, inputs, eps=1e-6, atol=1e-5)


# --------------------------------------------------------------------- RK4
# reference tests/unit/test_dynamics.py:261-298 (RK4 arm), :484-560


def _dd_circle_final(dt, N, rk4):
    cfg = AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=ControlMode.VELOCITY,
                      max_speed=5.0, max_ang_vel=5.0)
    s, w = 1.3, 0.9
    traj = run(world([cfg], dt, collisions=False, rk4=rk4), state_of([[0.2, -0.1]], theta=[0.3]),
               np.tile(np.array([s, w]), (N, 1, 1)))
    th = 0.3 + w * dt * N
    exact = np.array([0.2 + (s / w) * (np.sin(th) - np.sin(0.3)),
                      -0.1 - (s / w) * (np.cos(th) - np.cos(0.3))])
    return np.linalg.norm(traj[-1][0][0, 0].numpy() - exact)


def test_rk4_convergence_order():
    """On the circular diff-drive trajectory RK4 converges ~dt^4, Euler ~dt^1."""
    e_rk, e_rk2 = _dd_circle_final(2.0 / 100, 100, True), _dd_circle_final(2.0 / 200, 200, True)
    e_eu, e_eu2 = _dd_circle_final(2.0 / 100, 100, False), _dd_circle_final(2.0 / 200, 200, False)
    assert np.log2(e_rk / e_rk2) > 3.5
    assert 0.8 < np.log2(e_eu / e_eu2) < 1.3
    assert e_rk < e_eu * 1e-3


def test_rk4_matches_euler_on_straight_line():
    cfg = AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.VELOCITY, max_speed=2.0)
    acts = np.tile(np.array([0.7, -0.4]), (20, 1, 1))
    eu = run(world([cfg], 0.05, collisions=False), state_of([[0.0, 0.0]]), acts)
    rk = run(world([cfg], 0.05, collisions=False, rk4=True), state_of([[0.0, 0.0]]), acts)
    np.testing.assert_allclose(rk[-1][0].numpy(), eu[-1][0].numpy(), atol=1e-12)


def test_rk4_bicycle_min_speed_stops_but_creeps():
    """min_speed = 0 stops the car under full braking; RK4 applies limits to the combined
    result only, so (unlike Euler) its pose still moves after the speed reaches zero."""
    cfg = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=5.0, max_accel=1.0,
                      l_f=1.25, l_r=1.25, max_steer=0.6, min_speed=0.0)
    init = state_of([[0.0, 0.0]], vel=[[0.5, 0.0]], speed=[0.5])
    acts = np.tile(np.array([-1.0, 0.3]), (30, 1, 1))
    traj = run(world([cfg], 0.1, collisions=False, rk4=True), init, acts)
    speeds = np.array([s[3][0, 0].item() for s in traj])
    assert speeds.min() == 0.0 and speeds[-1] == 0.0
    rev = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=5.0, max_accel=1.0,
                      l_f=1.25, l_r=1.25, max_steer=0.6)
    traj_rev = run(world([rev], 0.1, collisions=False, rk4=True), init, acts)
    assert traj_rev[-1][3][0, 0].item() < 0.0


@pytest.mark.parametrize("model,mode", [
    (DynamicsModel.HOLONOMIC, ControlMode.VELOCITY), (DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION),
    (DynamicsModel.DIFF_DRIVE, ControlMode.VELOCITY), (DynamicsModel.DIFF_DRIVE, ControlMode.ACCELERATION),
    (DynamicsModel.DIFF_DRIVE, ControlMode.SERVO), (DynamicsModel.KINEMATIC_BICYCLE, ControlMode.VELOCITY)])
def test_gradcheck_oracle_rk4_step(model, mode):
    """reference tests/unit/test_gradients.py:77-108: the RK4 step is differentiable."""
    cfgs = [AgentConfig(model=model, ctrl_mode=mode, max_speed=BIG, max_accel=BIG, max_ang_vel=BIG,
                        max_ang_accel=BIG, max_steer=1.0, l_f=0.16, l_r=0.14) for _ in range(2)]
    w = world(cfgs, 0.1, collisions=False, rk4=True)
    g = torch.Generator().manual_seed(1)
    st = [torch.randn(2, 2, 2, generator=g, dtype=D), torch.randn(2, 2, generator=g, dtype=D),
          torch.randn(2, 2, 2, generator=g, dtype=D), torch.randn(2, 2, generator=g, dtype=D),
          torch.randn(2, 2, generator=g, dtype=D)]
    st = [x.requires_grad_(True) for x in st]
    a = (0.3 * torch.randn(2, 2, 2, generator=g, dtype=D)).requires_grad_(True)

    def fn(p, th, v, s, om, act):
        return R.step((p, th, v, s, om), act, w)[0]

    assert torch.autograd.gradcheck(fn, (*st, a), eps=1e-6, atol=1e-5)


# ------------------------------------------------- contact laws: finite differences
# The reference pins its contact gradients only where no contact is active
# (tests/unit/test_gradients.py:174-221); the oracle's autograd through the contact laws is
# pinned here by central finite differences (torch.autograd.gradcheck) on contact-active
# inputs held away from the laws' kinks (contact onset, the clamp of the coefficient at
# zero, the box's face switch and corner region, the wall's onset).


def _gc(fn, *xs):
    inputs = tuple(torch.as_tensor(x, dtype=D).clone().requires_grad_(True) for x in xs)
    assert torch.autograd.gradcheck(fn, inputs, eps=1e-7, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("max_overlap", [0.0, 0.03])
def test_pair_force_finite_differences(max_overlap):
    # overlap 0.12 - |d| > 0 in every row; k * ov - c * vn > 0 (repulsive, unclamped)
    dx = [0.05, -0.07, 0.01, 0.09]
    dy = [0.03, 0.02, -0.08, -0.01]
    rvx = [0.2, -0.1, 0.05, -0.3]
    rvy = [-0.1, 0.3, 0.1, 0.05]

    def fn(dx, dy, rvx, rvy):
        return R.pair_force(dx, dy, rvx, rvy, 0.12, 40.0, 0.5, 1.3, max_overlap)

    _gc(fn, dx, dy, rvx, rvy)


@pytest.mark.parametrize("inside", [False, True])
def test_box_force_finite_differences(inside):
    # outside: the point's closest box point on a face or a corner, within reach; inside:
    # the point past a face (the face with the larger q chosen, away from the tie)
    if inside:
        px, py = [0.05, -0.02, 0.01], [0.01, 0.06, -0.075]
    else:
        px, py = [0.17, -0.03, 0.16], [0.02, -0.13, 0.11]
    vx, vy = [0.1, -0.2, 0.05], [0.0, 0.1, -0.1]

    def fn(px, py, vx, vy, cx, cy, ang, vox, voy, om):
        return R.box_force(px, py, vx, vy, cx, cy, ang, 0.12, 0.08, 0.06, 40.0, 0.5, 1.2, 0.0,
                           vox, voy, om)

    _gc(fn, px, py, vx, vy, [0.01] * 3, [-0.01] * 3, [0.2] * 3, [0.05] * 3, [-0.02] * 3,
        [0.3] * 3)


def test_wall_law_finite_differences():
    # agents pressed into each of the four walls (and one into a corner), closing speeds
    # below k * penetration / c so the coefficient stays positive
    w = world(holo(5), 0.05, collisions=False, k=40.0, c=0.5, margin=0.02,
              bounds=(-1.0, 1.0, -1.0, 1.0), soft_walls=True)
    px = [-0.95, 0.96, 0.1, -0.2, 0.97]
    py = [0.1, -0.3, -0.94, 0.955, 0.96]
    vx = [-0.1, 0.2, 0.0, 0.05, 0.1]
    vy = [0.0, 0.05, -0.2, 0.1, 0.1]

    def fn(px, py, vx, vy):
        ra = torch.full_like(px, 0.07)
        return R.wall_forces(px, py, vx, vy, ra, w, torch.full_like(px, 1.2))

    _gc(fn, px, py, vx, vy)


def test_obstacle_step_gradcheck():
    # a full step with circle, box and segment obstacles in contact, through autograd
    cfgs = holo(3, mode=ControlMode.ACCELERATION)
    w = world(cfgs, 0.05, collisions=True, k=40.0, c=0.5, margin=0.02, neighbor_radius=0.3,
              bounds=(-1.0, 1.0, -1.0, 1.0), soft_walls=True)
    ob = R.RefObstacles(pos=torch.tensor([[[0.0, 0.0], [0.5, 0.5], [-0.5, 0.4]]], dtype=D),
                        angle=torch.tensor([[0.0, 0.3, -0.4]], dtype=D),
                        vel=torch.zeros(1, 3, 2, dtype=D), ang_vel=torch.zeros(1, 3, dtype=D),
                        radius=torch.tensor([0.1, 0.0, 0.02], dtype=D),
                        half=torch.tensor([[0.0, 0.0], [0.1, 0.06], [0.2, 0.0]], dtype=D),
                        shape=[0, 1, 2], kind=[0, 0, 0])
    st = state_of([[0.15, 0.03], [0.5, 0.63], [-0.48, 0.45]],
                  vel=[[-0.1, 0.0], [0.0, -0.1], [0.05, -0.05]])
    acts = 0.1 * torch.randn(1, 3, 2, dtype=D, generator=torch.Generator().manual_seed(1))

    def fn(pos, vel, act):
        out, _, _ = R.step((pos, st[1], vel, st[3], st[4]), act, w, ob)
        return out[0], out[2]

    fx, fy = R.obstacle_forces(st[0][..., 0], st[0][..., 1], st[2][..., 0], st[2][..., 1],
                               torch.full((1, 3), 0.08, dtype=D), ob, w,
                               torch.ones(1, 3, dtype=D))
    assert bool((fx.abs() + fy.abs() > 0).all()), "every agent touches its obstacle"
    _gc(fn, st[0], st[2], acts)
