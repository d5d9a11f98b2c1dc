"""The 6-DOF quadrotor drone in the CPU oracle, pinned by the reference's drone known
answers (ddebenedittis/swarp tests/unit/test_drone.py:120-234): hover equilibrium,
closed-form vertical climb, pure yaw torque, agreement with a plain numpy restatement of
the semi-implicit Euler recurrence, and a gradcheck; plus the RK4 drone's fourth-order
convergence, the one-sided thrust clamp and the 2-D fleet passing the 6-DOF fields
through (CPU only)."""

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.dynamics.base import AgentConfig, DynamicsModel, param_rows

D = torch.float64
MASS, ARM, IXX, IYY, IZZ, KAPPA, G, TMAX = 1.0, 0.15, 0.01, 0.01, 0.02, 0.02, 9.81, 20.0
HOVER = MASS * G / 4.0


def drone_cfg(**kw):
    base = dict(model=DynamicsModel.DRONE, mass=MASS, arm_length=ARM, inertia_xx=IXX,
                inertia_yy=IYY, inertia_zz=IZZ, torque_coeff=KAPPA, gravity=G, thrust_max=TMAX)
    base.update(kw)
    return AgentConfig(**base)


def world(cfgs, dt, rk4=False):
    return R.RefWorld(params=torch.tensor(param_rows(cfgs), dtype=D),
                      model_tag=[int(c.model) for c in cfgs], ctrl_mode=[int(c.ctrl_mode) for c in cfgs],
                      dt=dt, collisions=False, rk4=rk4)


def state9(p=(0.3, -0.2), z=1.0, v=(0.0, 0.0), vz=0.0, q=(0.0, 0.0, 0.0, 1.0), br=(0.0, 0.0, 0.0)):
    t = lambda x, shp: torch.tensor(np.asarray(x, dtype=np.float64)).reshape(shp)  # noqa: E731
    zero = torch.zeros(1, 1, dtype=D)
    return (t(p, (1, 1, 2)), zero.clone(), t(v, (1, 1, 2)), zero.clone(), zero.clone(),
            t(z, (1, 1)), t(vz, (1, 1)), t(q, (1, 1, 4)), t(br, (1, 1, 3)))


def run(st, thrusts, dt, rk4=False, cfgs=None):
    w = world(cfgs or [drone_cfg()], dt, rk4)
    traj = []
    for a in thrusts:
        st, _, _ = R.step(st, torch.as_tensor(np.asarray(a, dtype=np.float64)).reshape(1, -1, 4), w)
        traj.append(st)
    return traj


def np_euler(p, z, v, vz, q, br, thrusts, dt):
    """Plain numpy restatement of the drone's semi-implicit Euler recurrence."""
    p, v, q, br = (np.array(x, dtype=np.float64) for x in (p, v, q, br))
    for a in thrusts:
        f = np.clip(np.asarray(a, dtype=np.float64), 0.0, TMAX)
        u = q[:3]
        tv = np.array([0.0, 0.0, f.sum()])
        t = 2.0 * np.cross(u, tv)
        fw = tv + q[3] * t + np.cross(u, t)
        acc = fw / MASS - np.array([0.0, 0.0, G])
        tau = np.array([ARM * (f[1] - f[3]), ARM * (f[2] - f[0]), KAPPA * (f[0] - f[1] + f[2] - f[3])])
        coup = np.array([(IZZ - IYY) * br[1] * br[2], (IXX - IZZ) * br[2] * br[0],
                         (IYY - IXX) * br[0] * br[1]])
        br = br + (tau - coup) / np.array([IXX, IYY, IZZ]) * dt
        vz = vz + acc[2] * dt
        v = v + acc[:2] * dt
        wx, wy, wz = br
        x, y, zq, ww = q
        qd = 0.5 * np.array([ww * wx + y * wz - zq * wy, ww * wy - x * wz + zq * wx,
                             ww * wz + x * wy - y * wx, -x * wx - y * wy - zq * wz])
        q = q + qd * dt
        q = q / np.linalg.norm(q)
        p = p + v * dt
        z = z + vz * dt
    return p, z, v, vz, q, br


def fields(st):
    return (st[0][0, 0].numpy(), float(st[5][0, 0]), st[2][0, 0].numpy(), float(st[6][0, 0]),
            st[7][0, 0].numpy(), st[8][0, 0].numpy())


def test_hover_equilibrium():
    last = fields(run(state9(), np.full((50, 4), HOVER), 0.02)[-1])
    np.testing.assert_allclose(last[0], [0.3, -0.2], atol=1e-10)
    np.testing.assert_allclose(last[1], 1.0, atol=1e-10)
    np.testing.assert_allclose(last[4], [0.0, 0.0, 0.0, 1.0], atol=1e-10)
    np.testing.assert_allclose(last[5], [0.0, 0.0, 0.0], atol=1e-12)


def test_vertical_climb_closed_form():
    dt, T, f = 0.02, 40, HOVER + 0.5
    last = fields(run(state9(), np.full((T, 4), f), dt)[-1])
    az = 4.0 * f / MASS - G
    np.testing.assert_allclose(last[1], 1.0 + az * dt * dt * T * (T + 1) / 2.0, atol=1e-9)
    np.testing.assert_allclose(last[3], az * dt * T, atol=1e-10)
    np.testing.assert_allclose(last[4], [0.0, 0.0, 0.0, 1.0], atol=1e-12)
    np.testing.assert_allclose(last[0], [0.3, -0.2], atol=1e-12)


def test_pure_yaw_torque():
    dt, T, d = 0.01, 30, 0.5
    thrusts = np.tile([HOVER + d, HOVER - d, HOVER + d, HOVER - d], (T, 1))
    last = fields(run(state9(), thrusts, dt)[-1])
    np.testing.assert_allclose(last[1], 1.0, atol=1e-9)
    assert last[5][2] > 1e-3 and abs(last[4][2]) > 1e-3
    ref = np_euler([0.3, -0.2], 1.0, [0.0, 0.0], 0.0, [0, 0, 0, 1.0], [0, 0, 0], thrusts, dt)
    np.testing.assert_allclose(last[4], ref[4], atol=1e-9)


def test_general_thrusts_match_numpy_restatement():
    rng = np.random.default_rng(0)
    dt, T = 0.01, 60
    thrusts = HOVER + 0.4 * rng.standard_normal((T, 4))
    init = dict(p=(0.0, 0.0), z=0.5, v=(0.1, -0.05), vz=0.2, q=(0, 0, 0, 1.0), br=(0.05, -0.03, 0.1))
    last = fields(run(state9(**init), thrusts, dt)[-1])
    ref = np_euler(init["p"], init["z"], init["v"], init["vz"], init["q"], init["br"], thrusts, dt)
    for got, want in zip(last, ref):
        np.testing.assert_allclose(got, want, atol=1e-9)


def test_thrust_clamps_to_zero_and_thrust_max():
    dt = 0.02
    a = run(state9(), [[-5.0, -5.0, -5.0, -5.0]], dt)[-1]
    b = run(state9(), [[0.0, 0.0, 0.0, 0.0]], dt)[-1]
    c = run(state9(), [[TMAX, TMAX, TMAX, TMAX]], dt)[-1]
    d = run(state9(), [[3 * TMAX, 2 * TMAX, 5 * TMAX, TMAX + 1]], dt)[-1]
    for x, y in ((a, b), (c, d)):
        for f in range(9):
            torch.testing.assert_close(x[f], y[f], rtol=0, atol=0)


@pytest.mark.parametrize("rk4", [False, True], ids=["euler", "rk4"])
def test_gradcheck_drone_step(rk4):
    g = torch.Generator().manual_seed(1)
    st = [x.clone() for x in state9(v=(0.05, -0.02), vz=0.1, q=(0.1, -0.05, 0.2, 0.97),
                                    br=(0.02, -0.01, 0.03))]
    st = [x + 0.01 * torch.randn(x.shape, generator=g, dtype=D) for x in st]
    st = [x.requires_grad_(True) for x in st]
    acts = (HOVER + 0.3 * torch.randn(1, 1, 4, generator=g, dtype=D)).requires_grad_(True)
    w = world([drone_cfg()], 0.02, rk4)
    assert torch.autograd.gradcheck(lambda *x: R.step(tuple(x[:9]), x[9], w)[0], (*st, acts),
                                    eps=1e-6, atol=1e-6)


def test_rk4_drone_is_fourth_order():
    rng = np.random.default_rng(3)
    thrust = HOVER + 0.3 * rng.standard_normal(4)
    q = np.array([0.05, -0.02, 0.1, 0.99])
    init = dict(v=(0.2, -0.1), vz=0.3, q=q / np.linalg.norm(q), br=(0.4, -0.3, 0.5))
    horizon = 0.32

    def final(dt):
        n = int(round(horizon / dt))
        return fields(run(state9(**init), np.tile(thrust, (n, 1)), dt, rk4=True)[-1])

    fine = final(0.0025)
    errs = []
    for dt in (0.04, 0.02):
        got = final(dt)
        errs.append(max(float(np.max(np.abs(np.asarray(a) - np.asarray(b)))) for a, b in zip(got, fine)))
    assert 11.0 < errs[0] / errs[1] < 21.0  # ~2^4


def test_two_d_agents_pass_the_drone_fields_through():
    cfgs = [drone_cfg(), AgentConfig(model=DynamicsModel.DIFF_DRIVE, max_ang_vel=3.0)]
    st = list(state9())
    st = [torch.cat([x, x], 1) for x in st]
    st[7] = torch.tensor([[[0, 0, 0, 1.0], [0.1, 0.2, 0.3, 0.9]]], dtype=D)
    st[8] = torch.tensor([[[0, 0, 0.0], [1.0, 2.0, 3.0]]], dtype=D)
    st[5] = torch.tensor([[1.0, 7.0]], dtype=D)
    out = run(tuple(st), [[[HOVER] * 4, [0.5, 1.0, 9.0, 9.0]]], 0.02, cfgs=cfgs)[-1]
    for f in (5, 6, 7, 8):
        torch.testing.assert_close(out[f][:, 1], st[f][:, 1], rtol=0, atol=0)
    assert float(out[1][0, 1]) != 0.0  # the diff-drive turned
