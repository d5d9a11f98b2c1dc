"""Box agents in the CPU oracle, pinned by the reference's own known answers
(ddebenedittis/swarp tests/unit/test_box_agents.py:104-323): analytic face/corner/disc/
capsule contacts, invariance, third law, SAT crossing, walls at the support extents,
wall damping at the support vertex, the footprint clamp and a gradcheck (CPU only)."""

import math

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, param_rows

D = torch.float64
DT, K, MARGIN, BIG = 0.1, 100.0, 0.02, 100.0


def box(hx=0.2, hy=0.1, **kw):
    kw.setdefault("max_speed", BIG)
    return AgentConfig(shape="box", half_extents=(hx, hy), **kw)


def disc(r=0.1, **kw):
    kw.setdefault("max_speed", BIG)
    return AgentConfig(radius=r, **kw)


def world(cfgs, c=0.0, bounds=None, mode="soft"):
    reach = 2.0 * max(x.radius for x in cfgs) + MARGIN
    return R.RefWorld(params=torch.tensor(param_rows(cfgs), dtype=D),
                      model_tag=[int(x.model) for x in cfgs], ctrl_mode=[int(x.ctrl_mode) for x in cfgs],
                      dt=DT, k=K, c=c, margin=MARGIN, neighbor_radius=reach, max_neighbors=32,
                      bounds=bounds, soft_walls=bounds is not None and mode == "soft",
                      clamp_bounds=bounds is not None and mode == "clamp")


def state(pos, theta=None, vel=None, ang_vel=None):
    pos = torch.tensor(np.asarray(pos, dtype=np.float64))[None]
    n = pos.shape[1]
    sc = lambda x: torch.zeros(1, n, dtype=D) if x is None else torch.tensor(np.asarray(x, dtype=np.float64))[None]  # noqa: E731
    v = torch.zeros_like(pos) if vel is None else torch.tensor(np.asarray(vel, dtype=np.float64))[None]
    return (pos, sc(theta), v, sc(None), sc(ang_vel))


def obstacles(pos, radius, shape, half=None, angle=None, vel=None, ang_vel=None):
    n = len(radius)
    t = lambda x, shp: torch.zeros(shp, dtype=D) if x is None else torch.tensor(np.asarray(x, dtype=np.float64))  # noqa: E731
    return R.RefObstacles(pos=t(pos, (n, 2))[None], angle=t(angle, (n,))[None], vel=t(vel, (n, 2))[None],
                          ang_vel=t(ang_vel, (n,))[None], radius=t(radius, (n,)),
                          half=t(half, (n, 2)), shape=[int(x) for x in shape], kind=[0] * n)


def forces(cfgs, s, obs=None, **kw):
    out, _, _ = R.step(s, torch.zeros(1, len(cfgs), 2, dtype=D), world(cfgs, **kw), obs)
    return out[2][0] / DT


def close(a, b, atol=1e-10):
    np.testing.assert_allclose(np.asarray(a, dtype=np.float64), b, atol=atol, rtol=0)


@pytest.mark.parametrize("gap", [-0.01, 0.01])
def test_face_face(gap):
    f = forces([box(), box()], state([[0.0, 0.0], [0.4 + gap, 0.05]]))
    mag = K * (MARGIN - gap)
    close(f[0], [-mag, 0.0])
    close(f[1], [mag, 0.0])


@pytest.mark.parametrize("gap", [-0.005, 0.005])
def test_corner_face(gap):
    corner = 0.1 * math.sqrt(2.0)
    f = forces([box(0.1, 0.1), box(0.2, 0.2)],
               state([[0.0, 0.0], [corner + 0.2 + gap, 0.03]], theta=[math.pi / 4, 0.0]))
    close(f[0], [-K * (MARGIN - gap), 0.0])
    close(f[1], -f[0].numpy())


def test_disc_box_face_and_corner():
    f = forces([disc(), box()], state([[0.0, 0.0], [0.29, 0.0]]))
    close(f[0], [-K * 0.03, 0.0])
    close(f[1], [K * 0.03, 0.0])
    d = 0.05 * math.sqrt(2.0)
    f = forces([disc(), box()], state([[0.25, 0.15], [0.0, 0.0]]))
    mag = K * (0.1 + MARGIN - d)
    close(f[0], [mag / math.sqrt(2.0), mag / math.sqrt(2.0)])
    close(f[1], -f[0].numpy())


@pytest.mark.parametrize("phi", [0.2, 0.7, 1.2])
def test_capsule_end_cap_is_round(phi):
    seg = obstacles([[0.0, 0.0]], [0.05], [R.SEGMENT], half=[[0.3, 0.0]], angle=[0.0])
    corner = np.array([0.3 + 0.05 * math.cos(phi), 0.05 * math.sin(phi)])
    f = forces([box(0.1, 0.1)], state([corner + 0.1]), obs=seg)
    close(f[0], K * MARGIN * np.array([math.cos(phi), math.sin(phi)]))


def test_capsule_side_and_box_and_circle_obstacles():
    seg = obstacles([[0.0, 0.0]], [0.05], [R.SEGMENT], half=[[0.3, 0.0]], angle=[0.0])
    close(forces([box()], state([[0.05, 0.16]]), obs=seg)[0], [0.0, K * 0.01])
    obs = obstacles([[0.0, 0.0], [2.0, 0.0]], [0.0, 0.1], [R.BOX, R.CIRCLE],
                    half=[[0.3, 0.2], [0.0, 0.0]], angle=[0.0, 0.0])
    close(forces([box()], state([[0.49, 0.1]]), obs=obs)[0], [K * 0.03, 0.0])
    close(forces([box()], state([[2.0, -0.18]]), obs=obs)[0], [0.0, -K * 0.04])


def scene():
    cfgs = [box(0.2, 0.1), box(0.15, 0.06), box(0.1, 0.1), disc(0.08)]
    pos = np.array([[0.0, 0.0], [0.27, 0.12], [0.02, 0.2], [-0.24, -0.06]])
    theta = np.array([0.3, -0.4, 1.1, 0.0])
    vel = np.array([[0.2, -0.1], [-0.3, 0.05], [0.1, 0.2], [0.4, 0.0]])
    ang_vel = np.array([0.5, -1.0, 2.0, 0.0])
    obs = dict(pos=np.array([[0.2, -0.2], [-0.3, 0.2], [0.42, 0.3]]), radius=[0.0, 0.03, 0.1],
               shape=[R.BOX, R.SEGMENT, R.CIRCLE], half=[[0.15, 0.05], [0.2, 0.0], [0.0, 0.0]],
               angle=np.array([0.2, -0.5, 0.0]), vel=np.array([[0.1, 0.0], [0.0, -0.2], [0.0, 0.1]]),
               ang_vel=[0.3, -0.4, 1.0])
    return cfgs, pos, theta, vel, ang_vel, obs


def test_rotation_and_translation_invariance():
    cfgs, pos, theta, vel, ang_vel, obs = scene()
    f0 = forces(cfgs, state(pos, theta, vel, ang_vel), obs=obstacles(**obs), c=1.0)
    assert (f0.norm(dim=-1) > 1e-3).sum() >= 3
    a, shift = 0.7, np.array([0.3, -0.5])
    r = np.array([[math.cos(a), -math.sin(a)], [math.sin(a), math.cos(a)]])
    moved = dict(obs, pos=obs["pos"] @ r.T + shift, angle=obs["angle"] + a, vel=obs["vel"] @ r.T)
    f1 = forces(cfgs, state(pos @ r.T + shift, theta + a, vel @ r.T, ang_vel),
                obs=obstacles(**moved), c=1.0)
    close(f1, f0.numpy() @ r.T, atol=1e-9)


def test_agent_forces_cancel():
    rng = np.random.default_rng(3)
    cfgs = [box(0.2, 0.08), box(0.1, 0.1), box(0.15, 0.05), box(0.05, 0.2), disc(0.1), disc(0.06)]
    n = len(cfgs)
    f = forces(cfgs, state(rng.random((n, 2)) * 0.35, rng.uniform(-3, 3, n), rng.normal(size=(n, 2)),
                           rng.normal(size=n)), c=1.0)
    assert (f.norm(dim=-1) > 1e-3).sum() >= 4
    close(f.sum(0), [0.0, 0.0], atol=1e-12)


def test_plus_crossing_is_detected():
    f = forces([box(0.3, 0.02), box(0.3, 0.02)], state([[0.0, 0.0], [0.01, 0.02]],
                                                        theta=[0.0, math.pi / 2]))
    assert f[0].norm() > 10.0
    close(f[0] + f[1], [0.0, 0.0], atol=1e-12)
    assert min(abs(float(f[0, 0])), abs(float(f[0, 1]))) < 1e-9


def _extents(hx, hy, th):
    return (hx * abs(math.cos(th)) + hy * abs(math.sin(th)),
            hx * abs(math.sin(th)) + hy * abs(math.cos(th)))


def test_walls_see_the_support_extents():
    th = 0.5
    ex, ey = _extents(0.2, 0.1, th)
    f = forces([box()], state([[-1.0 + ex + 0.01, 1.0 - ey - 0.005]], theta=[th]),
               bounds=(-1.0, 1.0, -1.0, 1.0))
    close(f[0], [K * 0.01, -K * 0.015])


def test_wall_damping_reads_the_support_vertex_velocity():
    th, w, c = 0.5, 3.0, 1.0
    ex, _ = _extents(0.2, 0.1, th)
    r_y = -0.2 * math.sin(th) + 0.1 * math.cos(th)
    kw = dict(c=c, bounds=(-1.0, 1.0, -1.0, 1.0))
    f_still = forces([box()], state([[-1.0 + ex + 0.01, 0.0]], theta=[th]), **kw)
    f_spin = forces([box()], state([[-1.0 + ex + 0.01, 0.0]], theta=[th], ang_vel=[w]), **kw)
    close(f_still[0], [K * 0.01 / (1.0 + c * DT), 0.0])
    close(f_spin[0], [(K * 0.01 - c * (-w * r_y)) / (1.0 + c * DT), 0.0])


def test_clamp_holds_each_footprint_inside():
    w = 2.0
    cfgs = [box(model=DynamicsModel.DIFF_DRIVE, max_ang_vel=BIG), disc()]
    out, _, _ = R.step(state([[-1.5, 1.5], [1.5, -1.5]], theta=[0.3, 0.0]),
                       torch.tensor([[[0.0, w], [0.0, 0.0]]], dtype=D),
                       world(cfgs, bounds=(-1.0, 1.0, -1.0, 1.0), mode="clamp"))
    ex, ey = _extents(0.2, 0.1, 0.3 + w * DT)
    close(out[1][0, 0], 0.3 + w * DT, atol=1e-12)
    close(out[0][0, 0], [-1.0 + ex, 1.0 - ey], atol=1e-12)
    close(out[0][0, 1], [0.9, -0.9], atol=1e-12)


def test_gradcheck_through_box_contacts():
    ha, hb = (0.2, 0.1), (0.15, 0.08)
    tha, thb = 0.3, 1.0
    n = np.array([-math.sin(tha), math.cos(tha)])
    t = np.array([math.cos(tha), math.sin(tha)])
    ub0, ub1 = np.array([math.cos(thb), math.sin(thb)]), np.array([-math.sin(thb), math.cos(thb)])
    rb = hb[0] * abs(ub0 @ n) + hb[1] * abs(ub1 @ n)
    pos = np.array([[0.0, 0.0], n * (ha[1] + rb - 0.01), -n * (ha[1] + 0.06 - 0.01) + 0.05 * t])
    cfgs = [box(*ha, model=DynamicsModel.DIFF_DRIVE, max_ang_vel=BIG, max_accel=BIG),
            box(*hb, model=DynamicsModel.DIFF_DRIVE, max_ang_vel=BIG, max_accel=BIG,
                ctrl_mode=ControlMode.ACCELERATION, max_ang_accel=BIG),
            disc(0.06, max_accel=BIG)]
    w = world(cfgs, c=1.0)
    rng = np.random.default_rng(0)
    s = [x.clone().requires_grad_(True) for x in state(pos, [tha, thb, 0.0], 0.1 * rng.normal(size=(3, 2)),
                                                       0.5 * rng.normal(size=3))]
    acts = torch.tensor([[[0.1, 0.4], [0.05, -0.3], [0.1, 0.0]]], dtype=D, requires_grad=True)
    assert torch.autograd.gradcheck(lambda *x: R.step(tuple(x[:5]), x[5], w)[0], (*s, acts),
                                    eps=1e-6, atol=1e-5)
    out = R.step(tuple(s), acts, w)[0]
    (gth,) = torch.autograd.grad(out[0][0, 0].sum(), [s[1]])
    assert gth[0, 1].abs() > 1e-6


def test_gradcheck_through_the_footprint_clamp():
    """A box pinned against a wall by the footprint clamp: its position follows the
    support extent at the new heading, so the clamped coordinate carries a gradient into
    the heading (Warp's clamp adjoint routes it to the bound)."""
    cfgs = [box(0.2, 0.1, model=DynamicsModel.DIFF_DRIVE, max_ang_vel=BIG, max_accel=BIG)]
    w = world(cfgs, bounds=(-1.0, 1.0, -1.0, 1.0), mode="clamp")
    s = [x.clone().requires_grad_(True) for x in state([[-0.95, 0.97]], [0.9], [[-0.5, 0.3]], [1.0])]
    acts = torch.tensor([[[0.3, 0.8]]], dtype=D, requires_grad=True)
    out = R.step(tuple(s), acts, w)[0]
    ex, ey = _extents(0.2, 0.1, float(out[1][0, 0]))
    close(out[0][0, 0].detach(), [-1.0 + ex, 1.0 - ey], atol=1e-12)  # both coordinates clamped
    assert torch.autograd.gradcheck(lambda *x: R.step(tuple(x[:5]), x[5], w)[0], (*s, acts),
                                    eps=1e-6, atol=1e-5)
    (gth,) = torch.autograd.grad(out[0][0, 0, 0], [s[1]])
    assert gth.abs().max() > 0.05
