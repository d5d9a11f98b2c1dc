"""Box agents (AgentShape.BOX) on the CUDA path (GPU): the forward rollout against the
float64 oracle on the reference's box-agent known-answer scenes
(tests/unit/test_box_agents.py:104-323: face/corner/disc/capsule contacts, SAT crossing,
walls at the support extents, support-vertex damping, the footprint clamp) and on random
mixed box/disc fleets with every obstacle shape, walls, clamped bounds, truncated lists,
substeps and both integrators."""

import math

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, Integrator
from swarp_b200.interop.autograd import TorchState, rollout

from ref_bridge import ref_obstacles, ref_world
from test_gpu_parity import close, rand_actions

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = torch.float64
DT, K, MARGIN, BIG = 0.1, 100.0, 0.02, 100.0
NAMES = ["pos", "theta", "vel", "speed", "ang_vel"]


def box(hx=0.2, hy=0.1, **kw):
    kw.setdefault("max_speed", BIG)
    return AgentConfig(shape="box", half_extents=(hx, hy), **kw)


def disc(r=0.1, **kw):
    kw.setdefault("max_speed", BIG)
    return AgentConfig(radius=r, **kw)


def stepper(cfgs, dtype=D, c=0.0, bounds=None, mode="soft", dt=DT, substeps=1, rk4=False,
            max_neighbors=32, neighbor_radius=None):
    reach = 2.0 * max(x.radius for x in cfgs) + MARGIN
    world = WorldConfig(collision_k=K, collision_c=c, collision_margin=MARGIN,
                        neighbor_radius=neighbor_radius or reach, max_neighbors=max_neighbors,
                        bounds=bounds, bounds_mode=mode,
                        integrator=Integrator.RK4 if rk4 else Integrator.EULER)
    return Stepper(cfgs, dt=dt, substeps=substeps, device=DEV, dtype=dtype, world=world)


def obstacles(pos, radius, shape, half=None, angle=None, vel=None, ang_vel=None, E=1):
    n = len(radius)
    t = lambda x, shp: (torch.zeros(shp, dtype=D) if x is None  # noqa: E731
                        else torch.tensor(np.asarray(x, dtype=np.float64)).reshape(shp))
    rep = lambda x: x.unsqueeze(0).expand(E, *x.shape).contiguous()  # noqa: E731
    return Obstacles(pos=rep(t(pos, (n, 2))), radius=t(radius, (n,)),
                     shape=torch.tensor(shape, dtype=torch.int32), angle=rep(t(angle, (n,))),
                     half_extents=t(half, (n, 2)), vel=rep(t(vel, (n, 2))),
                     ang_vel=rep(t(ang_vel, (n,))))


def state(pos, theta=None, vel=None, ang_vel=None):
    pos = torch.tensor(np.asarray(pos, dtype=np.float64))
    if pos.dim() == 2:
        pos = pos[None]
    E, n = pos.shape[:2]
    sc = lambda x: (torch.zeros(E, n, dtype=D) if x is None  # noqa: E731
                    else torch.tensor(np.asarray(x, dtype=np.float64)).reshape(E, n))
    v = torch.zeros_like(pos) if vel is None else torch.tensor(
        np.asarray(vel, dtype=np.float64)).reshape(E, n, 2)
    return (pos, sc(theta), v, torch.zeros(E, n, dtype=D), sc(ang_vel))


def run_both(st, s5, acts, dtype=D):
    """Trajectories of the oracle and of the CUDA rollout (float64 on the CPU)."""
    _, traj, _ = R.rollout(tuple(t.clone() for t in s5), acts.clone(), ref_world(st),
                           ref_obstacles(st))
    ref = [torch.stack([traj[t][f] for t in range(len(traj))]) for f in range(5)]
    with torch.no_grad():
        _, tr = rollout(st, TorchState(*(t.to(DEV, dtype) for t in s5)), acts.to(DEV, dtype))
    got = [torch.stack([tr[t][f] for t in range(len(tr))]).cpu().double() for f in range(5)]
    return got, ref


def check_fwd(st, s5, acts, rtol=1e-10, dtype=D):
    got, ref = run_both(st, s5, acts, dtype)
    for f in range(5):
        close(got[f], ref[f], rtol, f"traj {NAMES[f]}")
    return got


def one_step_forces(cfgs, s5, obs=None, **kw):
    """Contact forces of one zero-action step from the CUDA rollout (velocity / dt), after
    checking the whole step against the oracle."""
    st = stepper(cfgs, **kw)
    if obs is not None:
        st.set_obstacles(obs)
    got = check_fwd(st, s5, torch.zeros(1, 1, len(cfgs), 2, dtype=D))
    return got[2][0, 0] / DT


def near(a, b, atol=1e-10):
    np.testing.assert_allclose(np.asarray(a, dtype=np.float64), b, atol=atol, rtol=0)


# ------------------------------------------------------------ known-answer scenes
@pytest.mark.parametrize("gap", [-0.01, 0.01])
def test_face_face(gap):
    f = one_step_forces([box(), box()], state([[0.0, 0.0], [0.4 + gap, 0.05]]))
    mag = K * (MARGIN - gap)
    near(f[0], [-mag, 0.0])
    near(f[1], [mag, 0.0])


@pytest.mark.parametrize("gap", [-0.005, 0.005])
def test_corner_face(gap):
    corner = 0.1 * math.sqrt(2.0)
    f = one_step_forces([box(0.1, 0.1), box(0.2, 0.2)],
                        state([[0.0, 0.0], [corner + 0.2 + gap, 0.03]], theta=[math.pi / 4, 0.0]))
    near(f[0], [-K * (MARGIN - gap), 0.0])
    near(f[1], -f[0].numpy())


def test_disc_box_face_and_corner():
    f = one_step_forces([disc(), box()], state([[0.0, 0.0], [0.29, 0.0]]))
    near(f[0], [-K * 0.03, 0.0])
    near(f[1], [K * 0.03, 0.0])
    d = 0.05 * math.sqrt(2.0)
    f = one_step_forces([disc(), box()], state([[0.25, 0.15], [0.0, 0.0]]))
    mag = K * (0.1 + MARGIN - d)
    near(f[0], [mag / math.sqrt(2.0), mag / math.sqrt(2.0)])
    near(f[1], -f[0].numpy())


@pytest.mark.parametrize("phi", [0.2, 0.7, 1.2])
def test_capsule_end_cap_is_round(phi):
    seg = obstacles([[0.0, 0.0]], [0.05], [R.SEGMENT], half=[[0.3, 0.0]], angle=[0.0])
    corner = np.array([0.3 + 0.05 * math.cos(phi), 0.05 * math.sin(phi)])
    f = one_step_forces([box(0.1, 0.1)], state([corner + 0.1]), obs=seg)
    near(f[0], K * MARGIN * np.array([math.cos(phi), math.sin(phi)]))


def test_capsule_side_and_box_and_circle_obstacles():
    seg = obstacles([[0.0, 0.0]], [0.05], [R.SEGMENT], half=[[0.3, 0.0]], angle=[0.0])
    near(one_step_forces([box()], state([[0.05, 0.16]]), obs=seg)[0], [0.0, K * 0.01])
    obs = obstacles([[0.0, 0.0], [2.0, 0.0]], [0.0, 0.1], [R.BOX, R.CIRCLE],
                    half=[[0.3, 0.2], [0.0, 0.0]], angle=[0.0, 0.0])
    near(one_step_forces([box()], state([[0.49, 0.1]]), obs=obs)[0], [K * 0.03, 0.0])
    near(one_step_forces([box()], state([[2.0, -0.18]]), obs=obs)[0], [0.0, -K * 0.04])


def test_moving_scene_rotation_invariance():
    cfgs = [box(0.2, 0.1), box(0.15, 0.06), box(0.1, 0.1), disc(0.08)]
    pos = np.array([[0.0, 0.0], [0.27, 0.12], [0.02, 0.2], [-0.24, -0.06]])
    theta = np.array([0.3, -0.4, 1.1, 0.0])
    vel = np.array([[0.2, -0.1], [-0.3, 0.05], [0.1, 0.2], [0.4, 0.0]])
    ang_vel = np.array([0.5, -1.0, 2.0, 0.0])
    o = dict(pos=np.array([[0.2, -0.2], [-0.3, 0.2], [0.42, 0.3]]), radius=[0.0, 0.03, 0.1],
             shape=[R.BOX, R.SEGMENT, R.CIRCLE], half=[[0.15, 0.05], [0.2, 0.0], [0.0, 0.0]],
             angle=np.array([0.2, -0.5, 0.0]), vel=np.array([[0.1, 0.0], [0.0, -0.2], [0.0, 0.1]]),
             ang_vel=[0.3, -0.4, 1.0])
    f0 = one_step_forces(cfgs, state(pos, theta, vel, ang_vel), obs=obstacles(**o), c=1.0)
    assert (f0.norm(dim=-1) > 1e-3).sum() >= 3
    a, shift = 0.7, np.array([0.3, -0.5])
    r = np.array([[math.cos(a), -math.sin(a)], [math.sin(a), math.cos(a)]])
    moved = dict(o, pos=o["pos"] @ r.T + shift, angle=o["angle"] + a, vel=o["vel"] @ r.T)
    f1 = one_step_forces(cfgs, state(pos @ r.T + shift, theta + a, vel @ r.T, ang_vel),
                         obs=obstacles(**moved), c=1.0)
    near(f1, f0.numpy() @ r.T, atol=1e-9)


def test_agent_forces_cancel():
    rng = np.random.default_rng(3)
    cfgs = [box(0.2, 0.08), box(0.1, 0.1), box(0.15, 0.05), box(0.05, 0.2), disc(0.1), disc(0.06)]
    n = len(cfgs)
    f = one_step_forces(cfgs, state(rng.random((n, 2)) * 0.35, rng.uniform(-3, 3, n),
                                    rng.normal(size=(n, 2)), rng.normal(size=n)), c=1.0)
    assert (f.norm(dim=-1) > 1e-3).sum() >= 4
    near(f.sum(0), [0.0, 0.0], atol=1e-12)


def test_plus_crossing_is_detected():
    f = one_step_forces([box(0.3, 0.02), box(0.3, 0.02)],
                        state([[0.0, 0.0], [0.01, 0.02]], theta=[0.0, math.pi / 2]))
    assert f[0].norm() > 10.0
    near(f[0] + f[1], [0.0, 0.0], atol=1e-12)


def _extents(hx, hy, th):
    return (hx * abs(math.cos(th)) + hy * abs(math.sin(th)),
            hx * abs(math.sin(th)) + hy * abs(math.cos(th)))


def test_walls_see_the_support_extents():
    th = 0.5
    ex, ey = _extents(0.2, 0.1, th)
    f = one_step_forces([box()], state([[-1.0 + ex + 0.01, 1.0 - ey - 0.005]], theta=[th]),
                        bounds=(-1.0, 1.0, -1.0, 1.0))
    near(f[0], [K * 0.01, -K * 0.015])


def test_wall_damping_reads_the_support_vertex_velocity():
    th, w, c = 0.5, 3.0, 1.0
    ex, _ = _extents(0.2, 0.1, th)
    r_y = -0.2 * math.sin(th) + 0.1 * math.cos(th)
    kw = dict(c=c, bounds=(-1.0, 1.0, -1.0, 1.0))
    f_still = one_step_forces([box()], state([[-1.0 + ex + 0.01, 0.0]], theta=[th]), **kw)
    f_spin = one_step_forces([box()], state([[-1.0 + ex + 0.01, 0.0]], theta=[th], ang_vel=[w]),
                             **kw)
    near(f_still[0], [K * 0.01 / (1.0 + c * DT), 0.0])
    near(f_spin[0], [(K * 0.01 - c * (-w * r_y)) / (1.0 + c * DT), 0.0])


def test_clamp_holds_each_footprint_inside():
    w = 2.0
    cfgs = [box(model=DynamicsModel.DIFF_DRIVE, max_ang_vel=BIG), disc()]
    st = stepper(cfgs, bounds=(-1.0, 1.0, -1.0, 1.0), mode="clamp")
    got = check_fwd(st, state([[-1.5, 1.5], [1.5, -1.5]], theta=[0.3, 0.0]),
                    torch.tensor([[[[0.0, w], [0.0, 0.0]]]], dtype=D))
    ex, ey = _extents(0.2, 0.1, 0.3 + w * DT)
    near(got[1][0, 0, 0], 0.3 + w * DT, atol=1e-12)
    near(got[0][0, 0, 0], [-1.0 + ex, 1.0 - ey], atol=1e-12)
    near(got[0][0, 0, 1], [0.9, -0.9], atol=1e-12)


# ------------------------------------------------------------ random fleets
def mixed_fleet(n, seed):
    rng = np.random.default_rng(seed)
    models = [(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION),
              (DynamicsModel.DIFF_DRIVE, ControlMode.ACCELERATION),
              (DynamicsModel.DIFF_DRIVE, ControlMode.VELOCITY),
              (DynamicsModel.KINEMATIC_BICYCLE, ControlMode.ACCELERATION),
              (DynamicsModel.HOLONOMIC, ControlMode.VELOCITY)]
    cfgs = []
    for i in range(n):
        model, mode = models[i % len(models)]
        kw = dict(model=model, ctrl_mode=mode, max_speed=1.5, max_accel=3.0, max_ang_vel=3.0,
                  max_ang_accel=6.0, max_steer=0.6, l_f=0.08, l_r=0.07)
        if i % 3 == 2:
            cfgs.append(disc(float(rng.uniform(0.04, 0.08)), **kw))
        else:
            cfgs.append(box(float(rng.uniform(0.03, 0.09)), float(rng.uniform(0.02, 0.06)), **kw))
    return cfgs


def rand_scene(E, A, seed, spread=0.35):
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1) * spread
    th = (torch.rand(E, A, generator=g, dtype=D) * 2 - 1) * 3.0
    v = torch.randn(E, A, 2, generator=g, dtype=D) * 0.4
    w = torch.randn(E, A, generator=g, dtype=D) * 0.8
    return (pos, th, v, torch.zeros(E, A, dtype=D), w)


def obstacle_mix(E, seed):
    g = torch.Generator().manual_seed(seed)
    N = 6
    return Obstacles(
        pos=(torch.rand(E, N, 2, generator=g, dtype=D) * 2 - 1) * 0.4,
        radius=torch.tensor([0.08, 0.05, 0.0, 0.0, 0.03, 0.02], dtype=D),
        shape=torch.tensor([0, 0, 1, 1, 2, 2], dtype=torch.int32),
        angle=torch.rand(E, N, generator=g, dtype=D) * 3.14,
        half_extents=torch.tensor([[0, 0], [0, 0], [0.1, 0.05], [0.04, 0.1], [0.15, 0],
                                   [0.1, 0]], dtype=D),
        vel=torch.randn(E, N, 2, generator=g, dtype=D) * 0.2,
        ang_vel=torch.randn(E, N, generator=g, dtype=D) * 0.5,
    )


@pytest.mark.parametrize("rk4", [False, True], ids=["euler", "rk4"])
@pytest.mark.parametrize("walls", ["soft", "clamp"])
def test_mixed_fleet_obstacles_walls_f64(rk4, walls):
    cfgs = mixed_fleet(9, 1)
    st = stepper(cfgs, c=1.0, bounds=(-0.45, 0.45, -0.45, 0.45), mode=walls, dt=0.05,
                 substeps=2, rk4=rk4)
    E = 5
    st.set_obstacles(obstacle_mix(E, 2))
    check_fwd(st, rand_scene(E, 9, 3), rand_actions(8, E, 9, 4, scale=1.5))


def test_truncated_lists_f64():
    cfgs = mixed_fleet(12, 5)
    st = stepper(cfgs, c=0.5, dt=0.05, max_neighbors=3, neighbor_radius=0.3)
    check_fwd(st, rand_scene(3, 12, 6, spread=0.2), rand_actions(6, 3, 12, 7))


def test_boxes_only_no_contacts_with_walls_f64():
    """Box agents with agent contacts off: walls and obstacles still see the box."""
    cfgs = [box(0.08, 0.04, model=DynamicsModel.DIFF_DRIVE, max_ang_vel=3.0)] * 4
    world = WorldConfig(collisions=False, collision_k=K, collision_c=1.0,
                        collision_margin=MARGIN, bounds=(-0.3, 0.3, -0.3, 0.3))
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=D, world=world)
    st.set_obstacles(obstacle_mix(3, 8))
    check_fwd(st, rand_scene(3, 4, 9, spread=0.28), rand_actions(6, 3, 4, 10, scale=2.0))


def test_sixteen_agent_fleet_f32():
    """The 16-agent float specialisation with box agents, against the float64 oracle."""
    cfgs = mixed_fleet(16, 11)
    st = stepper(cfgs, dtype=torch.float32, c=1.0, bounds=(-0.6, 0.6, -0.6, 0.6), dt=0.05)
    check_fwd(st, rand_scene(24, 16, 12, spread=0.55), rand_actions(4, 24, 16, 13),
              rtol=1e-5, dtype=torch.float32)


# ------------------------------------------------------------ adjoint
from test_gpu_parity import check  # noqa: E402


@pytest.mark.parametrize("rk4", [False, True], ids=["euler", "rk4"])
def test_grad_mixed_fleet_obstacles_soft_walls_f64(rk4):
    cfgs = mixed_fleet(9, 21)
    st = stepper(cfgs, c=1.0, bounds=(-0.45, 0.45, -0.45, 0.45), dt=0.05, rk4=rk4)
    E = 4
    st.set_obstacles(obstacle_mix(E, 22))
    check(st, rand_scene(E, 9, 23), rand_actions(6, E, 9, 24, scale=1.5), seed=25, final=True)


@pytest.mark.parametrize("rk4", [False, True], ids=["euler", "rk4"])
def test_grad_footprint_clamp_f64(rk4):
    """Boxes held inside the bounds by the footprint clamp: the clamped coordinates'
    gradients flow into the heading through the support extents."""
    cfgs = mixed_fleet(6, 31)
    st = stepper(cfgs, c=1.0, bounds=(-0.25, 0.25, -0.25, 0.25), mode="clamp", dt=0.05, rk4=rk4)
    check(st, rand_scene(5, 6, 32, spread=0.3), rand_actions(6, 5, 6, 33, scale=2.0), seed=34)


def test_grad_substeps_and_saturation_f64():
    cfgs = mixed_fleet(7, 41)
    reach = 2.0 * max(x.radius for x in cfgs) + MARGIN
    world = WorldConfig(collision_k=K, collision_c=1.0, collision_margin=MARGIN,
                        contact_max_overlap=0.02, neighbor_radius=reach,
                        bounds=(-0.4, 0.4, -0.4, 0.4))
    st = Stepper(cfgs, dt=0.06, substeps=3, device=DEV, dtype=D, world=world)
    st.set_obstacles(obstacle_mix(3, 42))
    check(st, rand_scene(3, 7, 43), rand_actions(5, 3, 7, 44), seed=45, final=True)


def test_grad_truncated_lists_f64():
    cfgs = mixed_fleet(12, 51)
    st = stepper(cfgs, c=0.5, dt=0.05, max_neighbors=3, neighbor_radius=0.3)
    check(st, rand_scene(3, 12, 52, spread=0.2), rand_actions(5, 3, 12, 53), seed=54)


def test_grad_reference_gradcheck_scene_f64():
    """The reference's gradcheck scene (two boxes on a face contact and a disc)."""
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
    st = stepper(cfgs, c=1.0)
    rng = np.random.default_rng(0)
    s5 = state(pos, [tha, thb, 0.0], 0.1 * rng.normal(size=(3, 2)), 0.5 * rng.normal(size=3))
    acts = torch.tensor([[[[0.1, 0.4], [0.05, -0.3], [0.1, 0.0]]]], dtype=D).repeat(3, 1, 1, 1)
    check(st, s5, acts, seed=61, final=True)


def test_grad_sixteen_agent_fleet_f32():
    """The 16-agent float instances' adjoint against the float64 oracle. Box contacts
    switch branch (vertex, SAT axis, contact on/off) discontinuously, so a float32
    gradient is ill-conditioned wherever a scene sits near such a tie; this scene was
    chosen so that the oracle's own float32 and float64 gradients agree within 2e-5."""
    cfgs = mixed_fleet(16, 85)
    st = stepper(cfgs, dtype=torch.float32, c=1.0, bounds=(-0.6, 0.6, -0.6, 0.6), dt=0.05)
    check(st, rand_scene(24, 16, 86, spread=0.6), rand_actions(3, 24, 16, 87), seed=88,
          dtype=torch.float32, rtol_f=1e-5, rtol_g=1e-4)


@pytest.mark.parametrize("shape", [0, 1, 2], ids=["circle-body", "box-body", "segment-body"])
def test_box_agents_push_movable_body_f64(shape):
    """Box and disc agents pushing one movable body (reference swarp/core/bodies.py:131-166,
    _reaction_box): the body takes the negated box-obstacle force each box agent feels, at
    the contact point, so off-centre pushes spin it. Forward against the oracle in float64."""
    from oracle import torch_ref as R
    from swarp_b200.interop.autograd import rollout_bodies

    from ref_bridge import ref_obstacles, ref_world

    E, A, T = 4, 6, 30
    cfgs = mixed_fleet(A, 31)
    # dt 0.05: the default body damping 10 / s leaves 1 - 10 dt = 0.5 of the body velocity
    # per step (at dt 0.1 it would leave none and the body could not move)
    st = stepper(cfgs, c=2.0, bounds=(-0.8, 0.8, -0.8, 0.8), dt=0.05)
    g = torch.Generator().manual_seed(32)
    half = {0: [0.0, 0.0], 1: [0.14, 0.07], 2: [0.16, 0.0]}[shape]
    obs = Obstacles(
        pos=(torch.rand(E, 1, 2, generator=g, dtype=D) - 0.5) * 0.1,
        radius=torch.tensor([{0: 0.1, 1: 0.0, 2: 0.04}[shape]], dtype=D),
        shape=torch.tensor([shape], dtype=torch.int32),
        angle=torch.rand(E, 1, generator=g, dtype=D),
        half_extents=torch.tensor([half], dtype=D),
        kind=torch.ones(1, dtype=torch.int32), mass=torch.tensor([1.2], dtype=D),
        inertia=torch.tensor([0.015], dtype=D))
    st.set_obstacles(obs)
    ang = torch.rand(E, A, generator=g, dtype=D) * 2 * math.pi
    rad = 0.2 + 0.06 * torch.rand(E, A, generator=g, dtype=D)
    pos = obs.pos + torch.stack([torch.cos(ang), torch.sin(ang)], -1) * rad[..., None]
    s5 = state(pos, theta=(torch.rand(E, A, generator=g, dtype=D) * 2 - 1) * 3.0)
    push = -(pos - obs.pos)  # toward the body
    push = push / push.norm(dim=-1, keepdim=True)
    acts = (push.unsqueeze(0).expand(T, E, A, 2)
            + 0.3 * torch.randn(T, E, A, 2, generator=g, dtype=D)).contiguous()
    w = ref_world(st)
    ob = ref_obstacles(st)
    with torch.no_grad():
        fin_r, traj_r, body_r = R.rollout(tuple(s5), acts, w, ob)
        fin, traj, body = rollout_bodies(st, TorchState(*(x.to(DEV) for x in s5)), acts.to(DEV))
    for f, name in enumerate(["pos", "theta", "vel", "speed", "ang_vel"]):
        ref = torch.stack([t[f] for t in traj_r])
        scale = max(float(ref.abs().max()), 1e-30)
        torch.testing.assert_close(traj.stacked[f].cpu(), ref, rtol=1e-10, atol=1e-10 * scale,
                                   msg=lambda m: f"traj {name}: {m}")
    for got, ref, name in [(body.pos[:, 0], body_r[-1].body_pos[:, 0], "pos"),
                           (body.angle[:, 0], body_r[-1].body_angle[:, 0], "angle"),
                           (body.vel[:, 0], body_r[-1].body_vel[:, 0], "vel"),
                           (body.ang_vel[:, 0], body_r[-1].body_ang_vel[:, 0], "ang_vel")]:
        torch.testing.assert_close(got.cpu(), ref, rtol=1e-10, atol=1e-12,
                                   msg=lambda m: f"body {name}: {m}")
    moved = (body.pos[:, 0].cpu() - obs.pos[:, 0]).norm(dim=-1)
    assert float(moved.max()) > 1e-3, "the agents pushed the body"
    if shape != 0:
        assert float((body.angle[:, 0].cpu() - obs.angle[:, 0]).abs().max()) > 1e-4  # it spun


def test_box_agents_with_bodies_in_grad_are_rejected():
    """The body adjoint covers disc agents only: a grad rollout that would move bodies
    pushed by box agents raises, while the reference rule (bodies frozen on taped steps)
    differentiates."""
    from swarp_b200.interop.autograd import rollout_bodies

    E, A, T = 2, 3, 4
    st = stepper(mixed_fleet(A, 3))
    st.set_obstacles(Obstacles(pos=torch.zeros(E, 1, 2, dtype=D), radius=torch.tensor([0.1], dtype=D),
                               kind=torch.ones(1, dtype=torch.int32)))
    s5 = [x.to(DEV) for x in rand_scene(E, A, 4)]
    acts = torch.zeros(T, E, A, 2, dtype=D, device=DEV, requires_grad=True)
    _, _, body = rollout_bodies(st, TorchState(*s5), acts)  # frozen: no body state returned
    assert body is None
    st.bodies_in_grad = True
    with pytest.raises(NotImplementedError):
        rollout_bodies(st, TorchState(*s5), acts)
