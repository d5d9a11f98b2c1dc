"""Movable compound rigid bodies on the CUDA path against the CPU oracle (GPU).

Forward: agent trajectory and body state against the torch restatement of the
reference's body pass (swarp/core/bodies.py:367-569) for circle, box and segment bodies,
compound bodies and several bodies per env, in float64. Adjoint: the gradient of a
loss on the final body pose w.r.t. actions and initial agent state against the
oracle's autograd (the reference has no body gradients; the oracle's is pinned by
finite differences in test_oracle_body_gradient_finite_differences). Behaviour ported
from the reference's tests/unit/test_obstacle_kinds.py is checked on the CUDA path.
"""

import math

import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.core.config import ObstacleKind, Obstacles, ObstacleShape, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel
from swarp_b200.interop.autograd import TorchState, rollout, rollout_bodies, warp_step

from ref_bridge import D, ref_obstacles, ref_world

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def transport_world(bounds=(-1.0, 1.0, -1.0, 1.0)):
    return WorldConfig(collision_k=100.0, collision_c=5.0, collision_margin=0.025, bounds=bounds,
                       bounds_mode="soft", neighbor_radius=0.125, max_neighbors=4)


def compound_body(E, seed, mass=2.5, extra=None):
    """One movable body of three circles on a line (config 4), optionally plus more shapes."""
    g = torch.Generator().manual_seed(seed)
    r, d = 0.08, 0.12
    inertia = mass * (0.5 * r * r + 2.0 * d * d / 3.0)
    ang = (torch.rand(E, generator=g, dtype=D) * 2 - 1) * 0.5
    cen = (torch.rand(E, 2, generator=g, dtype=D) * 2 - 1) * 0.3
    off = torch.tensor([[-d, 0.0], [0.0, 0.0], [d, 0.0]], dtype=D)
    ca, sa = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
    pos = torch.stack([cen[:, None, 0] + ca * off[:, 0] - sa * off[:, 1],
                       cen[:, None, 1] + sa * off[:, 0] + ca * off[:, 1]], -1)
    spec = dict(pos=pos, radius=torch.full((3,), r, dtype=D),
                shape=torch.zeros(3, dtype=torch.int32), angle=ang[:, None].expand(E, 3).clone(),
                kind=torch.full((3,), int(ObstacleKind.MOVABLE), dtype=torch.int32),
                mass=torch.full((3,), mass, dtype=D), inertia=torch.full((3,), inertia, dtype=D),
                body=torch.zeros(3, dtype=torch.int32), body_offset=off)
    if extra is not None:
        for k_, v in extra.items():
            spec[k_] = torch.cat([spec[k_], v], dim=1 if k_ in ("pos", "angle") else 0)
    spec["half_extents"] = torch.zeros(spec["radius"].shape[0], 2, dtype=D)
    return Obstacles(**spec)


def agents_around(E, A, seed, body_pos):
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand(E, A, generator=g, dtype=D) * 2 * math.pi
    rad = 0.2 + 0.08 * torch.rand(E, A, generator=g, dtype=D)
    c = body_pos[:, 1:2, :]  # middle circle
    pos = c + torch.stack([torch.cos(ang), torch.sin(ang)], -1) * rad[..., None]
    z = torch.zeros(E, A, dtype=D)
    return (pos, z, torch.zeros(E, A, 2, dtype=D), z.clone(), z.clone())


def push_actions(T, E, A, seed, pos0, target):
    g = torch.Generator().manual_seed(seed)
    dirn = target[:, None, :] - pos0
    dirn = dirn / dirn.norm(dim=-1, keepdim=True)
    base = dirn.unsqueeze(0).expand(T, E, A, 2)
    return (base + 0.3 * torch.randn(T, E, A, 2, generator=g, dtype=D)).contiguous()


def oracle_body_rollout(st, state5, acts, moving=True):
    w = ref_world(st)
    w.bodies_move = moving
    ob = ref_obstacles(st)
    return w, ob


def test_compound_circle_body_forward_and_adjoint_f64():
    E, A, T = 6, 4, 20
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float64, world=transport_world())
    obs = compound_body(E, 1)
    st.set_obstacles(obs)
    st.bodies_in_grad = True
    state5 = agents_around(E, A, 2, obs.pos)
    acts = push_actions(T, E, A, 3, state5[0], obs.pos[:, 1])
    goal = torch.tensor([0.4, -0.2], dtype=D)

    # oracle (before the CUDA rollout advances the stepper's body state)
    w = ref_world(st)
    ob = ref_obstacles(st)
    s_ref = [x.clone().requires_grad_(True) for x in state5]
    a_ref = acts.clone().requires_grad_(True)
    fin_r, traj_r, body_r = R.rollout(tuple(s_ref), a_ref, w, ob)
    loss_r = ((body_r[-1].body_pos[:, 0] - goal) ** 2).sum() + 0.3 * body_r[-1].body_angle[:, 0].sum() \
        + (fin_r[0] ** 2).sum()
    loss_r.backward()

    s = [x.to(DEV).requires_grad_(True) for x in state5]
    a = acts.to(DEV).requires_grad_(True)
    fin, traj, body = rollout_bodies(st, TorchState(*s), a)
    assert body is not None
    loss = ((body.pos[:, 0] - goal.to(DEV)) ** 2).sum() + 0.3 * body.angle[:, 0].sum() \
        + (fin.pos ** 2).sum()
    loss.backward()

    def close(x, y, rtol, what):
        scale = max(float(y.detach().abs().max()), 1e-30)
        torch.testing.assert_close(x.detach().cpu(), y.detach(), rtol=rtol, atol=rtol * scale,
                                   msg=lambda m: f"{what}: {m}")

    close(traj.stacked[0], torch.stack([t[0] for t in traj_r]), 1e-10, "agent pos")
    close(body.pos[:, 0], body_r[-1].body_pos[:, 0], 1e-10, "body pos")
    close(body.angle[:, 0], body_r[-1].body_angle[:, 0], 1e-10, "body angle")
    close(body.vel[:, 0], body_r[-1].body_vel[:, 0], 1e-10, "body vel")
    # the body moved
    assert float((body.pos[:, 0].detach().cpu() - ob.body_pos[:, 0]).norm(dim=-1).max()) > 1e-3
    close(a.grad, a_ref.grad, 1e-9, "grad actions")
    close(s[0].grad, s_ref[0].grad, 1e-9, "grad init pos")
    assert float(a.grad.abs().max()) > 0
    # the stepper carries the final body state
    close(st.body_state[0][:, 0], body_r[-1].body_pos[:, 0], 1e-10, "stepper body state")


def test_body_substeps_and_immovable_scenery_f64():
    """Two substeps; the body can hit an immovable circle and a segment wall."""
    E, A, T = 4, 4, 15
    cfgs = [AgentConfig(radius=0.05, max_speed=1.5, max_accel=2.0) for _ in range(A)]
    st = Stepper(cfgs, dt=0.05, substeps=2, device=DEV, dtype=torch.float64, world=transport_world())
    extra = dict(pos=torch.tensor([[[0.45, 0.0], [0.0, 0.5]]], dtype=D).expand(E, 2, 2).clone(),
                 radius=torch.tensor([0.1, 0.02], dtype=D),
                 shape=torch.tensor([0, 2], dtype=torch.int32),
                 angle=torch.zeros(E, 2, dtype=D),
                 kind=torch.zeros(2, dtype=torch.int32), mass=torch.ones(2, dtype=D),
                 inertia=torch.ones(2, dtype=D), body=torch.tensor([3, 4], dtype=torch.int32),
                 body_offset=torch.zeros(2, 2, dtype=D))
    obs = compound_body(E, 4, extra=extra)
    obs.half_extents = torch.tensor([[0, 0]] * 3 + [[0, 0], [0.4, 0]], dtype=D)
    st.set_obstacles(obs)
    st.bodies_in_grad = True
    state5 = agents_around(E, A, 5, obs.pos)
    acts = push_actions(T, E, A, 6, state5[0], torch.tensor([[0.6, 0.1]] * E, dtype=D))
    w = ref_world(st)
    ob = ref_obstacles(st)
    s_ref = [x.clone().requires_grad_(True) for x in state5]
    a_ref = acts.clone().requires_grad_(True)
    fin_r, _, body_r = R.rollout(tuple(s_ref), a_ref, w, ob)
    (body_r[-1].body_pos[:, 0].sum() + body_r[-1].body_vel[:, 0, 1].sum()).backward()
    a = acts.to(DEV).requires_grad_(True)
    fin, _, body = rollout_bodies(st, TorchState(*(x.to(DEV) for x in state5)), a)
    (body.pos[:, 0].sum() + body.vel[:, 0, 1].sum()).backward()
    torch.testing.assert_close(body.pos[:, 0].detach().cpu(), body_r[-1].body_pos[:, 0], rtol=1e-10,
                               atol=1e-12)
    scale = float(a_ref.grad.abs().max())
    torch.testing.assert_close(a.grad.cpu(), a_ref.grad, rtol=1e-9, atol=1e-9 * scale)


@pytest.mark.parametrize("shape", [ObstacleShape.BOX, ObstacleShape.SEGMENT])
def test_box_and_segment_bodies_forward_f64(shape):
    """Forward only (the adjoint differentiates circle bodies): off-centre pushes spin them."""
    E, A, T = 3, 4, 25
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float64, world=transport_world())
    g = torch.Generator().manual_seed(7)
    obs = Obstacles(
        pos=(torch.rand(E, 1, 2, generator=g, dtype=D) - 0.5) * 0.2,
        radius=torch.tensor([0.0 if shape == ObstacleShape.BOX else 0.04], dtype=D),
        shape=torch.tensor([int(shape)], dtype=torch.int32),
        angle=torch.rand(E, 1, generator=g, dtype=D),
        half_extents=torch.tensor([[0.15, 0.06] if shape == ObstacleShape.BOX else [0.15, 0.0]],
                                  dtype=D),
        kind=torch.ones(1, dtype=torch.int32), mass=torch.tensor([1.5], dtype=D),
        inertia=torch.tensor([0.02], dtype=D))
    st.set_obstacles(obs)
    state5 = agents_around(E, A, 8, torch.cat([obs.pos] * 3, 1))
    acts = push_actions(T, E, A, 9, state5[0], obs.pos[:, 0] + 0.05)
    w = ref_world(st)
    ob = ref_obstacles(st)
    with torch.no_grad():
        fin_r, _, body_r = R.rollout(state5, acts, w, ob)
        fin, _, body = rollout_bodies(st, TorchState(*(x.to(DEV) for x in state5)), acts.to(DEV))
    torch.testing.assert_close(fin.pos.cpu(), fin_r[0], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(body.pos.cpu()[:, 0], body_r[-1].body_pos[:, 0], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(body.angle.cpu()[:, 0], body_r[-1].body_angle[:, 0], rtol=1e-10,
                               atol=1e-12)
    assert float(body.angle[:, 0].sub(obs.angle[:, 0].to(DEV)).abs().max()) > 1e-4  # it spun


def test_reference_rule_freezes_bodies_on_grad_rollouts():
    """Default stepper: a taped rollout leaves movable bodies where they are (the
    reference's taped-step rule); an untaped one moves them."""
    E, A, T = 2, 4, 10
    cfgs = [AgentConfig(radius=0.05) for _ in range(A)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float64, world=transport_world())
    obs = compound_body(E, 11)
    st.set_obstacles(obs)
    state5 = agents_around(E, A, 12, obs.pos)
    acts = push_actions(T, E, A, 13, state5[0], obs.pos[:, 1]).to(DEV).requires_grad_(True)
    b0 = st.body_state[0].clone()
    fin, _, body = rollout_bodies(st, TorchState(*(x.to(DEV) for x in state5)), acts)
    assert body is None and torch.equal(st.body_state[0], b0)
    # and the agents were stopped by a static body: matches the oracle with frozen bodies
    w = ref_world(st)
    w.bodies_move = False
    with torch.no_grad():
        fin_r, _, _ = R.rollout(state5, acts.detach().cpu(), w, ref_obstacles(st))
    torch.testing.assert_close(fin.pos.detach().cpu(), fin_r[0], rtol=1e-10, atol=1e-12)
    with torch.no_grad():
        rollout(st, TorchState(*(x.to(DEV) for x in state5)), acts.detach())
    assert float((st.body_state[0] - b0).abs().max()) > 1e-4


def test_consecutive_rollouts_continue_bitwise():
    """Two rollouts of 5 steps equal one of 10 (body state and placed shapes carried)."""
    E, A = 3, 4
    cfgs = [AgentConfig(radius=0.05) for _ in range(A)]
    obs = compound_body(E, 21)
    state5 = agents_around(E, A, 22, obs.pos)
    acts = push_actions(10, E, A, 23, state5[0], obs.pos[:, 1]).to(DEV)
    s0 = TorchState(*(x.to(DEV) for x in state5))
    st1 = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float64, world=transport_world())
    st1.set_obstacles(obs)
    st2 = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float64, world=transport_world())
    st2.set_obstacles(obs)
    with torch.no_grad():
        f10, _ = rollout(st1, s0, acts)
        f5, _ = rollout(st2, s0, acts[:5])
        f55, _ = rollout(st2, f5, acts[5:])
    assert torch.equal(f10.pos, f55.pos)
    assert torch.equal(st1.body_state[0], st2.body_state[0])


def test_movable_pushed_along_and_compound_stays_rigid_f32():
    """Ported behaviour (reference tests/unit/test_obstacle_kinds.py): a head-on push
    moves the body along the push without deflecting it; a compound body keeps its shape."""
    cfgs = [AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.VELOCITY,
                        radius=0.05, max_speed=1.0)]
    world = WorldConfig(collisions=True, collision_k=1000.0, collision_c=20.0, collision_margin=0.01,
                        bounds=(-2.0, 2.0, -2.0, 2.0))
    st = Stepper(cfgs, dt=0.05, substeps=4, device=DEV, dtype=torch.float32, world=world)
    st.set_obstacles(Obstacles(
        pos=torch.zeros(2, 1, 2), radius=torch.full((1,), 0.1),
        kind=torch.ones(1, dtype=torch.int32), mass=torch.ones(1), inertia=torch.full((1,), 0.01)))
    pos = torch.tensor([[[-0.4, 0.0]]]).expand(2, 1, 2).contiguous().to(DEV)
    z = torch.zeros(2, 1, device=DEV)
    state = TorchState(pos, z, torch.zeros(2, 1, 2, device=DEV), z, z)
    act = torch.tensor([[[1.0, 0.0]]], device=DEV).expand(30, 2, 1, 2).contiguous()
    with torch.no_grad():
        rollout(st, state, act)
    o = st.obstacles
    assert float(o.pos[:, 0, 0].min()) > 0.05
    assert float(o.pos[:, 0, 1].abs().max()) < 1e-3
    assert float(o.vel[:, 0, 0].min()) > 0.0

    st2 = Stepper(cfgs, dt=0.05, substeps=4, device=DEV, dtype=torch.float32, world=world)
    off = torch.tensor([[0.0, 0.1], [0.0, -0.1]])
    st2.set_obstacles(Obstacles(
        pos=torch.tensor([[[0.0, 0.1], [0.0, -0.1]]]), radius=torch.full((2,), 0.08),
        angle=torch.zeros(1, 2), kind=torch.ones(2, dtype=torch.int32), mass=torch.ones(2),
        inertia=torch.full((2,), 0.02), body=torch.zeros(2, dtype=torch.int32), body_offset=off))
    state = TorchState(torch.tensor([[[-0.4, 0.06]]], device=DEV), z[:1], torch.zeros(1, 1, 2, device=DEV),
                       z[:1], z[:1])
    with torch.no_grad():
        rollout(st2, state, act[:, :1].contiguous().repeat(2, 1, 1, 1))
    p = st2.obstacles.pos
    assert abs(float((p[0, 0] - p[0, 1]).norm()) - 0.2) < 1e-5
    assert abs(float(st2.obstacles.angle[0, 0] - st2.obstacles.angle[0, 1])) < 1e-6
    assert float(p[0, :, 0].min()) > 0.02
    assert abs(float(st2.obstacles.angle[0, 0])) > 1e-4


def test_oracle_body_gradient_finite_differences():
    """Pins the oracle's body gradient (the reference has none): central differences of
    the final body x-position w.r.t. one action entry (float64, CPU)."""
    E, A, T = 1, 2, 8
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    from swarp_b200.dynamics.base import param_rows
    w = R.RefWorld(params=torch.tensor(param_rows(cfgs)), model_tag=[0] * A, ctrl_mode=[0] * A,
                   dt=0.05, k=100.0, c=5.0, margin=0.025, neighbor_radius=0.125, max_neighbors=4,
                   bounds=(-1.0, 1.0, -1.0, 1.0), soft_walls=True)
    spec = compound_body(E, 31)
    o = spec.resolve("cpu", D)
    ob = R.seed_bodies(R.RefObstacles(
        pos=o.pos, angle=o.angle, vel=o.vel, ang_vel=o.ang_vel, radius=o.radius, half=o.half_extents,
        shape=o.shape.tolist(), kind=o.kind.tolist(), mass=o.mass, inertia=o.inertia,
        body=o.body.tolist(), body_off=o.body_offset))
    state5 = agents_around(E, A, 32, o.pos)
    acts = push_actions(T, E, A, 33, state5[0], o.pos[:, 1]).clone().requires_grad_(True)
    _, _, body = R.rollout(state5, acts, w, ob)
    body[-1].body_pos[0, 0, 0].backward()
    h = 1e-6
    for idx in [(0, 0, 0, 0), (3, 0, 1, 1), (T - 1, 0, 0, 1)]:
        ap, am = acts.detach().clone(), acts.detach().clone()
        ap[idx] += h
        am[idx] -= h
        fp = R.rollout(state5, ap, w, ob)[2][-1].body_pos[0, 0, 0]
        fm = R.rollout(state5, am, w, ob)[2][-1].body_pos[0, 0, 0]
        fd = float((fp - fm) / (2 * h))
        assert abs(fd - float(acts.grad[idx])) <= 1e-6 + 1e-5 * abs(fd), (idx, fd, float(acts.grad[idx]))
