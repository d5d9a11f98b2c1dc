"""GraphedRollout (one CUDA graph per BPTT step) reproduces the eager drop-in path
bit for bit, before and after new inputs are copied in (GPU)."""

import pytest
import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig
from swarp_b200.interop.autograd import TorchState, rollout
from swarp_b200.interop.graphs import GraphedRollout

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(E, A, T, seed):
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g) * 1.8 - 0.9).to(DEV)
    goal = (torch.rand(E, A, 2, generator=g) * 1.8 - 0.9).to(DEV)
    acts = (torch.rand(T, E, A, 2, generator=g) * 2 - 1).to(DEV)
    z = torch.zeros(E, A, device=DEV)
    return TorchState(pos, z, torch.zeros(E, A, 2, device=DEV), z.clone(), z.clone()), goal, acts


def _eager(st, state, acts, goal):
    a = acts.clone().requires_grad_(True)
    s = TorchState(*(t.clone().requires_grad_(True) for t in state[:5]))
    fin, traj = rollout(st, s, a)
    loss = ((fin.pos - goal) ** 2).sum() + 0.1 * traj.stacked[2].square().sum()
    grads = torch.autograd.grad(loss, [a, *s[:5]])
    return loss.detach(), grads


def test_graphed_bptt_matches_eager_bitwise():
    E, A, T = 300, 16, 12
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft",
                        neighbor_radius=0.125, max_neighbors=16)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0)] * A, dt=0.05,
                 device=DEV, world=world)
    state, goal, acts = _inputs(E, A, T, 0)
    goal_buf = goal.clone()

    def loss_fn(fin, traj):
        return ((fin.pos - goal_buf) ** 2).sum() + 0.1 * traj.stacked[2].square().sum()

    # inputs that carry autograd history of their own must not leak into the capture
    gr = GraphedRollout(st, state, acts.clone().requires_grad_(True) * 1.0, loss_fn,
                        wrt_state=True)
    loss, g_act = gr()
    ref_loss, ref_g = _eager(st, state, acts, goal)
    assert torch.equal(loss, ref_loss) and torch.equal(g_act, ref_g[0])
    for a, b in zip(gr.grad_state, ref_g[1:]):
        assert torch.equal(a, b)
    assert gr.loss_and_grad_norm[0].item() == loss.item()
    assert gr.loss_and_grad_norm[1].item() == pytest.approx(
        float(ref_g[0].double().square().sum()), rel=1e-5)

    # new inputs, copied from pinned host memory; vel/speed/ang_vel keep their zeros
    state2, goal2, acts2 = _inputs(E, A, T, 1)
    goal_buf.copy_(goal2)
    host = [t.cpu().pin_memory() for t in (state2.pos, state2.theta, acts2)]
    loss, g_act = gr(TorchState(host[0], host[1], None, None, None), host[2])
    ref_loss, ref_g = _eager(st, state2, acts2, goal2)
    assert torch.equal(loss, ref_loss) and torch.equal(g_act, ref_g[0])
    gr.release()


def _body_world(E, dtype=torch.float32):
    """Four disc agents around a movable three-circle body (the transport shape)."""
    import numpy as np

    from swarp_b200.core.config import ObstacleKind, Obstacles

    world = WorldConfig(collision_k=100.0, collision_c=5.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft", neighbor_radius=0.125,
                        max_neighbors=4)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0)] * 4, dt=0.05,
                 device=DEV, dtype=dtype, world=world)
    rng = np.random.default_rng(4)
    ang = rng.uniform(-0.5, 0.5, E)
    cen = rng.uniform(-0.3, 0.3, (E, 2))
    off = np.array([[-0.12, 0.0], [0.0, 0.0], [0.12, 0.0]])
    ca, sa = np.cos(ang)[:, None], np.sin(ang)[:, None]
    opos = np.stack([cen[:, None, 0] + ca * off[:, 0] - sa * off[:, 1],
                     cen[:, None, 1] + sa * off[:, 0] + ca * off[:, 1]], -1)
    t = lambda x: torch.tensor(x, dtype=dtype)  # noqa: E731
    st.set_obstacles(Obstacles(
        pos=t(opos), radius=torch.full((3,), 0.08), shape=torch.zeros(3, dtype=torch.int32),
        angle=t(np.repeat(ang[:, None], 3, 1)),
        kind=torch.full((3,), int(ObstacleKind.MOVABLE), dtype=torch.int32),
        mass=torch.full((3,), 2.5), inertia=torch.full((3,), 0.03),
        body=torch.zeros(3, dtype=torch.int32), body_offset=t(off), half_extents=torch.zeros(3, 2)))
    st.bodies_in_grad = True
    a_ang = rng.uniform(0.0, 2 * np.pi, (E, 4))
    a_rad = rng.uniform(0.2, 0.28, (E, 4))
    pos = cen[:, None, :] + np.stack([np.cos(a_ang), np.sin(a_ang)], -1) * a_rad[..., None]
    goal = t(rng.uniform(-0.5, 0.5, (E, 2))).to(DEV)
    push = goal.cpu().numpy()[:, None, :] - pos
    push /= np.linalg.norm(push, axis=-1, keepdims=True)
    return st, t(pos).to(DEV), goal, push


def test_graphed_rollout_pushes_movable_bodies_bitwise():
    from swarp_b200.interop.autograd import rollout_bodies

    E, T = 64, 20
    st, pos, goal, push = _body_world(E)
    z = torch.zeros(E, 4, device=DEV)
    state = TorchState(pos, z, torch.zeros(E, 4, 2, device=DEV), z, z)
    g = torch.Generator().manual_seed(3)
    acts = (torch.from_numpy(push).float()[None] + 0.3 * torch.randn(T, E, 4, 2, generator=g))
    acts = acts.to(DEV)
    snap = st.bodies_snapshot()

    def loss_fn(fin, traj, body):
        return (body.pos[:, 0] - goal).norm(dim=-1).sum() + 0.01 * fin.vel.square().sum()

    def eager(a_in):
        st.restore_bodies(snap)
        a = a_in.clone().requires_grad_(True)
        fin, traj, body = rollout_bodies(st, state, a)
        loss = loss_fn(fin, traj, body)
        (ga,) = torch.autograd.grad(loss, [a])
        return loss.detach(), ga, body

    ref_loss, ref_g, ref_body = eager(acts)
    st.restore_bodies(snap)
    gr = GraphedRollout(st, state, acts, loss_fn)
    for _ in range(2):  # replays start from the same static body state
        loss, g_act = gr()
        assert torch.equal(loss, ref_loss) and torch.equal(g_act, ref_g)
        for x, y in zip(gr.final_bodies, ref_body):
            assert torch.equal(x, y)
    assert float(ref_g.abs().max()) > 0.0
    # new actions and a refilled body state
    acts2 = acts + 0.1
    ref_loss2, ref_g2, _ = eager(acts2)
    loss, g_act = gr(actions=acts2, bodies=snap[1])
    assert torch.equal(loss, ref_loss2) and torch.equal(g_act, ref_g2)
    gr.release()


def test_graphed_rollout_rejects_fused_loss_with_bodies():
    from swarp_b200.interop.autograd import FusedGoalLoss

    st, pos, goal, _ = _body_world(4)
    z = torch.zeros(4, 4, device=DEV)
    state = TorchState(pos, z, torch.zeros(4, 4, 2, device=DEV), z, z)
    acts = torch.zeros(3, 4, 4, 2, device=DEV)
    with pytest.raises(NotImplementedError):
        GraphedRollout(st, state, acts, FusedGoalLoss(torch.zeros(4, 4, 2, device=DEV)))


@pytest.mark.parametrize("dtype,substeps,A,K", [(torch.float32, 1, 16, 16), (torch.float64, 1, 40, 8),
                                                (torch.float32, 3, 8, 8), (torch.float64, 2, 5, 4)])
def test_fused_grad_sqnorm_matches_the_gradient(dtype, substeps, A, K):
    """The adjoint epilogue's sum(grad_actions^2) equals the norm of the returned gradient
    (fast path, truncating lists, substep recompute path)."""
    E, T = 37, 9
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft",
                        neighbor_radius=0.3, max_neighbors=K)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0)] * A, dt=0.05,
                 substeps=substeps, device=DEV, dtype=dtype, world=world)
    st.track_grad_norm = True
    state, goal, acts = _inputs(E, A, T, 3)
    state = TorchState(*(t.to(dtype) for t in state[:5]))
    a = acts.to(dtype).requires_grad_(True)
    fin, _ = rollout(st, state, a)
    (g,) = torch.autograd.grad(((fin.pos - goal.to(dtype)) ** 2).sum(), [a])
    want = float(g.double().square().sum())
    got = float(st.last_grad_sqnorm)
    assert got == pytest.approx(want, rel=1e-5 if dtype == torch.float32 else 1e-12)


def test_fused_norm_in_graph_pair():
    E, A, T = 64, 16, 8
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0)] * A, dt=0.05,
                 device=DEV, world=WorldConfig(collision_margin=0.025, neighbor_radius=0.125,
                                               max_neighbors=16))
    state, goal, acts = _inputs(E, A, T, 4)
    gr = GraphedRollout(st, state, acts, lambda f, t: ((f.pos - goal) ** 2).sum(),
                        grad_norm="fused")
    _, g = gr()
    torch.cuda.synchronize()
    assert gr.loss_and_grad_norm[1].item() == pytest.approx(float(g.double().square().sum()),
                                                            rel=1e-5)
    gr.release()
