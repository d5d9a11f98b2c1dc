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


def test_graphed_rollout_rejects_movable_bodies():
    from swarp_b200.core.config import ObstacleKind, Obstacles

    st = Stepper([AgentConfig()] * 2, dt=0.05, device=DEV, world=WorldConfig())
    st.set_obstacles(Obstacles(pos=torch.zeros(2, 1, 2), radius=torch.full((1,), 0.1),
                               kind=torch.full((1,), int(ObstacleKind.MOVABLE),
                                               dtype=torch.int32)))
    state, _, acts = _inputs(2, 2, 3, 0)
    with pytest.raises(NotImplementedError):
        GraphedRollout(st, state, acts, lambda f, t: f.pos.sum())


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
