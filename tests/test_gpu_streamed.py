"""StreamedRollout: BPTT over a batch in pinned host memory, pipelined over env chunks.

Envs are independent, so the gradient each chunk brings back must equal the whole-batch
rollout's for the same envs bit for bit, and the chunk losses must sum to its loss. Two
consecutive calls (the second overlapping the first) on different inputs both check out.
"""

import pytest
import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig
from swarp_b200.interop.autograd import TorchState, rollout
from swarp_b200.interop.streamed import StreamedRollout

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_streamed_equals_whole_batch():
    E, A, H = 600, 16, 9
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=16)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)],
                 dt=0.05, device=DEV, world=world)

    def loss_fn(fin, _traj, goal):
        return torch.nn.functional.mse_loss(fin.pos, goal, reduction="sum")

    inputs = []
    for seed in (0, 1):
        g = torch.Generator().manual_seed(seed)
        pos = (torch.rand(E, A, 2, generator=g) * 1.6 - 0.8).pin_memory()
        th = torch.zeros(E, A).pin_memory()
        acts = (torch.rand(H, E, A, 2, generator=g) * 2 - 1).pin_memory()
        goal = (torch.rand(E, A, 2, generator=g) * 1.6 - 0.8).pin_memory()
        inputs.append((pos, th, acts, goal))
    sr = StreamedRollout(st, E, H, 2, loss_fn, aux_like=[inputs[0][3]], chunks=4)
    assert sr.n_chunks == 4
    outs = []
    for pos, th, acts, goal in inputs:
        grad = torch.empty(H, E, A, 2).pin_memory()
        loss = torch.zeros(sr.n_chunks, dtype=torch.float64).pin_memory()
        sr(TorchState(pos, th, None, None, None), acts, [goal], grad, loss)
        outs.append((grad, loss))
    sr.synchronize()
    for (pos, th, acts, goal), (grad, loss) in zip(inputs, outs, strict=True):
        z = torch.zeros(E, A, device=DEV)
        a = acts.to(DEV).requires_grad_(True)
        fin, traj = rollout(st, TorchState(pos.to(DEV), th.to(DEV), torch.zeros(E, A, 2,
                                                                                   device=DEV),
                                           z, z), a)
        ref_loss = loss_fn(fin, traj, goal.to(DEV))
        (ref_g,) = torch.autograd.grad(ref_loss, [a])
        assert torch.equal(grad, ref_g.cpu())
        assert float(loss.sum()) == pytest.approx(float(ref_loss.detach()), rel=1e-5)
    sr.release()


def test_streamed_with_per_env_obstacles_equals_whole_batch():
    """Per-env obstacle poses: every chunk steps its own envs' obstacles."""
    from swarp_b200.core.config import Obstacles

    E, A, H = 64, 8, 6
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=8)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)],
                 dt=0.05, device=DEV, world=world)
    g = torch.Generator().manual_seed(3)
    st.set_obstacles(Obstacles(pos=torch.rand(E, 3, 2, generator=g) * 1.6 - 0.8,
                               radius=torch.tensor([0.1, 0.0, 0.03]),
                               shape=torch.tensor([0, 1, 2], dtype=torch.int32),
                               angle=torch.rand(E, 3, generator=g) * 3.0,
                               half_extents=torch.tensor([[0.0, 0.0], [0.1, 0.05], [0.15, 0.0]])))
    pos = (torch.rand(E, A, 2, generator=g) * 1.6 - 0.8).pin_memory()
    th = torch.zeros(E, A).pin_memory()
    acts = (torch.rand(H, E, A, 2, generator=g) * 2 - 1).pin_memory()
    goal = (torch.rand(E, A, 2, generator=g) * 1.6 - 0.8).pin_memory()
    sr = StreamedRollout(st, E, H, 2, "goal", aux_like=[goal], chunks=4)
    assert sr.per_chunk
    grad = torch.empty(H, E, A, 2).pin_memory()
    loss = torch.zeros(sr.n_chunks, dtype=torch.float64).pin_memory()
    sr(TorchState(pos, th, None, None, None), acts, [goal], grad, loss)
    sr.synchronize()
    z = torch.zeros(E, A, device=DEV)
    a = acts.to(DEV).requires_grad_(True)
    fin, _ = rollout(st, TorchState(pos.to(DEV), th.to(DEV), torch.zeros(E, A, 2, device=DEV), z,
                                    z), a)
    ref_loss = ((fin.pos - goal.to(DEV)) ** 2).sum()
    (ref_g,) = torch.autograd.grad(ref_loss, [a])
    assert torch.equal(grad, ref_g.cpu())
    assert float(loss.sum()) == pytest.approx(float(ref_loss.detach()), rel=1e-5)
    sr.release()
