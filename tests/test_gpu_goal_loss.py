"""The fused goal loss (rollout_goal_loss, swarp_goal_loss_t) against the same loss in torch.

``rollout_goal_loss`` reduces sum |pos_T - goal|^2 in the forward kernel and seeds its
gradient 2 (pos_T - goal) inside the adjoint kernel. The seed is exactly what torch's
backward of ``((final.pos - goal) ** 2).sum()`` hands the adjoint for a unit cotangent, so
the gradients must be bitwise those of the unfused path; the loss value is the same sum
in another order (per CTA, then in double), so it agrees to rounding.
"""

import pytest
import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig
from swarp_b200.interop.autograd import FusedGoalLoss, TorchState, rollout, rollout_goal_loss
from swarp_b200.interop.graphs import GraphedRollout

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def scene(E, A, T, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, device=DEV) * 1.6 - 0.8).to(dtype)
    z = torch.zeros(E, A, device=DEV, dtype=dtype)
    state = (pos, z, torch.zeros(E, A, 2, device=DEV, dtype=dtype), z.clone(), z.clone())
    acts = (torch.rand(T, E, A, 2, generator=g, device=DEV) * 2 - 1).to(dtype)
    goal = (torch.rand(E, A, 2, generator=g, device=DEV) * 1.6 - 0.8).to(dtype)
    return state, acts, goal


def stepper(A, K, dtype, substeps=1):
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=K)
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    return Stepper(cfgs, dt=0.05, substeps=substeps, device=DEV, dtype=dtype, world=world)


# 16 agents in float32 take the two-agents-per-thread kernels; the others the generic ones
CASES = [(torch.float32, 16, 16, 1), (torch.float32, 12, 4, 1), (torch.float64, 16, 16, 1),
         (torch.float32, 16, 16, 2)]


@pytest.mark.parametrize("dtype,A,K,S", CASES, ids=["f32-x2", "f32-trunc", "f64", "f32-sub2"])
def test_fused_goal_loss_matches_torch_loss(dtype, A, K, S):
    E, T = 301, 9  # E not a multiple of the envs per CTA
    st = stepper(A, K, dtype, S)
    state, acts, goal = scene(E, A, T, dtype, seed=A + K)

    def unfused():
        s = [t.clone().requires_grad_(True) for t in state]
        a = acts.clone().requires_grad_(True)
        fin, _ = rollout(st, TorchState(*s), a)
        loss = ((fin.pos - goal) ** 2).sum()
        grads = torch.autograd.grad(loss, [a, s[0], s[2]])
        return loss.detach(), grads

    def fused():
        s = [t.clone().requires_grad_(True) for t in state]
        a = acts.clone().requires_grad_(True)
        loss = rollout_goal_loss(st, TorchState(*s), a, goal)
        grads = torch.autograd.grad(loss, [a, s[0], s[2]])
        return loss.detach(), grads

    l_ref, g_ref = unfused()
    l_fus, g_fus = fused()
    rtol = 1e-12 if dtype == torch.float64 else 1e-5
    torch.testing.assert_close(l_fus, l_ref, rtol=rtol, atol=0.0)
    for x, y in zip(g_fus, g_ref, strict=True):
        assert torch.equal(x, y)
    # a scaled cotangent scales the seed
    s = [t.clone() for t in state]
    a = acts.clone().requires_grad_(True)
    (3.0 * rollout_goal_loss(st, TorchState(*s), a, goal)).backward()
    tol = 1e-5 if dtype == torch.float32 else 1e-13  # the adjoint is linear, up to rounding
    torch.testing.assert_close(a.grad, 3.0 * g_ref[0], rtol=tol,
                               atol=tol * float(g_ref[0].abs().max()))
    # without grad: the value only
    with torch.no_grad():
        torch.testing.assert_close(rollout_goal_loss(st, TorchState(*state), acts, goal), l_ref,
                                   rtol=rtol, atol=0.0)


def test_graphed_fused_goal_loss_equals_graphed_torch_loss():
    E, A, T = 512, 16, 12
    st = stepper(A, 16, torch.float32)
    state, acts, goal = scene(E, A, T, torch.float32, seed=5)
    ref = GraphedRollout(st, TorchState(*state), acts,
                         lambda fin, _t: ((fin.pos - goal) ** 2).sum(), grad_norm=False)
    fus = GraphedRollout(st, TorchState(*state), acts, FusedGoalLoss(goal), grad_norm=False)
    for seed in (6, 7):  # new inputs through the static buffers
        state2, acts2, _ = scene(E, A, T, torch.float32, seed=seed)
        l1, g1 = ref(TorchState(*state2), acts2)
        l2, g2 = fus(TorchState(*state2), acts2)
        torch.testing.assert_close(l2, l1, rtol=1e-5, atol=0.0)
        assert torch.equal(g1, g2)
    ref.release()
    fus.release()


def test_goal_shape_is_checked():
    st = stepper(16, 16, torch.float32)
    state, acts, goal = scene(8, 16, 3, torch.float32, seed=1)
    with pytest.raises(ValueError):
        rollout_goal_loss(st, TorchState(*state), acts, goal[:, :8])
