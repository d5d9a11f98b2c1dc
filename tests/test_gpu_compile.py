"""The ``swarp::step`` custom op (torch.compile front end) on the CUDA path (GPU):
same results as ``warp_step``, no graph break under ``torch.compile(fullgraph=True)``,
and the op registration passes ``torch.library.opcheck`` (reference
swarp/interop/compile.py)."""

import pytest
import torch

from swarp_b200.core.config import ObstacleKind, Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel
from swarp_b200.interop.autograd import TorchState, fill_state_defaults, warp_step
from swarp_b200.interop.compile import compiled_warp_step, register_stepper

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _stepper(dtype=torch.float64):
    cfgs = [AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=ControlMode.ACCELERATION,
                        radius=0.05),
            AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0)] * 3
    world = WorldConfig(collision_k=100.0, collision_margin=0.025, neighbor_radius=0.2,
                        max_neighbors=6, bounds=(-0.4, 0.4, -0.4, 0.4), bounds_mode="soft")
    return Stepper(cfgs, dt=0.05, device=DEV, dtype=dtype, world=world)


def _state(E, A, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    f = lambda *s: (torch.rand(*s, generator=g, dtype=dtype) - 0.5).to(DEV)  # noqa: E731
    return TorchState(0.6 * f(E, A, 2), 3 * f(E, A), f(E, A, 2), f(E, A), f(E, A)), 3 * f(E, A, 2)


def test_op_matches_warp_step_values_and_grads():
    st = _stepper()
    s0, a0 = _state(5, 6, torch.float64, 0)
    out = []
    for fn in (warp_step, compiled_warp_step):
        s = TorchState(*(t.clone().requires_grad_(True) for t in s0[:5]))
        a = a0.clone().requires_grad_(True)
        nxt = fn(st, s, a)
        loss = (nxt.pos ** 2).sum() + nxt.theta.sin().sum() + (nxt.vel * 0.3).sum()
        grads = torch.autograd.grad(loss, [a, *s[:5]])
        out.append((tuple(nxt[:5]), grads))
    for x, y in zip(out[0][0] + out[0][1], out[1][0] + out[1][1], strict=True):
        assert torch.equal(x, y)


def test_torch_compile_fullgraph_multi_step():
    st = _stepper(torch.float32)
    s0, a0 = _state(8, 6, torch.float32, 1)
    goal = torch.full((8, 6, 2), 0.1, device=DEV)

    def episode(s, a, step):
        for _ in range(3):
            s = step(st, s, a)
        return ((s.pos - goal) ** 2).sum()

    compiled = torch.compile(lambda s, a: episode(s, a, compiled_warp_step), fullgraph=True,
                             backend="aot_eager")
    res = []
    for fn in (lambda s, a: episode(s, a, warp_step), compiled):
        a = a0.clone().requires_grad_(True)
        loss = fn(s0, a)
        (g,) = torch.autograd.grad(loss, [a])
        res.append((loss.detach(), g))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])


def test_opcheck():
    st = _stepper()
    s0, a0 = _state(3, 6, torch.float64, 2)
    s = fill_state_defaults(s0)
    args = (register_stepper(st), a0.requires_grad_(True),
            *(t.clone().requires_grad_(True) for t in s))
    torch.library.opcheck(torch.ops.swarp.step.default, args,
                          test_utils=("test_schema", "test_autograd_registration",
                                      "test_faketensor"))


def test_movable_bodies_rejected():
    st = _stepper()
    st.set_obstacles(Obstacles(pos=torch.zeros(3, 1, 2), radius=torch.full((1,), 0.1),
                               kind=torch.full((1,), int(ObstacleKind.MOVABLE),
                                               dtype=torch.int32)))
    s0, a0 = _state(3, 6, torch.float64, 3)
    with pytest.raises(NotImplementedError):
        compiled_warp_step(st, s0, a0)
