"""``torch.compile``-compatible step: the functional custom op ``swarp::step``.

Drop-in for the reference's ``swarp/interop/compile.py`` (``register_stepper`` ``:62-77``,
``swarp::step`` ``:92-120``, its fake ``:123-135`` and autograd rule ``:138-171``,
``compiled_warp_step`` ``:174-179``): same op name, argument list (a stepper handle, the
actions and the nine state fields) and outputs (nine fresh tensors). Dynamo and
AOTAutograd see one opaque differentiable operator instead of graph-breaking on the
autograd Function.

Forward: one launch of the fused rollout kernel with T = 1; in a fleet without drones the
drone fields are passed through as copies, with drones the kernel steps all nine. Backward: a second opaque op, ``swarp::step_backward``, runs the
forward kernel again from the saved inputs (it also rebuilds the contact checkpoint the
adjoint reads) and then the adjoint kernel; nothing survives between the forward and
backward calls, which is the functional contract the op promises. Steppers with movable bodies are not accepted here: their
state advances on the host between steps, which a functional op cannot express.
"""

from __future__ import annotations

import torch

from swarp_b200.core.stepper import Stepper, stepper_by_handle
from swarp_b200.interop.autograd import TorchState, fill_state_defaults, warp_step

def register_stepper(stepper: Stepper) -> int:
    """The stable int handle of ``stepper`` (assigned at construction; held weakly)."""
    return stepper.handle


def _check(stepper: Stepper) -> None:
    if stepper.any_movable:
        raise NotImplementedError("swarp::step does not take steppers with movable bodies; "
                                  "use warp_step / rollout_bodies")


@torch.library.custom_op("swarp::step", mutates_args=())
def _step_op(
    stepper_id: int,
    actions: torch.Tensor,
    pos: torch.Tensor,
    theta: torch.Tensor,
    vel: torch.Tensor,
    speed: torch.Tensor,
    ang_vel: torch.Tensor,
    z: torch.Tensor,
    vz: torch.Tensor,
    attitude: torch.Tensor,
    body_rates: torch.Tensor,
) -> list[torch.Tensor]:
    st = stepper_by_handle(stepper_id)
    _check(st)
    full = (pos, theta, vel, speed, ang_vel, z, vz, attitude, body_rates)
    state = tuple(t.contiguous() for t in full[:st.n_state])
    _, fin, _, _ = st.rollout_forward(state, actions.contiguous().unsqueeze(0), final=True)
    return [*fin, *(t.clone() for t in full[st.n_state:])]


@_step_op.register_fake
def _step_op_fake(stepper_id, actions, pos, theta, vel, speed, ang_vel, z, vz, attitude,
                  body_rates):
    # fresh contiguous outputs (the real op never returns an input's strides)
    return [torch.empty(t.shape, dtype=t.dtype, device=t.device)
            for t in (pos, theta, vel, speed, ang_vel, z, vz, attitude, body_rates)]


def _setup_context(ctx, inputs, output):
    stepper_id, actions, *state = inputs
    ctx.stepper_id = stepper_id
    ctx.save_for_backward(actions, *state)


@torch.library.custom_op("swarp::step_backward", mutates_args=())
def _step_backward_op(
    stepper_id: int,
    actions: torch.Tensor,
    pos: torch.Tensor,
    theta: torch.Tensor,
    vel: torch.Tensor,
    speed: torch.Tensor,
    ang_vel: torch.Tensor,
    z: torch.Tensor,
    vz: torch.Tensor,
    attitude: torch.Tensor,
    body_rates: torch.Tensor,
    g_pos: torch.Tensor | None,
    g_theta: torch.Tensor | None,
    g_vel: torch.Tensor | None,
    g_speed: torch.Tensor | None,
    g_ang_vel: torch.Tensor | None,
    g_z: torch.Tensor | None,
    g_vz: torch.Tensor | None,
    g_attitude: torch.Tensor | None,
    g_body_rates: torch.Tensor | None,
) -> list[torch.Tensor]:
    """Adjoint of one step: recompute the forward (trajectory and contact checkpoint)
    from the inputs, then run the adjoint kernel. Returns the action gradient and the
    gradients of the stepped state fields (five, or nine in a fleet with drones)."""
    st = stepper_by_handle(stepper_id)
    n = st.n_state
    state = tuple(t.contiguous() for t in (pos, theta, vel, speed, ang_vel, z, vz, attitude,
                                          body_rates)[:n])
    acts = actions.contiguous().unsqueeze(0)
    traj, _, _, rec = st.rollout_forward(state, acts, final=False)
    grads = (g_pos, g_theta, g_vel, g_speed, g_ang_vel, g_z, g_vz, g_attitude, g_body_rates)[:n]
    gtraj = tuple(None if g is None else g.contiguous().unsqueeze(0) for g in grads)
    g_act, g_init = st.rollout_backward(state, acts, traj, gtraj, (None,) * n, rec)
    return [g_act[0], *g_init]


@_step_backward_op.register_fake
def _step_backward_fake(stepper_id, actions, pos, theta, vel, speed, ang_vel, z, vz, attitude,
                        body_rates, *grads):
    n = stepper_by_handle(stepper_id).n_state
    return [torch.empty(t.shape, dtype=t.dtype, device=t.device)
            for t in (actions, pos, theta, vel, speed, ang_vel, z, vz, attitude, body_rates)[:n + 1]]


def _backward(ctx, *grad_outputs):
    grads = grad_outputs[0] if len(grad_outputs) == 1 else grad_outputs
    actions, *state = ctx.saved_tensors
    n = stepper_by_handle(ctx.stepper_id).n_state
    g_act, *g_init = torch.ops.swarp.step_backward(ctx.stepper_id, actions, *state, *grads[:9])
    passthrough = tuple(None if g is None else g.clone() for g in grads[n:9])
    return (None, g_act, *g_init, *passthrough)


_step_op.register_autograd(_backward, setup_context=_setup_context)


def compiled_warp_step(stepper: Stepper, state: TorchState, actions: torch.Tensor) -> TorchState:
    """``warp_step`` routed through the ``swarp::step`` custom op (torch.compile-safe)."""
    _check(stepper)
    state = fill_state_defaults(state)
    outs = torch.ops.swarp.step(stepper.handle, actions, *state)
    return TorchState(*outs)


__all__ = ["compiled_warp_step", "register_stepper", "warp_step"]
