"""PyTorch autograd bridge: ``warp_step`` and ``rollout`` as differentiable torch ops.

Drop-in for the reference's ``swarp/interop/autograd.py`` (``TorchState`` ``:29-45``,
``fill_state_defaults`` ``:48-68``, ``GradRing`` ``:184-226``, ``warp_step``
``:299-338``, ``rollout`` ``:341-369``). Same signatures and return values; what
differs is underneath: the reference records a Warp tape per step and replays Warp's
generated adjoints step by step from a Python loop, while here ``rollout`` is ONE
autograd node whose forward is one fused CUDA kernel over the whole horizon (the
trajectory it returns doubles as the checkpoint) and whose backward is one fused
adjoint kernel.

The four 6-DOF drone fields are carried through unchanged (2-D fleets only on this
path), exactly as the reference's full integrate kernel passes them through for 2-D
agents; their gradient is therefore the identity.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import NamedTuple

import torch

from swarp_b200.core.stepper import Stepper


class TorchState(NamedTuple):
    """World state as torch tensors (``[n_envs, n_agents]`` leading dims)."""

    pos: torch.Tensor
    theta: torch.Tensor
    vel: torch.Tensor
    speed: torch.Tensor
    ang_vel: torch.Tensor
    z: torch.Tensor | None = None
    vz: torch.Tensor | None = None
    attitude: torch.Tensor | None = None
    body_rates: torch.Tensor | None = None


def fill_state_defaults(state: TorchState) -> TorchState:
    """Materialise absent drone fields as zeros (identity attitude), freshly allocated on
    every call with the batch shape, device and dtype of ``pos`` (reference
    ``swarp/interop/autograd.py:48-68``): the tensors a state returns are its own, so a
    caller may edit them in place without touching any other state.
    """
    if all(t is not None for t in state):
        return state
    ref = state.pos
    E, A = ref.shape[0], ref.shape[1]
    opts = {"device": ref.device, "dtype": ref.dtype}
    z = state.z if state.z is not None else torch.zeros(E, A, **opts)
    vz = state.vz if state.vz is not None else torch.zeros(E, A, **opts)
    if state.attitude is not None:
        att = state.attitude
    else:
        att = torch.zeros(E, A, 4, **opts)
        att[..., 3] = 1.0
    br = state.body_rates if state.body_rates is not None else torch.zeros(E, A, 3, **opts)
    return state._replace(z=z, vz=vz, attitude=att, body_rates=br)


class Trajectory(Sequence):
    """``trajectory[t]`` is the :class:`TorchState` after step ``t``: views of the stacked
    ``[T, ...]`` rollout outputs, built on access (a T-step list of views costs more host
    time than the fused rollout itself at large horizons). Behaves as a read-only list."""

    def __init__(self, stacked: tuple[torch.Tensor, ...], extra: tuple) -> None:
        self.stacked = stacked
        self.extra = extra

    def __len__(self) -> int:
        return self.stacked[0].shape[0]

    def __getitem__(self, t):
        if isinstance(t, slice):
            return [self[i] for i in range(*t.indices(len(self)))]
        return TorchState(*(f[t] for f in self.stacked), *self.extra)


class BodyState(NamedTuple):
    """Movable-body state per obstacle slot (only body-root slots are meaningful)."""

    pos: torch.Tensor  # [n_envs, n_obstacles, 2]
    angle: torch.Tensor  # [n_envs, n_obstacles]
    vel: torch.Tensor  # [n_envs, n_obstacles, 2]
    ang_vel: torch.Tensor  # [n_envs, n_obstacles]


class _RolloutFn(torch.autograd.Function):
    """``(actions [T,E,A,D], n state tensors) -> (final n, trajectory n [T,...], final body
    state four)`` with n = ``stepper.n_state`` (five, nine with the drone fields); the body
    outputs are empty when no body moves."""

    @staticmethod
    def forward(ctx, stepper: Stepper, moving: bool, actions, *state):
        state5 = tuple(t.contiguous() for t in state)
        acts = actions.contiguous()
        traj, fin, _, rec = stepper.rollout_forward(state5, acts, final=True, moving_bodies=moving)
        ctx.stepper = stepper
        ctx.rec = rec
        ctx.n = len(state5)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(acts, *state5, *traj)
        if rec.moving:
            body = tuple(x[-1] for x in rec.body_traj)
        else:
            body = tuple(acts.new_empty(0) for _ in range(4))
            ctx.mark_non_differentiable(*body)
        return (*fin, *traj, *body)

    @staticmethod
    def backward(ctx, *grads):
        acts, *rest = ctx.saved_tensors
        n = ctx.n
        state5, traj5 = tuple(rest[:n]), tuple(rest[n:2 * n])
        gfin = tuple(None if g is None else g.contiguous() for g in grads[:n])
        gtraj = tuple(None if g is None else g.contiguous() for g in grads[n:2 * n])
        gb = grads[2 * n:2 * n + 4]
        gbody = gb if ctx.rec.moving and any(g is not None for g in gb) else None
        g_act, g_init = ctx.stepper.rollout_backward(state5, acts, traj5, gtraj, gfin, ctx.rec,
                                                     gbody_final=gbody)
        return (None, None, g_act, *g_init)


def _run(stepper: Stepper, state: TorchState, actions_seq: torch.Tensor):
    state = fill_state_defaults(state)
    n = stepper.n_state
    core = tuple(state[:n])
    stepper._check_inputs(core, actions_seq, horizon_dim=True)
    grad_mode = torch.is_grad_enabled() and (
        actions_seq.requires_grad or any(t.requires_grad for t in core)
    )
    extra = tuple(state[n:])
    # Reference rule: movable bodies advance on untaped steps; on taped ones only when
    # the stepper opts in (bodies_in_grad), which also makes them differentiable.
    moving = stepper.any_movable and (not grad_mode or stepper.bodies_in_grad)
    if moving and grad_mode and stepper.box_agents:
        raise NotImplementedError(
            "gradients through movable bodies pushed by box agents are not built (the forward "
            "is: step without grad, or keep bodies_in_grad False to freeze bodies on taped "
            "steps as the reference does)")
    if grad_mode:
        out = _RolloutFn.apply(stepper, moving, actions_seq, *core)
        fin, traj, body = out[:n], out[n:2 * n], out[2 * n:2 * n + 4]
    else:
        with torch.no_grad():
            core_c = tuple(t.contiguous() for t in core)
            traj, fin, _, rec = stepper.rollout_forward(core_c, actions_seq.contiguous(), final=True,
                                                        moving_bodies=moving)
            body = tuple(x[-1] for x in rec.body_traj) if rec.moving else None
    body_state = BodyState(*body) if moving else None
    return TorchState(*fin, *extra), traj, extra, body_state


def warp_step(stepper: Stepper, state: TorchState, actions: torch.Tensor, slot=None) -> TorchState:
    """Differentiable env step: ``state, actions [E,A,act_dim] -> next state``."""
    fin, _, _, _ = _run(stepper, state, actions.unsqueeze(0))
    return fin


def rollout(
    stepper: Stepper,
    state: TorchState,
    actions_seq: torch.Tensor,
    ring: GradRing | None = None,
) -> tuple[TorchState, list[TorchState]]:
    """Backprop-through-time rollout over ``actions_seq [T, n_envs, n_agents, act_dim]``.

    Returns ``(final_state, trajectory)``; ``trajectory[t]`` is the state after step
    ``t`` (a read-only sequence of :class:`TorchState`; ``trajectory.stacked`` holds the
    five ``[T, ...]`` tensors). Gradients flow to ``state`` and ``actions_seq``.
    """
    T = actions_seq.shape[0]
    if ring is not None:
        ring.reset()
        for _ in range(T):
            ring.acquire()
    fin, traj, extra, _ = _run(stepper, state, actions_seq)
    return fin, Trajectory(tuple(traj), extra)


def rollout_bodies(
    stepper: Stepper,
    state: TorchState,
    actions_seq: torch.Tensor,
) -> tuple[TorchState, Trajectory, BodyState | None]:
    """:func:`rollout` that also returns the movable bodies' final state.

    With ``stepper.bodies_in_grad`` (or under ``torch.no_grad()``) the bodies advance
    through the rollout, and in grad mode their final state is differentiable: a loss
    on it back-propagates through the body dynamics and the agent contacts into the
    actions and the initial agent state (bodies made of circle shapes). The body state
    the rollout starts from is ``stepper.body_state``, which the rollout advances.
    ``None`` is returned when no body moves.
    """
    fin, traj, extra, body = _run(stepper, state, actions_seq)
    return fin, Trajectory(tuple(traj), extra), body


class _GoalLossFn(torch.autograd.Function):
    """``(goal, actions [T,E,A,D], n state tensors) -> loss`` (0-d): the goal loss
    sum |pos_T - goal|^2 reduced in the forward kernel's epilogue, its cotangent seeded in
    the adjoint kernel's prologue (no torch ops between the two kernels)."""

    @staticmethod
    def forward(ctx, stepper: Stepper, goal, actions, *state):
        state5 = tuple(t.contiguous() for t in state)
        acts = actions.contiguous()
        loss = torch.empty((), dtype=stepper.dtype, device=stepper.device)
        traj, _, _, rec = stepper.rollout_forward(state5, acts, final=False, moving_bodies=False,
                                                  goal=goal, loss_out=loss)
        ctx.stepper, ctx.rec, ctx.n = stepper, rec, len(state5)
        ctx.save_for_backward(acts, goal, *state5, *traj)
        return loss

    @staticmethod
    def backward(ctx, g_loss):
        acts, goal, *rest = ctx.saved_tensors
        n = ctx.n
        state5, traj5 = tuple(rest[:n]), tuple(rest[n:2 * n])
        g_act, g_init = ctx.stepper.rollout_backward(
            state5, acts, traj5, (None,) * n, (None,) * n, ctx.rec, goal=goal,
            loss_grad=g_loss.detach().to(ctx.stepper.dtype).contiguous())
        return (None, None, g_act, *g_init)


def rollout_goal_loss(stepper: Stepper, state: TorchState, actions_seq: torch.Tensor,
                      goal: torch.Tensor) -> torch.Tensor:
    """``sum over envs and agents of ||pos_T - goal||^2`` after a rollout of ``actions_seq``
    ``[T, E, A, act_dim]`` from ``state``, differentiable w.r.t. the actions and the
    initial state (``goal`` ``[E, A, 2]`` is a constant).

    The same value and gradients as ``((rollout(...)[0].pos - goal) ** 2).sum()``, with the
    loss reduced in the forward kernel (per-CTA partials, fixed order) and its gradient
    seeded inside the adjoint kernel: a BPTT step is then two rollout kernels and one
    small reduction, with no elementwise torch ops between them. A fused fast path of
    this library; the reference's callers write such losses in torch. Fleets with
    movable bodies are not accepted (use ``rollout_bodies``).
    """
    if stepper.any_movable:
        raise NotImplementedError("rollout_goal_loss does not take movable bodies")
    state = fill_state_defaults(state)
    n = stepper.n_state
    core = tuple(state[:n])
    stepper._check_inputs(core, actions_seq, horizon_dim=True)
    E, A = core[0].shape[0], core[0].shape[1]
    if tuple(goal.shape) != (E, A, 2):
        raise ValueError(f"goal must be [{E}, {A}, 2]; got {tuple(goal.shape)}")
    goal = goal.detach().to(device=stepper.device, dtype=stepper.dtype).contiguous()
    if torch.is_grad_enabled() and (actions_seq.requires_grad or
                                    any(t.requires_grad for t in core)):
        return _GoalLossFn.apply(stepper, goal, actions_seq, *core)
    with torch.no_grad():
        loss = torch.empty((), dtype=stepper.dtype, device=stepper.device)
        stepper.rollout_forward(tuple(t.contiguous() for t in core), actions_seq.contiguous(),
                                final=False, moving_bodies=False, goal=goal, loss_out=loss)
    return loss


class FusedGoalLoss:
    """Marker for :class:`~swarp_b200.interop.graphs.GraphedRollout` (and
    :class:`~swarp_b200.interop.streamed.StreamedRollout`): take the step's loss from
    :func:`rollout_goal_loss` with this ``goal`` instead of a torch loss on the rollout."""

    def __init__(self, goal: torch.Tensor) -> None:
        self.goal = goal


class _CheckpointedFn(torch.autograd.Function):
    """``(actions [T,E,A,D], n state tensors) -> final n``, keeping only the state at
    every ``every``-th step: the forward runs the fused rollout kernel one segment of
    ``every`` steps at a time and drops each segment's trajectory; the backward re-runs
    each segment from its checkpoint (the same kernels on the same inputs reproduce it bit
    for bit) and runs the adjoint kernel over it, last segment first, handing the
    cotangent of each segment's initial state to the segment before."""

    @staticmethod
    def forward(ctx, stepper: Stepper, every: int, actions, *state):
        acts = actions.contiguous()
        cur = tuple(t.contiguous() for t in state)
        checkpoints = [cur]
        T = acts.shape[0]
        for t0 in range(0, T, every):
            _, fin, _, _ = stepper.rollout_forward(cur, acts[t0:t0 + every], final=True,
                                                   moving_bodies=False)
            cur = fin
            checkpoints.append(cur)
        ctx.stepper, ctx.every, ctx.n = stepper, every, len(cur)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(acts, *(t for cp in checkpoints[:-1] for t in cp))
        return cur

    @staticmethod
    def backward(ctx, *g_final):
        acts, *flat = ctx.saved_tensors
        n, every, st = ctx.n, ctx.every, ctx.stepper
        checkpoints = [tuple(flat[i:i + n]) for i in range(0, len(flat), n)]
        g = tuple(None if x is None else x.contiguous() for x in g_final)
        g_act = torch.empty_like(acts)
        for i in reversed(range(len(checkpoints))):
            t0 = i * every
            seg = acts[t0:t0 + every]
            traj, _, _, rec = st.rollout_forward(checkpoints[i], seg, final=False,
                                                 moving_bodies=False)
            ga, g = st.rollout_backward(checkpoints[i], seg, traj, (None,) * n, g, rec)
            g_act[t0:t0 + every] = ga
        return (None, None, g_act, *g)


def rollout_checkpointed(stepper: Stepper, state: TorchState, actions_seq: torch.Tensor,
                         every: int = 8) -> TorchState:
    """BPTT rollout that returns only the final state and keeps the state of every
    ``every``-th step for the backward pass instead of the whole trajectory.

    Memory for a T-step rollout is T/every checkpoints plus one ``every``-step segment,
    against T steps for :func:`rollout`; the price is a second forward pass over the
    horizon inside the backward. Gradients (w.r.t. ``state`` and ``actions_seq``) are the
    same as :func:`rollout`'s for a loss on the final state, bit for bit. Fleets with
    movable bodies are not accepted (their state advances on the host between rollouts).
    """
    if every < 1:
        raise ValueError(f"every must be >= 1, got {every}")
    if stepper.any_movable:
        raise NotImplementedError("rollout_checkpointed does not take movable bodies; use "
                                  "rollout_bodies")
    state = fill_state_defaults(state)
    n = stepper.n_state
    core = tuple(state[:n])
    stepper._check_inputs(core, actions_seq, horizon_dim=True)
    extra = tuple(state[n:])
    if torch.is_grad_enabled() and (actions_seq.requires_grad or
                                    any(t.requires_grad for t in core)):
        fin = _CheckpointedFn.apply(stepper, int(every), actions_seq, *core)
    else:
        with torch.no_grad():
            _, fin, _, _ = stepper.rollout_forward(tuple(t.contiguous() for t in core),
                                                   actions_seq.contiguous(), final=True,
                                                   moving_bodies=False)
    return TorchState(*fin, *extra)


@dataclass
class StepGradSlot:
    """One reserved step of a :class:`GradRing` (API compatibility)."""

    index: int


class GradRing:
    """Capacity bookkeeping of the reference's reusable BPTT scratch ring.

    The fused rollout allocates its trajectory/checkpoint buffers once per call from
    torch's caching allocator, so no per-step scratch exists to recycle; the ring
    keeps the reference contract (``reset``, ``acquire``, ``RuntimeError`` when a
    rollout is longer than ``capacity``).
    """

    def __init__(self, stepper: Stepper, n_envs: int, act_dim: int, capacity: int) -> None:
        self.stepper = stepper
        self.n_envs = n_envs
        self.act_dim = act_dim
        self.capacity = capacity
        self._idx = 0
        self.slots = [StepGradSlot(i) for i in range(capacity)]

    def reset(self) -> None:
        self._idx = 0

    def acquire(self) -> StepGradSlot:
        if self._idx >= self.capacity:
            raise RuntimeError(
                f"GradRing capacity {self.capacity} exhausted; size it to the rollout length T"
            )
        slot = self.slots[self._idx]
        self._idx += 1
        return slot
