"""A whole BPTT step captured in one CUDA graph.

One eager BPTT step through :func:`~swarp_b200.interop.autograd.rollout` is two fused
kernels on the device but a few hundred microseconds of host work (autograd bookkeeping,
the loss ops, the adjoint's engine hand-off). At the benchmark sizes that host time is
the same order as the kernels, so a training loop, and every rank of a multi-GPU job, is
then limited by Python. :class:`GraphedRollout` records the step once (forward kernel,
the user's loss, ``autograd.grad``, the adjoint kernel, the squared gradient norm) and
replays it with one graph launch. This is the B200-side counterpart of the reference's
CUDA-graph runtime (``swarp/core/stepper.py`` persistent buffers + ``wp.capture_*``),
which captures the forward step only.

Shapes, the stepper's configuration and the loss are fixed at capture; inputs are
copied into the graph's static buffers on each call.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from swarp_b200.core.stepper import Stepper
from swarp_b200.interop.autograd import (BodyState, FusedGoalLoss, TorchState, Trajectory,
                                         fill_state_defaults, rollout, rollout_bodies,
                                         rollout_goal_loss)


class GraphedRollout:
    """``loss_fn(final, trajectory) -> scalar`` differentiated w.r.t. the actions (and,
    with ``wrt_state``, the five initial-state fields), captured as one CUDA graph.
    ``loss_fn`` may also be a :class:`~swarp_b200.interop.autograd.FusedGoalLoss`: the
    goal loss computed inside the rollout kernels (its goal tensor is read at every
    replay, so it can be refilled in place between calls).

    ``state`` / ``actions`` give the shapes and the first inputs. Calling the object
    (optionally with new inputs, device or pinned host tensors of the same shapes) replays
    the graph and returns ``(loss, grad_actions)``: static tensors overwritten by the
    next call. With ``grad_norm`` (default), ``loss_and_grad_norm`` is a static
    ``[loss, ||grad_actions||^2]`` pair in the stepper's dtype, ready for a single
    all-reduce across ranks (``None`` otherwise). ``grad_norm="fused"`` takes the norm
    from the adjoint kernel's epilogue instead of a second pass over the gradient; it
    equals the exact norm when the loss depends on the actions only through the rollout.
    With ``all_reduce`` (and an initialised process group), the pair is summed across ranks
    by one NCCL all-reduce captured in the same graph, in stream order after the adjoint:
    a collective that overlapped the next step's forward kernel would take SM resources
    from it (one wave of it fills every SM's register file) and slow the step more than
    the all-reduce's own ~20 us. Release such a graph before destroying the process group.

    Movable bodies: with ``stepper.bodies_in_grad`` the captured step pushes the bodies
    (``rollout_bodies``) and ``loss_fn`` is called as ``loss_fn(final, trajectory,
    bodies)`` with the final :class:`~swarp_b200.interop.autograd.BodyState`. Every replay
    starts the bodies from the static state ``self.bodies`` (a copy of the stepper's body
    state and obstacle poses at construction; ``bodies=`` of a call refills it) and leaves
    the final body state in ``self.final_bodies``; replays do not advance the stepper's own
    body state. Without ``bodies_in_grad`` a taped step freezes the bodies (the reference's
    rule) and the world captures like one with static obstacles.
    """

    def __init__(self, stepper: Stepper, state: TorchState, actions: torch.Tensor,
                 loss_fn: Callable[[TorchState, Trajectory], torch.Tensor], *,
                 wrt_state: bool = False, grad_norm: bool | str = True,
                 warmup: int = 3, all_reduce: bool = False, group=None) -> None:
        self.bodies: BodyState | None = None
        self.final_bodies: BodyState | None = None
        self._moving = stepper.any_movable and stepper.bodies_in_grad
        if self._moving:
            if isinstance(loss_fn, FusedGoalLoss):
                raise NotImplementedError("the fused goal loss does not take movable bodies")
            if stepper.box_agents:
                raise NotImplementedError("gradients through movable bodies pushed by box agents "
                                          "are not built")
            # the static body state every replay starts from, and the obstacle set (with its
            # placed shape poses) the captured world description points at
            self.bodies = BodyState(*(t.detach().clone() for t in stepper.body_state))
            self._obstacles0 = stepper.obstacles
            self._from_bodies0 = stepper._poses_from_bodies
        if stepper.has_drones:
            raise NotImplementedError("GraphedRollout captures 2-D fleets; run a fleet with "
                                      "drones through rollout eagerly")
        dev = stepper.device
        self.stepper = stepper
        self.loss_fn = loss_fn
        self.wrt_state = wrt_state
        if grad_norm not in (True, False, "fused"):
            raise ValueError(f"grad_norm must be True, False or 'fused'; got {grad_norm!r}")
        self.grad_norm = grad_norm
        self.all_reduce = bool(all_reduce) and grad_norm is not False
        self.group = group
        if grad_norm == "fused":
            stepper.track_grad_norm = True
        # Static leaves, detached from any history the given inputs carry: a backward that
        # reached back into the caller's graph would leave the capture stream.
        self.actions = actions.detach().to(dev, copy=True).requires_grad_(True)
        self.state = TorchState(*(t.detach().to(dev, copy=True) for t in tuple(state)[:5]))
        # the drone fields a 2-D fleet passes through, materialised once outside the capture
        # (the graph then holds no allocation or fill of them)
        self.state = fill_state_defaults(self.state)
        if wrt_state:
            for t in self.state[:5]:
                t.requires_grad_(True)
        # the unit cotangent of the loss, allocated once: autograd would otherwise fill a
        # fresh one inside the graph at every replay
        self._one = torch.ones((), device=dev, dtype=stepper.dtype)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._install_bodies()
                self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        self._install_bodies()
        with torch.cuda.graph(self.graph):
            self.loss, self.grads, self.loss_and_grad_norm = self._body()
        self._install_bodies()
        self.grad_actions = self.grads[0]
        self.grad_state = TorchState(*self.grads[1:6]) if wrt_state else None

    def _install_bodies(self) -> None:
        """Point the stepper at the static body state and the obstacle set of construction
        (a body rollout replaces both attributes with its outputs)."""
        if not self._moving:
            return
        st = self.stepper
        st.obstacles = self._obstacles0
        st.body_state = tuple(self.bodies)
        st._poses_from_bodies = self._from_bodies0
        st._wc_cache.clear()

    def _body(self):
        if isinstance(self.loss_fn, FusedGoalLoss):
            loss = rollout_goal_loss(self.stepper, self.state, self.actions, self.loss_fn.goal)
        elif self._moving:
            fin, traj, body = rollout_bodies(self.stepper, self.state, self.actions)
            self.final_bodies = body
            loss = self.loss_fn(fin, traj, body)
        else:
            fin, traj = rollout(self.stepper, self.state, self.actions)
            loss = self.loss_fn(fin, traj)
        wrt = [self.actions] + (list(self.state[:5]) if self.wrt_state else [])
        one = self._one if loss.dtype == self._one.dtype else torch.ones_like(loss)
        grads = torch.autograd.grad(loss, wrt, grad_outputs=one)
        pair = None
        if self.grad_norm == "fused":
            pair = torch.stack([loss.detach(), self.stepper.last_grad_sqnorm])
        elif self.grad_norm:
            g = grads[0].reshape(-1)
            pair = torch.stack([loss.detach(), torch.dot(g, g)])
        dist = torch.distributed
        if self.all_reduce and dist.is_available() and dist.is_initialized():
            dist.all_reduce(pair, group=self.group)
        return loss.detach(), grads, pair

    def __call__(self, state: TorchState | None = None, actions: torch.Tensor | None = None,
                 bodies: BodyState | None = None):
        with torch.no_grad():
            if bodies is not None:
                if self.bodies is None:
                    raise ValueError("this graph pushes no movable bodies")
                for dst, src in zip(self.bodies, tuple(bodies), strict=True):
                    dst.copy_(src, non_blocking=True)
            if actions is not None:
                self.actions.copy_(actions, non_blocking=True)
            if state is not None:
                for dst, src in zip(self.state[:5], tuple(state)[:5], strict=True):
                    if src is not None:  # None keeps that field's current contents
                        dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.loss, self.grad_actions

    def release(self) -> None:
        """Free the graph (and its memory pool) now rather than at garbage collection."""
        self.graph.reset()
        self.graph = None
