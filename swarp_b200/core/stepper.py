"""Stepper: owns the agent parameters, the obstacle set and the substep pipeline.

Drop-in for ``swarp.core.stepper.Stepper`` (reference ``swarp/core/stepper.py:66-240``,
``set_obstacles`` ``:295-344``, ``set_agent_params_per_env`` ``:362-452``): same
constructor arguments and validation. Instead of launching Warp kernels per substep it
describes the world once (``swarp_world_t``) and runs whole rollouts through the C ABI
of ``libswarp_b200.so``: one kernel for the forward horizon, one for its adjoint.

``dtype`` accepts a torch dtype (``torch.float32``/``torch.float64``) or its name; the
reference's Warp dtype argument has no meaning without Warp.
"""

from __future__ import annotations

import ctypes as C
import itertools
import weakref
from dataclasses import dataclass, replace

import numpy as np
import torch

from swarp_b200 import _lib
from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.dynamics.base import (
    NUM_PARAMS,
    P_RADIUS,
    P_SHAPE,
    AgentConfig,
    AgentShape,
    DynamicsModel,
    Integrator,
    param_rows,
)

_DTYPES = {
    torch.float32: torch.float32, torch.float64: torch.float64,
    "float32": torch.float32, "float64": torch.float64,
    "f32": torch.float32, "f64": torch.float64,
}


def _as_torch_dtype(dtype) -> torch.dtype:
    if dtype in _DTYPES:
        return _DTYPES[dtype]
    name = getattr(dtype, "__name__", str(dtype)).lower()
    for key in ("float64", "float32"):
        if key in name:
            return _DTYPES[key]
    raise TypeError(f"unsupported dtype {dtype!r}; use torch.float32 or torch.float64")


@dataclass
class RolloutRecord:
    """What a forward rollout hands to its adjoint: the exact C world it ran with, and
    the buffers that world points to (kept alive until the adjoint has run)."""

    wc: _lib.WorldC
    workspace: torch.Tensor
    obstacles: object
    body_init: tuple | None
    body_traj: tuple | None
    moving: bool


# Live steppers by integer handle (weak): the handle is how an op that cannot carry Python
# objects (the ``swarp::step`` custom op) names its stepper. Assigned at construction so
# that a traced program only ever reads ``stepper.handle``.
_REGISTRY: "weakref.WeakValueDictionary[int, Stepper]" = weakref.WeakValueDictionary()
_NEXT_HANDLE = itertools.count()


def stepper_by_handle(handle: int) -> Stepper:
    try:
        return _REGISTRY[handle]
    except KeyError:
        raise RuntimeError(
            f"no live Stepper has handle {handle}: it was garbage-collected; keep the "
            "Environment/World (or the Stepper) alive while a compiled step uses it") from None


class Stepper:
    """Owns per-agent parameters, interaction config and the rollout launches."""

    def __init__(
        self,
        configs: list[AgentConfig],
        dt: float = 0.1,
        substeps: int = 1,
        device: str = "cuda:0",
        dtype=torch.float32,
        world: WorldConfig | None = None,
    ) -> None:
        # A bare Stepper is collision-free unless a config asks (reference stepper.py:97-101).
        world = world if world is not None else WorldConfig(collisions=False)
        if substeps < 1:
            raise ValueError("substeps must be >= 1")
        if not configs:
            raise ValueError("a Stepper needs at least one agent")
        self.configs = list(configs)
        self.n_agents = len(configs)
        self.dt = float(dt)
        self.substeps = int(substeps)
        self.sub_dt = self.dt / self.substeps
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError(
                f"swarp_b200 steps only on CUDA devices (got {device!r}); there is no CPU path"
            )
        if self.device.index is None:  # "cuda" means the current device, as in torch
            self.device = torch.device(
                "cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
        self.dtype = _as_torch_dtype(dtype)
        self.torch_dtype = self.dtype
        self.world = world
        self.handle = next(_NEXT_HANDLE)
        _REGISTRY[self.handle] = self
        if self.n_agents > _lib.MAX_AGENTS:
            raise ValueError(f"{self.n_agents} agents per env exceed the {_lib.MAX_AGENTS} this "
                             "build runs (one env per cluster of 8 CTAs)")
        # 6-DOF drones carry four more state fields (z, vz, attitude, body rates)
        self.has_drones = any(c.model == DynamicsModel.DRONE for c in self.configs)
        self.n_state = 9 if self.has_drones else 5
        if world.integrator not in (Integrator.EULER, Integrator.RK4):
            raise NotImplementedError(f"integrator {world.integrator} is not on the CUDA path")
        if world.wheel_contacts:
            raise NotImplementedError("wheel contacts are not on the CUDA path")
        if world.obstacle_friction > 0.0:
            raise NotImplementedError("floor friction of movable bodies (obstacle_friction) is "
                                      "not on the CUDA path")
        # Every method is served by the brute-force (ascending-index) lists of the fused
        # kernels. With collisions on (the reference then builds a NeighborGrid), the radius,
        # method and bins are checked as NeighborGrid checks them
        # (swarp/core/neighbors.py:376-379, 391-394).
        if world.collisions:
            reach = 2.0 * max(c.radius for c in self.configs) + world.collision_margin
            if not (world.neighbor_radius or reach) > 0.0:
                raise ValueError("radius must be positive")
            if world.neighbor_method not in ("auto", "grid", "brute", "uniform_grid"):
                raise ValueError('method must be "auto", "grid", "brute", or "uniform_grid"')
            if world.uniform_bins is not None and world.uniform_bins < 1:
                raise ValueError("uniform_bins must be >= 1")
        self.box_agents = any(c.shape == AgentShape.BOX for c in self.configs)
        if self.has_drones and self.box_agents:
            raise NotImplementedError("box agents and drones in one fleet are not on the CUDA path")
        if self.n_agents > _lib.MAX_CTA_AGENTS and (self.has_drones or self.box_agents):
            raise NotImplementedError(f"box agents and drones run in envs of at most "
                                      f"{_lib.MAX_CTA_AGENTS} agents")
        self.params = torch.tensor(param_rows(self.configs), dtype=self.dtype, device=self.device)
        self.params_per_env: torch.Tensor | None = None
        self.model_tag = torch.tensor([int(c.model) for c in self.configs], dtype=torch.int32,
                                      device=self.device)
        self.ctrl_mode = torch.tensor([int(c.ctrl_mode) for c in self.configs],
                                      dtype=torch.int32, device=self.device)
        self.fleet_models = 0
        self.fleet_modes = 0
        for c in self.configs:
            self.fleet_models |= 1 << int(c.model)
            self.fleet_modes |= 1 << int(c.ctrl_mode)

        self.collisions = bool(world.collisions)
        self.max_agent_radius = max(c.radius for c in self.configs)
        self.neighbor_radius = 0.0
        if self.collisions:
            reach = 2.0 * self.max_agent_radius + world.collision_margin
            self.neighbor_radius = world.neighbor_radius or reach
            if self.neighbor_radius < reach:
                raise ValueError(
                    f"neighbor_radius={self.neighbor_radius} is smaller than the collision "
                    f"reach {reach} (= 2 * max radius + margin); collisions would be missed."
                )
        self._soft_walls = world.bounds is not None and world.bounds_mode == "soft"
        self._clamp = world.bounds is not None and world.bounds_mode == "clamp"
        self.n_obstacles = 0
        self.obstacles: Obstacles | None = None
        self.any_movable = False
        #: Bitmask (1 << ObstacleShape) of the shapes belonging to movable bodies.
        self.movable_shapes = 0
        #: Whether movable bodies advance on grad (taped) rollouts. False (default) is the
        #: reference's rule: a taped step freezes them (swarp/core/stepper.py:593-601)
        #: and only no-grad steps integrate them. True integrates them on grad rollouts
        #: as well and differentiates through them (bodies of circle shapes).
        self.bodies_in_grad = False
        #: When set, every rollout also records, per agent, the largest uncapped in-radius
        #: neighbor count over its substeps (``last_true_count_max`` [E, A] int32);
        #: :meth:`rollout_overflow` compares it with ``max_neighbors``.
        self.track_neighbor_overflow = False
        self.last_true_count_max: torch.Tensor | None = None
        #: When set, every adjoint rollout also reduces sum(grad_actions^2) in its epilogue
        #: into ``last_grad_sqnorm`` (a 0-d tensor of the stepper's dtype): the squared norm
        #: of the gradient that flows into the actions through the rollout, without a
        #: second pass over it.
        self.track_grad_norm = False
        self.last_grad_sqnorm: torch.Tensor | None = None
        #: Body state per obstacle slot (pos [E,N,2], angle [E,N], vel [E,N,2],
        #: ang_vel [E,N]); only body-root slots are meaningful.
        self.body_state: tuple[torch.Tensor, ...] | None = None
        self._poses_from_bodies = False
        # (n_envs, act_dim) -> filled swarp_world_t; cleared whenever an input it points to
        # is replaced (obstacles, per-env parameters).
        self._wc_cache: dict[tuple[int, int], _lib.WorldC] = {}

    # ----------------------------------------------------------------- set-up
    def set_obstacles(self, obstacles: Obstacles) -> None:
        """Install (or refresh) an obstacle set; absent fields take their defaults."""
        obs = obstacles.resolve(self.device, self.dtype)
        self._wc_cache.clear()
        self.obstacles = obs
        self.n_obstacles = obs.n_obstacles
        moving = obs.kind[obs.body.long()] != 0  # shapes whose body root is movable
        self.any_movable = bool(moving.any().item())
        if self.any_movable and self.n_agents > _lib.MAX_CTA_AGENTS:
            raise NotImplementedError(f"movable obstacles run in envs of at most "
                                      f"{_lib.MAX_CTA_AGENTS} agents")
        self.movable_shapes = 0
        self._poses_from_bodies = False
        if self.any_movable:
            for st in obs.shape[moving].unique().tolist():
                self.movable_shapes |= 1 << int(st)
            self.body_state = self._body_seed(obs)
        else:
            self.body_state = None

    def _body_seed(self, obs: Obstacles) -> tuple[torch.Tensor, ...]:
        """Body state per shape slot derived from the root shapes' world poses."""
        root = obs.body.long()
        r_ang = obs.angle[:, root]
        r_off = obs.body_offset[root]
        ca, sa = torch.cos(r_ang), torch.sin(r_ang)
        wx = ca * r_off[:, 0] - sa * r_off[:, 1]
        wy = sa * r_off[:, 0] + ca * r_off[:, 1]
        b_pos = (obs.pos[:, root] - torch.stack([wx, wy], dim=-1)).contiguous()
        return (b_pos, r_ang.contiguous(), obs.vel[:, root].contiguous(),
                obs.ang_vel[:, root].contiguous())

    def set_agent_params_per_env(self, floats) -> None:
        """Install a per-env ``[n_envs, n_agents, NUM_PARAMS]`` parameter override."""
        t = torch.as_tensor(np.asarray(floats) if not torch.is_tensor(floats) else floats)
        if t.dim() != 3 or tuple(t.shape[1:]) != (self.n_agents, NUM_PARAMS):
            raise ValueError(
                f"per-env params must have shape [n_envs, n_agents={self.n_agents}, "
                f"NUM_PARAMS={NUM_PARAMS}]; got {tuple(t.shape)}"
            )
        shared = torch.tensor([float(c.shape) for c in self.configs], dtype=torch.float64)
        if not torch.equal(t[..., P_SHAPE].detach().double().cpu(), shared.expand(t.shape[0], -1)):
            raise ValueError("per-env params must not change the P_SHAPE column: an agent's "
                             "AgentShape is structural and fixed by its AgentConfig.")
        if self.collisions:
            max_r = float(t[..., P_RADIUS].max())
            reach = 2.0 * max_r + self.world.collision_margin
            if self.neighbor_radius < reach:
                raise ValueError(
                    f"per-env radius up to {max_r} needs neighbor_radius >= {reach}, but "
                    f"neighbor_radius={self.neighbor_radius}; set WorldConfig.neighbor_radius."
                )
        self._wc_cache.clear()
        self.params_per_env = t.detach().to(device=self.device, dtype=self.dtype).contiguous()

    def env_slice(self, start: int, stop: int) -> Stepper:
        """A stepper for envs ``[start, stop)`` of this one's batch: the same agents and
        world, the obstacle poses and per-env parameters of those envs (views). Stepping
        it on the slice of a batch gives that slice of the batch's results bit for bit
        (envs are independent). Movable bodies are not sliced (their state is per call)."""
        if self.any_movable:
            raise NotImplementedError("env_slice does not carry movable-body state")
        st = Stepper(self.configs, dt=self.dt, substeps=self.substeps, device=self.device,
                     dtype=self.dtype, world=self.world)
        if self.obstacles is not None:
            st.set_obstacles(self.obstacles.env_slice(start, stop))
        if self.params_per_env is not None:
            st.set_agent_params_per_env(self.params_per_env[start:stop])
        st.track_neighbor_overflow = self.track_neighbor_overflow
        return st

    # ------------------------------------------------------------- C world
    def world_c(self, n_envs: int, act_dim: int) -> _lib.WorldC:
        key = (n_envs, act_dim)
        wc = self._wc_cache.get(key)
        if wc is None:
            wc = self._build_world_c(n_envs, act_dim)
            self._wc_cache[key] = wc
        return wc

    def _build_world_c(self, n_envs: int, act_dim: int) -> _lib.WorldC:
        w = self.world
        wc = _lib.WorldC()
        wc.dtype = 0 if self.dtype == torch.float32 else 1
        wc.n_envs = n_envs
        wc.n_agents = self.n_agents
        wc.act_dim = act_dim
        wc.substeps = self.substeps
        wc.dt = self.dt
        wc.collisions = int(self.collisions)
        wc.k = w.collision_k
        wc.c = w.collision_c
        wc.margin = w.collision_margin
        wc.max_overlap = w.contact_max_overlap
        wc.neighbor_radius = self.neighbor_radius
        wc.max_neighbors = w.max_neighbors
        wc.bounds_mode = 1 if self._soft_walls else (2 if self._clamp else 0)
        wc.integrator = 1 if w.integrator == Integrator.RK4 else 0
        wc.box_agents = int(self.box_agents)
        b = w.bounds if w.bounds is not None else (0.0, 0.0, 0.0, 0.0)
        wc.bounds = (C.c_double * 4)(*b)
        wc.lin_damping = w.obstacle_linear_damping
        wc.ang_damping = w.obstacle_angular_damping
        if self.params_per_env is not None:
            if self.params_per_env.shape[0] != n_envs:
                raise ValueError(f"per-env params were installed for {self.params_per_env.shape[0]}"
                                 f" envs, stepping {n_envs}")
            wc.params = self.params_per_env.data_ptr()
            wc.params_env_stride = self.n_agents * NUM_PARAMS
        else:
            wc.params = self.params.data_ptr()
            wc.params_env_stride = 0
        wc.model_tag = self.model_tag.data_ptr()
        wc.ctrl_mode = self.ctrl_mode.data_ptr()
        wc.fleet_models = self.fleet_models
        wc.fleet_modes = self.fleet_modes
        o = self.obstacles
        if o is not None and self.n_obstacles > 0:
            if o.n_envs != n_envs:
                raise ValueError(f"obstacles were installed for {o.n_envs} envs, stepping {n_envs}")
            oc = wc.obstacles
            oc.n_obstacles = self.n_obstacles
            oc.pos, oc.angle = o.pos.data_ptr(), o.angle.data_ptr()
            oc.vel, oc.ang_vel = o.vel.data_ptr(), o.ang_vel.data_ptr()
            oc.radius, oc.half = o.radius.data_ptr(), o.half_extents.data_ptr()
            oc.shape, oc.kind = o.shape.data_ptr(), o.kind.data_ptr()
            oc.mass, oc.inertia = o.mass.data_ptr(), o.inertia.data_ptr()
            oc.body, oc.body_off = o.body.data_ptr(), o.body_offset.data_ptr()
            oc.any_movable = int(self.any_movable)
            oc.bodies_move = int(self.any_movable)
            oc.movable_shapes = self.movable_shapes
            oc.poses_from_bodies = int(self._poses_from_bodies)
        return wc

    def rollout_overflow(self) -> torch.Tensor | None:
        """Bool ``[E, A]``: the agent had more in-radius neighbors than ``max_neighbors``
        on some substep of the last rollout (needs ``track_neighbor_overflow``)."""
        if self.last_true_count_max is None:
            return None
        return self.last_true_count_max > self.world.max_neighbors

    def bodies_snapshot(self):
        """Opaque copy of the movable-body state (body poses/velocities and the placed
        shapes) that :meth:`restore_bodies` reinstates, e.g. to restart an episode."""
        bs = None if self.body_state is None else tuple(t.clone() for t in self.body_state)
        return (self.obstacles, bs, self._poses_from_bodies)

    def restore_bodies(self, snapshot) -> None:
        obstacles, bs, from_bodies = snapshot
        self.obstacles = obstacles
        self.body_state = None if bs is None else tuple(t.clone() for t in bs)
        self._poses_from_bodies = from_bodies
        self._wc_cache.clear()

    def _advance_bodies(self, body_traj) -> None:
        """After a rollout that moved the bodies: the final body state becomes the stepper's,
        and the moving shapes are re-placed on it (as the reference's body pass leaves its
        obstacle arrays). The next rollout places them from the body state itself."""
        bpos, bang, bvel, bom = (x[-1].clone() for x in body_traj)
        self.body_state = (bpos, bang, bvel, bom)
        o = self.obstacles
        root = o.body.long()
        moving = (o.kind[root] != 0).view(1, -1)
        ang = bang[:, root]
        ca, sa = torch.cos(ang), torch.sin(ang)
        offx, offy = o.body_offset[:, 0], o.body_offset[:, 1]
        owx = ca * offx - sa * offy
        owy = sa * offx + ca * offy
        om = bom[:, root]
        pos = torch.stack([bpos[:, root, 0] + owx, bpos[:, root, 1] + owy], -1)
        vel = torch.stack([bvel[:, root, 0] - om * owy, bvel[:, root, 1] + om * owx], -1)
        m2 = moving.unsqueeze(-1)
        new = replace(o, pos=torch.where(m2, pos, o.pos).contiguous(),
                      angle=torch.where(moving, ang, o.angle).contiguous(),
                      vel=torch.where(m2, vel, o.vel).contiguous(),
                      ang_vel=torch.where(moving, om, o.ang_vel).contiguous())
        new._resolved_for = o._resolved_for
        self.obstacles = new
        self._poses_from_bodies = True
        self._wc_cache.clear()

    # -------------------------------------------------------------- launches
    def _check_inputs(self, state, actions: torch.Tensor, horizon_dim: bool):
        exp = 4 if horizon_dim else 3
        if actions.dim() != exp:
            raise ValueError(f"actions must be {exp}-D, got shape {tuple(actions.shape)}")
        if actions.dtype != self.dtype:
            raise TypeError(f"actions dtype {actions.dtype} != stepper dtype {self.dtype}")
        if actions.device != self.device:
            raise ValueError(f"actions on {actions.device}, stepper on {self.device}")
        E = actions.shape[-3]
        if actions.shape[-2] != self.n_agents or actions.shape[-1] < 2:
            raise ValueError(f"actions must be [..., n_envs, {self.n_agents}, act_dim>=2]; got "
                             f"{tuple(actions.shape)}")
        A = self.n_agents
        shapes = [(E, A, 2), (E, A), (E, A, 2), (E, A), (E, A), (E, A), (E, A), (E, A, 4),
                  (E, A, 3)][:self.n_state]
        for t, shp in zip(state, shapes, strict=True):
            if tuple(t.shape) != shp:
                raise ValueError(f"state field of shape {tuple(t.shape)}, expected {shp}")
            if t.dtype != self.dtype or t.device != self.device:
                raise TypeError(f"state field {t.dtype}/{t.device} != stepper "
                                f"{self.dtype}/{self.device}")
        return E

    def workspace_bytes(self, n_envs: int, act_dim: int, horizon: int) -> int:
        lib = _lib.load()
        wc = self.world_c(n_envs, act_dim)
        return int(lib.swarp_rollout_workspace_bytes(C.byref(wc), horizon))

    def rollout_forward(self, state5, actions: torch.Tensor, *, final: bool = True,
                        out=None, true_count: bool = False, moving_bodies: bool = True,
                        goal: torch.Tensor | None = None, loss_out: torch.Tensor | None = None):
        """Run the forward rollout kernel.

        ``state5`` are the ``n_state`` contiguous initial-state tensors (five, or nine with
        the drone fields z, vz, attitude, body_rates when the fleet has drones), ``actions``
        is ``[T, E, A, act_dim]``. Movable bodies (if any) advance when ``moving_bodies``; the
        stepper then carries their final state. Returns ``(traj5, final5 | None,
        true_max | None, record)`` with ``traj5`` stacked ``[T, E, A(,k)]`` and ``record``
        the :class:`RolloutRecord` the adjoint needs. With ``goal`` ``[E, A, 2]`` the kernel
        also reduces the goal loss sum |pos_T - goal|^2 into ``loss_out`` (a 0-d tensor of
        the stepper's dtype).
        """
        lib = _lib.load()
        H, E, _, D = actions.shape
        moving = bool(self.any_movable and moving_bodies)
        wc = self.world_c(E, D)
        if self.n_obstacles > 0:
            wc.obstacles.bodies_move = int(moving)
        opts = {"device": self.device, "dtype": self.dtype}
        if out is None:
            A = self.n_agents
            traj = (torch.empty(H, E, A, 2, **opts), torch.empty(H, E, A, **opts),
                    torch.empty(H, E, A, 2, **opts), torch.empty(H, E, A, **opts),
                    torch.empty(H, E, A, **opts))
            if self.has_drones:
                traj = traj + (torch.empty(H, E, A, **opts), torch.empty(H, E, A, **opts),
                               torch.empty(H, E, A, 4, **opts), torch.empty(H, E, A, 3, **opts))
        else:
            traj = out
        fin = tuple(torch.empty_like(t[0]) for t in traj) if final else None
        true_count = true_count or self.track_neighbor_overflow
        tmax = (torch.empty(E, self.n_agents, dtype=torch.int32, device=self.device)
                if true_count and self.collisions else None)
        self.last_true_count_max = tmax
        nbytes = int(lib.swarp_rollout_workspace_bytes(C.byref(wc), H))
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=self.device)
        bi = bt = None
        if moving:
            N = self.n_obstacles
            bi = self.body_state
            bt = (torch.empty(H, E, N, 2, **opts), torch.empty(H, E, N, **opts),
                  torch.empty(H, E, N, 2, **opts), torch.empty(H, E, N, **opts))
        rec = RolloutRecord(type(wc).from_buffer_copy(wc), ws, self.obstacles, bi, bt, moving)
        rc = lib.swarp_rollout_fwd(
            C.byref(rec.wc), H, _lib.state_c(state5), actions.data_ptr(), _lib.state_c(traj),
            _lib.state_c(fin) if fin else _lib.State(), _lib.ptr(tmax),
            _lib.Bodies(*(_lib.ptr(x) for x in bi)) if bi else _lib.Bodies(),
            _lib.Bodies(*(_lib.ptr(x) for x in bt)) if bt else _lib.Bodies(),
            _lib.GoalLoss(_lib.ptr(goal), _lib.ptr(loss_out), None),
            ws.data_ptr(), nbytes, _lib.stream_ptr(self.device),
        )
        _lib.check(rc, "swarp_rollout_fwd")
        if moving:
            self._advance_bodies(bt)
        return traj, fin, tmax, rec

    def rollout_backward(self, state5, actions, traj5, gtraj5, gfin5, record: RolloutRecord,
                         gbody_final=None, goal: torch.Tensor | None = None,
                         loss_grad: torch.Tensor | None = None):
        """Adjoint of :meth:`rollout_forward` for the same inputs and its ``record``.

        ``gbody_final``: cotangents of the final body state (pos, angle, vel, ang_vel;
        entries may be None). With ``goal``, ``loss_grad`` (a 0-d device tensor, the
        cotangent of the goal loss) seeds that loss's gradient in the kernel. Returns
        ``(grad_actions, grad_init5)``.
        """
        lib = _lib.load()
        g_act = torch.empty_like(actions)
        g_init = tuple(torch.empty_like(t) for t in state5)
        rec = record
        ws = rec.workspace
        gb = _lib.Bodies()
        keep = ()
        if gbody_final is not None:
            keep = tuple(None if x is None else x.contiguous() for x in gbody_final)
            gb = _lib.Bodies(*(_lib.ptr(x) for x in keep))
        sq = None
        if self.track_grad_norm:
            sq = torch.empty((), dtype=self.dtype, device=self.device)
            self.last_grad_sqnorm = sq
        rc = lib.swarp_rollout_bwd(
            C.byref(rec.wc), actions.shape[0], _lib.state_c(state5), actions.data_ptr(),
            _lib.state_c(traj5), _lib.state_c(gtraj5), _lib.state_c(gfin5),
            _lib.Bodies(*(_lib.ptr(x) for x in rec.body_init)) if rec.body_init else _lib.Bodies(),
            _lib.Bodies(*(_lib.ptr(x) for x in rec.body_traj)) if rec.body_traj else _lib.Bodies(),
            gb, g_act.data_ptr(), _lib.state_c(g_init), _lib.ptr(sq),
            _lib.GoalLoss(_lib.ptr(goal), None, _lib.ptr(loss_grad)), ws.data_ptr(), ws.numel(),
            _lib.stream_ptr(self.device),
        )
        _lib.check(rc, "swarp_rollout_bwd")
        del keep
        return g_act, g_init

    def neighbors(self, pos: torch.Tensor):
        """Padded within-radius lists of ``pos [E, A, 2]``: ``(idx, count, true_count)``."""
        if not self.collisions:
            raise RuntimeError("neighbor lists require WorldConfig.collisions=True")
        lib = _lib.load()
        E = pos.shape[0]
        wc = self.world_c(E, 2)
        K = self.world.max_neighbors
        idx = torch.zeros(E, self.n_agents, K, dtype=torch.int32, device=self.device)
        cnt = torch.empty(E, self.n_agents, dtype=torch.int32, device=self.device)
        tru = torch.empty_like(cnt)
        pos = pos.detach().contiguous()
        rc = lib.swarp_neighbors(C.byref(wc), pos.data_ptr(), idx.data_ptr(), cnt.data_ptr(),
                                 tru.data_ptr(), _lib.stream_ptr(self.device))
        _lib.check(rc, "swarp_neighbors")
        return idx, cnt, tru
