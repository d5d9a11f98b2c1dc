"""World configuration and the batched obstacle description.

Field names, defaults and validation mirror the reference
(``swarp/core/config.py``: ``ObstacleShape`` ``:118-127``, ``ObstacleKind``
``:130-141``, ``Obstacles`` ``:144-283``, ``WorldConfig`` ``:286-427``) because they
are the public configuration surface scenarios pass in. Options that select paths
this package does not run on the GPU (``wheel_contacts``, floor friction, the
``grid``/``uniform_grid`` neighbor backends) are accepted
for compatibility and rejected by :class:`~swarp_b200.core.stepper.Stepper` when
they would change the physics.
"""

from __future__ import annotations

from dataclasses import dataclass, field, fields, replace
from enum import IntEnum

import torch

from swarp_b200.dynamics.base import Integrator


class ObstacleShape(IntEnum):
    CIRCLE = 0
    BOX = 1
    SEGMENT = 2


class ObstacleKind(IntEnum):
    IMMOVABLE = 0
    MOVABLE = 1


@dataclass
class Obstacles:
    """One batched obstacle set (``E`` envs, ``N`` shapes).

    ``pos [E,N,2]`` and ``radius [N]`` are required; ``shape [N]``, ``angle [N]`` or
    ``[E,N]``, ``half_extents [N,2]``, ``vel [E,N,2]``, ``ang_vel [E,N]``, ``kind [N]``,
    ``mass [N]``, ``inertia [N]``, ``body [N]`` (index of each shape's body root) and
    ``body_offset [N,2]`` are optional, ``None`` meaning the documented default
    (circle, 0, 0, 0, 0, immovable, 1, 1, own root, 0).
    """

    pos: torch.Tensor
    radius: torch.Tensor
    shape: torch.Tensor | None = None
    angle: torch.Tensor | None = None
    half_extents: torch.Tensor | None = None
    vel: torch.Tensor | None = None
    ang_vel: torch.Tensor | None = None
    kind: torch.Tensor | None = None
    mass: torch.Tensor | None = None
    inertia: torch.Tensor | None = None
    body: torch.Tensor | None = None
    body_offset: torch.Tensor | None = None
    _resolved_for: tuple | None = field(default=None, init=False, repr=False, compare=False)

    def __post_init__(self) -> None:
        if self.pos.dim() != 3 or self.pos.shape[-1] != 2:
            raise ValueError(f"obstacle pos must be [n_envs, n_obstacles, 2]; got {self.pos.shape}")
        n = self.pos.shape[1]
        if self.radius.dim() != 1 or self.radius.shape[0] != n:
            raise ValueError(
                f"obstacle radius must be [n_obstacles={n}]; got {tuple(self.radius.shape)}"
            )
        if self.angle is not None and self.angle.dim() not in (1, 2):
            raise ValueError(
                "obstacle angle must be [n_obstacles] or [n_envs, n_obstacles]; got "
                f"{tuple(self.angle.shape)}"
            )

    @property
    def n_envs(self) -> int:
        return self.pos.shape[0]

    @property
    def n_obstacles(self) -> int:
        return self.pos.shape[1]

    def env_slice(self, start: int, stop: int) -> Obstacles:
        """The set of envs ``[start, stop)``: per-env fields sliced (views), per-shape
        constants shared."""
        def cut(t):
            return t if t is None or t.dim() < 2 else t[start:stop]

        angle = self.angle if self.angle is None or self.angle.dim() == 1 else self.angle[start:stop]
        return Obstacles(pos=self.pos[start:stop], radius=self.radius, shape=self.shape,
                         angle=angle, half_extents=self.half_extents, vel=cut(self.vel),
                         ang_vel=cut(self.ang_vel), kind=self.kind, mass=self.mass,
                         inertia=self.inertia, body=self.body, body_offset=self.body_offset)

    def resolve(self, device, dtype: torch.dtype) -> Obstacles:
        """Every field materialised, contiguous, on ``device`` in ``dtype`` (int32 tags)."""
        key = (str(device), dtype)
        if self._resolved_for == key:
            return self
        E, N = self.n_envs, self.n_obstacles

        def f(t, shape, fill=0.0):
            if t is None:
                return torch.full(shape, fill, device=device, dtype=dtype)
            return t.detach().to(device=device, dtype=dtype).contiguous()

        def i(t, default):
            if t is None:
                return default.to(device=device, dtype=torch.int32)
            return t.detach().to(device=device, dtype=torch.int32).contiguous()

        angle = f(self.angle, (E, N))
        if angle.dim() == 1:
            angle = angle.unsqueeze(0).expand(E, -1).contiguous()
        out = Obstacles(
            pos=f(self.pos, (E, N, 2)),
            radius=f(self.radius, (N,)),
            shape=i(self.shape, torch.zeros(N)),
            angle=angle,
            half_extents=f(self.half_extents, (N, 2)),
            vel=f(self.vel, (E, N, 2)),
            ang_vel=f(self.ang_vel, (E, N)),
            kind=i(self.kind, torch.zeros(N)),
            mass=f(self.mass, (N,), 1.0),
            inertia=f(self.inertia, (N,), 1.0),
            body=i(self.body, torch.arange(N)),
            body_offset=f(self.body_offset, (N, 2)),
        )
        out._resolved_for = key
        return out

    @property
    def any_movable(self) -> bool:
        return self.kind is not None and bool((self.kind != 0).any().item())


@dataclass
class WorldConfig:
    """Interaction and boundary settings shared by all envs (reference defaults)."""

    collisions: bool = True
    collision_k: float = 100.0
    collision_c: float = 1.0
    collision_margin: float = 0.02
    obstacle_linear_damping: float = 10.0
    obstacle_angular_damping: float = 10.0
    obstacle_friction: float = 0.0
    gravity: float = 9.81
    wheel_contacts: bool = False
    wheel_lateral_friction: float = 0.2
    wheel_turn_torque: float = 0.0
    obstacle_friction_speed: float = 0.005
    obstacle_friction_grid: int = 6
    contact_max_overlap: float = 0.0
    bounds: tuple[float, float, float, float] | None = None
    bounds_mode: str = "soft"
    neighbor_radius: float | None = None
    max_neighbors: int = 32
    neighbor_method: str = "auto"
    grid_dim: int = 128
    uniform_bins: int | None = None
    integrator: Integrator = Integrator.EULER
    neighbor_reuse: bool = True

    def override_with(self, other: WorldConfig | None) -> WorldConfig:
        """This config with ``other``'s non-default fields applied on top."""
        if other is None:
            return self
        default = WorldConfig()
        changed = {
            f.name: getattr(other, f.name)
            for f in fields(self)
            if getattr(other, f.name) != getattr(default, f.name)
        }
        return replace(self, **changed) if changed else self

    def __post_init__(self) -> None:
        if self.bounds_mode not in ("soft", "clamp"):
            raise ValueError('bounds_mode must be "soft" or "clamp"')
        if self.bounds is not None:
            x_min, x_max, y_min, y_max = self.bounds
            if x_min >= x_max or y_min >= y_max:
                raise ValueError("bounds must satisfy x_min < x_max and y_min < y_max")
        if self.collision_k < 0.0 or self.collision_c < 0.0 or self.collision_margin < 0.0:
            raise ValueError("collision constants must be non-negative")
        if self.obstacle_friction < 0.0 or self.obstacle_friction_speed <= 0.0:
            raise ValueError("obstacle_friction must be >= 0 and obstacle_friction_speed > 0")
        if self.wheel_lateral_friction < 0.0 or self.wheel_turn_torque < 0.0:
            raise ValueError("wheel_lateral_friction and wheel_turn_torque must be >= 0")
        if self.obstacle_friction_grid < 1:
            raise ValueError("obstacle_friction_grid must be >= 1")
        if self.obstacle_linear_damping < 0.0 or self.obstacle_angular_damping < 0.0:
            raise ValueError("obstacle damping must be non-negative")
        if self.contact_max_overlap < 0.0:
            raise ValueError("contact_max_overlap must be non-negative (0 disables)")
