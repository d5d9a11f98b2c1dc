"""Agent models, control modes and the packed per-agent parameter rows.

Interface parity with the reference: ``swarp/dynamics/base.py`` (``DynamicsModel``
``:13-19``, ``ControlMode`` ``:61-79``, ``AgentShape`` ``:82-94``, ``Integrator``
``:97-101``, ``PARAM_FIELDS`` ``:114-169``, ``AgentConfig`` ``:172-286``,
``action_bounds`` ``:310-331``). The enum values and the column order of the
parameter row are a data format shared with the reference (scenarios build per-env
parameter tensors by column index), so they are kept identical; everything else is
written for this package.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from enum import Enum, IntEnum

import numpy as np


class DynamicsModel(IntEnum):
    """Motion model tag, stored per agent and read by the integrate phase."""

    HOLONOMIC = 0
    DIFF_DRIVE = 1
    KINEMATIC_BICYCLE = 2
    DRONE = 3


class ControlMode(IntEnum):
    """How the first two action slots are read (see the integrate phase)."""

    VELOCITY = 0
    ACCELERATION = 1
    SERVO = 2


class AgentShape(IntEnum):
    """Agent footprint tag: a disc of ``radius`` or an oriented box of half extents
    ``half_extents`` (both run on the CUDA path)."""

    DISC = 0
    BOX = 1


class Integrator(Enum):
    """Time integrator of every substep: semi-implicit ``EULER`` or classic ``RK4`` (both
    run on the CUDA path)."""

    EULER = "euler"
    RK4 = "rk4"


#: Action arity of each model; the env-level action width is the fleet maximum.
MODEL_ACTION_DIM = {"HOLONOMIC": 2, "DIFF_DRIVE": 2, "KINEMATIC_BICYCLE": 2, "DRONE": 4}


def _coerce(enum_cls, val, argname: str):
    """Accept an enum member, its (case/dash-insensitive) name, or its value."""
    if isinstance(val, enum_cls):
        return val
    if isinstance(val, str):
        key = val.strip().upper().replace("-", "_")
        try:
            return enum_cls[key]
        except KeyError:
            valid = ", ".join(m.name.lower() for m in enum_cls)
            raise ValueError(f"unknown {argname} {val!r}; valid names are {valid}") from None
    return enum_cls(val)


def action_dim(model) -> int:
    """Number of action slots ``model`` reads."""
    return MODEL_ACTION_DIM[_coerce(DynamicsModel, model, "model").name]


#: Column layout of the ``[n_agents, NUM_PARAMS]`` parameter matrix (same order as
#: the reference, so per-env parameter tensors built for it index identically).
PARAM_FIELDS: tuple[str, ...] = (
    "radius",
    "mass",
    "max_speed",
    "max_accel",
    "max_ang_vel",
    "max_ang_accel",
    "l_f",
    "l_r",
    "max_steer",
    "thrust_max",
    "arm_length",
    "inertia_xx",
    "inertia_yy",
    "inertia_zz",
    "torque_coeff",
    "gravity",
    "min_speed",
    "shape",
    "half_x",
    "half_y",
    "cmd_gain_v",
    "cmd_gain_w",
)
NUM_PARAMS = len(PARAM_FIELDS)
_COL = {name: i for i, name in enumerate(PARAM_FIELDS)}
P_RADIUS = _COL["radius"]
P_MASS = _COL["mass"]
P_MAX_SPEED = _COL["max_speed"]
P_MAX_ACCEL = _COL["max_accel"]
P_MAX_ANG_VEL = _COL["max_ang_vel"]
P_MAX_ANG_ACCEL = _COL["max_ang_accel"]
P_LF = _COL["l_f"]
P_LR = _COL["l_r"]
P_MAX_STEER = _COL["max_steer"]
P_THRUST_MAX = _COL["thrust_max"]
P_ARM = _COL["arm_length"]
P_IXX = _COL["inertia_xx"]
P_IYY = _COL["inertia_yy"]
P_IZZ = _COL["inertia_zz"]
P_KAPPA = _COL["torque_coeff"]
P_GRAVITY = _COL["gravity"]
P_MIN_SPEED = _COL["min_speed"]
P_SHAPE = _COL["shape"]
P_HALF_X = _COL["half_x"]
P_HALF_Y = _COL["half_y"]
P_CMD_GAIN_V = _COL["cmd_gain_v"]
P_CMD_GAIN_W = _COL["cmd_gain_w"]


@dataclass
class AgentConfig:
    """Static definition of one agent: model, control mode, footprint and limits.

    Defaults and validation follow the reference dataclass
    (``swarp/dynamics/base.py:172-286``): a disc's radius defaults to 0.05, a box's
    radius is its circumscribed one, limits must be positive, ``SERVO`` is a
    diff-drive mode and ``min_speed`` (bicycle) defaults to ``-max_speed``.
    """

    model: DynamicsModel | str | int = DynamicsModel.HOLONOMIC
    ctrl_mode: ControlMode | str | int = ControlMode.VELOCITY
    radius: float | None = None
    mass: float = 1.0
    max_speed: float = 1.0
    max_accel: float = 1.0
    max_ang_vel: float = math.pi
    max_ang_accel: float = 2.0 * math.pi
    l_f: float = 0.1
    l_r: float = 0.1
    max_steer: float = math.pi / 4
    min_speed: float | None = None
    thrust_max: float = 10.0
    arm_length: float = 0.15
    inertia_xx: float = 0.01
    inertia_yy: float = 0.01
    inertia_zz: float = 0.02
    torque_coeff: float = 0.02
    gravity: float = 9.81
    shape: AgentShape | str | int = AgentShape.DISC
    half_extents: tuple[float, float] = (0.0, 0.0)
    cmd_gain_v: float = 1.0
    cmd_gain_w: float = 1.0

    def __post_init__(self) -> None:
        self.model = _coerce(DynamicsModel, self.model, "model")
        self.ctrl_mode = _coerce(ControlMode, self.ctrl_mode, "ctrl_mode")
        self.shape = _coerce(AgentShape, self.shape, "shape")
        self.half_extents = tuple(float(h) for h in self.half_extents)
        if len(self.half_extents) != 2:
            raise ValueError("AgentConfig.half_extents must be a pair (hx, hy).")
        if self.shape == AgentShape.BOX:
            hx, hy = self.half_extents
            if hx <= 0.0 or hy <= 0.0:
                raise ValueError("A box agent needs positive half_extents (hx, hy).")
            if self.model == DynamicsModel.DRONE:
                raise ValueError("A drone cannot be a box agent; its footprint is a disc.")
            circ = math.hypot(hx, hy)
            if self.radius is not None and not math.isclose(
                self.radius, circ, rel_tol=1e-9, abs_tol=1e-12
            ):
                raise ValueError(
                    f"A box agent's radius is derived from its half_extents ({circ}); "
                    f"got radius={self.radius}. Leave radius unset (None)."
                )
            self.radius = circ
        else:
            if self.half_extents != (0.0, 0.0):
                raise ValueError(
                    "AgentConfig.half_extents is only meaningful for shape=AgentShape.BOX."
                )
            if self.radius is None:
                self.radius = 0.05
        if self.l_f + self.l_r <= 0.0:
            raise ValueError("Bicycle wheelbase l_f + l_r must be positive.")
        for name in (
            "radius", "mass", "max_speed", "max_accel", "max_ang_vel", "max_ang_accel",
            "cmd_gain_v", "cmd_gain_w",
        ):
            if getattr(self, name) <= 0.0:
                raise ValueError(f"AgentConfig.{name} must be positive.")
        if self.ctrl_mode == ControlMode.SERVO and self.model != DynamicsModel.DIFF_DRIVE:
            raise ValueError(
                f"ControlMode.SERVO is a diff-drive mode; got model {self.model.name}."
            )
        if self.min_speed is not None and not -self.max_speed <= self.min_speed <= self.max_speed:
            raise ValueError("AgentConfig.min_speed must lie in [-max_speed, max_speed].")

    @property
    def half_x(self) -> float:
        return self.half_extents[0]

    @property
    def half_y(self) -> float:
        return self.half_extents[1]

    def to_row(self) -> list[float]:
        """This config as one parameter row in ``PARAM_FIELDS`` order."""
        row = {name: getattr(self, name) for name in PARAM_FIELDS}
        if row["min_speed"] is None:
            row["min_speed"] = -self.max_speed
        return [float(row[name]) for name in PARAM_FIELDS]


#: Limit field clamped against per action slot, per (model, mode); ``None`` low is the
#: negated high. Same table as the reference (``swarp/dynamics/base.py:289-307``).
_ACTION_LIMITS = {
    ("HOLONOMIC", "VELOCITY"): ((None, "max_speed"), (None, "max_speed")),
    ("HOLONOMIC", "ACCELERATION"): ((None, "max_accel"), (None, "max_accel")),
    ("DIFF_DRIVE", "VELOCITY"): ((None, "max_speed"), (None, "max_ang_vel")),
    ("DIFF_DRIVE", "ACCELERATION"): ((None, "max_accel"), (None, "max_ang_accel")),
    ("DIFF_DRIVE", "SERVO"): ((None, "max_speed"), (None, "max_ang_vel")),
    ("KINEMATIC_BICYCLE", "VELOCITY"): ((None, "max_accel"), (None, "max_steer")),
    ("KINEMATIC_BICYCLE", "ACCELERATION"): ((None, "max_accel"), (None, "max_steer")),
    ("DRONE", "VELOCITY"): ((0.0, "thrust_max"),) * 4,
    ("DRONE", "ACCELERATION"): ((0.0, "thrust_max"),) * 4,
}


def action_bounds(cfg: AgentConfig) -> tuple[list[float], list[float]]:
    """Per-slot physical action box ``(low, high)`` the integrate phase clamps to."""
    key = (DynamicsModel(cfg.model).name, ControlMode(cfg.ctrl_mode).name)
    slots = _ACTION_LIMITS[key]
    high = [getattr(cfg, field) for _, field in slots]
    low = [-h if lo is None else lo for (lo, _), h in zip(slots, high, strict=True)]
    return low, high


def param_rows(configs: list[AgentConfig]) -> np.ndarray:
    """``[n_agents, NUM_PARAMS]`` float64 rows for ``configs``."""
    return np.array([c.to_row() for c in configs], dtype=np.float64)


def per_env_float_template(configs: list[AgentConfig], n_envs: int) -> np.ndarray:
    """``[n_envs, n_agents, NUM_PARAMS]`` float64 rows, every env a copy of ``configs``."""
    rows = param_rows(configs)
    return np.broadcast_to(rows, (n_envs, *rows.shape)).copy()
