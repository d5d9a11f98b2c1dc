"""swarp_b200 — B200-native differentiable batched multi-robot physics step.

A drop-in for the step / BPTT path of ddebenedittis/swarp: ``make`` builds an
:class:`Environment`; :func:`warp_step` and :func:`rollout` are the differentiable step
and backprop-through-time rollout over a :class:`Stepper`. The compute runs in
hand-written sm_100a CUDA kernels behind a C ABI (include/swarp_b200.h); importing this
package needs no GPU, stepping does.

    import swarp_b200 as swarp
    env = swarp.make("navigation", n_envs=4096, n_agents=8, device="cuda:0")
"""

from __future__ import annotations

import difflib
import inspect

from swarp_b200.core.config import ObstacleKind, Obstacles, ObstacleShape, WorldConfig
from swarp_b200.core.environment import Environment
from swarp_b200.core.stepper import Stepper
from swarp_b200.core.world import World
from swarp_b200.dynamics.base import (
    NUM_PARAMS,
    P_HALF_X,
    P_HALF_Y,
    P_LF,
    P_LR,
    P_MASS,
    P_MAX_ACCEL,
    P_MAX_ANG_ACCEL,
    P_MAX_ANG_VEL,
    P_MAX_SPEED,
    P_MAX_STEER,
    P_MIN_SPEED,
    P_RADIUS,
    P_SHAPE,
    PARAM_FIELDS,
    AgentConfig,
    AgentShape,
    ControlMode,
    DynamicsModel,
    Integrator,
    action_bounds,
    per_env_float_template,
)
from swarp_b200.interop.autograd import (
    BodyState,
    GradRing,
    TorchState,
    rollout,
    rollout_bodies,
    rollout_checkpointed,
    warp_step,
)
from swarp_b200.core.sharding import PairReducer, env_shard, reduce_loss_and_grad_norm
from swarp_b200.interop.compile import compiled_warp_step, register_stepper
from swarp_b200.interop.graphs import GraphedRollout
from swarp_b200.scenarios import SCENARIOS, NavigationScenario, make_scenario, scenario_class

__version__ = "0.1.0"

_ENV_KWARGS = frozenset(inspect.signature(Environment.__init__).parameters) - {
    "self", "scenario", "n_envs",
}


def make(name: str, n_envs: int, **kwargs) -> Environment:
    """Build an :class:`Environment` for a registered scenario (reference
    ``swarp/__init__.py:95-121``): Environment keywords go to the environment, every
    other keyword to the scenario constructor; an unknown keyword is a ``TypeError``."""
    env_kwargs = {k: v for k, v in kwargs.items() if k in _ENV_KWARGS}
    scen_kwargs = {k: v for k, v in kwargs.items() if k not in _ENV_KWARGS}
    params = inspect.signature(scenario_class(name).__init__).parameters
    valid = sorted(set(params) - {"self"})
    for key in scen_kwargs:
        if key not in valid:
            msg = (f"{key!r} is not a keyword of scenario {name!r} or of Environment. "
                   f"Scenario keywords: {', '.join(valid)}.")
            close = difflib.get_close_matches(key, _ENV_KWARGS, n=1)
            if close:
                msg += f" Did you mean Environment's {close[0]!r}?"
            raise TypeError(msg)
    return Environment(make_scenario(name, **scen_kwargs), n_envs=n_envs, **env_kwargs)


__all__ = [
    "AgentConfig", "AgentShape", "BodyState", "ControlMode", "DynamicsModel", "Environment",
    "GradRing", "GraphedRollout", "PairReducer", "compiled_warp_step", "env_shard",
    "reduce_loss_and_grad_norm", "register_stepper", "Integrator", "NUM_PARAMS", "NavigationScenario", "ObstacleKind", "ObstacleShape",
    "Obstacles", "PARAM_FIELDS", "P_HALF_X", "P_HALF_Y", "P_LF", "P_LR", "P_MASS", "P_MAX_ACCEL",
    "P_MAX_ANG_ACCEL", "P_MAX_ANG_VEL", "P_MAX_SPEED", "P_MAX_STEER", "P_MIN_SPEED", "P_RADIUS",
    "P_SHAPE", "SCENARIOS", "Stepper", "TorchState", "World", "WorldConfig", "action_bounds",
    "make", "make_scenario", "per_env_float_template", "rollout", "rollout_bodies", "rollout_checkpointed",
    "scenario_class", "warp_step", "__version__",
]
