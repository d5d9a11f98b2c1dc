"""Build the CPU oracle's world description from a product Stepper (test helper)."""

from __future__ import annotations

import torch

from oracle import torch_ref as R
from swarp_b200.dynamics.base import Integrator

D = torch.float64


def ref_world(stepper, n_envs: int | None = None) -> R.RefWorld:
    w = stepper.world
    params = stepper.params_per_env if stepper.params_per_env is not None else stepper.params
    return R.RefWorld(
        params=params.detach().to("cpu", D),
        model_tag=[int(c.model) for c in stepper.configs],
        ctrl_mode=[int(c.ctrl_mode) for c in stepper.configs],
        dt=stepper.dt,
        substeps=stepper.substeps,
        collisions=stepper.collisions,
        k=w.collision_k,
        c=w.collision_c,
        margin=w.collision_margin,
        max_overlap=w.contact_max_overlap,
        neighbor_radius=stepper.neighbor_radius,
        max_neighbors=w.max_neighbors,
        bounds=w.bounds,
        soft_walls=stepper._soft_walls,
        clamp_bounds=stepper._clamp,
        lin_damping=w.obstacle_linear_damping,
        ang_damping=w.obstacle_angular_damping,
        rk4=w.integrator == Integrator.RK4,
    )


def ref_obstacles(stepper) -> R.RefObstacles | None:
    o = stepper.obstacles
    if o is None or stepper.n_obstacles == 0:
        return None
    cpu = lambda t: t.detach().to("cpu", D)  # noqa: E731
    obs = R.RefObstacles(
        pos=cpu(o.pos), angle=cpu(o.angle), vel=cpu(o.vel), ang_vel=cpu(o.ang_vel),
        radius=cpu(o.radius), half=cpu(o.half_extents), shape=o.shape.cpu().tolist(),
        kind=o.kind.cpu().tolist(), mass=cpu(o.mass), inertia=cpu(o.inertia),
        body=o.body.cpu().tolist(), body_off=cpu(o.body_offset),
    )
    return R.seed_bodies(obs)


def to_ref(t):
    return t.detach().to("cpu", D)
