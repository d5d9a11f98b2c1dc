"""Golden-fixture case specs and their builders (test infrastructure).

Each case is a small seeded rollout described in plain JSON-able terms (agent configs,
world constants, obstacles). ``make_golden.py`` runs it through the float64 CPU oracle
(oracle/torch_ref.py, itself pinned by the reference's known-answer tests) and stores
inputs, trajectories and gradients under tests/golden/*.npz; the tests replay the same
inputs through the CUDA path and compare.
"""

from __future__ import annotations

import json
import math
import os

import numpy as np
import torch

from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel, param_rows

HERE = os.path.dirname(os.path.abspath(__file__))
D = torch.float64


def _body3(E, seed, mass=2.0):
    """One movable body of three circles on a line, placed at a seeded pose per env."""
    g = np.random.default_rng(seed)
    r, d = 0.08, 0.12
    ang = g.uniform(-0.5, 0.5, E)
    cen = g.uniform(-0.1, 0.1, (E, 2))
    off = np.array([[-d, 0.0], [0.0, 0.0], [d, 0.0]])
    ca, sa = np.cos(ang)[:, None], np.sin(ang)[:, None]
    pos = np.stack([cen[:, None, 0] + ca * off[:, 0] - sa * off[:, 1],
                    cen[:, None, 1] + sa * off[:, 0] + ca * off[:, 1]], -1)
    return {"pos": pos.tolist(), "radius": [r] * 3, "shape": [0, 0, 0],
            "angle": np.repeat(ang[:, None], 3, 1).tolist(), "kind": [1, 1, 1],
            "mass": [mass] * 3, "inertia": [mass * (0.5 * r * r + 2 * d * d / 3)] * 3,
            "body": [0, 0, 0], "body_offset": off.tolist(), "half_extents": [[0.0, 0.0]] * 3}


def _scenery(E, seed):
    """A circle, a box and a segment, per-env poses (immovable)."""
    g = np.random.default_rng(seed)
    return {"pos": g.uniform(-0.35, 0.35, (E, 3, 2)).tolist(), "radius": [0.08, 0.0, 0.02],
            "shape": [0, 1, 2], "angle": g.uniform(0, math.pi, (E, 3)).tolist(),
            "half_extents": [[0.0, 0.0], [0.09, 0.05], [0.12, 0.0]],
            "vel": (0.1 * g.standard_normal((E, 3, 2))).tolist(),
            "ang_vel": (0.2 * g.standard_normal((E, 3))).tolist()}


CASES = {
    "holonomic_velocity_contacts_walls": dict(
        E=3, T=8, seed=11, spread=0.45,
        agents=[dict(model="HOLONOMIC", ctrl_mode="VELOCITY", radius=0.05, max_speed=1.0,
                     max_accel=2.0)] * 6,
        world=dict(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                   neighbor_radius=0.3, max_neighbors=6, bounds=[-0.5, 0.5, -0.5, 0.5],
                   bounds_mode="soft")),
    "diff_drive_acceleration_obstacles": dict(
        E=2, T=8, seed=12, spread=0.4,
        agents=[dict(model="DIFF_DRIVE", ctrl_mode="ACCELERATION", radius=0.06, max_speed=0.8,
                     max_accel=1.5, max_ang_vel=2.0, max_ang_accel=4.0)] * 5,
        world=dict(collision_k=80.0, collision_c=2.0, collision_margin=0.02,
                   neighbor_radius=0.25, max_neighbors=5, bounds=[-0.5, 0.5, -0.5, 0.5],
                   bounds_mode="soft"),
        obstacles="scenery"),
    "bicycle_substeps_clamped": dict(
        E=2, T=6, seed=13, spread=0.3, substeps=3,
        agents=[dict(model="KINEMATIC_BICYCLE", ctrl_mode="VELOCITY", radius=0.05,
                     max_speed=1.2, max_accel=2.0, l_f=0.08, l_r=0.12, max_steer=0.6)] * 4,
        world=dict(collision_k=120.0, collision_c=1.0, collision_margin=0.02,
                   neighbor_radius=0.2, max_neighbors=4, bounds=[-0.35, 0.35, -0.35, 0.35],
                   bounds_mode="clamp")),
    "mixed_fleet_servo_truncated_lists": dict(
        E=2, T=6, seed=14, spread=0.25,
        agents=[dict(model="HOLONOMIC", ctrl_mode="ACCELERATION", radius=0.05, max_accel=2.0),
                dict(model="DIFF_DRIVE", ctrl_mode="SERVO", radius=0.05, max_speed=1.0),
                dict(model="KINEMATIC_BICYCLE", ctrl_mode="VELOCITY", radius=0.05),
                dict(model="DIFF_DRIVE", ctrl_mode="VELOCITY", radius=0.04)] * 3,
        world=dict(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                   neighbor_radius=0.4, max_neighbors=3, bounds=[-0.4, 0.4, -0.4, 0.4],
                   bounds_mode="soft", contact_max_overlap=0.03)),
    "movable_compound_body": dict(
        E=2, T=10, seed=15, spread=0.3, bodies_in_grad=True,
        agents=[dict(model="HOLONOMIC", ctrl_mode="VELOCITY", radius=0.05, max_speed=1.0,
                     max_accel=2.0)] * 3,
        world=dict(collision_k=100.0, collision_c=5.0, collision_margin=0.025,
                   neighbor_radius=0.125, max_neighbors=3, bounds=[-0.6, 0.6, -0.6, 0.6],
                   bounds_mode="soft"),
        obstacles="body3"),
}


def agent_configs(spec):
    out = []
    for a in spec["agents"]:
        a = dict(a)
        out.append(AgentConfig(model=DynamicsModel[a.pop("model")],
                               ctrl_mode=ControlMode[a.pop("ctrl_mode")], **a))
    return out


def world_config(spec):
    w = dict(spec["world"])
    w["bounds"] = tuple(w["bounds"])
    return WorldConfig(**w)


def obstacle_spec(spec):
    kind = spec.get("obstacles")
    if kind is None:
        return None
    return _scenery(spec["E"], spec["seed"] + 100) if kind == "scenery" else _body3(
        spec["E"], spec["seed"] + 100)


def obstacles(ospec, dtype=D):
    if ospec is None:
        return None
    f = {k: torch.tensor(v, dtype=dtype) for k, v in ospec.items()
         if k not in ("shape", "kind", "body")}
    i = {k: torch.tensor(v, dtype=torch.int32) for k, v in ospec.items()
         if k in ("shape", "kind", "body")}
    return Obstacles(**f, **i)


def inputs(spec):
    """Seeded initial state (five fields) and actions, float64 numpy."""
    E, T, A = spec["E"], spec["T"], len(spec["agents"])
    g = np.random.default_rng(spec["seed"])
    s = spec["spread"]
    pos = g.uniform(-s, s, (E, A, 2))
    th = g.uniform(-math.pi, math.pi, (E, A))
    vel = 0.3 * g.standard_normal((E, A, 2))
    sp = 0.3 * g.standard_normal((E, A))
    om = 0.3 * g.standard_normal((E, A))
    acts = g.uniform(-1.5, 1.5, (T, E, A, 2))
    w_fin = g.standard_normal((E, A, 2))      # loss weights: final positions
    w_traj = g.standard_normal((T, E, A))     # loss weights: trajectory headings
    w_body = g.standard_normal((E, 2))        # loss weights: final body position (slot 0)
    return [pos, th, vel, sp, om], acts, w_fin, w_traj, w_body


def oracle_world(spec):
    """The float64 oracle world for a case (the Stepper's derivations, restated)."""
    from oracle import torch_ref as R

    cfgs = agent_configs(spec)
    w = world_config(spec)
    reach = 2.0 * max(c.radius for c in cfgs) + w.collision_margin
    return R.RefWorld(
        params=torch.tensor(param_rows(cfgs), dtype=D), model_tag=[int(c.model) for c in cfgs],
        ctrl_mode=[int(c.ctrl_mode) for c in cfgs], dt=0.05, substeps=spec.get("substeps", 1),
        collisions=w.collisions, k=w.collision_k, c=w.collision_c, margin=w.collision_margin,
        max_overlap=w.contact_max_overlap, neighbor_radius=w.neighbor_radius or reach,
        max_neighbors=w.max_neighbors, bounds=w.bounds, soft_walls=w.bounds_mode == "soft",
        clamp_bounds=w.bounds_mode == "clamp", lin_damping=w.obstacle_linear_damping,
        ang_damping=w.obstacle_angular_damping, bodies_move=True)


def oracle_obstacles(ospec):
    from oracle import torch_ref as R

    o = obstacles(ospec)
    if o is None:
        return None
    r = o.resolve("cpu", D)
    ob = R.RefObstacles(pos=r.pos, angle=r.angle, vel=r.vel, ang_vel=r.ang_vel, radius=r.radius,
                        half=r.half_extents, shape=r.shape.tolist(), kind=r.kind.tolist(),
                        mass=r.mass, inertia=r.inertia, body=r.body.tolist(),
                        body_off=r.body_offset)
    return R.seed_bodies(ob)


def run_oracle(spec):
    """Oracle rollout and the gradient of the case's loss; returns the fixture dict."""
    from oracle import torch_ref as R

    init, acts, w_fin, w_traj, w_body = inputs(spec)
    ospec = obstacle_spec(spec)
    st = [torch.tensor(x, dtype=D, requires_grad=True) for x in init]
    a = torch.tensor(acts, dtype=D, requires_grad=True)
    fin, traj, body_traj = R.rollout(tuple(st), a, oracle_world(spec), oracle_obstacles(ospec))
    th_traj = torch.stack([s[1] for s in traj])
    loss = (fin[0] * torch.tensor(w_fin)).sum() + (th_traj * torch.tensor(w_traj)).sum()
    moving = ospec is not None and any(k != 0 for k in ospec.get("kind", []))
    if moving:
        loss = loss + (body_traj[-1].body_pos[:, 0] * torch.tensor(w_body)).sum()
    grads = torch.autograd.grad(loss, [a, *st])
    out = {"spec": np.array(json.dumps(spec)), "acts": acts, "w_fin": w_fin, "w_traj": w_traj,
           "w_body": w_body, "loss": np.array(float(loss.detach())), "grad_acts": grads[0].numpy()}
    for i, name in enumerate(("pos", "theta", "vel", "speed", "ang_vel")):
        out[f"init_{name}"] = init[i]
        out[f"traj_{name}"] = torch.stack([s[i] for s in traj]).detach().numpy()
        out[f"grad_init_{name}"] = grads[1 + i].numpy()
    if moving:
        out["body_pos_final"] = body_traj[-1].body_pos.detach().numpy()
        out["body_angle_final"] = body_traj[-1].body_angle.detach().numpy()
    return out


def load(name):
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    d["spec"] = json.loads(str(d["spec"]))
    return d
