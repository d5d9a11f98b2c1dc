"""Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py from the
float64 oracle): the oracle and the C restatement reproduce them on CPU; the CUDA path
matches them in float64 (1e-10) and, from float32 inputs, within float32 tolerances."""

import numpy as np
import pytest
import torch

from golden.cases import CASES, agent_configs, load, obstacle_spec, obstacles, run_oracle
from golden.cases import world_config

NAMES = sorted(CASES)
FIELDS = ("pos", "theta", "vel", "speed", "ang_vel")


@pytest.mark.parametrize("name", NAMES)
def test_oracle_reproduces_golden(name):
    gold = load(name)
    assert gold["spec"] == CASES[name]
    out = run_oracle(CASES[name])
    for k in gold:
        if k == "spec":
            continue
        np.testing.assert_allclose(out[k], gold[k], rtol=1e-12, atol=1e-14, err_msg=k)


@pytest.mark.parametrize("name", [n for n in NAMES if CASES[n].get("obstacles") != "body3"])
def test_cpu_port_trajectories_match_golden(name):
    from oracle import cpu_port
    from swarp_b200.dynamics.base import param_rows

    gold = load(name)
    spec = gold["spec"]
    cfgs, w = agent_configs(spec), world_config(spec)
    o = obstacles(obstacle_spec(spec))
    obs = None
    if o is not None:
        r = o.resolve("cpu", torch.float64)
        obs = {"pos": r.pos.numpy(), "angle": r.angle.numpy(), "vel": r.vel.numpy(),
               "ang_vel": r.ang_vel.numpy(), "radius": r.radius.numpy(),
               "half": r.half_extents.numpy(), "shape": r.shape.numpy()}
    traj, _, _ = cpu_port.rollout(
        params=param_rows(cfgs), model_tag=[int(c.model) for c in cfgs],
        ctrl_mode=[int(c.ctrl_mode) for c in cfgs], dt=0.05, substeps=spec.get("substeps", 1),
        collisions=True, k=w.collision_k, c=w.collision_c, margin=w.collision_margin,
        max_overlap=w.contact_max_overlap, neighbor_radius=w.neighbor_radius,
        max_neighbors=w.max_neighbors, bounds_mode=1 if w.bounds_mode == "soft" else 2,
        bounds=w.bounds, init=[gold[f"init_{f}"] for f in FIELDS], actions=gold["acts"],
        obstacles=obs, threads=1, dtype=np.float64)
    for i, f in enumerate(FIELDS):
        np.testing.assert_allclose(traj[i], gold[f"traj_{f}"], rtol=1e-10, atol=1e-12, err_msg=f)


def _cuda_run(gold, dtype):
    from swarp_b200.core.stepper import Stepper
    from swarp_b200.interop.autograd import TorchState, rollout_bodies

    spec = gold["spec"]
    dev = "cuda:0"
    st = Stepper(agent_configs(spec), dt=0.05, substeps=spec.get("substeps", 1), device=dev,
                 dtype=dtype, world=world_config(spec))
    o = obstacles(obstacle_spec(spec))
    if o is not None:
        st.set_obstacles(o)
    st.bodies_in_grad = bool(spec.get("bodies_in_grad", False))
    t = lambda x: torch.tensor(x, dtype=dtype, device=dev)  # noqa: E731
    s = [t(gold[f"init_{f}"]).requires_grad_(True) for f in FIELDS]
    a = t(gold["acts"]).requires_grad_(True)
    fin, traj, body = rollout_bodies(st, TorchState(*s), a)
    loss = (fin.pos * t(gold["w_fin"])).sum() + (traj.stacked[1] * t(gold["w_traj"])).sum()
    if body is not None:
        loss = loss + (body.pos[:, 0] * t(gold["w_body"])).sum()
    grads = torch.autograd.grad(loss, [a, *s])
    out = {"loss": loss.detach(), "grad_acts": grads[0]}
    for i, f in enumerate(FIELDS):
        out[f"traj_{f}"] = traj.stacked[i].detach()
        out[f"grad_init_{f}"] = grads[1 + i]
    if body is not None:
        out["body_pos_final"] = body.pos.detach()
        out["body_angle_final"] = body.angle.detach()
    return {k: v.double().cpu().numpy() for k, v in out.items()}


def _check(out, gold, rtol_state, atol_state, rtol_grad, rel_grad_floor, rel_state_floor=0.0):
    for k, v in out.items():
        ref = gold[k]
        scale = max(np.abs(ref).max(), 1e-30)
        if k.startswith("grad"):
            np.testing.assert_allclose(v, ref, rtol=rtol_grad, atol=rel_grad_floor * scale,
                                       err_msg=k)
        else:
            np.testing.assert_allclose(v, ref, rtol=rtol_state,
                                       atol=max(atol_state, rel_state_floor * scale), err_msg=k)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_cuda_float64_matches_golden(name):
    gold = load(name)
    _check(_cuda_run(gold, torch.float64), gold, 1e-10, 1e-12, 1e-10, 1e-10)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_cuda_float32_within_tolerance_of_golden(name):
    """float32 from the same inputs (rounded to float32) at the north-star bars: states
    within 1e-5 relative (plus 1e-5 of the field's largest entry), gradients within 1e-4
    relative plus 1e-4 of their largest entry (the golden answers are float64)."""
    gold = load(name)
    _check(_cuda_run(gold, torch.float32), gold, 1e-5, 0.0, 1e-4, 1e-4, rel_state_floor=1e-5)
