"""Float32 parity at the benchmark configurations, against the float64 oracle.

The north-star bars are forward states within 1e-5 relative and gradients w.r.t. actions
within 1e-4 relative in float32. The workloads are ``bench.build_workload``'s configs 2
(16 holonomic agents, walls, agent contacts, H=64), 3 (32-agent mixed fleet, 10
circle/box/segment obstacles, K=32, H=50) and 5 (256 agents in a dense Gaussian cluster,
R=0.15, K=32, one env per CTA with eight mask words, H=32), on a few envs each. Float32
contact dynamics amplify rounding differences along a trajectory, so each configuration
is checked three ways:

1. step by step over the whole horizon from identical inputs: the oracle steps every
   state the float32 kernel visited (cast to float64) with the same action, and its
   vector-Jacobian product runs on the same states and cotangents (the step's gradient
   w.r.t. action and state); both must meet the bars at every step;
2. free running: the float32 rollout against the float64 rollout from the same start.
   The test asserts the bar for the first ``HOLD_STEPS`` steps; the report gives the step
   at which the difference, grown by the dynamics, first exceeds it;
3. BPTT: the gradient of sum ||pos_h - goal||^2 w.r.t. all actions for growing h, at the
   bar up to ``HOLD_H``.

Relative errors: ``rel_max`` = max |got - ref| / max |ref| over a field; ``rel_elem`` =
max over the elements with |ref| >= 1e-2 max |ref| of |got - ref| / |ref|. Both are
checked. Where the reference's arithmetic itself cannot meet a bar in float32 (the
oracle evaluated in float32 on the same inputs misses it too: the mixed fleet's obstacle
contacts are ill-conditioned at their kinks, config 3), the kernel must stay within twice
that float32 evaluation's own error; the report gives both. Setting
``SWARP_PARITY_REPORT=<file>`` appends the measured profile as JSON lines.
"""

from __future__ import annotations

import dataclasses
import json
import os

import pytest
import torch

from bench import build_workload
from oracle import torch_ref as R
from swarp_b200.core.config import Obstacles
from swarp_b200.core.stepper import Stepper
from swarp_b200.interop.autograd import TorchState, rollout, warp_step

from ref_bridge import D, ref_obstacles, ref_world

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
F32 = torch.float32
RTOL_STATE, RTOL_GRAD = 1e-5, 1e-4

ENVS = {2: 32, 3: 8, 5: 2}
# Free-running steps within RTOL_STATE and BPTT horizons within RTOL_GRAD (max-normalised)
# that each configuration keeps on its seeded inputs, with a margin below the measured
# break-points (B200: config 2 first over the state bar at step 57 of 64, config 3 at 42
# of 50, config 5 at 4 of 32; BPTT gradients within 1e-4 at H = 64, 50 and 16).
HOLD_STEPS = {2: 48, 3: 36, 5: 3}
HOLD_H = {2: 64, 3: 50, 5: 8}
NAMES = ["pos", "theta", "vel", "speed", "ang_vel"]


def rel_max(got, ref) -> float:
    return float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def rel_elem(got, ref, floor=1e-2) -> float:
    big = ref.abs() >= floor * ref.abs().max()
    if not bool(big.any()):
        return 0.0
    return float(((got - ref).abs()[big] / ref.abs()[big]).max())


def report(entry: dict) -> None:
    print(json.dumps(entry))
    path = os.environ.get("SWARP_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(entry) + "\n")


_CACHE: dict = {}


def case(cid: int):
    """(stepper, float64 initial state of float32 values, actions, goal) of config cid."""
    if cid not in _CACHE:
        wl = build_workload(cid, n_envs=ENVS[cid], dev=DEV)
        st = wl.stepper
        E, A = wl.E, wl.A
        pos = torch.from_numpy(wl.pos).to(D)
        th = torch.from_numpy(wl.theta).to(D)
        state = (pos, th, torch.zeros(E, A, 2, dtype=D), torch.zeros(E, A, dtype=D),
                 torch.zeros(E, A, dtype=D))
        _CACHE[cid] = (st, state, torch.from_numpy(wl.acts).to(D), torch.from_numpy(wl.goal).to(D))
    return _CACHE[cid]


def tiled(st: Stepper, n: int) -> Stepper:
    """The same world with every env's obstacles repeated n times along the env axis."""
    if st.obstacles is None:
        return st
    o = st.obstacles
    t = Stepper(st.configs, dt=st.dt, substeps=st.substeps, device=DEV, dtype=st.dtype,
                world=st.world)
    t.set_obstacles(Obstacles(
        pos=o.pos.repeat(n, 1, 1), radius=o.radius, shape=o.shape,
        angle=o.angle.repeat(n, 1) if o.angle.dim() == 2 else o.angle,
        half_extents=o.half_extents, vel=o.vel.repeat(n, 1, 1), ang_vel=o.ang_vel.repeat(n, 1),
        kind=o.kind, mass=o.mass, inertia=o.inertia, body=o.body, body_offset=o.body_offset))
    return t


def obs_to(ob, dtype):
    """The oracle's obstacle set with every floating field in dtype (None stays None)."""
    if ob is None:
        return None
    return dataclasses.replace(ob, **{f.name: getattr(ob, f.name).to(dtype)
                                      for f in dataclasses.fields(ob)
                                      if torch.is_tensor(getattr(ob, f.name))})


def cuda_rollout(st, state, acts):
    with torch.no_grad():
        fin, traj = rollout(st, TorchState(*(t.to(DEV, F32) for t in state)), acts.to(DEV, F32))
    return [tuple(x.cpu().to(D) for x in traj[t][:5]) for t in range(acts.shape[0])]


@pytest.mark.parametrize("cid", [2, 3, 5])
def test_teacher_forced_steps_f32(cid):
    """Every step of the float32 trajectory, forward and VJP, from identical inputs."""
    st, state, acts, _ = case(cid)
    H, E = acts.shape[0], acts.shape[1]
    traj = cuda_rollout(st, state, acts)
    inputs = [state] + traj[:-1]
    x = tuple(torch.cat([inp[f] for inp in inputs]) for f in range(5))  # [H*E, A, ...]
    a = acts.reshape(H * E, *acts.shape[2:])
    big = tiled(st, H)
    g = torch.Generator().manual_seed(100 + cid)
    cot = [torch.randn(t.shape, generator=g, dtype=D) for t in x]

    def oracle(dtype):
        """The oracle's step (outputs) and VJP (gradients) at every visited state."""
        w, ob = ref_world(big), ref_obstacles(big)
        if dtype != D:
            w = dataclasses.replace(w, params=w.params.to(dtype))
            ob = obs_to(ob, dtype)
        xs = [t.to(dtype).requires_grad_(True) for t in x]
        ar = a.to(dtype).requires_grad_(True)
        out, _, _ = R.step(tuple(xs), ar, w, ob)
        gr = torch.autograd.grad(sum((c.to(dtype) * o).sum() for c, o in zip(cot, out)),
                                 [ar, *xs], allow_unused=True)
        return ([o.detach().to(D) for o in out], [None if q is None else q.to(D) for q in gr])

    ref_out, ref_g = oracle(D)
    o32_out, o32_g = oracle(F32)
    # the kernel: its own next states, and its VJP at the same states and cotangents
    got = tuple(torch.cat([s[f] for s in traj]) for f in range(5))
    xc = [t.to(DEV, F32).requires_grad_(True) for t in x]
    ac = a.to(DEV, F32).requires_grad_(True)
    outc = warp_step(big, TorchState(*xc), ac)
    got_g = torch.autograd.grad(sum((c.to(DEV, F32) * o).sum() for c, o in zip(cot, outc)),
                                [ac, *xc], allow_unused=True)
    got_g = [None if q is None else q.cpu().to(D) for q in got_g]
    rows = []  # (what, kernel (max, elem), float32 oracle (max, elem), bar)
    for f in range(5):
        if float(ref_out[f].abs().max()) > 0:
            rows.append((f"step {NAMES[f]}", (rel_max(got[f], ref_out[f]),
                                              rel_elem(got[f], ref_out[f])),
                         (rel_max(o32_out[f], ref_out[f]), rel_elem(o32_out[f], ref_out[f])),
                         RTOL_STATE))
    for n, gc, gr, go in zip(["actions", *NAMES], got_g, ref_g, o32_g):
        if gr is not None and float(gr.abs().max()) > 0:
            rows.append((f"vjp {n}", (rel_max(gc, gr), rel_elem(gc, gr)),
                         (rel_max(go, gr), rel_elem(go, gr)), RTOL_GRAD))
    report({"config": cid, "check": "teacher_forced", "envs": E, "horizon": H,
            "rows": {w: {"kernel": k, "oracle_f32": o, "bar": b} for w, k, o, b in rows}})
    for what, k, o, bar in rows:
        for i, kind in enumerate(("max-normalised", "elementwise")):
            allowed = max(bar, 2.0 * o[i])
            assert k[i] <= allowed, (f"config {cid} {what} {kind}: {k[i]:.3g} > {allowed:.3g} "
                                     f"(float32 oracle {o[i]:.3g})")


@pytest.mark.parametrize("cid", [2, 3, 5])
def test_free_running_divergence_f32(cid):
    """Float32 rollout vs float64 rollout from the same start; reports where they part."""
    st, state, acts, _ = case(cid)
    H = acts.shape[0]
    traj = cuda_rollout(st, state, acts)
    _, ref, _ = R.rollout(state, acts, ref_world(st), ref_obstacles(st))

    def profile(tr):
        return [max(rel_max(tr[t][f], ref[t][f]) for f in range(5)
                    if float(ref[t][f].abs().max()) > 0) for t in range(H)]

    def first_over(prof):
        return next((t + 1 for t, e in enumerate(prof) if e > RTOL_STATE), None)

    prof = profile(traj)
    first_break = first_over(prof)
    # the same rollout in float32 through the oracle: how soon float32 itself departs
    w32 = dataclasses.replace(ref_world(st), params=ref_world(st).params.float())
    ob = obs_to(ref_obstacles(st), F32)
    _, r32, _ = R.rollout(tuple(t.float() for t in state), acts.float(), w32, ob)
    prof32 = profile([tuple(x.to(D) for x in r32[t]) for t in range(H)])
    report({"config": cid, "check": "free_running", "horizon": H, "first_step_over_bar":
            first_break, "oracle_f32_first_step_over_bar": first_over(prof32),
            "rel_max_by_step": [float(f"{e:.3g}") for e in prof],
            "oracle_f32_rel_max_by_step": [float(f"{e:.3g}") for e in prof32]})
    held = H if first_break is None else first_break - 1
    assert held >= HOLD_STEPS[cid], f"config {cid}: bar held for {held} steps"


@pytest.mark.parametrize("cid", [2, 3, 5])
def test_bptt_gradients_f32(cid):
    """Gradient of sum ||pos_h - goal||^2 w.r.t. the actions, float32 vs float64."""
    st, state, acts, goal = case(cid)
    H = acts.shape[0]
    hs = sorted({1, 2, 4, 8, 16, 32, H} & set(range(1, H + 1)))
    w32 = dataclasses.replace(ref_world(st), params=ref_world(st).params.float())
    ob32 = obs_to(ref_obstacles(st), F32)
    errs, errs32 = {}, {}
    for h in hs:
        a_r = acts[:h].clone().requires_grad_(True)
        fin, _, _ = R.rollout(state, a_r, ref_world(st), ref_obstacles(st))
        (g_ref,) = torch.autograd.grad(((fin[0] - goal) ** 2).sum(), [a_r])
        a_c = acts[:h].to(DEV, F32).requires_grad_(True)
        fc, _ = rollout(st, TorchState(*(t.to(DEV, F32) for t in state)), a_c)
        (g_c,) = torch.autograd.grad(((fc.pos - goal.to(DEV, F32)) ** 2).sum(), [a_c])
        g_c = g_c.cpu().to(D)
        errs[h] = (rel_max(g_c, g_ref), rel_elem(g_c, g_ref))
        # the reference's arithmetic in float32 (the oracle run in float32)
        a_o = acts[:h].float().requires_grad_(True)
        f32, _, _ = R.rollout(tuple(t.float() for t in state), a_o, w32, ob32)
        (g_o,) = torch.autograd.grad(((f32[0] - goal.float()) ** 2).sum(), [a_o])
        errs32[h] = (rel_max(g_o.to(D), g_ref), rel_elem(g_o.to(D), g_ref))
    first_break = next((h for h in hs if errs[h][0] > RTOL_GRAD), None)
    report({"config": cid, "check": "bptt", "horizons": hs,
            "rel_max": [float(f"{errs[h][0]:.3g}") for h in hs],
            "rel_elem": [float(f"{errs[h][1]:.3g}") for h in hs],
            "oracle_f32_rel_max": [float(f"{errs32[h][0]:.3g}") for h in hs],
            "oracle_f32_rel_elem": [float(f"{errs32[h][1]:.3g}") for h in hs],
            "first_horizon_over_bar": first_break})
    for h in hs:
        if h <= HOLD_H[cid]:
            assert errs[h][0] <= RTOL_GRAD, f"config {cid} H={h}: {errs[h]}"
            # elementwise: the bar, or (chaos) four times float32's own error
            allowed = max(RTOL_GRAD, 4.0 * errs32[h][1])
            assert errs[h][1] <= allowed, f"config {cid} H={h}: {errs[h]} vs {errs32[h]}"
