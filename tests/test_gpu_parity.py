"""CUDA rollout (forward + adjoint) against the CPU oracle, through the public API.

Every test here drives ``swarp_b200`` (ctypes -> libswarp_b200.so, sm_100a) and checks
it against ``oracle/torch_ref.py`` (float64 restatement of the reference, autograd
gradients). Tolerances follow the north-star contract: float64 forward and gradients
within 1e-10 (relative, with an absolute floor scaled to the largest magnitude);
float32 forward within 1e-5 and gradients within 1e-4 relative to the float64 oracle.
"""

import numpy as np
import pytest
import torch

from oracle import torch_ref as R
from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel
from swarp_b200.interop.autograd import TorchState, rollout, warp_step

from ref_bridge import D, ref_obstacles, ref_world

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BIG = 100.0


def cfgs_of(model, mode, n, radius=0.1, **kw):
    base = dict(model=model, ctrl_mode=mode, radius=radius, max_speed=BIG, max_accel=BIG,
                max_ang_vel=BIG, max_ang_accel=BIG, max_steer=1.0, l_f=0.16, l_r=0.14)
    base.update(kw)
    return [AgentConfig(**base) for _ in range(n)]


def rand_state(E, A, seed, spread=0.3, vel=0.5):
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1) * spread
    th = (torch.rand(E, A, generator=g, dtype=D) * 2 - 1) * 3.0
    v = torch.randn(E, A, 2, generator=g, dtype=D) * vel
    s = torch.randn(E, A, generator=g, dtype=D) * vel
    w = torch.randn(E, A, generator=g, dtype=D) * vel
    return (pos, th, v, s, w)


def rand_actions(T, E, A, seed, scale=0.5, D_=2):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(T, E, A, D_, generator=g, dtype=D) * 2 - 1) * scale


def loss_weights(T, E, A, seed):
    g = torch.Generator().manual_seed(seed)
    shp = [(T, E, A, 2), (T, E, A), (T, E, A, 2), (T, E, A), (T, E, A)]
    return [torch.randn(*s, generator=g, dtype=D) for s in shp]


def run_oracle(stepper, state5, acts, weights, final_w=None):
    w = ref_world(stepper)
    ob = ref_obstacles(stepper)
    st = [t.clone().requires_grad_(True) for t in state5]
    a = acts.clone().requires_grad_(True)
    fin, traj, _ = R.rollout(tuple(st), a, w, ob)
    loss = sum((wf[t] * traj[t][f]).sum() for t in range(len(traj)) for f, wf in enumerate(weights))
    if final_w is not None:
        loss = loss + sum((wf * fin[f]).sum() for f, wf in enumerate(final_w))
    grads = torch.autograd.grad(loss, [a, *st], allow_unused=True)
    traj_t = [torch.stack([traj[t][f] for t in range(len(traj))]).detach() for f in range(5)]
    return traj_t, [g if g is not None else torch.zeros_like(x) for g, x in zip(grads, [a, *st])]


def run_cuda(stepper, state5, acts, weights, dtype, final_w=None):
    st = [t.to(DEV, dtype).clone().requires_grad_(True) for t in state5]
    a = acts.to(DEV, dtype).clone().requires_grad_(True)
    fin, traj = rollout(stepper, TorchState(*st), a)
    loss = sum((wf.to(DEV, dtype)[t] * traj[t][f]).sum() for t in range(len(traj))
               for f, wf in enumerate(weights))
    if final_w is not None:
        loss = loss + sum((wf.to(DEV, dtype) * fin[f]).sum() for f, wf in enumerate(final_w))
    grads = torch.autograd.grad(loss, [a, *st], allow_unused=True)
    traj_t = [torch.stack([traj[t][f] for t in range(len(traj))]).detach().cpu().double()
              for f in range(5)]
    return traj_t, [(g if g is not None else torch.zeros_like(x)).cpu().double()
                    for g, x in zip(grads, [a, *st])]


def close(got, ref, rtol, what):
    """Max-normalised: |got - ref| <= rtol * (|ref| + max|ref|). At the float64 bars
    (rtol <= 1e-9) also elementwise: every element with |ref| >= 1e-2 max|ref| within
    10 rtol of itself. (Float32 elementwise errors are compared with float32's own error on
    the same inputs in test_gpu_parity_f32.py.)"""
    scale = max(float(ref.abs().max()), 1e-30)
    torch.testing.assert_close(got, ref, rtol=rtol, atol=rtol * scale, msg=lambda m: f"{what}: {m}")
    big = ref.abs() >= 1e-2 * scale
    if rtol <= 1e-9 and bool(big.any()):
        worst = float(((got - ref).abs()[big] / ref.abs()[big]).max())
        assert worst <= 10 * rtol, f"{what}: elementwise relative error {worst:.3g}"


def check(stepper, state5, acts, seed=0, dtype=torch.float64, rtol_f=1e-10, rtol_g=1e-10,
          final=False):
    T, E, A, _ = acts.shape
    wts = loss_weights(T, E, A, seed + 100)
    fw = [w[-1] for w in loss_weights(1, E, A, seed + 200)] if final else None
    tr, gr = run_oracle(stepper, state5, acts, wts, fw)
    tc, gc = run_cuda(stepper, state5, acts, wts, dtype, fw)
    names = ["pos", "theta", "vel", "speed", "ang_vel"]
    for f in range(5):
        close(tc[f], tr[f], rtol_f, f"traj {names[f]}")
    for i, n in enumerate(["actions", *names]):
        close(gc[i], gr[i], rtol_g, f"grad {n}")


MODEL_CASES = [
    ("holonomic-vel", DynamicsModel.HOLONOMIC, ControlMode.VELOCITY),
    ("holonomic-acc", DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION),
    ("diffdrive-vel", DynamicsModel.DIFF_DRIVE, ControlMode.VELOCITY),
    ("diffdrive-acc", DynamicsModel.DIFF_DRIVE, ControlMode.ACCELERATION),
    ("diffdrive-servo", DynamicsModel.DIFF_DRIVE, ControlMode.SERVO),
    ("bicycle", DynamicsModel.KINEMATIC_BICYCLE, ControlMode.ACCELERATION),
]


@pytest.mark.parametrize("name,model,mode", MODEL_CASES, ids=[c[0] for c in MODEL_CASES])
def test_models_with_contacts_and_walls_f64(name, model, mode):
    world = WorldConfig(collision_k=30.0, collision_c=1.0, collision_margin=0.05,
                        bounds=(-0.4, 0.4, -0.4, 0.4), bounds_mode="soft")
    st = Stepper(cfgs_of(model, mode, 5, max_speed=1.5, max_accel=2.0, max_ang_vel=2.0,
                         max_ang_accel=4.0), dt=0.05, device=DEV, dtype=torch.float64, world=world)
    check(st, rand_state(3, 5, 1), rand_actions(6, 3, 5, 2, scale=2.0), seed=3)


def test_limits_saturating_f64():
    """Actions beyond the limits (clamp kinks active) for every model in one fleet."""
    cfgs = [AgentConfig(model=DynamicsModel.HOLONOMIC, radius=0.08, max_speed=1.0),
            AgentConfig(model=DynamicsModel.DIFF_DRIVE, radius=0.08, max_speed=1.0, max_ang_vel=1.0),
            AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, radius=0.08, max_speed=1.0,
                        max_accel=1.0, max_steer=0.5, min_speed=0.0)]
    world = WorldConfig(collision_k=50.0, collision_c=2.0, collision_margin=0.02)
    st = Stepper(cfgs, dt=0.1, device=DEV, dtype=torch.float64, world=world)
    check(st, rand_state(4, 3, 5, spread=0.15), rand_actions(8, 4, 3, 6, scale=3.0), seed=7)


def test_substeps_f64():
    world = WorldConfig(collision_k=30.0, collision_c=1.0, collision_margin=0.05,
                        bounds=(-0.5, 0.5, -0.5, 0.5))
    cfgs = (cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION, 2)
            + cfgs_of(DynamicsModel.DIFF_DRIVE, ControlMode.VELOCITY, 2)
            + cfgs_of(DynamicsModel.KINEMATIC_BICYCLE, ControlMode.ACCELERATION, 2))
    st = Stepper(cfgs, dt=0.06, substeps=3, device=DEV, dtype=torch.float64, world=world)
    check(st, rand_state(2, 6, 11), rand_actions(5, 2, 6, 12), seed=13, final=True)


def test_clamp_bounds_f64():
    world = WorldConfig(collision_k=30.0, collision_margin=0.02, bounds=(-0.3, 0.3, -0.3, 0.3),
                        bounds_mode="clamp")
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.VELOCITY, 4, max_speed=3.0), dt=0.1,
                 device=DEV, dtype=torch.float64, world=world)
    check(st, rand_state(3, 4, 21, spread=0.25), rand_actions(6, 3, 4, 22, scale=3.0), seed=23)


def _obstacle_set(E, seed):
    g = torch.Generator().manual_seed(seed)
    N = 6
    pos = (torch.rand(E, N, 2, generator=g, dtype=D) * 2 - 1) * 0.35
    ang = torch.rand(E, N, generator=g, dtype=D) * 3.14
    return Obstacles(
        pos=pos,
        radius=torch.tensor([0.1, 0.07, 0.0, 0.0, 0.03, 0.02], dtype=D),
        shape=torch.tensor([0, 0, 1, 1, 2, 2], dtype=torch.int32),
        angle=ang,
        half_extents=torch.tensor([[0, 0], [0, 0], [0.1, 0.06], [0.05, 0.12], [0.2, 0],
                                   [0.12, 0]], dtype=D),
        vel=torch.randn(E, N, 2, generator=g, dtype=D) * 0.2,
        ang_vel=torch.randn(E, N, generator=g, dtype=D) * 0.5,
    )


def test_obstacles_f64():
    world = WorldConfig(collision_k=40.0, collision_c=1.0, collision_margin=0.02,
                        bounds=(-0.6, 0.6, -0.6, 0.6))
    cfgs = (cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION, 3, radius=0.06)
            + cfgs_of(DynamicsModel.DIFF_DRIVE, ControlMode.ACCELERATION, 2, radius=0.06)
            + cfgs_of(DynamicsModel.KINEMATIC_BICYCLE, ControlMode.ACCELERATION, 2, radius=0.06))
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float64, world=world)
    st.set_obstacles(_obstacle_set(4, 31))
    check(st, rand_state(4, 7, 32, spread=0.4), rand_actions(8, 4, 7, 33, scale=1.0), seed=34)


def test_truncated_lists_f64():
    """A dense cluster with max_neighbors below the in-radius count (overflow)."""
    world = WorldConfig(collision_k=20.0, collision_c=0.5, collision_margin=0.02,
                        neighbor_radius=0.35, max_neighbors=3)
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION, 12, radius=0.06),
                 dt=0.05, device=DEV, dtype=torch.float64, world=world)
    check(st, rand_state(3, 12, 41, spread=0.18), rand_actions(5, 3, 12, 42), seed=43)


def test_two_chunk_agents_f64():
    """More than 32 agents per env (the neighbor mask spans two words), E not a multiple
    of the envs per CTA, truncation on."""
    world = WorldConfig(collision_k=20.0, collision_c=0.5, collision_margin=0.02,
                        neighbor_radius=0.3, max_neighbors=8, bounds=(-1.0, 1.0, -1.0, 1.0))
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.VELOCITY, 40, radius=0.05,
                         max_speed=1.0), dt=0.05, device=DEV, dtype=torch.float64, world=world)
    check(st, rand_state(5, 40, 51, spread=0.5), rand_actions(4, 5, 40, 52, scale=1.2), seed=53)


def test_single_agent_and_wide_actions_f64():
    world = WorldConfig(collisions=True, bounds=(-0.2, 0.2, -0.2, 0.2))
    st = Stepper(cfgs_of(DynamicsModel.DIFF_DRIVE, ControlMode.ACCELERATION, 1), dt=0.1, device=DEV,
                 dtype=torch.float64, world=world)
    acts = rand_actions(4, 7, 1, 61, D_=3)
    check(st, rand_state(7, 1, 60, spread=0.2), acts, seed=62)


def test_navigation_like_f32():
    """Config-2 physics at a small batch in float32 against the float64 oracle."""
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=16)
    cfgs = [AgentConfig(model=DynamicsModel.HOLONOMIC, radius=0.05, max_speed=1.0, max_accel=2.0)
            for _ in range(16)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float32, world=world)
    state = rand_state(64, 16, 71, spread=0.95, vel=0.3)
    acts = rand_actions(3, 64, 16, 72, scale=1.0)
    check(st, state, acts, seed=73, dtype=torch.float32, rtol_f=1e-5, rtol_g=1e-4)


def test_gradcheck_step_f64():
    world = WorldConfig(collision_k=10.0, collision_c=1.0, collision_margin=0.02,
                        bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft")
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION, 2), dt=0.1, substeps=2,
                 device=DEV, dtype=torch.float64, world=world)
    pos = torch.tensor([[[0.0, 0.0], [0.18, 0.02]]], dtype=D, device=DEV)
    vel = torch.tensor([[[0.1, 0.0], [-0.1, 0.05]]], dtype=D, device=DEV)
    z = torch.zeros(1, 2, dtype=D, device=DEV)
    acts = 0.1 * torch.randn(1, 2, 2, dtype=D, generator=torch.Generator().manual_seed(0))
    inputs = tuple(t.clone().requires_grad_(True) for t in (pos, z, vel, z, z, acts.to(DEV)))

    def fn(p, th, v, s, w, a):
        return tuple(warp_step(st, TorchState(p, th, v, s, w), a))[:5]

    assert torch.autograd.gradcheck(fn, inputs, eps=1e-6, atol=1e-5)


def test_gradcheck_rollout_f64():
    cfgs = [AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=BIG, max_accel=BIG,
                        max_steer=1.0, l_f=0.16, l_r=0.14),
            AgentConfig(model=DynamicsModel.DIFF_DRIVE, max_speed=BIG, max_ang_vel=BIG)]
    st = Stepper(cfgs, dt=0.1, device=DEV, dtype=torch.float64)
    state = [t.to(DEV).requires_grad_(True) for t in rand_state(1, 2, 3, spread=0.5)]
    acts = (0.3 * torch.randn(5, 1, 2, 2, dtype=D)).to(DEV).requires_grad_(True)

    def fn(p, th, v, s, w, a):
        final, _ = rollout(st, TorchState(p, th, v, s, w), a)
        return final.pos, final.theta

    assert torch.autograd.gradcheck(fn, (*state, acts), eps=1e-6, atol=1e-5)


def test_bptt_analytic_holonomic():
    T, dt = 6, 0.1
    st = Stepper([AgentConfig(model=DynamicsModel.HOLONOMIC, max_speed=BIG)], dt=dt, device=DEV,
                 dtype=torch.float64)
    state = TorchState(*(t.to(DEV) for t in rand_state(1, 1, 4)))
    acts = (0.2 * torch.randn(T, 1, 1, 2, dtype=D)).to(DEV).requires_grad_(True)
    final, _ = rollout(st, state, acts)
    final.pos[0, 0, 0].backward()
    expected = torch.zeros_like(acts)
    expected[:, 0, 0, 0] = dt
    torch.testing.assert_close(acts.grad, expected)


def test_bptt_analytic_holonomic_accel():
    dt = 0.1
    st = Stepper([AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.ACCELERATION,
                              max_speed=BIG, max_accel=BIG)], dt=dt, device=DEV,
                 dtype=torch.float64)
    state = TorchState(*(t.to(DEV) for t in rand_state(1, 1, 5)))
    acts = (0.2 * torch.randn(2, 1, 1, 2, dtype=D)).to(DEV).requires_grad_(True)
    final, _ = rollout(st, state, acts)
    final.pos[0, 0, 0].backward()
    torch.testing.assert_close(acts.grad[0, 0, 0, 0].cpu(), torch.tensor(2 * dt * dt, dtype=D))


def test_saturated_actions_zero_finite_grads():
    st = Stepper([AgentConfig(model=DynamicsModel.DIFF_DRIVE, max_speed=1.0, max_ang_vel=1.0)],
                 dt=0.1, device=DEV, dtype=torch.float64)
    state = TorchState(*(t.to(DEV) for t in rand_state(1, 1, 6)))
    acts = torch.full((1, 1, 2), 50.0, dtype=D, device=DEV, requires_grad=True)
    warp_step(st, state, acts).pos.sum().backward()
    assert torch.isfinite(acts.grad).all() and acts.grad.abs().sum() == 0.0


def test_grad_and_nograd_forward_match():
    world = WorldConfig(collision_k=30.0, collision_c=1.0, collision_margin=0.05)
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION, 3), dt=0.05,
                 substeps=3, device=DEV, dtype=torch.float64, world=world)
    state = [t.to(DEV) for t in rand_state(1, 3, 8, spread=0.15)]
    acts = torch.zeros(1, 3, 2, dtype=D, device=DEV)
    out_g = warp_step(st, TorchState(*(t.clone().requires_grad_(True) for t in state)),
                      acts.clone().requires_grad_(True))
    with torch.no_grad():
        out_f = warp_step(st, TorchState(*state), acts)
    for a, b in zip(out_g, out_f, strict=True):
        assert torch.equal(a.detach(), b)
    assert not out_f.pos.requires_grad


def test_run_twice_bitwise_identical():
    world = WorldConfig(collision_k=100.0, collision_margin=0.025, bounds=(-1.0, 1.0, -1.0, 1.0))
    cfgs = [AgentConfig(radius=0.05) for _ in range(16)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float32, world=world)
    state = [t.to(DEV, torch.float32) for t in rand_state(200, 16, 9, spread=0.6)]
    acts = rand_actions(10, 200, 16, 10).to(DEV, torch.float32)

    def once():
        s = [t.clone().requires_grad_(True) for t in state]
        a = acts.clone().requires_grad_(True)
        fin, traj = rollout(st, TorchState(*s), a)
        (fin.pos.square().sum() + traj[3].vel.sum()).backward()
        return [fin.pos.detach(), fin.vel.detach(), a.grad, s[0].grad, s[2].grad]

    for x, y in zip(once(), once(), strict=True):
        assert torch.equal(x, y)


def test_neighbor_lists_match_oracle():
    world = WorldConfig(neighbor_radius=0.3, max_neighbors=5, collision_margin=0.02)
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.VELOCITY, 20, radius=0.05), dt=0.1,
                 device=DEV, dtype=torch.float32, world=world)
    pos = rand_state(6, 20, 81, spread=0.5)[0]
    idx, cnt, tru = st.neighbors(pos.to(DEV, torch.float32))
    in_list, ridx, rcnt, rtru = R.brute_neighbors(pos.float().double(), 0.3, 5)
    assert torch.equal(cnt.cpu().long(), rcnt)
    assert torch.equal(tru.cpu().long(), rtru)
    for e in range(6):
        for a in range(20):
            n = int(rcnt[e, a])
            assert idx[e, a, :n].cpu().tolist() == ridx[e, a, :n].tolist()


def test_overflow_flag_cluster():
    pos = torch.zeros(1, 5, 2, dtype=torch.float32)
    pos[0, :, 0] = torch.linspace(0.0, 0.04, 5)
    cfg = cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.VELOCITY, 5, radius=0.01)
    st = Stepper(cfg, dt=0.1, device=DEV, world=WorldConfig(neighbor_radius=0.5, max_neighbors=2))
    _, cnt, tru = st.neighbors(pos.to(DEV))
    assert torch.equal(tru.cpu(), torch.full((1, 5), 4, dtype=torch.int32))
    assert (tru > cnt).all()
    st8 = Stepper(cfg, dt=0.1, device=DEV, world=WorldConfig(neighbor_radius=0.5, max_neighbors=8))
    _, cnt8, tru8 = st8.neighbors(pos.to(DEV))
    assert not (tru8 > cnt8).any()


def test_env_independence_full_size_f32():
    """Config-2 size (16000 envs x 16 agents, H=64): every env evolves independently, so a
    subset of envs stepped alone reproduces the full batch bit for bit (forward and
    gradients), and the first step matches the float64 oracle on that subset."""
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=16)
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(16)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float32, world=world)
    E, A, T = 16000, 16, 64
    g = torch.Generator(device=DEV).manual_seed(0)
    pos = (torch.rand(E, A, 2, generator=g, device=DEV) * 1.9 - 0.95)
    z = torch.zeros(E, A, device=DEV)
    state = [pos, z, torch.zeros(E, A, 2, device=DEV), z, z]
    acts = torch.rand(T, E, A, 2, generator=g, device=DEV) * 2 - 1
    goal = torch.rand(E, A, 2, generator=g, device=DEV) * 1.9 - 0.95

    def grads(sel):
        s = [t[sel].clone().requires_grad_(True) for t in state]
        a = acts[:, sel].clone().requires_grad_(True)
        fin, traj = rollout(st, TorchState(*s), a)
        ((fin.pos - goal[sel]) ** 2).sum().backward()
        return fin.pos.detach(), traj[0].pos.detach(), a.grad, s[0].grad

    full = grads(slice(None))
    sub_idx = torch.tensor([0, 1, 777, 8191, 15999], device=DEV)
    sub = grads(sub_idx)
    for f, s_ in zip(full, sub, strict=True):
        assert torch.equal(f[sub_idx] if f.dim() == 3 else f[:, sub_idx], s_)
    assert torch.isfinite(full[2]).all()
    # first step vs oracle on the subset
    w = ref_world(st)
    st0 = tuple(t[sub_idx].detach().cpu().double() for t in state)
    r1, _, _ = R.step(st0, acts[0, sub_idx].cpu().double(), w)
    close(full[1][sub_idx].cpu().double(), r1[0], 1e-5, "step-1 pos")


def test_bare_cuda_device_string():
    """device="cuda" names the current device, as in torch."""
    st = Stepper(cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.VELOCITY, 3), dt=0.05, device="cuda",
                 dtype=torch.float64, world=WorldConfig())
    assert st.device == torch.device("cuda", torch.cuda.current_device())
    s = TorchState(*(t.to(DEV) for t in rand_state(2, 3, 91)))
    fin, traj = rollout(st, s, rand_actions(2, 2, 3, 92).to(DEV))
    assert traj[-1][0].shape == (2, 3, 2)
