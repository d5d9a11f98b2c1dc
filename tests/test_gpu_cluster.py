"""Envs wider than one CTA (more than 1024 agents per env): the thread-block-cluster
kernels (swarp_b200/csrc/rollout_cluster.cuh) and the wide-env neighbor lists.

The reference builds neighbor lists and steps envs of any agent count
(swarp/core/neighbors.py:135-254 grids them; the taped path is the layered brute build
plus force and integrate kernels, swarp/core/stepper.py:784-1011). Here envs of 1025 to
4096 agents run one env per cluster of up to 8 CTAs. Checked:

- 2048-agent envs against the C restatement of the reference (oracle/cpu_port.c, float64,
  hand-written adjoint): trajectories within 1e-12 and gradients within 1e-10;
- lists, counts and uncapped counts of 2048- and 1501-agent envs bit for bit against the
  reference's membership rule restated in numpy, and the rollout's uncapped counts;
- a float32 2048-agent goal-loss case: bitwise across 4- and 8-CTA clusters, and against
  the float32 and float64 restatements within the float32 problem's own sensitivity;
- small envs forced through the cluster kernels (SWARP_CLUSTER_MIN_AGENTS /
  SWARP_CLUSTER_CTA_THREADS): bitwise the single-CTA kernels' trajectories and gradients
  (same device arithmetic in the same order), over models, RK4, substeps, truncation,
  obstacles, the fused goal loss and the gradient-norm epilogue.
"""

from __future__ import annotations

import contextlib
import os

import numpy as np
import pytest
import torch

from oracle import cpu_port
from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import (AgentConfig, ControlMode, DynamicsModel, Integrator,
                                      param_rows)
from swarp_b200.interop.autograd import TorchState, rollout, rollout_goal_loss

from test_gpu_neighbor_boundary import truth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = torch.float64


@contextlib.contextmanager
def cluster_env(min_agents: int, cta_threads: int):
    """Route envs of >= min_agents agents through the cluster kernels, cta_threads per CTA."""
    old = {k: os.environ.get(k) for k in ("SWARP_CLUSTER_MIN_AGENTS", "SWARP_CLUSTER_CTA_THREADS")}
    os.environ["SWARP_CLUSTER_MIN_AGENTS"] = str(min_agents)
    os.environ["SWARP_CLUSTER_CTA_THREADS"] = str(cta_threads)
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def swarm(E, A, seed, spread=1.0):
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1) * spread
    th = (torch.rand(E, A, generator=g, dtype=D) * 2 - 1) * 3.0
    vel = torch.randn(E, A, 2, generator=g, dtype=D) * 0.3
    sp = torch.randn(E, A, generator=g, dtype=D) * 0.3
    om = torch.randn(E, A, generator=g, dtype=D) * 0.3
    return [pos, th, vel, sp, om]


def obstacle_set(E, seed):
    rng = np.random.default_rng(seed)
    shapes = [0, 1, 2, 0, 1]
    N = len(shapes)
    o = dict(pos=rng.uniform(-0.8, 0.8, (E, N, 2)), angle=rng.uniform(-3, 3, (E, N)),
             vel=rng.normal(0, 0.1, (E, N, 2)), ang_vel=rng.normal(0, 0.1, (E, N)),
             radius=rng.uniform(0.03, 0.08, N), half=rng.uniform(0.03, 0.1, (N, 2)),
             shape=np.array(shapes, np.int32))
    return o


def to_obstacles(o) -> Obstacles:
    t = lambda x: torch.tensor(x, dtype=D)  # noqa: E731
    return Obstacles(pos=t(o["pos"]), radius=t(o["radius"]), shape=torch.tensor(o["shape"]),
                     angle=t(o["angle"]), half_extents=t(o["half"]), vel=t(o["vel"]),
                     ang_vel=t(o["ang_vel"]))


@pytest.mark.parametrize("substeps,K,with_obs", [(1, 4, True), (2, 64, False)])
def test_2048_agents_match_cpu_restatement_f64(substeps, K, with_obs):
    """2048 agents per env (4 CTAs of 512): forward and adjoint against oracle/cpu_port.c."""
    E, A, T = 2, 2048, 4
    cfgs = ([AgentConfig(radius=0.015, max_speed=2.0, max_accel=4.0) for _ in range(A // 2)]
            + [AgentConfig(model=DynamicsModel.DIFF_DRIVE, ctrl_mode=ControlMode.ACCELERATION,
                           radius=0.012, max_speed=2.0, max_accel=4.0, max_ang_vel=5.0,
                           max_ang_accel=10.0) for _ in range(A // 2)])
    bounds = (-1.0, 1.0, -1.0, 1.0)
    world = WorldConfig(collision_k=60.0, collision_c=0.8, collision_margin=0.005,
                        bounds=bounds, neighbor_radius=0.06, max_neighbors=K)
    st = Stepper(cfgs, dt=0.05, substeps=substeps, device=DEV, dtype=D, world=world)
    obs = obstacle_set(E, 7) if with_obs else None
    if obs is not None:
        st.set_obstacles(to_obstacles(obs))
    st.track_neighbor_overflow = True
    state = swarm(E, A, 11)
    g = torch.Generator().manual_seed(12)
    acts = (torch.rand(T, E, A, 2, generator=g, dtype=D) * 2 - 1) * 1.5
    gf = torch.randn(E, A, 2, generator=g, dtype=D)

    s_gpu = [x.to(DEV).requires_grad_(True) for x in state]
    a_gpu = acts.to(DEV).requires_grad_(True)
    fin, traj = rollout(st, TorchState(*s_gpu), a_gpu)
    (fin.pos * gf.to(DEV)).sum().backward()
    tmax = st.last_true_count_max.cpu().numpy()
    assert tmax.max() > K or K >= 64  # the truncating case does truncate

    traj_c, ga_c, gi_c = cpu_port.rollout(
        params=param_rows(cfgs), model_tag=[int(c.model) for c in cfgs],
        ctrl_mode=[int(c.ctrl_mode) for c in cfgs], dt=0.05, substeps=substeps,
        collisions=True, k=60.0, c=0.8, margin=0.005, max_overlap=0.0, neighbor_radius=0.06,
        max_neighbors=K, bounds_mode=1, bounds=bounds, init=[x.numpy() for x in state],
        actions=acts.numpy(), grad_final_pos=gf.numpy(), obstacles=obs, threads=0,
        dtype=np.float64)
    for f in range(5):
        got = traj.stacked[f].detach().cpu().numpy()
        np.testing.assert_allclose(got, traj_c[f], rtol=1e-12,
                                   atol=1e-12 * np.abs(traj_c[f]).max(), err_msg=f"field {f}")
    sc = np.abs(ga_c).max()
    np.testing.assert_allclose(a_gpu.grad.cpu().numpy(), ga_c, rtol=1e-10, atol=1e-10 * sc)
    for f in range(5):
        ref = gi_c[f]
        np.testing.assert_allclose(s_gpu[f].grad.cpu().numpy(), ref, rtol=1e-10,
                                   atol=1e-10 * max(np.abs(ref).max(), 1e-30))
    # uncapped counts: the reference's rule on every substep's input state (one substep)
    if substeps == 1:
        pos_in = np.concatenate([state[0].numpy()[None], traj.stacked[0].detach().cpu().numpy()])
        want = np.zeros((E, A), np.int64)
        for t in range(T):
            _, cnt, _ = truth(pos_in[t], st.neighbor_radius, K)
            want = np.maximum(want, cnt)
        np.testing.assert_array_equal(tmax, want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("A,K", [(2048, 12), (1501, 3000)])
def test_wide_env_neighbor_lists(dtype, A, K):
    """Lists, counts and uncapped counts of envs above one CTA, bit for bit."""
    E = 3
    f = np.float32 if dtype == torch.float32 else np.float64
    rng = np.random.default_rng(A)
    pos = rng.uniform(-1.0, 1.0, (E, A, 2)).astype(f)
    R_nb = 0.07
    world = WorldConfig(neighbor_radius=R_nb, max_neighbors=K, bounds=(-1, 1, -1, 1))
    cfgs = [AgentConfig(radius=0.02) for _ in range(A)]
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=dtype, world=world)
    idx, cnt, tru = st.neighbors(torch.from_numpy(pos).to(DEV))
    lists, true_count, _ = truth(pos, R_nb, K)
    idx, cnt, tru = idx.cpu().numpy(), cnt.cpu().numpy(), tru.cpu().numpy()
    np.testing.assert_array_equal(tru, true_count)
    for e in range(E):
        for a in range(A):
            want = lists[e][a]
            assert cnt[e, a] == len(want)
            assert list(idx[e, a, :len(want)]) == want, (e, a)


def _bitwise_case(cfgs, world, dtype, E, T, seed, obs=None, substeps=1, goal=False):
    A = len(cfgs)
    state = swarm(E, A, seed, spread=0.5)
    g = torch.Generator().manual_seed(seed + 1)
    acts = (torch.rand(T, E, A, 2, generator=g, dtype=D) * 2 - 1) * 1.5
    gt = torch.randn(E, A, 2, generator=g, dtype=D)

    def run():
        st = Stepper(cfgs, dt=0.05, substeps=substeps, device=DEV, dtype=dtype, world=world)
        if obs is not None:
            st.set_obstacles(to_obstacles(obs))
        st.track_neighbor_overflow = True
        st.track_grad_norm = True
        s = [x.to(DEV, dtype).requires_grad_(True) for x in state]
        a = acts.to(DEV, dtype).requires_grad_(True)
        sums = []
        if goal:
            loss = rollout_goal_loss(st, TorchState(*s), a, gt.to(DEV, dtype))
            sums.append(loss.detach().clone())
            out = []
        else:
            fin, traj = rollout(st, TorchState(*s), a)
            loss = sum((x * (i + 1)).sum() for i, x in enumerate(traj.stacked))
            out = [x.detach().clone() for x in traj.stacked]
        loss.backward()
        sums.append(st.last_grad_sqnorm.clone())
        return out + [a.grad, *[x.grad for x in s], st.last_true_count_max], sums

    ref, ref_sums = run()
    with cluster_env(2, 128):
        got, got_sums = run()
    for i, (x, y) in enumerate(zip(got, ref)):
        assert torch.equal(x, y), f"output {i} differs"
    # the goal loss and the gradient norm are sums of per-CTA partials: the cluster
    # kernels group the agents into other CTAs, so only the rounding of the sum may differ
    rtol = 1e-5 if dtype == torch.float32 else 1e-13
    for x, y in zip(got_sums, ref_sums):
        torch.testing.assert_close(x, y, rtol=rtol, atol=0.0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_cluster_bitwise_single_cta_holonomic(dtype):
    """300 agents as 3 CTAs of 128 (the last with 44 live threads) vs one CTA of 300."""
    cfgs = [AgentConfig(radius=0.03, max_speed=2.0, max_accel=4.0) for _ in range(300)]
    world = WorldConfig(collision_k=80.0, bounds=(-0.6, 0.6, -0.6, 0.6), neighbor_radius=0.1,
                        max_neighbors=6)
    _bitwise_case(cfgs, world, dtype, E=5, T=6, seed=3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_cluster_bitwise_single_cta_mixed_rk4_substeps_obstacles(dtype):
    A = 257  # odd: the scan table's pad slot
    models = [DynamicsModel.HOLONOMIC, DynamicsModel.DIFF_DRIVE, DynamicsModel.KINEMATIC_BICYCLE]
    modes = [ControlMode.VELOCITY, ControlMode.ACCELERATION, ControlMode.SERVO]
    cfgs = [AgentConfig(model=models[i % 3],
                        ctrl_mode=modes[(i // 3) % (3 if models[i % 3] == DynamicsModel.DIFF_DRIVE
                                                    else 2)], radius=0.025,
                        max_speed=1.5, max_accel=3.0, max_ang_vel=4.0, max_ang_accel=8.0,
                        max_steer=0.6, l_f=0.1, l_r=0.1) for i in range(A)]
    world = WorldConfig(collision_k=80.0, bounds=(-0.6, 0.6, -0.6, 0.6), neighbor_radius=0.09,
                        max_neighbors=A, integrator=Integrator.RK4)
    _bitwise_case(cfgs, world, dtype, E=3, T=4, seed=5, obs=obstacle_set(3, 1), substeps=2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_cluster_bitwise_single_cta_goal_loss(dtype):
    cfgs = [AgentConfig(radius=0.03, max_speed=2.0, max_accel=4.0) for _ in range(200)]
    world = WorldConfig(collision_k=80.0, bounds=(-0.6, 0.6, -0.6, 0.6), neighbor_radius=0.1,
                        max_neighbors=8)
    _bitwise_case(cfgs, world, dtype, E=4, T=5, seed=9, goal=True)


def test_oversized_and_unsupported_wide_envs():
    with pytest.raises(ValueError):
        Stepper([AgentConfig(radius=0.01)] * 4097, dt=0.05, device=DEV, dtype=torch.float32,
                world=WorldConfig(neighbor_radius=0.05, max_neighbors=8))
    with pytest.raises(NotImplementedError):
        from swarp_b200.dynamics.base import AgentShape
        Stepper([AgentConfig(shape=AgentShape.BOX, half_extents=(0.01, 0.01))] * 1100,
                dt=0.05, device=DEV, dtype=torch.float32,
                world=WorldConfig(neighbor_radius=0.05, max_neighbors=8))


def _f32_wide_case(E, A, T, K, seed):
    cfgs = [AgentConfig(radius=0.01, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.06, max_neighbors=K)
    g = torch.Generator().manual_seed(seed)
    pos = (torch.randn(E, A, 2, generator=g, dtype=D) * 0.3).clamp(-0.95, 0.95)
    z = torch.zeros(E, A, dtype=D)
    state = [pos, z, torch.zeros(E, A, 2, dtype=D), z, z]
    acts = torch.rand(T, E, A, 2, generator=g, dtype=D) * 2 - 1
    goal = torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1
    return cfgs, world, state, acts, goal


def _f32_wide_run(cfgs, world, state, acts, goal):
    f32 = lambda x: x.to(DEV, torch.float32)  # noqa: E731
    st = Stepper(cfgs, dt=0.05, device=DEV, dtype=torch.float32, world=world)
    st.track_neighbor_overflow = True
    a_gpu = f32(acts).requires_grad_(True)
    loss = rollout_goal_loss(st, TorchState(*map(f32, state)), a_gpu, f32(goal))
    (ga,) = torch.autograd.grad(loss, [a_gpu])
    _, traj = rollout(st, TorchState(*map(f32, state)), f32(acts))
    return ([x.detach().cpu() for x in traj.stacked], ga.cpu(), float(loss),
            int(st.last_true_count_max.max()))


def test_2048_agents_f32_goal_loss_against_cpu_restatement():
    """Float32, 2048 agents per env, holonomic velocity fleet, the fused goal loss.

    At 512 threads per CTA (4 CTAs) the forward's dynamic shared memory is exactly 48 KB,
    so the launch must raise the kernel's shared-memory limit; at 256 threads (8 CTAs, the
    portable maximum) the trajectories and gradients must be bitwise those of 4 CTAs (the
    same arithmetic in the same order whatever the cluster shape).

    Against the C restatement, with the float32 bars of the float32 parity tests (states
    1e-5, action gradients 1e-4 of the field's largest magnitude) where the problem allows
    them. This dense random swarm is ill-conditioned in float32 in two ways:
    - at the second step two agents of env 1 (1512 and 2038) are 3e-8 inside their contact
      distance in float64 and 2e-8 outside it in float32; the contact law's damping term
      is nonzero at touch, so the float32 evaluations (kernel and restatement alike) end
      1.3e-3 (positions) and 1% (velocities) away from float64 for those agents;
    - the closest pairs start about 1e-4 apart, so their contact normals amplify ulp-level
      differences about a thousandfold in the states, and more in the gradients (the
      normal's derivative scales with 1/|d|): moving the float32 restatement's start
      positions by one ulp moves its action gradient by up to 4% of the largest component.
    So states must lie within the larger of the bar and twice the float32 restatement's
    own distance from float64, and within 1e-4 of the float32 restatement; the action
    gradient within the larger of the bar, twice the float32 restatement's distance from
    float64, and twice the largest change that one-ulp moves of the start positions make
    in the float32 restatement's gradient (four seeded draws). The cluster adjoint's
    gradients are pinned to 1e-10 in float64 by the 2048-agent test above."""
    E, A, T, K = 4, 2048, 3, 128
    cfgs, world, state, acts, goal = _f32_wide_case(E, A, T, K, 21)
    with cluster_env(1025, 512):
        got, ga, loss, tmax = _f32_wide_run(cfgs, world, state, acts, goal)
    with cluster_env(1025, 256):
        got8, ga8, _, tmax8 = _f32_wide_run(cfgs, world, state, acts, goal)
    assert 0 < tmax <= K and tmax8 == tmax, "listed neighbors, no truncation"
    for f in range(5):
        assert torch.equal(got[f], got8[f]), f"field {f}: 4 vs 8 CTAs"
    assert torch.equal(ga, ga8)

    def restated(dt_, pos0):
        init = [pos0] + [x.numpy() for x in state[1:]]
        common = dict(params=param_rows(cfgs), model_tag=[int(c.model) for c in cfgs],
                      ctrl_mode=[int(c.ctrl_mode) for c in cfgs], dt=0.05, substeps=1,
                      collisions=True, k=100.0, c=1.0, margin=0.025, max_overlap=0.0,
                      neighbor_radius=0.06, max_neighbors=K, bounds_mode=1,
                      bounds=(-1.0, 1.0, -1.0, 1.0), init=init, actions=acts.numpy(),
                      obstacles=None, threads=0, dtype=dt_)
        tr, _, _ = cpu_port.rollout(**common)
        tr = [np.asarray(x, np.float64) for x in tr]
        _, gr, _ = cpu_port.rollout(**common, grad_final_pos=2.0 * (tr[0][-1] - goal.numpy()))
        return tr, np.asarray(gr, np.float64)

    def err(x, y):
        return float(np.abs(np.asarray(x, np.float64) - y).max())

    p32 = state[0].numpy().astype(np.float32)
    r64, g64 = restated(np.float64, state[0].numpy())
    r32, g32 = restated(np.float32, p32.astype(np.float64))
    for f in range(5):
        scale = max(np.abs(r64[f]).max(), 1e-12)
        assert err(got[f], r64[f]) <= max(1e-5 * scale, 2 * err(r32[f], r64[f])), \
            f"field {f} vs float64"
        assert err(got[f], r32[f]) <= 1e-4 * scale, f"field {f} vs float32 restatement"
    fin32 = r32[0][-1]
    assert loss == pytest.approx(float(((fin32 - goal.numpy()) ** 2).sum()), rel=1e-4)

    rng = np.random.default_rng(0)
    spread = 0.0
    for _ in range(4):
        sign = rng.choice([-1, 1], size=p32.shape).astype(np.float32)
        p1 = np.nextafter(p32, p32 + sign)
        spread = max(spread, err(restated(np.float32, p1.astype(np.float64))[1], g32))
    assert err(ga, g64) <= max(1e-4 * np.abs(g64).max(), 2 * err(g32, g64), 2 * spread)
