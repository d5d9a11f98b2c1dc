"""The oracle's restatement of the reference's radix-sort uniform grid
(oracle/torch_ref.py ``uniform_grid_neighbors``), which ``neighbor_method="auto"`` picks
above 512 agents per env (swarp/core/neighbors.py:388-389).

Pinned by the reference's own uniform-grid tests, restated (tests/unit/test_neighbors.py:
79-135): without truncation the grid's counts, true counts and sets equal brute force's,
with the frame from the batch or pinned to a world rectangle, and for points outside that
rectangle. Then the list order: the grid lists in (3 x 3 block cell, index) order, so a
truncating list keeps a different set than brute force's ascending-index one; that
difference is the one the CUDA path (ascending index for every method) has against the
reference for truncating lists in envs above 512 agents. The C restatement
(oracle/cpu_port.c, ``grid=``) lists in the same grid order with a static frame, and the
two restatements agree through a truncating rollout and its adjoint.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import torch_ref as R


def make_positions(seed, n_envs, n_agents, extent=2.0):
    rng = np.random.default_rng(seed)
    return torch.from_numpy((rng.random((n_envs, n_agents, 2)) * 2.0 - 1.0) * extent)


def sets(idx, cnt):
    E, A, _ = idx.shape
    return [[set(idx[e, a, : cnt[e, a]].tolist()) for a in range(A)] for e in range(E)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("n_envs,n_agents", [(1, 8), (4, 32), (2, 128), (2, 600)])
@pytest.mark.parametrize("radius", [0.15, 0.5])
@pytest.mark.parametrize("bounds", [None, (-2.0, 2.0, -2.0, 2.0)])
def test_uniform_grid_matches_brute_force(dtype, n_envs, n_agents, radius, bounds):
    pos = make_positions(42, n_envs, n_agents).to(dtype)
    _, u_idx, u_cnt, u_true = R.uniform_grid_neighbors(pos, radius, 128, bounds=bounds)
    _, b_idx, b_cnt, b_true = R.brute_neighbors(pos, radius, 128)
    assert torch.equal(u_cnt, b_cnt) and torch.equal(u_true, b_true)
    assert not (b_true > 128).any(), "config truncated; widen max_neighbors"
    assert sets(u_idx, u_cnt) == sets(b_idx, b_cnt)


def test_static_frame_holds_for_points_outside_the_rectangle():
    pos = make_positions(11, 3, 64, extent=3.0).to(torch.float32)
    _, u_idx, u_cnt, u_true = R.uniform_grid_neighbors(pos, 0.3, 128, bounds=(-1, 1, -1, 1))
    _, b_idx, b_cnt, b_true = R.brute_neighbors(pos, 0.3, 128)
    assert torch.equal(u_cnt, b_cnt) and torch.equal(u_true, b_true)
    assert sets(u_idx, u_cnt) == sets(b_idx, b_cnt)


def test_frame_and_bins():
    assert R.default_uniform_bins(8) == 4 and R.default_uniform_bins(600) == 25
    assert R.default_uniform_bins(2048) == 46 and R.default_uniform_bins(10 ** 6) == 128
    assert R.auto_neighbor_method(512) == "brute"
    assert R.auto_neighbor_method(513) == "uniform_grid"
    pos = make_positions(3, 2, 16).to(torch.float32)
    origin, cell = R.uniform_grid_frame(pos, 0.1, 4, bounds=(-1.0, 1.0, -0.5, 0.5))
    assert origin.tolist() == [-1.0, -0.5] and float(cell) == pytest.approx(0.5)
    origin, cell = R.uniform_grid_frame(pos, 0.1, 4)  # the batch's own corner and extent
    lo = pos.reshape(-1, 2).min(0).values
    ext = float((pos.reshape(-1, 2).max(0).values - lo).max())
    assert torch.equal(origin, lo) and float(cell) == pytest.approx(ext / 4, rel=1e-6)


def test_grid_list_order_and_truncation():
    """Every list is the in-radius set sorted by (block cell, index), cut at K; with K
    below the true counts the kept sets differ from the ascending-index ones."""
    pos = make_positions(5, 2, 600).to(torch.float32)
    radius, K, bins = 0.3, 6, R.default_uniform_bins(600)
    origin, cell = R.uniform_grid_frame(pos, radius, bins, bounds=(-2, 2, -2, 2))
    c = ((pos - origin) / cell).to(torch.int32).clamp(0, bins - 1)
    _, u_idx, u_cnt, u_true = R.uniform_grid_neighbors(pos, radius, K, bounds=(-2, 2, -2, 2))
    _, b_idx, b_cnt, b_true = R.brute_neighbors(pos, radius, K)
    assert torch.equal(u_cnt, b_cnt) and torch.equal(u_true, b_true)
    assert int((b_true > K).sum()) > 100, "the case truncates"
    for e in range(2):
        for a in range(0, 600, 7):
            lst = u_idx[e, a, : u_cnt[e, a]].tolist()
            keys = [((int(c[e, b, 1]) - int(c[e, a, 1]) + 1) * 3
                     + int(c[e, b, 0]) - int(c[e, a, 0]) + 1, b) for b in lst]
            assert all(0 <= k[0] <= 8 for k in keys)
            assert keys == sorted(keys), "cell-major, ascending index within a cell"
    differ = sum(s != t for su, sb in zip(sets(u_idx, u_cnt), sets(b_idx, b_cnt))
                 for s, t in zip(su, sb))
    assert differ > 0, "truncated lists keep different sets in grid and index order"


def _grid_rollouts(E, A, T, K, seed, bins, bounds=(-1.0, 1.0, -1.0, 1.0), R_=0.12):
    """One truncating case through both restatements with grid-ordered lists, float64."""
    from oracle import cpu_port
    from swarp_b200.dynamics.base import AgentConfig, param_rows

    cfgs = [AgentConfig(radius=0.03, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    D = torch.float64
    g = torch.Generator().manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, dtype=D) * 2 - 1) * 0.9
    z = torch.zeros(E, A, dtype=D)
    vel = torch.randn(E, A, 2, generator=g, dtype=D) * 0.3
    acts = (torch.rand(T, E, A, 2, generator=g, dtype=D) * 2 - 1)
    gf = torch.randn(E, A, 2, generator=g, dtype=D)
    params = param_rows(cfgs)
    tags = [int(c.model) for c in cfgs]
    modes = [int(c.ctrl_mode) for c in cfgs]
    out = {}
    for method in ("uniform_grid", "brute"):
        w = R.RefWorld(params=torch.tensor(params), model_tag=tags, ctrl_mode=modes, dt=0.05,
                       k=60.0, c=1.0, margin=0.02, neighbor_radius=R_, max_neighbors=K,
                       bounds=bounds, soft_walls=True, neighbor_method=method,
                       uniform_bins=bins)
        st = [x.clone().requires_grad_(True) for x in (pos, z, vel, z, z)]
        a = acts.clone().requires_grad_(True)
        fin, traj, _ = R.rollout(tuple(st), a, w, None)
        (fin[0] * gf).sum().backward()
        ref = [torch.stack([traj[t][f] for t in range(T)]).detach().numpy() for f in range(5)]
        out[method] = (ref, a.grad.numpy())
    traj_c, ga_c, _ = cpu_port.rollout(
        params=params, model_tag=tags, ctrl_mode=modes, dt=0.05, substeps=1, collisions=True,
        k=60.0, c=1.0, margin=0.02, max_overlap=0.0, neighbor_radius=R_, max_neighbors=K,
        bounds_mode=1, bounds=bounds, init=[x.numpy() for x in (pos, z, vel, z, z)],
        actions=acts.numpy(), grad_final_pos=gf.numpy(), threads=2, dtype=np.float64,
        grid=(bins, bounds))
    return out, traj_c, ga_c


def test_cpu_port_grid_order_matches_torch_oracle():
    """The C restatement's grid-ordered lists (static frame) against the torch oracle's,
    through a truncating rollout and its adjoint; and the grid order changes the result
    against ascending-index lists (the lists truncate)."""
    out, traj_c, ga_c = _grid_rollouts(E=2, A=300, T=3, K=4, seed=9, bins=17)
    ref, ga = out["uniform_grid"]
    for f in range(5):
        np.testing.assert_allclose(traj_c[f], ref[f], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(ga_c, ga, rtol=1e-9, atol=1e-9 * np.abs(ga).max())
    idx_ref, _ = out["brute"]
    assert np.abs(idx_ref[2] - ref[2]).max() > 1e-3, "grid and index order keep other members"
