"""Neighbor membership at the radius, bit for bit.

The reference keeps b in a's list when ``wp.length(p_b - p_a) <= radius``
(swarp/core/neighbors.py:91): in the working precision, sqrt(dx*dx + dy*dy) <= R with
every operation rounded (no contraction). These tests place agents on a circle of radius
R around a centre agent, on the axes, the diagonals and random directions, each
coordinate moved by up to two ulps, so that pairs fall exactly on, just inside and just
outside the threshold, and compare the kernels' lists, counts and uncapped counts
with that rule restated in numpy in the same precision.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig
from swarp_b200.interop.autograd import TorchState, rollout

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
R_NB = 0.125


def ring_positions(E: int, A: int, R: float, ftype, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    f = ftype
    pos = np.empty((E, A, 2), f)
    for e in range(E):
        # dyadic centres in the first envs (exactly representable offsets on the axes)
        c = (np.array([0.25, -0.375]) if e < 2 else rng.uniform(-0.6, 0.6, 2)).astype(f)
        pos[e, 0] = c
        for a in range(1, A):
            k = int(rng.integers(0, 12))
            phi = k * np.pi / 4 if k < 8 else rng.uniform(0.0, 2 * np.pi)
            b = np.array([c[0] + R * np.cos(phi), c[1] + R * np.sin(phi)]).astype(f)
            if e >= 1:  # env 0 keeps the exact ring
                for i in range(2):
                    n = int(rng.integers(-2, 3))
                    for _ in range(abs(n)):
                        b[i] = np.nextafter(b[i], f(np.inf) if n > 0 else f(-np.inf))
            pos[e, a] = b
    return pos


def truth(pos: np.ndarray, R: float, K: int):
    """The reference's rule in pos.dtype: lists (ascending, capped at K), counts, true counts."""
    f = pos.dtype.type
    d = pos[:, None, :, :] - pos[:, :, None, :]  # [E, a, b, 2] = p_b - p_a
    s = d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]
    inr = np.sqrt(s) <= f(R)
    E, A = pos.shape[:2]
    inr &= ~np.eye(A, dtype=bool)[None]
    lists = [[list(np.nonzero(inr[e, a])[0][:K]) for a in range(A)] for e in range(E)]
    return lists, inr.sum(-1), s


def exact_hits(pos, R):
    """How many pairs sit exactly on the threshold (s == largest value with sqrt <= R)."""
    f = pos.dtype.type
    _, _, s = truth(pos, R, 1)
    thr = f(R) * f(R)
    while np.sqrt(np.nextafter(thr, f(np.inf))) <= f(R):
        thr = np.nextafter(thr, f(np.inf))
    while np.sqrt(thr) > f(R):
        thr = np.nextafter(thr, f(-np.inf))
    return int((s == thr).sum()), int((np.abs(s - thr) <= 4 * np.spacing(thr)).sum())


def stepper(A: int, K: int, dtype) -> Stepper:
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        neighbor_radius=R_NB, max_neighbors=K, bounds=(-1.0, 1.0, -1.0, 1.0))
    cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
    return Stepper(cfgs, dt=0.05, device=DEV, dtype=dtype, world=world)


@pytest.mark.parametrize("dtype,A,K", [(torch.float32, 16, 16), (torch.float32, 12, 4),
                                       (torch.float32, 40, 8), (torch.float64, 16, 16),
                                       (torch.float64, 40, 8)])
def test_neighbor_lists_at_the_radius(dtype, A, K):
    ft = np.float32 if dtype == torch.float32 else np.float64
    pos = ring_positions(96, A, R_NB, ft, seed=A + K)
    on, near = exact_hits(pos, R_NB)
    assert near > 50, "the generator must put pairs within a few ulps of the threshold"
    lists, tru, _ = truth(pos, R_NB, K)
    st = stepper(A, K, dtype)
    idx, cnt, tc = st.neighbors(torch.from_numpy(pos).to(DEV))
    idx, cnt, tc = idx.cpu().numpy(), cnt.cpu().numpy(), tc.cpu().numpy()
    assert np.array_equal(tc, tru)
    assert np.array_equal(cnt, np.minimum(tru, K))
    for e in range(pos.shape[0]):
        for a in range(A):
            assert list(idx[e, a, :cnt[e, a]]) == lists[e][a], (e, a)
    if dtype == torch.float32 and A == 16:
        assert on > 0, "no pair exactly on the float32 threshold"


@pytest.mark.parametrize("dtype,A,K", [(torch.float32, 16, 16), (torch.float32, 12, 4),
                                       (torch.float32, 40, 8), (torch.float64, 16, 16)])
def test_rollout_counts_at_the_radius(dtype, A, K):
    """The rollout kernels' own scan (the two-agents-per-thread float kernel at 16 agents,
    the one-agent kernels otherwise): the uncapped count of the first substep equals the
    reference rule's at the initial positions."""
    ft = np.float32 if dtype == torch.float32 else np.float64
    pos = ring_positions(96, A, R_NB, ft, seed=7 * A + K)
    _, tru, _ = truth(pos, R_NB, K)
    st = stepper(A, K, dtype)
    st.track_neighbor_overflow = True
    E = pos.shape[0]
    p = torch.from_numpy(pos).to(DEV)
    z = torch.zeros(E, A, dtype=dtype, device=DEV)
    state = TorchState(p, z, torch.zeros(E, A, 2, dtype=dtype, device=DEV), z, z)
    acts = torch.zeros(1, E, A, 2, dtype=dtype, device=DEV)
    with torch.no_grad():
        rollout(st, state, acts)
    assert np.array_equal(st.last_true_count_max.cpu().numpy(), tru)
