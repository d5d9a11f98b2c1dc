"""rollout_checkpointed (GPU): the state kept every `every` steps instead of the whole
trajectory. Final state and gradients equal rollout's bit for bit (ragged last segments,
substeps, obstacles, the paired 16-agent kernels, drones), and the peak device memory of a
long horizon drops with the trajectory."""

import pytest
import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel
from swarp_b200.interop.autograd import TorchState, rollout, rollout_checkpointed

from test_gpu_boxes import obstacle_mix
from test_gpu_drone import fleet as drone_fleet, state9, thrusts
from test_gpu_parity import cfgs_of, rand_actions, rand_state

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def grads(st, s, acts, every):
    leaves = [t.clone().requires_grad_(True) for t in s]
    a = acts.clone().requires_grad_(True)
    if every is None:
        fin, _ = rollout(st, TorchState(*leaves), a)
    else:
        fin = rollout_checkpointed(st, TorchState(*leaves), a, every=every)
    fin = tuple(fin)[:len(leaves)]
    g = torch.Generator(device=DEV).manual_seed(3)
    loss = sum((torch.randn(f.shape, generator=g, device=DEV, dtype=f.dtype) * f).sum() for f in fin)
    return [f.detach() for f in fin], torch.autograd.grad(loss, [a, *leaves])


def same(st, s, acts, everies):
    ref_fin, ref_g = grads(st, s, acts, None)
    for every in everies:
        fin, g = grads(st, s, acts, every)
        for x, y in zip(fin, ref_fin):
            assert torch.equal(x, y), every
        for x, y in zip(g, ref_g):
            assert torch.equal(x, y), every


def test_sixteen_agent_fleet_f32():
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=16)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0)] * 16, dt=0.05, device=DEV,
                 dtype=torch.float32, world=world)
    s = [t.to(DEV, torch.float32) for t in rand_state(64, 16, 1, spread=0.9)]
    same(st, s, rand_actions(20, 64, 16, 2).to(DEV, torch.float32), [1, 3, 8, 20, 64])


def test_mixed_fleet_obstacles_substeps_f64():
    world = WorldConfig(collision_k=40.0, collision_c=1.0, collision_margin=0.02,
                        bounds=(-0.6, 0.6, -0.6, 0.6))
    cfgs = (cfgs_of(DynamicsModel.HOLONOMIC, ControlMode.ACCELERATION, 3, radius=0.06)
            + cfgs_of(DynamicsModel.DIFF_DRIVE, ControlMode.SERVO, 2, radius=0.06)
            + cfgs_of(DynamicsModel.KINEMATIC_BICYCLE, ControlMode.ACCELERATION, 2, radius=0.06))
    st = Stepper(cfgs, dt=0.05, substeps=2, device=DEV, dtype=torch.float64, world=world)
    st.set_obstacles(obstacle_mix(4, 9))
    same(st, [t.to(DEV) for t in rand_state(4, 7, 10, spread=0.4)],
         rand_actions(11, 4, 7, 11).to(DEV), [2, 4, 5])


def test_drone_fleet_f64():
    world = WorldConfig(collision_k=40.0, collision_c=1.0, collision_margin=0.02,
                        bounds=(-0.5, 0.5, -0.5, 0.5))
    st = Stepper(drone_fleet(6), dt=0.02, device=DEV, dtype=torch.float64, world=world)
    same(st, [t.to(DEV) for t in state9(3, 6, 12, spread=0.4)], thrusts(9, 3, 6, 13).to(DEV),
         [2, 4])


def test_long_horizon_memory():
    """A 256-step horizon at 4000 x 16 agents: the plain rollout keeps 256 trajectory
    steps for the backward, the checkpointed one 16 checkpoints and one 16-step segment."""
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=16)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0)] * 16, dt=0.05, device=DEV,
                 dtype=torch.float32, world=world)
    s = [t.to(DEV, torch.float32) for t in rand_state(4000, 16, 21, spread=0.9)]
    acts = rand_actions(256, 4000, 16, 22).to(DEV, torch.float32)
    peaks = []
    for every in (None, 16):
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(DEV)
        base = torch.cuda.memory_allocated(DEV)
        grads(st, s, acts, every)
        torch.cuda.synchronize()
        peaks.append(torch.cuda.max_memory_allocated(DEV) - base)
    assert peaks[1] < 0.6 * peaks[0], peaks
