"""Host-side API contract (CPU only): keyword routing of ``make``, loud failure without
CUDA (no CPU fallback), configuration validation mirrored from the reference."""

import pytest
import torch

import swarp_b200 as swarp
from swarp_b200.core.config import WorldConfig
from swarp_b200.dynamics.base import AgentConfig, AgentShape, ControlMode, DynamicsModel


def test_make_rejects_unknown_scenario():
    with pytest.raises(ValueError, match="unknown scenario"):
        swarp.make("no-such-scenario", n_envs=4)


def test_make_rejects_unknown_keyword_and_suggests_environment_keyword():
    with pytest.raises(TypeError, match="not a keyword"):
        swarp.make("navigation", n_envs=4, n_agnets=3)
    with pytest.raises(TypeError, match="Did you mean Environment's 'device'"):
        swarp.make("navigation", n_envs=4, devcie="cuda:0")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_no_cpu_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        swarp.Stepper([AgentConfig()], device="cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        swarp.make("navigation", n_envs=2, device="cuda:0")


def test_agent_config_validation_matches_reference():
    with pytest.raises(ValueError, match="diff-drive mode"):
        AgentConfig(model=DynamicsModel.HOLONOMIC, ctrl_mode=ControlMode.SERVO)
    with pytest.raises(ValueError, match="min_speed"):
        AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=2.0, min_speed=-3.0)
    assert AgentConfig(model="diff-drive").model == DynamicsModel.DIFF_DRIVE
    box = AgentConfig(shape=AgentShape.BOX, half_extents=(3.0, 4.0))
    assert box.radius == 5.0
    row = AgentConfig(model=DynamicsModel.KINEMATIC_BICYCLE, max_speed=2.0).to_row()
    assert row[swarp.P_MIN_SPEED] == -2.0 and len(row) == swarp.NUM_PARAMS


def test_world_config_validation_and_override():
    with pytest.raises(ValueError):
        WorldConfig(bounds_mode="bouncy")
    with pytest.raises(ValueError):
        WorldConfig(bounds=(1.0, -1.0, 0.0, 1.0))
    base = WorldConfig(collision_k=100.0, bounds=(-1, 1, -1, 1))
    over = base.override_with(WorldConfig(collision_k=50.0))
    assert over.collision_k == 50.0 and over.bounds == (-1, 1, -1, 1)


def test_neighbor_method_validation_matches_reference():
    """swarp/core/neighbors.py:376-379, 391-394: with collisions on, a zero list radius,
    unknown methods and bins below 1 raise (checked before anything touches the device)."""
    with pytest.raises(ValueError, match="method must be"):
        swarp.Stepper([AgentConfig()], device="cuda:0",
                      world=WorldConfig(neighbor_method="octree"))
    with pytest.raises(ValueError, match="uniform_bins"):
        swarp.Stepper([AgentConfig()], device="cuda:0",
                      world=WorldConfig(neighbor_method="uniform_grid", uniform_bins=0))
    with pytest.raises(ValueError, match="radius must be positive"):
        swarp.Stepper([AgentConfig(radius=0.0)], device="cuda:0",
                      world=WorldConfig(collision_margin=0.0))


def test_action_bounds_table():
    lo, hi = swarp.action_bounds(AgentConfig(model=DynamicsModel.DIFF_DRIVE, max_speed=2.0,
                                             max_ang_vel=3.0))
    assert lo == [-2.0, -3.0] and hi == [2.0, 3.0]


def test_streamed_chunk_count():
    """StreamedRollout splits the batch into the most equal env chunks up to the asked
    count (equal chunks replay one captured step)."""
    from swarp_b200.interop.streamed import _chunks

    assert _chunks(16000, 2) == 2 and _chunks(16000, 3) == 2 and _chunks(12, 5) == 4
    assert _chunks(7, 4) == 1 and _chunks(3, 8) == 3 and _chunks(1, 1) == 1
