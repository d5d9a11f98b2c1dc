"""Host side of bench.py (no GPU): the seeded workloads of configs 1-5, the config-5 agent
override used to profile the cluster kernels, the command-line checks, and the CPU
restatement samples that the reference arm and the cpu_baseline leg time."""

from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

SHAPES = {1: (8, 32), 2: (16, 64), 3: (32, 50), 4: (4, 100), 5: (256, 32)}  # A, H


@pytest.mark.parametrize("cid", [1, 2, 3, 4, 5])
def test_workload_shapes_and_bytes(cid):
    wl = bench.build_workload(cid, n_envs=3, make_stepper=False)
    A, H = SHAPES[cid]
    assert (wl.E, wl.A, wl.H) == (3, A, H)
    assert wl.acts.shape[:3] == (H, 3, A) and wl.acts.dtype == np.float32
    assert wl.pos.shape == (3, A, 2)
    assert wl.name.startswith(f"config{cid}:")
    assert wl.algo_bytes_per_env_step == 80 * A + (48 if cid == 4 else 0)
    again = bench.build_workload(cid, n_envs=3, make_stepper=False)
    assert np.array_equal(wl.acts, again.acts) and np.array_equal(wl.pos, again.pos)
    other = bench.build_workload(cid, rank=1, n_envs=3, make_stepper=False)
    assert not np.array_equal(wl.acts, other.acts), "ranks draw their own inputs"


def test_config5_agent_override():
    wl = bench.build_workload(5, n_envs=2, n_agents=2048, make_stepper=False)
    assert (wl.E, wl.A) == (2, 2048)
    assert "2 envs x 2048 agents" in wl.name
    assert wl.acts.shape == (32, 2, 2048, 2)
    with pytest.raises(ValueError):
        bench.build_workload(2, n_envs=2, n_agents=2048, make_stepper=False)


@pytest.mark.parametrize("argv", [["--config", "2", "--agents", "10"],
                                  ["--impl", "reference", "--config", "5", "--agents", "2048"]])
def test_cli_rejects_agents_outside_config5(argv):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *argv],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 2
    assert "--agents applies to config 5" in r.stderr


def test_config_block_and_traffic():
    wl = bench.build_workload(1, n_envs=4, make_stepper=False)
    cfg = bench.config_block(wl, 2)
    assert cfg["n_envs_per_gpu"] == 4 and cfg["n_agents"] == 8 and cfg["horizon"] == 32
    assert cfg["parallelism"] == "env-sharded dp2"
    assert cfg["l2"].startswith("inputs smaller than L2")
    # the committed config-2 ncu summary carries both kernels' DRAM bytes per launch
    assert bench.profile_traffic(2, "fwd") > 0 and bench.profile_traffic(2, "bwd") > 0
    assert bench.profile_traffic(5, "fwd") is None


@pytest.mark.parametrize("cid", [1, 2, 3, 4, 5])
def test_cpu_samples_run(cid):
    """The samples the reference arm and the cpu_baseline leg time: inputs prepared
    untimed, the returned callable times only the restatement's rollout + adjoint."""
    s = bench.cpu_prepare(cid, 2)
    assert (s.cid, s.E, s.H) == (cid, 2, SHAPES[cid][1])
    assert s.run(1) > 0.0
