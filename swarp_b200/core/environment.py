"""VMAS-style vectorized Environment over a scenario.

Drop-in for the reference's ``swarp/core/environment.py`` (``Environment`` ``:18-749``):
constructor keywords, ``reset``/``reset_at``, and ``step(actions) -> (obs, reward,
terminated, truncated, info)`` with the same shape (``ValueError``) and dtype
(``TypeError``) checks (``:604-611``), ``max_steps`` truncation and masked
``auto_reset``. The physics step is the fused CUDA rollout kernel (T = 1); observation
and reward assembly are torch ops of the scenario. ``use_graph`` and ``fused`` are
accepted for compatibility: the step is already a single launch, and scenario
observations run on the torch path.
"""

from __future__ import annotations

from typing import Any

import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.dynamics.base import action_bounds


class Environment:
    def __init__(
        self,
        scenario,
        n_envs: int,
        device: str = "cuda:0",
        dt: float = 0.1,
        substeps: int = 1,
        dtype: torch.dtype = torch.float32,
        max_steps: int | None = None,
        seed: int = 0,
        auto_reset: bool = False,
        use_graph: bool | str = "auto",
        clone_outputs: bool = False,
        fused: bool | str = "auto",
        world_config: WorldConfig | None = None,
    ) -> None:
        if n_envs < 1:
            raise ValueError(f"n_envs must be >= 1, got {n_envs}")
        self.scenario = scenario
        self.n_envs = n_envs
        self.device = str(device)
        if not self.device.startswith("cuda") or not torch.cuda.is_available():
            raise RuntimeError(
                f"device {self.device!r}: swarp_b200 steps on a CUDA device only (no CPU path)"
            )
        self.dtype = dtype
        self.max_steps = max_steps
        self.auto_reset = auto_reset
        self.clone_outputs = clone_outputs
        self.world = scenario.make_world(n_envs=n_envs, device=self.device, dt=dt,
                                         substeps=substeps, dtype=dtype, world_config=world_config)
        self.n_agents = self.world.n_agents
        self._step_count = torch.zeros(n_envs, dtype=torch.int64, device=self.device)
        self._never_truncated = torch.zeros(n_envs, dtype=torch.bool, device=self.device)
        self.seed(seed)

    # ------------------------------------------------------------------ setup
    def seed(self, seed: int) -> None:
        self.world.generator = torch.Generator(device=self.device).manual_seed(seed)

    @property
    def action_dim(self) -> int:
        return self.world.act_dim

    @property
    def action_bounds(self) -> tuple[torch.Tensor, torch.Tensor]:
        """``(low, high)`` per agent and action slot, ``[n_agents, act_dim]``."""
        lo = torch.zeros(self.n_agents, self.world.act_dim, dtype=self.dtype)
        hi = torch.zeros(self.n_agents, self.world.act_dim, dtype=self.dtype)
        for i, cfg in enumerate(self.world.agent_configs):
            low, high = action_bounds(cfg)
            lo[i, : len(low)] = torch.tensor(low, dtype=self.dtype)
            hi[i, : len(high)] = torch.tensor(high, dtype=self.dtype)
        return lo.to(self.device), hi.to(self.device)

    # ------------------------------------------------------------------ reset
    def reset(self, seed: int | None = None) -> torch.Tensor:
        if seed is not None:
            self.seed(seed)
        with torch.no_grad():
            self.scenario.reset_world(None)
        self._step_count.zero_()
        return self.scenario.observations()

    def reset_at(self, env_mask: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            self.scenario.reset_world(env_mask)
        self._step_count.masked_fill_(env_mask, 0)
        return self.scenario.observations()

    # ------------------------------------------------------------------ step
    def step(self, actions: torch.Tensor):
        act_dim = self.world.act_dim
        if actions.shape != (self.n_envs, self.n_agents, act_dim):
            raise ValueError(f"actions must have shape {(self.n_envs, self.n_agents, act_dim)}, "
                             f"got {tuple(actions.shape)}")
        if actions.dtype != self.dtype:
            raise TypeError(f"actions dtype {actions.dtype} != env dtype {self.dtype}")
        self.world.action = actions
        self.world.step(actions)
        self.scenario.post_step()
        reward = self.scenario.rewards()
        self._step_count += 1
        terminated = self.scenario.done()
        if self.max_steps is not None:
            truncated = self._step_count >= self.max_steps
        else:
            truncated = self._never_truncated
        info: dict[str, Any] = self.scenario.info()
        if self.auto_reset:
            ended = terminated | truncated
            with torch.no_grad():
                self.scenario.reset_world(ended, obs_only=True)
            self._step_count.masked_fill_(ended, 0)
        obs = self.scenario.observations()
        if self.clone_outputs:
            obs, reward = obs.clone(), reward.clone()
            terminated, truncated = terminated.clone(), truncated.clone()
            info = {k: v.clone() if torch.is_tensor(v) else v for k, v in info.items()}
        return obs, reward, terminated, truncated, info

    def radius_graph(self) -> torch.Tensor:
        """COO edge index ``[2, n_edges]`` of the current within-radius neighbor graph."""
        return self.world.edge_index()
