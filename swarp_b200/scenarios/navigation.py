"""Navigation scenario (the caller of the hot path in the reference's benchmarks).

World construction follows ``NavigationScenario.make_world`` of the reference
(``swarp/scenarios/navigation.py:127-200``: contact constants k = 100, c = 1, margin
0.5 r, soft walls at +-world_size, neighbor radius max(user, 2 r + margin),
max_neighbors min(32, max(4, n_agents))). Resets draw separated spawns and goals with the
reference's stratified jittered-cell construction (``_sample_separated``, ``:222-272``);
observations, shaped rewards, termination and info follow its torch path
(``:671-839``). These are torch ops around the fused CUDA step; they are not the hot
path and have no CUDA kernels of their own.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from swarp_b200.core.config import WorldConfig
from swarp_b200.core.world import World
from swarp_b200.dynamics.base import AgentConfig, ControlMode, DynamicsModel


class NavigationScenario:
    def __init__(
        self,
        n_agents: int = 4,
        agent_radius: float = 0.05,
        model: DynamicsModel = DynamicsModel.HOLONOMIC,
        ctrl_mode: ControlMode = ControlMode.VELOCITY,
        max_speed: float = 1.0,
        world_size: float = 1.0,
        n_obstacles: int = 0,
        obstacle_radius: float = 0.1,
        neighbor_obs: int = 2,
        neighbor_radius: float | None = None,
        shared_reward: bool = False,
        pos_shaping_factor: float = 1.0,
        collision_penalty: float = -1.0,
        final_reward: float = 5.0,
        goal_tolerance: float | None = None,
        min_spawn_separation: float | None = None,
        neighbor_method: str = "auto",
    ) -> None:
        self.n_agents = n_agents
        self.agent_radius = agent_radius
        self.model = model
        self.ctrl_mode = ctrl_mode
        self.max_speed = max_speed
        self.world_size = world_size
        self.n_obstacles = n_obstacles
        self.obstacle_radius = obstacle_radius
        self.neighbor_obs = neighbor_obs
        self.neighbor_radius = neighbor_radius
        self.shared_reward = shared_reward
        self.pos_shaping_factor = pos_shaping_factor
        self.collision_penalty = collision_penalty
        self.final_reward = final_reward
        self.goal_tolerance = goal_tolerance if goal_tolerance is not None else agent_radius
        self.min_spawn_separation = (
            min_spawn_separation if min_spawn_separation is not None else 3.0 * agent_radius
        )
        self.neighbor_method = neighbor_method
        self._k_obs = min(self.neighbor_obs, min(32, max(4, self.n_agents)))
        self.world: World | None = None
        self._cache: dict[str, Any] | None = None
        self._prev_dist: torch.Tensor | None = None

    @property
    def obs_dim(self) -> int:
        return 9 + 5 * self._k_obs

    def _agent_configs(self) -> list[AgentConfig]:
        return [AgentConfig(model=self.model, ctrl_mode=self.ctrl_mode, radius=self.agent_radius,
                            max_speed=self.max_speed, max_accel=2.0 * self.max_speed)
                for _ in range(self.n_agents)]

    def make_world(self, n_envs, device, dt, substeps, dtype, world_config=None) -> World:
        margin = 0.5 * self.agent_radius
        reach = 2.0 * self.agent_radius + margin
        cfg = WorldConfig(
            collisions=True, collision_k=100.0, collision_c=1.0, collision_margin=margin,
            bounds=(-self.world_size, self.world_size, -self.world_size, self.world_size),
            bounds_mode="soft", neighbor_radius=max(self.neighbor_radius or 0.0, reach),
            max_neighbors=min(32, max(4, self.n_agents)), neighbor_method=self.neighbor_method,
        ).override_with(world_config)
        self.world = World(self._agent_configs(), cfg, n_envs=n_envs, device=device, dt=dt,
                           substeps=substeps, dtype=dtype)
        self.world.goals = torch.zeros(n_envs, self.n_agents, 2, device=device, dtype=dtype)
        self._k_obs = min(self.neighbor_obs, cfg.max_neighbors)
        if self.n_obstacles > 0:
            from swarp_b200.core.config import Obstacles

            tt = {"device": device, "dtype": dtype}
            self.world.set_obstacles(Obstacles(torch.zeros(n_envs, self.n_obstacles, 2, **tt),
                                               torch.full((self.n_obstacles,), self.obstacle_radius,
                                                          **tt)))
        return self.world

    # ----------------------------------------------------------------- reset
    def _sample_separated(self, n_envs: int, n_points: int, min_dist: float) -> torch.Tensor:
        """Spawn points with pairwise separation >= min_dist (stratified jittered cells)."""
        w = self.world
        lim = self.world_size - 2.0 * self.agent_radius
        shape = (n_envs, n_points, 2)
        if n_points == 1 or min_dist <= 0.0:
            return w.sample_uniform(shape, -lim, lim)
        side = 2.0 * lim
        g = math.ceil(math.sqrt(n_points * 8))
        g = min(g, int(side // (2.0 * min_dist)))
        g = max(g, math.ceil(math.sqrt(n_points)))
        if side / g <= min_dist:
            return w.sample_uniform(shape, -lim, lim)
        s = side / g
        jitter = s - min_dist
        cell = w.sample_uniform((n_envs, g * g), 0.0, 1.0).argsort(dim=-1)[:, :n_points]
        col = (cell % g).to(w.dtype)
        row = torch.div(cell, g, rounding_mode="floor").to(w.dtype)
        centers = torch.stack([col, row], dim=-1) * s + (0.5 * s - lim)
        return centers + (w.sample_uniform(shape, 0.0, 1.0) - 0.5) * jitter

    def reset_world(self, env_mask: torch.Tensor | None = None, *, obs_only: bool = False) -> None:
        w = self.world
        E = w.n_envs
        pos = self._sample_separated(E, self.n_agents, self.min_spawn_separation)
        goals = self._sample_separated(E, self.n_agents, self.min_spawn_separation)
        theta = w.sample_uniform((E, self.n_agents), -math.pi, math.pi)
        z = torch.zeros(E, self.n_agents, device=w.device, dtype=w.dtype)
        w.write_state(env_mask, pos=pos, theta=theta, vel=torch.zeros_like(pos), speed=z,
                      ang_vel=z)
        if env_mask is None:
            w.goals.copy_(goals)
        else:
            w.goals.copy_(torch.where(env_mask.view(-1, 1, 1), goals, w.goals))
        if self.n_obstacles > 0:
            lim = self.world_size - self.obstacle_radius
            obs_pos = w.sample_uniform((E, self.n_obstacles, 2), -lim, lim)
            cur = w.obstacles.pos
            w.obstacles.pos = obs_pos if env_mask is None else torch.where(
                env_mask.view(-1, 1, 1), obs_pos, cur)
            w.obstacles._resolved_for = None
            w.set_obstacles(w.obstacles)
        self._refresh(reset_mask=env_mask if env_mask is not None else
                      torch.ones(E, dtype=torch.bool, device=w.device))

    def post_step(self) -> None:
        self._refresh(None)

    # --------------------------------------------------------- obs / rewards
    def _refresh(self, reset_mask: torch.Tensor | None) -> None:
        w = self.world
        pos, vel = w.state.pos, w.state.vel
        idx, cnt = w.neighbors()
        idx_long = idx.long()
        k_all = idx.shape[-1]
        k = min(self.neighbor_obs, k_all)
        arange_k = torch.arange(k_all, device=pos.device)
        valid = arange_k.view(1, 1, -1) < cnt.long().unsqueeze(-1)
        flat = idx_long.reshape(w.n_envs, -1)
        npos = torch.gather(pos, 1, flat.unsqueeze(-1).expand(-1, -1, 2)).view(
            w.n_envs, w.n_agents, k_all, 2)
        rel_all = npos - pos.unsqueeze(2)
        r = w.agent_radius
        touching = ((rel_all.norm(dim=-1) < r.view(1, -1, 1) + r[idx_long]) & valid).sum(-1).to(w.dtype)
        rel_pos = rel_all[:, :, :k] * valid[:, :, :k].unsqueeze(-1)
        flat_k = idx_long[:, :, :k].reshape(w.n_envs, -1)
        nvel = torch.gather(vel, 1, flat_k.unsqueeze(-1).expand(-1, -1, 2)).view(
            w.n_envs, w.n_agents, k, 2)
        rel_vel = (nvel - vel.unsqueeze(2)) * valid[:, :, :k].unsqueeze(-1)
        dist = (pos - w.goals).norm(dim=-1)
        if self._prev_dist is None:
            self._prev_dist = dist.detach().clone()
        shaping = (self._prev_dist - dist) * self.pos_shaping_factor
        if reset_mask is None:
            self._prev_dist = dist.detach().clone()
        else:
            m = reset_mask.unsqueeze(-1)
            shaping = torch.where(m, torch.zeros_like(shaping), shaping)
            self._prev_dist = torch.where(m, dist.detach(), self._prev_dist)
        self._cache = {"rel_pos": rel_pos, "rel_vel": rel_vel, "valid": valid, "touching": touching,
                       "dist_to_goal": dist, "on_goal": dist < self.goal_tolerance,
                       "pos_shaping": shaping, "neighbor_overflow": w.neighbor_overflow()}

    def observations(self) -> torch.Tensor:
        w = self.world
        s = w.state
        c = self._cache
        feats = [s.pos, s.vel, torch.cos(s.theta).unsqueeze(-1), torch.sin(s.theta).unsqueeze(-1),
                 s.ang_vel.unsqueeze(-1), w.goals - s.pos]
        k = min(self.neighbor_obs, c["rel_pos"].shape[2])
        if k > 0:
            E, A = w.n_envs, w.n_agents
            feats += [c["rel_pos"][:, :, :k].reshape(E, A, -1),
                      c["rel_vel"][:, :, :k].reshape(E, A, -1), c["valid"][:, :, :k].to(w.dtype)]
        return torch.cat(feats, dim=-1)

    def rewards(self) -> torch.Tensor:
        c = self._cache
        rew = self.collision_penalty * c["touching"]
        if self.shared_reward:
            rew = rew + c["pos_shaping"].sum(dim=-1, keepdim=True)
        else:
            rew = rew + c["pos_shaping"]
        final = self.final_reward * c["on_goal"].all(dim=-1).to(self.world.dtype)
        return rew + final.unsqueeze(-1)

    def done(self) -> torch.Tensor:
        return self._cache["on_goal"].all(dim=-1)

    def info(self) -> dict[str, Any]:
        c = self._cache
        return {"dist_to_goal": c["dist_to_goal"], "on_goal": c["on_goal"],
                "collisions": c["touching"], "neighbor_overflow": c["neighbor_overflow"]}
