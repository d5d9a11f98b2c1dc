"""World: one batched multi-agent world ([n_envs, n_agents] on one CUDA device).

Drop-in for the reference's ``swarp/core/world.py`` (``World`` ``:35-491``): the
state tensors, ``step``, the reset primitive ``write_state``, obstacle install and live
views, and the neighbor-list views (``neighbors``, ``neighbor_overflow``,
``edge_index``). Stepping goes through :func:`~swarp_b200.interop.autograd.warp_step`
(one fused CUDA launch per step, or its adjoint under autograd). The reference's
persistent-buffer / CUDA-graph runtime (``enable_persistent``) is a Warp launch-overhead
workaround; here it is accepted and is a no-op, the step being a single launch already.
"""

from __future__ import annotations

import torch

from swarp_b200.core.config import Obstacles, WorldConfig
from swarp_b200.core.stepper import Stepper
from swarp_b200.dynamics.base import AgentConfig, action_dim
from swarp_b200.interop.autograd import TorchState, warp_step


class World:
    def __init__(
        self,
        agent_configs: list[AgentConfig],
        world_config: WorldConfig | None = None,
        n_envs: int = 1,
        device: str = "cuda:0",
        dt: float = 0.1,
        substeps: int = 1,
        dtype: torch.dtype = torch.float32,
    ) -> None:
        if n_envs < 1:
            raise ValueError(f"n_envs must be >= 1, got {n_envs}")
        if dtype not in (torch.float32, torch.float64):
            raise TypeError(f"unsupported dtype {dtype!r} for World; supported: torch.float32, "
                            "torch.float64")
        self.n_envs = n_envs
        self.n_agents = len(agent_configs)
        self.device = str(device)
        self.dtype = dtype
        self.agent_configs = agent_configs
        self.act_dim = max(action_dim(c.model) for c in agent_configs)
        self.config = world_config
        self.stepper = Stepper(agent_configs, dt=dt, substeps=substeps, device=device, dtype=dtype,
                               world=world_config)
        self.state: TorchState = self.zero_state()
        self.action: torch.Tensor | None = None
        self.goals: torch.Tensor | None = None
        self.obstacles: Obstacles | None = None
        self.generator: torch.Generator | None = None
        self.agent_radius = torch.tensor([c.radius for c in agent_configs], device=device,
                                         dtype=dtype)
        self._nbr_version = -1
        self._state_version = 0
        self._nbr: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None
        self.ran_post_physics = False

    # ------------------------------------------------------------------ state
    def zero_state(self) -> TorchState:
        e, a = self.n_envs, self.n_agents

        def z(*shape):
            return torch.zeros(*shape, device=self.device, dtype=self.dtype)

        return TorchState(pos=z(e, a, 2), theta=z(e, a), vel=z(e, a, 2), speed=z(e, a),
                          ang_vel=z(e, a))

    def step(self, actions: torch.Tensor) -> None:
        """Advance one step (differentiable when grads are enabled)."""
        self.state = warp_step(self.stepper, self.state, actions)
        self._state_version += 1

    def enable_persistent(self, use_graph: bool = True, *, graph_requested: bool = True) -> None:
        """Accepted for API compatibility; the fused step needs no persistent runtime."""

    def write_state(self, mask: torch.Tensor | None = None, *, pos=None, theta=None, vel=None,
                    speed=None, ang_vel=None) -> None:
        """Write agent state fields in place, optionally only into the masked envs."""
        for name, value in (("pos", pos), ("theta", theta), ("vel", vel), ("speed", speed),
                            ("ang_vel", ang_vel)):
            if value is None:
                continue
            dst = getattr(self.state, name).data
            if mask is None:
                dst.copy_(value.expand_as(dst) if torch.is_tensor(value) else value)
            else:
                m = mask.view(-1, *([1] * (dst.dim() - 1)))
                dst.copy_(torch.where(m, value, dst))
        if pos is not None:
            self.mark_pos_dirty()

    def reset_state(self) -> None:
        self.state = self.zero_state()
        self.mark_pos_dirty()

    def sample_uniform(self, shape, low: float, high: float) -> torch.Tensor:
        u = torch.rand(shape, generator=self.generator, device=self.device, dtype=self.dtype)
        return u * (high - low) + low

    # -------------------------------------------------------------- obstacles
    def set_obstacles(self, obstacles: Obstacles) -> None:
        obs = obstacles.resolve(self.device, self.dtype)
        self.obstacles = obs
        self.stepper.set_obstacles(obs)

    @property
    def obstacle_pos(self):
        return None if self.obstacles is None else self.obstacles.pos

    def obstacle_state_views(self, body: bool = False):
        """Live ``(pos, angle, vel, ang_vel)`` per shape (or per body slot with ``body``)."""
        st = self.stepper
        if body:
            return st.body_state
        o = st.obstacles
        return o.pos, o.angle, o.vel, o.ang_vel

    # -------------------------------------------------------------- neighbors
    def build_neighbors(self) -> None:
        if not self.stepper.collisions:
            raise RuntimeError("neighbor lists require WorldConfig.collisions=True")
        if self._nbr_version != self._state_version or self._nbr is None:
            self._nbr = self.stepper.neighbors(self.state.pos.detach())
            self._nbr_version = self._state_version

    def neighbors(self) -> tuple[torch.Tensor, torch.Tensor]:
        """``(neighbor_idx [E, A, K] int32, neighbor_count [E, A] int32)`` of the current state."""
        self.build_neighbors()
        return self._nbr[0], self._nbr[1]

    def mark_pos_dirty(self) -> None:
        self._nbr_version = -1

    def neighbor_overflow(self) -> torch.Tensor:
        """Bool ``[E, A]``: in-radius count above ``max_neighbors`` on the last build."""
        self.build_neighbors()
        return self._nbr[2] > self._nbr[1]

    def edge_index(self, rebuild: bool = True) -> torch.Tensor:
        """Radius graph as COO ``[2, n_edges]`` (sender, receiver), global node ids."""
        if rebuild or self._nbr is None:
            self.build_neighbors()
        idx, cnt = self._nbr[0].long(), self._nbr[1].long()
        E, A, K = idx.shape
        ar = torch.arange(K, device=idx.device)
        mask = ar.view(1, 1, -1) < cnt.unsqueeze(-1)
        off = torch.arange(E, device=idx.device).view(-1, 1, 1) * A
        senders = (idx + off)[mask]
        receivers = (torch.arange(A, device=idx.device).view(1, -1, 1) + off).expand(-1, -1, K)[mask]
        return torch.stack([senders, receivers], dim=0)
