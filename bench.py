"""Benchmark: forward + adjoint (BPTT) env-steps/s of the fused B200 rollout.

One "step" is one full BPTT pass of the hot path over one batch: ``rollout`` of H env
steps, then the gradient of the config's loss w.r.t. all actions, through the public API
(``swarp_b200.interop.autograd.rollout`` / ``rollout_bodies`` + ``torch.autograd.grad``).
The default workload is config 2 of the reference's benchmark set (the headline): 16,000
navigation envs x 16 holonomic agents, H=64, loss sum(||pos_H - goal||^2). ``--config``
selects configs 1-5 (config 1: 1024 x 8, H=32; 3: heterogeneous fleet 8192 x 32 with 10
circle/box/segment obstacles per env, H=50; 4: 4096 x 4 agents pushing one movable
3-circle body, H=100, loss sum ||body_pos_H - goal||; 5: dense swarm 2048 x 256, H=32,
K=32 within 0.15, overflow flag tracked). Inputs are synthetic and seeded.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl reference]

N > 1 runs under torchrun, one rank per GPU, each rank stepping its own batch of envs
(weak scaling); the only collective is one NCCL all-reduce of (loss, ||grad||^2) per
step. ``--impl reference`` times the CPU restatement of the reference (oracle/cpu_port.c,
all host threads) on the same workload, metric and unit.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass, field

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

UNIT = "env-steps/s"
FWD_BYTES, BWD_BYTES = 36, 44  # algorithmic fp32 bytes per agent-step: fwd 8 + 28, adjoint 8 + 28 + 8
BYTES_PER_AGENT_STEP = FWD_BYTES + BWD_BYTES
BODY_BYTES_PER_ENV_STEP = 48  # config 4: body pos/angle/vel/ang_vel written fwd, read bwd
DT = 0.05
HEADLINE_METRIC = "fwd+bwd env-steps/s, 16k envs×16 agents, BPTT H=64; % of HBM roofline"


@dataclass
class Workload:
    """One benchmark configuration: stepper, seeded host inputs and the loss."""

    cid: int
    name: str
    E: int
    A: int
    H: int
    stepper: object
    pos: np.ndarray
    theta: np.ndarray
    goal: np.ndarray
    acts: np.ndarray
    body: bool = False
    cpu_spec: dict = field(default_factory=dict)

    @property
    def metric(self) -> str:
        if self.cid == 2:
            return HEADLINE_METRIC
        return f"fwd+bwd env-steps/s, config {self.cid}, BPTT H={self.H}"

    @property
    def algo_bytes_per_env_step(self) -> int:
        return BYTES_PER_AGENT_STEP * self.A + (BODY_BYTES_PER_ENV_STEP if self.body else 0)


def nav_world(A: int, radius: float = 0.05, neighbor_radius: float | None = None,
              max_neighbors: int | None = None):
    """NavigationScenario.make_world constants (reference swarp/scenarios/navigation.py:127-141):
    margin 0.5 r, reach 2 r + margin, soft walls at +-1, K = min(32, max(4, A))."""
    from swarp_b200.core.config import WorldConfig

    margin = 0.5 * radius
    return WorldConfig(collisions=True, collision_k=100.0, collision_c=1.0, collision_margin=margin,
                       bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft",
                       neighbor_radius=neighbor_radius or 2 * radius + margin,
                       max_neighbors=max_neighbors or min(32, max(4, A)))


def build_workload(cid: int, rank: int = 0, dev="cuda:0", n_envs: int | None = None,
                   make_stepper: bool = True, n_agents: int | None = None) -> Workload:
    """The seeded synthetic inputs of config ``cid`` (rank-dependent seeds). ``n_agents``
    widens config 5's dense swarm (same start distribution, radius and list length) to more
    agents per env: a profiling case for the thread-block-cluster kernels, not a bench line."""
    from swarp_b200.core.config import ObstacleKind, Obstacles, WorldConfig
    from swarp_b200.core.stepper import Stepper
    from swarp_b200.dynamics.base import AgentConfig, DynamicsModel

    rng = np.random.default_rng(7919 * cid + rank)
    f32 = np.float32
    obstacles = None
    body = False
    if cid in (1, 2, 5):
        E, A, H = {1: (1024, 8, 32), 2: (16000, 16, 64), 5: (2048, 256, 32)}[cid]
        E = n_envs or E
        if n_agents is not None:
            if cid != 5:
                raise ValueError("n_agents overrides config 5 only")
            A = n_agents
        cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
        if cid == 5:
            world = nav_world(A, neighbor_radius=0.15, max_neighbors=32)
            pos = np.clip(rng.normal(0.0, 0.6, (E, A, 2)), -1.0, 1.0).astype(f32)
            name = (f"config5: dense swarm, holonomic VELOCITY, {E} envs x {A} agents, "
                    "N(0, 0.6^2) starts, R=0.15, K=32, H=32")
        else:
            world = nav_world(A)
            pos = rng.uniform(-0.95, 0.95, (E, A, 2)).astype(f32)
            name = (f"config{cid}: navigation, holonomic VELOCITY, {E} envs x {A} agents, "
                    f"H={H}, dt=0.05, soft walls, agent contacts, K={A}")
        theta = np.zeros((E, A), f32)
        goal = rng.uniform(-0.95, 0.95, (E, A, 2)).astype(f32)
        acts = rng.uniform(-1.0, 1.0, (H, E, A, 2)).astype(f32)
    elif cid == 3:
        E, A, H = n_envs or 8192, 32, 50
        models = rng.permutation(np.arange(A) % 3)
        kinds = [DynamicsModel.HOLONOMIC, DynamicsModel.DIFF_DRIVE, DynamicsModel.KINEMATIC_BICYCLE]
        cfgs = [AgentConfig(model=kinds[m]) for m in models]
        world = nav_world(A)
        pos = rng.uniform(-0.95, 0.95, (E, A, 2)).astype(f32)
        theta = rng.uniform(-math.pi, math.pi, (E, A)).astype(f32)
        goal = rng.uniform(-0.95, 0.95, (E, A, 2)).astype(f32)
        acts = rng.uniform(-1.0, 1.0, (H, E, A, 2)).astype(f32)
        # 4 circles, 2 boxes, 4 segments; sizes per obstacle index (shared by envs),
        # poses per env (reference obstacle layout, swarp/core/config.py:155-166).
        shape = np.array([0, 0, 0, 0, 1, 1, 2, 2, 2, 2], np.int32)
        radius = np.concatenate([rng.uniform(0.05, 0.15, 4), np.zeros(2), np.full(4, 0.02)])
        half = np.zeros((10, 2))
        half[4:6] = rng.uniform(0.05, 0.15, (2, 2))
        half[6:, 0] = rng.uniform(0.1, 0.3, 4)
        obstacles = Obstacles(
            pos=torch.from_numpy(rng.uniform(-1.0, 1.0, (E, 10, 2)).astype(f32)),
            radius=torch.from_numpy(radius.astype(f32)), shape=torch.from_numpy(shape),
            angle=torch.from_numpy(rng.uniform(0.0, math.pi, (E, 10)).astype(f32)),
            half_extents=torch.from_numpy(half.astype(f32)))
        name = ("config3: heterogeneous fleet (1/3 holonomic, diff-drive, bicycle), 8192 envs x "
                "32 agents, 4 circle + 2 box + 4 segment obstacles per env, H=50, K=32")
    elif cid == 4:
        E, A, H = n_envs or 4096, 4, 100
        body = True
        cfgs = [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)]
        world = WorldConfig(collisions=True, collision_k=100.0, collision_c=5.0,
                            collision_margin=0.025, bounds=(-1.0, 1.0, -1.0, 1.0),
                            bounds_mode="soft", neighbor_radius=0.125, max_neighbors=4)
        r, d = 0.08, 0.12
        mass = float(rng.uniform(1.0, 5.0))
        inertia = mass * (0.5 * r * r + 2.0 * d * d / 3.0)  # parallel-axis sum of 3 discs
        ang = rng.uniform(-0.5, 0.5, E)
        cen = rng.uniform(-0.3, 0.3, (E, 2))
        off = np.array([[-d, 0.0], [0.0, 0.0], [d, 0.0]])
        ca, sa = np.cos(ang)[:, None], np.sin(ang)[:, None]
        opos = np.stack([cen[:, None, 0] + ca * off[:, 0] - sa * off[:, 1],
                         cen[:, None, 1] + sa * off[:, 0] + ca * off[:, 1]], -1)
        obstacles = Obstacles(
            pos=torch.from_numpy(opos.astype(f32)), radius=torch.full((3,), r),
            shape=torch.zeros(3, dtype=torch.int32),
            angle=torch.from_numpy(np.repeat(ang[:, None], 3, 1).astype(f32)),
            kind=torch.full((3,), int(ObstacleKind.MOVABLE), dtype=torch.int32),
            mass=torch.full((3,), mass), inertia=torch.full((3,), inertia),
            body=torch.zeros(3, dtype=torch.int32), body_offset=torch.from_numpy(off.astype(f32)),
            half_extents=torch.zeros(3, 2))
        a_ang = rng.uniform(0.0, 2 * math.pi, (E, A))
        a_rad = rng.uniform(0.2, 0.28, (E, A))
        pos = (cen[:, None, :] + np.stack([np.cos(a_ang), np.sin(a_ang)], -1) * a_rad[..., None])
        pos = pos.astype(f32)
        theta = np.zeros((E, A), f32)
        goal = rng.uniform(-0.5, 0.5, (E, 2)).astype(f32)
        push = goal[:, None, :] - pos
        push /= np.linalg.norm(push, axis=-1, keepdims=True)
        acts = (push[None] + 0.3 * rng.standard_normal((H, E, A, 2))).astype(f32)
        name = ("config4: transport pushing, 4096 envs x 4 holonomic agents + one movable "
                "3-circle body (mass U[1,5]), H=100, loss sum ||body_pos_H - goal||")
    else:
        raise ValueError(f"unknown config {cid}")
    st = None
    if make_stepper:
        st = Stepper(cfgs, dt=DT, device=dev, dtype=torch.float32, world=world)
        if obstacles is not None:
            st.set_obstacles(obstacles)
        if body:
            st.bodies_in_grad = True
        if cid == 5:
            st.track_neighbor_overflow = True
    cpu_spec = {"configs": cfgs, "world": world, "obstacles": obstacles}
    return Workload(cid, name, E, A, H, st, pos, theta, goal, acts, body, cpu_spec)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        t0 = time.monotonic()  # nvidia-smi takes a moment to start: wait for its first sample
        while not self.lines and self.proc.poll() is None and time.monotonic() - t0 < 5.0:
            time.sleep(0.01)
        self._first = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # samples taken during the timed region (plus the one just before it)
        for line in self.lines[max(0, getattr(self, "_first", 0) - 1):]:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


class _Null:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


# ------------------------------------------------------------------ CPU side
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


@dataclass
class CpuSample:
    """The inputs of one CPU fwd+adjoint rollout of E envs of a config, generated before
    any timing starts."""

    cid: int
    E: int
    H: int
    run: object  # callable(threads) -> seconds of the rollout + adjoint alone


def cpu_prepare(cid: int, E: int, seed: int = 0) -> CpuSample:
    """Seeded inputs of E envs of config ``cid`` for the CPU restatement (untimed).

    Configs 1, 2, 3, 5 run the OpenMP C restatement (oracle/cpu_port.c). Config 4 (movable
    bodies, which that port does not model) runs the float32 torch restatement
    (oracle/torch_ref.py) with torch's intra-op threads."""
    wl = build_workload(cid, rank=seed, n_envs=E, make_stepper=False)
    rng = np.random.default_rng(1000 + seed)
    if cid == 4:
        return CpuSample(cid, E, wl.H, _torch_oracle_prep(wl))
    from oracle import cpu_port
    from swarp_b200.dynamics.base import param_rows

    w = wl.cpu_spec["world"]
    cfgs = wl.cpu_spec["configs"]
    obs = None
    o = wl.cpu_spec["obstacles"]
    if o is not None:
        r = o.resolve("cpu", torch.float64)
        obs = {"pos": r.pos.numpy(), "angle": r.angle.expand(E, -1).numpy(),
               "vel": r.vel.numpy(), "ang_vel": r.ang_vel.numpy(), "radius": r.radius.numpy(),
               "half": r.half_extents.numpy(), "shape": r.shape.numpy()}
    z = np.zeros((wl.E, wl.A), np.float32)
    init = [wl.pos, wl.theta, np.zeros_like(wl.pos), z, z]
    # the adjoint's cotangent: seeded, nonzero (its work does not depend on the values:
    # the C adjoint has no value-dependent early exit)
    g_final = rng.standard_normal(wl.pos.shape).astype(np.float32)
    kw = dict(params=param_rows(cfgs), model_tag=[int(c.model) for c in cfgs],
              ctrl_mode=[int(c.ctrl_mode) for c in cfgs], dt=DT, substeps=1, collisions=True,
              k=w.collision_k, c=w.collision_c, margin=w.collision_margin, max_overlap=0.0,
              neighbor_radius=w.neighbor_radius, max_neighbors=w.max_neighbors, bounds_mode=1,
              bounds=w.bounds, init=init, actions=wl.acts, grad_final_pos=g_final,
              obstacles=obs, dtype=np.float32)

    def run(threads: int) -> float:
        t0 = time.perf_counter()
        cpu_port.rollout(threads=threads, **kw)
        return time.perf_counter() - t0

    return CpuSample(cid, E, wl.H, run)


def _torch_oracle_prep(wl: Workload):
    from oracle import torch_ref as R
    from swarp_b200.dynamics.base import param_rows

    cfgs, w, o = wl.cpu_spec["configs"], wl.cpu_spec["world"], wl.cpu_spec["obstacles"]
    f = torch.float32
    ro = o.resolve("cpu", f)
    rw = R.RefWorld(params=torch.tensor(param_rows(cfgs), dtype=f),
                    model_tag=[int(c.model) for c in cfgs], ctrl_mode=[int(c.ctrl_mode) for c in cfgs],
                    dt=DT, substeps=1, collisions=True, k=w.collision_k, c=w.collision_c,
                    margin=w.collision_margin, max_overlap=0.0, neighbor_radius=w.neighbor_radius,
                    max_neighbors=w.max_neighbors, bounds=w.bounds, soft_walls=True,
                    clamp_bounds=False, lin_damping=w.obstacle_linear_damping,
                    ang_damping=w.obstacle_angular_damping, bodies_move=True)
    rob = R.RefObstacles(pos=ro.pos, angle=ro.angle.expand(wl.E, -1), vel=ro.vel, ang_vel=ro.ang_vel,
                         radius=ro.radius, half=ro.half_extents, shape=ro.shape.tolist(),
                         kind=ro.kind.tolist(), mass=ro.mass, inertia=ro.inertia,
                         body=ro.body.tolist(), body_off=ro.body_offset)
    rob = R.seed_bodies(rob)
    pos = torch.from_numpy(wl.pos)
    z = torch.zeros(wl.E, wl.A)
    goal = torch.from_numpy(wl.goal)
    acts0 = torch.from_numpy(wl.acts)

    def run(threads: int) -> float:
        torch.set_num_threads(threads)
        acts = acts0.clone().requires_grad_(True)
        t0 = time.perf_counter()
        _, _, body_traj = R.rollout((pos, z, torch.zeros_like(pos), z, z), acts, rw, rob)
        loss = (body_traj[-1].body_pos[:, 0] - goal).norm(dim=-1).sum()
        loss.backward()
        return time.perf_counter() - t0

    return run


def cpu_envs_for(cid: int, seconds: float, threads: int, e_max: int) -> int:
    """Envs of config ``cid`` whose fwd+adjoint rollout takes about ``seconds`` on
    ``threads`` threads (at most e_max), from timed calibration samples."""
    E = max(threads, 8)
    while True:
        sample = cpu_prepare(cid, min(E, e_max))
        dt = sample.run(threads)
        if dt >= seconds / 4 or E >= e_max:
            return min(e_max, max(1, int(min(E, e_max) * seconds / max(dt, 1e-6))))
        E *= 4


def cpu_baseline_block(wl: Workload, target_s: float = 2.0, repeats: int = 3) -> dict:
    """The CPU restatement on all host threads and on one, in this run (rank 0, N=1)."""
    threads = host_threads()
    out = {}
    for label, th in (("all", threads), ("one", 1)):
        E = cpu_envs_for(wl.cid, target_s, th, wl.E)
        samples = [cpu_prepare(wl.cid, E, seed=i) for i in range(repeats)]
        times = [smp.run(th) for smp in samples]
        out[label] = (E, E * wl.H / statistics.median(times))
    port = ("float32 torch restatement (oracle/torch_ref.py)" if wl.cid == 4 else
            "C restatement (oracle/cpu_port.c, OpenMP)")
    return {"value": out["all"][1], "unit": UNIT, "cores": threads, "kind": "port",
            "threads": threads, "value_1core": out["one"][1], "cpu_model": cpu_model(),
            "sample": f"{out['all'][0]} envs x {wl.A} agents x H={wl.H} on {threads} threads, "
                      f"{out['one'][0]} envs on 1 thread; fwd+adjoint, float32, {port}; "
                      f"inputs generated before timing; median of {repeats}"}


def run_reference(args, rank: int, world: int) -> None:
    """The CPU restatement of the reference's rollout + adjoint (the reference's own Warp
    path cannot be installed here), all host threads, on this arm's workload: each step one
    rollout of the config's full env count, unless that would not let ``--steps`` +
    ``--warmup`` steps end within about two minutes (then a bounded env sample, stated in
    ``cpu_baseline.sample``). Inputs are generated before the timed loop; only the
    rollout + adjoint calls are timed."""
    if rank != 0:
        return
    threads = host_threads()
    wl = build_workload(args.config, make_stepper=False, n_envs=args.envs)
    budget = min(1.5, 120.0 / max(1, args.steps + args.warmup))
    E = cpu_envs_for(args.config, budget, threads, wl.E)
    samples = [cpu_prepare(args.config, E, seed=i) for i in range(2)]
    for i in range(args.warmup):
        samples[i % 2].run(threads)
    times = [samples[i % 2].run(threads) for i in range(args.steps)]
    dt = sum(times)
    value = E * wl.H * args.steps / dt
    full = E == wl.E
    line = {
        "impl": "reference", "metric": wl.metric, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": config_block(wl, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "threads": threads,
                         "kind": "port", "cpu_model": cpu_model(),
                         "sample": (f"{E} envs per step ({'the full workload' if full else 'a bounded sample of the workload'}), "
                                    "CPU restatement of the reference (oracle/cpu_port.c; "
                                    "the reference's Warp path cannot be installed here), "
                                    "inputs generated before timing")},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(wl: Workload, world: int) -> dict:
    agent_steps = wl.E * wl.A * wl.H
    return {"workload": wl.name, "config_id": wl.cid, "n_envs_per_gpu": wl.E, "n_agents": wl.A,
            "horizon": wl.H, "parallelism": f"env-sharded dp{world}",
            "l2": "inputs larger than L2" if wl.acts.nbytes + 28 * agent_steps > 126e6 else
                  "inputs smaller than L2 (small config; no flush)"}


# ------------------------------------------------------------------ GPU side
def profile_traffic(cid: int, kernel: str):
    """DRAM bytes per launch of the forward ("fwd") or adjoint ("bwd") kernel, from the ncu
    capture summarised in profiles/ (dram__bytes_read.sum + dram__bytes_write.sum of a
    half-size capture, doubled: traffic grows with the envs), if one exists for cid."""
    path = os.path.join(ROOT, "profiles", "rollout_kernels_config2.md")
    key = f"traffic_bytes_per_launch_config{cid}_{kernel}:"
    try:
        for line in open(path):
            if line.startswith(key):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--impl", default="swarp_b200", choices=["swarp_b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--e2e-chunks", type=int, default=2,
                    help="env chunks the end-to-end leg pipelines host copies over")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--envs", type=int, default=None,
                    help="override the config's envs per GPU (smaller cases for profiling)")
    ap.add_argument("--agents", type=int, default=None,
                    help="config 5 with this many agents per env (a profiling case for envs "
                         "wider than one CTA; no CPU baseline, no reference arm)")
    args = ap.parse_args()
    if args.agents is not None and (args.config != 5 or args.impl == "reference"):
        ap.error("--agents applies to config 5 of this implementation only")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl" if args.impl != "reference" else "gloo",
                                timeout=datetime.timedelta(seconds=120))
    if args.impl == "reference":
        run_reference(args, rank, world)
        if dist is not None:
            dist.destroy_process_group()
        return

    from swarp_b200.core.sharding import PairReducer, reduce_loss_and_grad_norm
    from swarp_b200.interop.autograd import FusedGoalLoss, TorchState, rollout, rollout_bodies
    from swarp_b200.interop.graphs import GraphedRollout

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl = build_workload(args.config, rank=rank, dev=dev, n_envs=args.envs,
                        n_agents=args.agents)
    st, E, A, H = wl.stepper, wl.E, wl.A, wl.H
    pos = torch.from_numpy(wl.pos).to(dev)
    theta = torch.from_numpy(wl.theta).to(dev)
    goal = torch.from_numpy(wl.goal).to(dev)
    acts = torch.from_numpy(wl.acts).to(dev).requires_grad_(True)
    zero = torch.zeros(E, A, device=dev)
    state = TorchState(pos, theta, torch.zeros(E, A, 2, device=dev), zero, zero)
    snap = st.bodies_snapshot() if wl.body else None

    def loss_fn(final, _traj):
        # sum ||pos_H - goal||^2 as one fused op (and one fused op in the backward)
        return torch.nn.functional.mse_loss(final.pos, goal, reduction="sum")

    def eager_step(state, acts):
        """The drop-in path: rollout (or rollout_bodies) + autograd.grad, all eager."""
        if wl.body:
            st.restore_bodies(snap)  # every step pushes the same body from the same pose
            _, _, body = rollout_bodies(st, state, acts)
            loss = (body.pos[:, 0] - goal).norm(dim=-1).sum()
        else:
            final, traj = rollout(st, state, acts)
            loss = loss_fn(final, traj)
        (g,) = torch.autograd.grad(loss, [acts])
        if dist is not None:
            loss = reduce_loss_and_grad_norm(loss, g)[0]
        return loss

    for _ in range(args.warmup):
        eager_step(state, acts)
    torch.cuda.synchronize()

    # ---- per-kernel device time: the two rollout kernels back to back (GPU-bound loop)
    s5 = tuple(state[:5])
    a_d = acts.detach()
    n_k = max(20, min(args.steps, 200))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_k)]
    for i in range(n_k + 3):
        if wl.body:
            st.restore_bodies(snap)
        if i >= 3:
            ev[i - 3][0].record()
        traj, fin, _, rec = st.rollout_forward(s5, a_d, final=True)
        if i >= 3:
            ev[i - 3][1].record()
        # cotangent only on the final positions, as the BPTT loss gives
        st.rollout_backward(s5, a_d, traj, (None,) * 5, (fin[0], None, None, None, None), rec)
        if i >= 3:
            ev[i - 3][2].record()
    torch.cuda.synchronize()
    t_fwd = statistics.median(e[0].elapsed_time(e[1]) for e in ev)
    t_bwd = statistics.median(e[1].elapsed_time(e[2]) for e in ev)

    # ---- the timed step: one CUDA-graph replay of the whole BPTT step (one launch from
    # the host), then the (loss, ||g||^2) all-reduce across ranks
    graphed = reducer = None
    if not wl.body:
        # the same loss fused into the rollout kernels (rollout_goal_loss): the step is the
        # forward kernel, one small reduction and the adjoint kernel. With ranks, the
        # (loss, ||g||^2) all-reduce is either captured in the same graph, in stream order
        # after the adjoint, or started asynchronously on NCCL's stream so that it overlaps
        # the next step (PairReducer); which costs less depends on the box (measured at
        # 2 GPUs: 0.017 vs 0.060 ms per step on one box, 0.019 vs 0.009 ms on another), so
        # the bench times both before the timed region and all ranks take the faster.
        graphed = GraphedRollout(st, state, acts, FusedGoalLoss(goal),
                                 grad_norm="fused" if dist is not None else False, warmup=3,
                                 all_reduce=dist is not None)

    else:
        # movable bodies: the same step (rollout_bodies, the body loss, autograd.grad) captured
        # in one graph; every replay pushes the bodies from the same initial pose
        def body_loss(_final, _traj, body):
            return (body.pos[:, 0] - goal).norm(dim=-1).sum()

        st.restore_bodies(snap)
        graphed = GraphedRollout(st, state, acts, body_loss,
                                 grad_norm=True if dist is not None else False, warmup=3,
                                 all_reduce=dist is not None)

    def step():
        graphed()

    def timed_loop(fn, n, sample_clocks, finish=None, start=None):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) if sample_clocks else _Null() as clk:
            e0.record()
            if start is not None:
                start()  # work on other streams is ordered after e0
            for _ in range(n):
                fn()
            if finish is not None:
                finish()  # the compute stream waits for work still on other streams
            e1.record()
            torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        return e0.elapsed_time(e1), clk

    schedule, finish, plain, cal = "in-graph", None, None, None
    if dist is not None and not wl.body:
        plain = GraphedRollout(st, state, acts, FusedGoalLoss(goal), grad_norm="fused",
                               warmup=3)
        reducer = PairReducer(plain.loss_and_grad_norm, depth=8)

        def step_async():
            plain()
            reducer(plain.loss_and_grad_norm)

        n_cal = max(20, min(args.steps, 200))
        for fn in (step, step_async):
            for _ in range(3):
                fn()
        t_sync, _ = timed_loop(step, n_cal, False)
        t_async, _ = timed_loop(step_async, n_cal, False, finish=reducer.drain)
        cal_t = torch.tensor([t_sync / n_cal, t_async / n_cal], device=dev, dtype=torch.float64)
        dist.all_reduce(cal_t, op=dist.ReduceOp.MAX)  # every rank takes the same schedule
        cal = {"ms_per_step_in_graph": float(cal_t[0]), "ms_per_step_async": float(cal_t[1]),
               "steps": n_cal}
        if float(cal_t[1]) < float(cal_t[0]):
            schedule, finish = "async", reducer.drain
            step = step_async  # noqa: F811
    for _ in range(args.warmup):
        step()
    if finish is not None:
        finish()
    torch.cuda.synchronize()

    ms, clocks = timed_loop(step, args.steps, True, finish=finish)
    n_eager = max(20, min(args.steps, 200))
    for _ in range(3):
        eager_step(state, acts)
    ms_eager, _ = timed_loop(lambda: eager_step(state, acts), n_eager, False)
    ms_t = torch.tensor([ms, t_fwd, t_bwd, ms_eager], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, t_fwd, t_bwd, ms_eager = (float(x) for x in ms_t.cpu())
    ms_per_step = ms / args.steps
    value = world * E * H / (ms_per_step / 1e3)
    value_eager = world * E * H / (ms_eager / n_eager / 1e3)
    overflow = None
    if st.track_neighbor_overflow:
        ov = st.rollout_overflow()
        overflow = {"agents_over_K": int(ov.sum()), "max_true_count":
                    int(st.last_true_count_max.max()), "K": st.world.max_neighbors}

    # ---- collective: device time of the (loss, ||g||^2) all-reduce alone, back to back,
    # and the two schedules' step times that chose the timed one
    allreduce = None
    if dist is not None and not wl.body:
        buf = torch.zeros(2, device=dev, dtype=torch.float32)
        for _ in range(20):
            dist.all_reduce(buf)
        n_ar = 100
        ar_ms, _ = timed_loop(lambda: dist.all_reduce(buf), n_ar, False)
        plain.release()
        ar_t = torch.tensor([ar_ms / n_ar * 1e3], device=dev, dtype=torch.float64)
        dist.all_reduce(ar_t, op=dist.ReduceOp.MAX)
        allreduce = {"us_per_allreduce_back_to_back": float(ar_t[0]), "calibration": cal,
                     "timed_step": ("all-reduce captured in the step's graph, in stream order"
                                    if schedule == "in-graph" else
                                    "all-reduce started asynchronously on NCCL's stream after "
                                    "each replay, overlapping the next step (8 in flight)"),
                     "bytes": 8, "backend": "nccl"}

    # ---- end to end through the public API with host buffers: every step copies its
    # inputs (actions, start positions and headings, goals) from pinned host memory and
    # its result (the action gradient and the loss) back to pinned host memory
    pin = [torch.from_numpy(x).pin_memory() for x in (wl.acts, wl.pos, wl.theta, wl.goal)]
    h2d = sum(p.numel() * p.element_size() for p in pin)
    grad_h = torch.empty(wl.acts.shape, dtype=torch.float32).pin_memory()
    streamed = None
    if not wl.body:
        from swarp_b200.interop.streamed import StreamedRollout

        streamed = StreamedRollout(st, E, H, 2, "goal", aux_like=[goal], chunks=args.e2e_chunks)
        loss_h = torch.zeros(streamed.n_chunks, dtype=torch.float64).pin_memory()
        d2h = grad_h.numel() * grad_h.element_size() + loss_h.numel() * 8

        def e2e_step():
            streamed(TorchState(pin[1], pin[2], None, None, None), pin[0], [pin[3]], grad_h,
                     loss_h)

        def e2e_begin():
            streamed.begin()

        def e2e_end():
            streamed.end()
    else:
        # the captured body step: inputs copied into its static buffers, gradient and loss out
        loss_h = torch.zeros(1, dtype=torch.float64).pin_memory()
        d2h = grad_h.numel() * grad_h.element_size() + 8

        def e2e_step():
            goal.copy_(pin[3], non_blocking=True)
            graphed(TorchState(pin[1], pin[2], None, None, None), pin[0])
            grad_h.copy_(graphed.grad_actions, non_blocking=True)
            loss_h.copy_(graphed.loss.double().reshape(1), non_blocking=True)

        e2e_begin = e2e_end = None

    for _ in range(3):
        if e2e_begin:
            e2e_begin()
        e2e_step()
        if e2e_end:
            e2e_end()
    torch.cuda.synchronize()
    e2e_total, _ = timed_loop(e2e_step, args.e2e_steps, False, finish=e2e_end, start=e2e_begin)
    e2e_ms = torch.tensor([e2e_total / args.e2e_steps], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = world * E * H / (float(e2e_ms.item()) / 1e3)
    # the gradient that came back equals the device-timed step's (same envs, same inputs)
    goal.copy_(pin[3])
    graphed(TorchState(pin[1].to(dev), pin[2].to(dev), None, None, None), pin[0].to(dev))
    e2e_grad_ok = bool(torch.equal(graphed.grad_actions.cpu(), grad_h))
    if streamed is not None:
        streamed.release()

    graphed.release()  # before the process group goes: the graph follows NCCL work
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        peak = json.load(open(peaks_path))["hbm_gbs"]
        peak_src = "measured"
    else:
        peak = 6650.0
        peak_src = "fallback"
    agent_steps = E * A * H
    body_b = (BODY_BYTES_PER_ENV_STEP // 2) * E * H if wl.body else 0
    bwd_gbs = (BWD_BYTES * agent_steps + body_b) / (t_bwd / 1e3) / 1e9
    fwd_gbs = (FWD_BYTES * agent_steps + body_b) / (t_fwd / 1e3) / 1e9
    step_gbs = wl.algo_bytes_per_env_step * E * H / ((t_fwd + t_bwd) / 1e3) / 1e9
    dom = "bwd" if t_bwd >= t_fwd else "fwd"
    # 16-agent float worlds without moving bodies take the two-agents-per-thread instances
    x2 = A == 16 and not wl.body and (dom == "fwd" or st.substeps == 1)
    variant = "x2_" if x2 else "cl_" if A > 1024 else ""  # envs above 1024 agents: clusters
    roof = {"bound": "hbm", "kernel": f"rollout_{dom}_{variant}kernel<...>",
            "achieved": bwd_gbs if dom == "bwd" else fwd_gbs, "peak": peak, "unit": "GB/s",
            "peak_source": peak_src}
    roof["frac"] = roof["achieved"] / peak
    roof["traffic"] = profile_traffic(args.config, dom)
    roof["traffic_source"] = ("ncu capture summarised in profiles/rollout_kernels_config2.md"
                              if roof["traffic"] is not None else None)
    cfg = config_block(wl, world)
    line = {
        "metric": wl.metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": cfg,
        "roofline": roof,
        "roofline_step": {"bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s",
                          "frac": step_gbs / peak,
                          "bytes_per_env_step": wl.algo_bytes_per_env_step,
                          "fwd_ms": t_fwd, "bwd_ms": t_bwd, "fwd_gbs": fwd_gbs,
                          "bwd_gbs": bwd_gbs},
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": (f"StreamedRollout: {streamed.n_chunks if streamed else 1} env chunks, "
                         "host-to-device copies, captured BPTT step and device-to-host copies "
                         "of the action gradient and loss on three streams"
                         if streamed is not None else
                         "inputs copied into the captured body step (GraphedRollout), action "
                         "gradient and loss copied back"),
                "grad_matches_device_step": e2e_grad_ok},
        # forward + loss reduction + adjoint per step, plus the fused-norm reduction when
        # ranks all-reduce it
        # (body worlds: the two rollout kernels; the body loss and the body-state hand-over
        # are torch ops in the same graph)
        "gpu_launches": (2 if wl.body else (4 if dist is not None else 3)) * args.steps,
        "timed_path": ("one CUDA-graph replay of the whole BPTT step per step "
                       "(swarp_b200.interop.graphs.GraphedRollout with the goal loss fused into "
                       "the rollout kernels, rollout_goal_loss)" if not wl.body else
                       "one CUDA-graph replay per step of rollout_bodies + the body loss + "
                       "autograd.grad (swarp_b200.interop.graphs.GraphedRollout)"),
        "value_eager": value_eager,
    }
    if overflow is not None:
        line["neighbor_overflow"] = overflow
    if allreduce is not None:
        line["allreduce"] = allreduce
    if world == 1 and not args.no_cpu_baseline and args.agents is None:
        line["cpu_baseline"] = cpu_baseline_block(wl)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
