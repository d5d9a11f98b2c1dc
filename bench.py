"""Benchmark: forward + adjoint (BPTT) env-steps/s of the fused B200 rollout.

One "step" is one full BPTT pass of the hot path over one batch: ``rollout`` of H=64 env
steps for 16,000 navigation envs x 16 holonomic agents (config 2 of the reference's
benchmark set), then the gradient of sum(||pos_H - goal||^2) w.r.t. all actions, through
the public API (``swarp_b200.interop.autograd.rollout`` + ``torch.autograd.grad``).
Inputs are synthetic and seeded (uniform starts/goals in the arena, uniform [-1, 1]
actions); every step's inputs and outputs exceed L2 (actions 131 MB, trajectory 459 MB).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun, one rank per GPU, each rank stepping its own 16,000 envs
(weak scaling); the only collective is one NCCL all-reduce of (loss, ||grad||^2) per
step. ``--impl reference`` times the CPU restatement of the reference (oracle/cpu_port.c,
all host threads) on the same workload, metric and unit.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

E_PER_GPU, N_AGENTS, HORIZON, DT = 16000, 16, 64, 0.05
METRIC = "fwd+bwd env-steps/s, 16k envs x 16 agents, BPTT H=64"
UNIT = "env-steps/s"
BYTES_PER_AGENT_STEP = 80  # algorithmic: fwd 8 + 28, adjoint 8 + 28 + 8 (fp32)
FWD_BYTES, BWD_BYTES = 36, 44


def world_config():
    from swarp_b200.core.config import WorldConfig

    # NavigationScenario.make_world defaults at radius 0.05 (reference
    # swarp/scenarios/navigation.py:127-141): margin 0.5 r, reach 2 r + margin, soft walls.
    r = 0.05
    margin = 0.5 * r
    return WorldConfig(collisions=True, collision_k=100.0, collision_c=1.0, collision_margin=margin,
                       bounds=(-1.0, 1.0, -1.0, 1.0), bounds_mode="soft",
                       neighbor_radius=2 * r + margin, max_neighbors=min(32, max(4, N_AGENTS)))


def agent_configs():
    from swarp_b200.dynamics.base import AgentConfig

    return [AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(N_AGENTS)]


def synthetic_inputs(E: int, seed: int):
    """Starts/goals U[-0.95, 0.95]^2, actions U[-1, 1] (numpy, float32)."""
    rng = np.random.default_rng(seed)
    pos = rng.uniform(-0.95, 0.95, (E, N_AGENTS, 2)).astype(np.float32)
    goal = rng.uniform(-0.95, 0.95, (E, N_AGENTS, 2)).astype(np.float32)
    acts = rng.uniform(-1.0, 1.0, (HORIZON, E, N_AGENTS, 2)).astype(np.float32)
    return pos, goal, acts


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
        for line in self.lines:
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


# ------------------------------------------------------------------ CPU side
def cpu_rollout_sample(E: int, threads: int, seed: int = 0):
    """One fwd+adjoint rollout of E envs on the C restatement; returns seconds."""
    from oracle import cpu_port

    pos, goal, acts = synthetic_inputs(E, seed)
    z = np.zeros((E, N_AGENTS), np.float32)
    from swarp_b200.dynamics.base import param_rows

    w = world_config()
    t0 = time.perf_counter()
    traj, _, _ = cpu_port.rollout(
        params=param_rows(agent_configs()), model_tag=[0] * N_AGENTS, ctrl_mode=[0] * N_AGENTS,
        dt=DT, substeps=1, collisions=True, k=w.collision_k, c=w.collision_c,
        margin=w.collision_margin, max_overlap=0.0, neighbor_radius=w.neighbor_radius,
        max_neighbors=w.max_neighbors, bounds_mode=1, bounds=w.bounds,
        init=[pos, z, np.zeros_like(pos), z, z], actions=acts,
        grad_final_pos=np.zeros_like(pos), threads=threads, dtype=np.float32)
    # The adjoint's work does not depend on the cotangent values, so the sample seeds it
    # with zeros instead of 2 (pos_H - goal) (which would need the forward first).
    return time.perf_counter() - t0


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def calibrate_cpu(target_s: float, threads: int) -> int:
    E = max(threads, 8)
    while True:
        dt = cpu_rollout_sample(E, threads)
        if dt >= target_s / 4 or E >= E_PER_GPU:
            return min(E_PER_GPU, max(1, int(E * target_s / max(dt, 1e-6))))
        E *= 4


def cpu_baseline_block(target_s: float = 2.0, repeats: int = 3) -> dict:
    threads = host_threads()
    E = calibrate_cpu(target_s, threads)
    times = [cpu_rollout_sample(E, threads, seed=i) for i in range(repeats)]
    t = statistics.median(times)
    return {"value": E * HORIZON / t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{E} envs x {N_AGENTS} agents x H={HORIZON}, fwd+adjoint, float32, "
                      f"C restatement (oracle/cpu_port.c, OpenMP {threads} threads), median of "
                      f"{repeats}"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = host_threads()
    E = calibrate_cpu(0.05, threads)  # ~50 ms per step keeps --steps runs to minutes
    for i in range(args.warmup):
        cpu_rollout_sample(E, threads, seed=i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cpu_rollout_sample(E, threads, seed=i)
    dt = time.perf_counter() - t0
    value = E * HORIZON * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "config2-sample: navigation, holonomic, 16 agents/env, H=64, "
                               f"{E} envs per step (bounded CPU sample)",
                   "n_agents": N_AGENTS, "horizon": HORIZON, "dt": DT},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{E} envs per step, C restatement of the reference "
                                   "(the reference's Warp path cannot be installed here)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU side
def profile_traffic():
    """DRAM bytes per launch of the adjoint kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "rollout_bwd_config2.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch_config2:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="swarp_b200", choices=["swarp_b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()

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

    from swarp_b200.core.stepper import Stepper
    from swarp_b200.interop.autograd import TorchState, rollout

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    st = Stepper(agent_configs(), dt=DT, device=dev, dtype=torch.float32, world=world_config())
    E = E_PER_GPU
    pos_h, goal_h, acts_h = synthetic_inputs(E, seed=1000 + rank)
    pos = torch.from_numpy(pos_h).to(dev)
    goal = torch.from_numpy(goal_h).to(dev)
    acts = torch.from_numpy(acts_h).to(dev).requires_grad_(True)
    zero = torch.zeros(E, N_AGENTS, device=dev)
    state = TorchState(pos, zero, torch.zeros(E, N_AGENTS, 2, device=dev), zero, zero)
    red = torch.zeros(2, device=dev)

    # per-kernel device time: events around the two rollout launches
    kern = {"fwd": [], "bwd": []}
    record = {"on": False}
    f_fwd, f_bwd = st.rollout_forward, st.rollout_backward

    def timed(name, fn):
        def wrap(*a, **k):
            if not record["on"]:
                return fn(*a, **k)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*a, **k)
            e1.record()
            kern[name].append((e0, e1))
            return out
        return wrap

    st.rollout_forward = timed("fwd", f_fwd)
    st.rollout_backward = timed("bwd", f_bwd)

    def bptt_step(state, acts, goal):
        final, _ = rollout(st, state, acts)
        loss = ((final.pos - goal) ** 2).sum()
        (g,) = torch.autograd.grad(loss, [acts])
        if dist is not None:
            red[0] = loss.detach()
            red[1] = g.square().sum()
            dist.all_reduce(red)
        return loss, g

    for _ in range(args.warmup):
        bptt_step(state, acts, goal)
    torch.cuda.synchronize()

    # ---- timed region (device time, max over ranks)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        record["on"] = True
        ev0.record()
        for _ in range(args.steps):
            bptt_step(state, acts, goal)
        ev1.record()
        torch.cuda.synchronize()
        record["on"] = False
    if dist is not None:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    t_fwd = statistics.mean(a.elapsed_time(b) for a, b in kern["fwd"])
    t_bwd = statistics.mean(a.elapsed_time(b) for a, b in kern["bwd"])
    ms_t = torch.tensor([ms, t_fwd, t_bwd], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, t_fwd, t_bwd = (float(x) for x in ms_t.cpu())
    ms_per_step = ms / args.steps
    value = world * E * HORIZON / (ms_per_step / 1e3)

    # ---- end to end: host inputs (pinned) -> device, step, loss -> host
    pin_acts = torch.from_numpy(acts_h).pin_memory()
    pin_pos = torch.from_numpy(pos_h).pin_memory()
    pin_goal = torch.from_numpy(goal_h).pin_memory()
    d_acts = torch.empty_like(acts)
    h2d = pin_acts.numel() * 4 + pin_pos.numel() * 4 + pin_goal.numel() * 4
    d2h = 8
    losses = []
    for i in range(args.e2e_steps + 3):
        if i == 3:
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize()
            e2e0 = torch.cuda.Event(enable_timing=True)
            e2e0.record()
        d_acts.copy_(pin_acts, non_blocking=True)
        p = pin_pos.to(dev, non_blocking=True)
        gl = pin_goal.to(dev, non_blocking=True)
        a = d_acts.detach().requires_grad_(True)
        s0 = TorchState(p, zero, torch.zeros_like(p), zero, zero)
        loss, _ = bptt_step(s0, a, gl)
        losses.append(float(loss.detach().to("cpu", torch.float64)))
    e2e1 = torch.cuda.Event(enable_timing=True)
    e2e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e2e0.elapsed_time(e2e1) / args.e2e_steps], device=dev,
                          dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = world * E * HORIZON / (float(e2e_ms.item()) / 1e3)

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
    agent_steps = E * N_AGENTS * HORIZON
    bwd_gbs = BWD_BYTES * agent_steps / (t_bwd / 1e3) / 1e9
    fwd_gbs = FWD_BYTES * agent_steps / (t_fwd / 1e3) / 1e9
    step_gbs = BYTES_PER_AGENT_STEP * agent_steps / ((t_fwd + t_bwd) / 1e3) / 1e9
    dom = "bwd" if t_bwd >= t_fwd else "fwd"
    traffic = profile_traffic()
    roof = {"bound": "hbm", "kernel": f"rollout_{dom}_kernel<float,...>",
            "achieved": bwd_gbs if dom == "bwd" else fwd_gbs, "peak": peak, "unit": "GB/s",
            "peak_source": peak_src}
    roof["frac"] = roof["achieved"] / peak
    roof["traffic"] = traffic if dom == "bwd" else None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2: navigation, holonomic VELOCITY, 16000 envs x 16 agents "
                               "per GPU, H=64, dt=0.05, soft walls, agent contacts",
                   "n_envs_per_gpu": E, "n_agents": N_AGENTS, "horizon": HORIZON,
                   "parallelism": f"env-sharded dp{world}",
                   "l2": "inputs larger than L2 (actions 131 MB, trajectory 459 MB per step)"},
        "roofline": roof,
        "roofline_step": {"bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s",
                          "frac": step_gbs / peak,
                          "bytes_per_agent_step": BYTES_PER_AGENT_STEP,
                          "fwd_ms": t_fwd, "bwd_ms": t_bwd, "fwd_gbs": fwd_gbs,
                          "bwd_gbs": bwd_gbs},
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": 2 * args.steps,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_block()
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
