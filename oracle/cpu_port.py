"""ctypes wrapper of the C restatement (oracle/cpu_port.c). TEST INFRASTRUCTURE / CPU
BASELINE ONLY: imported by tests/ and bench.py's CPU-baseline leg, never by swarp_b200."""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

from oracle import build_cpu


class CpuWorld(C.Structure):
    _fields_ = [
        ("n_envs", C.c_int), ("n_agents", C.c_int), ("act_dim", C.c_int), ("substeps", C.c_int),
        ("horizon", C.c_int), ("dt", C.c_double), ("collisions", C.c_int),
        ("k", C.c_double), ("c", C.c_double), ("margin", C.c_double), ("max_overlap", C.c_double),
        ("neighbor_radius", C.c_double), ("max_neighbors", C.c_int), ("bounds_mode", C.c_int),
        ("bounds", C.c_double * 4), ("params", C.c_void_p), ("params_env_stride", C.c_long),
        ("model_tag", C.c_void_p), ("ctrl_mode", C.c_void_p), ("n_obstacles", C.c_int),
        ("obs_pos", C.c_void_p), ("obs_angle", C.c_void_p), ("obs_vel", C.c_void_p),
        ("obs_ang_vel", C.c_void_p), ("obs_radius", C.c_void_p), ("obs_half", C.c_void_p),
        ("obs_shape", C.c_void_p), ("threads", C.c_int),
        ("list_order", C.c_int), ("grid_bins", C.c_int), ("grid_origin", C.c_double * 2),
        ("grid_cell", C.c_double),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_cpu.LIB if os.path.exists(build_cpu.LIB) else build_cpu.build()
        _lib = C.CDLL(path)
        for sfx in ("f32", "f64"):
            fn = getattr(_lib, f"swarp_cpu_rollout_{sfx}")
            fn.restype = C.c_int
            fn.argtypes = [C.POINTER(CpuWorld)] + [C.c_void_p] * 18
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def rollout(*, params, model_tag, ctrl_mode, dt, substeps, collisions, k, c, margin, max_overlap,
            neighbor_radius, max_neighbors, bounds_mode, bounds, init, actions, grad_final_pos=None,
            obstacles=None, threads=0, dtype=np.float32, grid=None):
    """Forward rollout (+ adjoint of <grad_final_pos, final pos> when given).

    ``init``: five arrays (pos [E,A,2], theta, vel [E,A,2], speed, ang_vel);
    ``actions`` [T,E,A,D]. Returns ``(traj5, grad_actions | None, grad_init5 | None)``.
    ``grid=(bins, (x_min, x_max, y_min, y_max))`` lists neighbors in the order of the
    reference's uniform grid with that static frame (origin at the rectangle's lower
    corner, cell ``max(neighbor_radius, extent / bins)``); ``None`` in ascending index.
    """
    T, E, A, D = actions.shape
    keep = []

    def arr(x, dt_=dtype):
        a = np.ascontiguousarray(x, dtype=dt_)
        keep.append(a)
        return a

    w = CpuWorld()
    w.n_envs, w.n_agents, w.act_dim, w.substeps, w.horizon = E, A, D, substeps, T
    w.dt, w.collisions = dt, int(collisions)
    w.k, w.c, w.margin, w.max_overlap = k, c, margin, max_overlap
    w.neighbor_radius, w.max_neighbors, w.bounds_mode = neighbor_radius, max_neighbors, bounds_mode
    w.bounds = (C.c_double * 4)(*(bounds or (0.0, 0.0, 0.0, 0.0)))
    pr = arr(params, np.float64)
    w.params = _p(pr)
    w.params_env_stride = A * 22 if pr.ndim == 3 else 0
    w.model_tag = _p(arr(model_tag, np.int32))
    w.ctrl_mode = _p(arr(ctrl_mode, np.int32))
    if grid is not None:
        bins, (x0, x1, y0, y1) = grid
        w.list_order, w.grid_bins = 1, int(bins)
        w.grid_origin = (C.c_double * 2)(x0, y0)
        w.grid_cell = max(neighbor_radius, max(x1 - x0, y1 - y0) / bins)
    if obstacles is not None:
        w.n_obstacles = obstacles["pos"].shape[1]
        for name in ("pos", "angle", "vel", "ang_vel", "radius", "half"):
            setattr(w, f"obs_{name}", _p(arr(obstacles[name], np.float64)))
        w.obs_shape = _p(arr(obstacles["shape"], np.int32))
    w.threads = threads
    st = [arr(x) for x in init]
    acts = arr(actions)
    traj = [np.empty((T, *x.shape), dtype=dtype) for x in st]
    if grad_final_pos is not None:
        gf = arr(grad_final_pos)
        g_act = np.empty_like(acts)
        g_init = [np.empty_like(x) for x in st]
    else:
        gf, g_act, g_init = None, None, [None] * 5
    fn = getattr(lib(), "swarp_cpu_rollout_" + ("f32" if dtype == np.float32 else "f64"))
    rc = fn(C.byref(w), *[_p(x) for x in st], _p(acts), *[_p(x) for x in traj], _p(gf), _p(g_act),
            *[_p(x) for x in g_init])
    if rc != 0:
        raise RuntimeError(f"swarp_cpu_rollout failed: {rc}")
    return traj, g_act, (g_init if g_act is not None else None)
