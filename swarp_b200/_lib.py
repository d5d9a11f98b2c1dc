"""ctypes binding of ``libswarp_b200.so`` (the C ABI declared in include/swarp_b200.h).

The library is the only compute path: there is no CPU fallback. Loading fails loudly
when the library has not been built or no CUDA device is visible.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libswarp_b200.so")

SWARP_OK = 0
ERRORS = {
    -1: "invalid argument",
    -2: "unsupported model or option",
    -3: "too many agents",
    -4: "CUDA launch failed",
    -5: "workspace missing or too small",
    -6: "rollout needs more workspace than the allocation-free entry point's static scratch",
}
MAX_AGENTS = 4096
MAX_CTA_AGENTS = 1024  # larger envs run one env per thread-block cluster


class State(C.Structure):
    _fields_ = [("pos", C.c_void_p), ("theta", C.c_void_p), ("vel", C.c_void_p),
                ("speed", C.c_void_p), ("ang_vel", C.c_void_p),
                ("z", C.c_void_p), ("vz", C.c_void_p), ("attitude", C.c_void_p),
                ("body_rates", C.c_void_p)]


class ObstaclesC(C.Structure):
    _fields_ = [
        ("n_obstacles", C.c_int32),
        ("pos", C.c_void_p), ("angle", C.c_void_p), ("vel", C.c_void_p), ("ang_vel", C.c_void_p),
        ("radius", C.c_void_p), ("half", C.c_void_p),
        ("shape", C.c_void_p), ("kind", C.c_void_p),
        ("mass", C.c_void_p), ("inertia", C.c_void_p),
        ("body", C.c_void_p), ("body_off", C.c_void_p),
        ("any_movable", C.c_int32), ("bodies_move", C.c_int32), ("movable_shapes", C.c_int32),
        ("poses_from_bodies", C.c_int32),
    ]


class Bodies(C.Structure):
    _fields_ = [("pos", C.c_void_p), ("angle", C.c_void_p), ("vel", C.c_void_p),
                ("ang_vel", C.c_void_p)]


class GoalLoss(C.Structure):
    _fields_ = [("goal", C.c_void_p), ("loss", C.c_void_p), ("loss_grad", C.c_void_p)]


class WorldC(C.Structure):
    _fields_ = [
        ("dtype", C.c_int32), ("n_envs", C.c_int32), ("n_agents", C.c_int32),
        ("act_dim", C.c_int32), ("substeps", C.c_int32),
        ("dt", C.c_double),
        ("collisions", C.c_int32),
        ("k", C.c_double), ("c", C.c_double), ("margin", C.c_double),
        ("max_overlap", C.c_double), ("neighbor_radius", C.c_double),
        ("max_neighbors", C.c_int32), ("bounds_mode", C.c_int32),
        ("bounds", C.c_double * 4),
        ("lin_damping", C.c_double), ("ang_damping", C.c_double),
        ("params", C.c_void_p), ("params_env_stride", C.c_int64),
        ("model_tag", C.c_void_p), ("ctrl_mode", C.c_void_p),
        ("fleet_models", C.c_int32), ("fleet_modes", C.c_int32),
        ("obstacles", ObstaclesC),
        ("integrator", C.c_int32),
        ("box_agents", C.c_int32),
    ]


#: exported symbol -> (restype, argtypes); every entry point the header declares
SIGNATURES = {
    "swarp_rollout_workspace_bytes": (C.c_size_t, [C.POINTER(WorldC), C.c_int32]),
    "swarp_rollout_fwd": (C.c_int, [C.POINTER(WorldC), C.c_int32, State, C.c_void_p, State, State,
                                    C.c_void_p, Bodies, Bodies, GoalLoss, C.c_void_p, C.c_size_t,
                                    C.c_void_p]),
    "swarp_rollout_bwd": (C.c_int, [C.POINTER(WorldC), C.c_int32, State, C.c_void_p, State, State,
                                    State, Bodies, Bodies, Bodies, C.c_void_p, State, C.c_void_p,
                                    GoalLoss, C.c_void_p, C.c_size_t, C.c_void_p]),
    "swarp_neighbors": (C.c_int, [C.POINTER(WorldC), C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p]),
    "swarp_rollout_noalloc": (C.c_int, [C.POINTER(WorldC), C.c_int32, State, C.c_void_p, State,
                                        State, State, State, C.c_void_p, State, C.c_void_p]),
    "swarp_copy_rows": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t,
                                  C.c_size_t, C.c_void_p]),
    "swarp_error_string": (C.c_char_p, [C.c_int]),
    "swarp_abi_version": (C.c_int32, []),
}

_lib = None


def load(require_cuda: bool = True):
    """The loaded library. Raises if it is missing or (by default) CUDA is unavailable."""
    global _lib
    if require_cuda and not torch.cuda.is_available():
        raise RuntimeError(
            "swarp_b200 runs only on a CUDA device (sm_100a); no CUDA device is visible and "
            "there is no CPU fallback"
        )
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m swarp_b200.build` "
                "(there is no CPU fallback)"
            )
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != SWARP_OK:
        msg = _lib.swarp_error_string(rc).decode() if _lib is not None else ERRORS.get(rc, "?")
        if rc == -2:
            raise NotImplementedError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed with code {rc}: {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def state_c(fields) -> State:
    """``State`` of five (2-D) or nine (with the drone fields) tensors or Nones."""
    return State(*(ptr(t) for t in fields))


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
