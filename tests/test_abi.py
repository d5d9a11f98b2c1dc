"""The C-ABI library loads and exports every entry point include/swarp_b200.h declares,
and the ctypes mirrors of its structs have the C layout (checked with gcc). CPU only:
no compute call is made here."""

import ctypes as C
import os
import re
import subprocess

import pytest

from swarp_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "swarp_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(swarp_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return C.CDLL(_lib.LIB_PATH)


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert "swarp_rollout_fwd" in names and "swarp_rollout_bwd" in names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"


def test_bindings_cover_the_header():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_error_strings_and_version(lib):
    lib.swarp_error_string.restype = C.c_char_p
    assert lib.swarp_error_string(0) == b"ok"
    assert b"unsupported" in lib.swarp_error_string(-2)
    assert lib.swarp_abi_version() == 7


def test_invalid_world_is_rejected_without_a_gpu(lib):
    """Argument validation happens before any CUDA call."""
    fn = lib.swarp_rollout_workspace_bytes
    fn.restype = C.c_size_t
    fn.argtypes = [C.POINTER(_lib.WorldC), C.c_int32]
    w = _lib.WorldC()
    assert fn(C.byref(w), 4) == 0  # all-zero world is invalid -> 0
    fwd = lib.swarp_rollout_fwd
    fwd.restype = C.c_int
    fwd.argtypes = _lib.SIGNATURES["swarp_rollout_fwd"][1]
    rc = fwd(None, 4, _lib.State(), None, _lib.State(), _lib.State(), None, _lib.Bodies(),
             _lib.Bodies(), _lib.GoalLoss(), None, 0, None)
    assert rc == -1
    w.dtype, w.n_envs, w.n_agents, w.act_dim, w.substeps, w.dt = 0, 2, 3, 2, 1, 0.1
    w.params, w.model_tag, w.ctrl_mode = 8, 8, 8  # non-null placeholders, never dereferenced
    w.fleet_models, w.fleet_modes = 1 << 4, 1  # an unknown model tag
    rc = fwd(C.byref(w), 4, _lib.State(), None, _lib.State(), _lib.State(), None, _lib.Bodies(),
             _lib.Bodies(), _lib.GoalLoss(), None, 0, None)
    assert rc == -2
    w.fleet_models = 1 << 3  # a drone fleet without its drone state fields
    rc = fwd(C.byref(w), 4, _lib.State(), None, _lib.State(), _lib.State(), None, _lib.Bodies(),
             _lib.Bodies(), _lib.GoalLoss(), None, 0, None)
    assert rc == -1
    w.fleet_models = 1
    w.n_agents = 5000
    rc = fwd(C.byref(w), 4, _lib.State(), None, _lib.State(), _lib.State(), None, _lib.Bodies(),
             _lib.Bodies(), _lib.GoalLoss(), None, 0, None)
    assert rc == -3


LAYOUT_C = r"""
#include <stdio.h>
#include <stddef.h>
#include "swarp_b200.h"
#define F(T, f) printf(#T "." #f " %zu\n", offsetof(T, f))
int main(void) {
  printf("swarp_world_t %zu\n", sizeof(swarp_world_t));
  printf("swarp_obstacles_t %zu\n", sizeof(swarp_obstacles_t));
  printf("swarp_state_t %zu\n", sizeof(swarp_state_t));
  printf("swarp_bodies_t %zu\n", sizeof(swarp_bodies_t));
  F(swarp_world_t, dt); F(swarp_world_t, collisions); F(swarp_world_t, k);
  F(swarp_world_t, max_neighbors); F(swarp_world_t, bounds); F(swarp_world_t, params);
  F(swarp_world_t, params_env_stride); F(swarp_world_t, fleet_models);
  F(swarp_world_t, obstacles); F(swarp_obstacles_t, pos); F(swarp_obstacles_t, any_movable);
  F(swarp_obstacles_t, bodies_move); F(swarp_obstacles_t, movable_shapes);
  F(swarp_obstacles_t, poses_from_bodies); F(swarp_world_t, integrator);
  F(swarp_world_t, box_agents); F(swarp_state_t, z); F(swarp_state_t, body_rates);
  return 0;
}
"""


def test_ctypes_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(LAYOUT_C)
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    out = dict(line.rsplit(" ", 1) for line in subprocess.check_output([str(exe)]).decode().split("\n")
               if line)
    assert int(out["swarp_world_t"]) == C.sizeof(_lib.WorldC)
    assert int(out["swarp_obstacles_t"]) == C.sizeof(_lib.ObstaclesC)
    assert int(out["swarp_state_t"]) == C.sizeof(_lib.State)
    assert int(out["swarp_bodies_t"]) == C.sizeof(_lib.Bodies)
    for key, val in out.items():
        if "." not in key:
            continue
        struct, field = key.split(".")
        cls = {"swarp_world_t": _lib.WorldC, "swarp_state_t": _lib.State}.get(struct, _lib.ObstaclesC)
        assert getattr(cls, field).offset == int(val), key


def _world(A, K, box=False):
    w = _lib.WorldC()
    w.dtype, w.n_envs, w.n_agents, w.act_dim, w.substeps, w.dt = 0, 100, A, 2, 2, 0.05
    w.params, w.model_tag, w.ctrl_mode = 8, 8, 8  # non-null placeholders, never dereferenced
    w.fleet_models, w.fleet_modes = 1, 1
    w.collisions, w.max_neighbors, w.neighbor_radius = 1, K, 0.2
    w.box_agents = int(box)
    return w


@pytest.mark.parametrize("A,K,box,masks_off,nw,trunc", [
    (16, 16, False, False, 1, False),   # contact masks, one word
    (16, 8, False, False, 1, True),     # truncating lists: masks and cutoffs
    (40, 64, False, False, 2, False),   # two mask words
    (40, 64, False, True, 0, False),    # SWARP_CONTACT_MASKS=0: the rescan path
    (256, 32, False, False, 8, True),   # the config-5 shape
    (300, 8, False, False, 0, True),    # above 256 agents: cutoffs only
    (40, 64, True, False, 0, False),    # box agents beyond 32: no masks
])
def test_workspace_holds_the_contact_checkpoint(lib, monkeypatch, A, K, box, masks_off, nw,
                                                trunc):
    """The workspace the forward fills for its adjoint: ceil(A/32) mask words per agent and
    substep where masks are checkpointed, int16 list cutoffs where lists can truncate, then
    one partial sum per CTA (host logic only, no GPU)."""
    if masks_off:
        monkeypatch.setenv("SWARP_CONTACT_MASKS", "0")
    fn = lib.swarp_rollout_workspace_bytes
    fn.restype = C.c_size_t
    fn.argtypes = [C.POINTER(_lib.WorldC), C.c_int32]
    H = 6
    w = _world(A, K, box)
    cells = H * 2 * 100 * A
    align = lambda b: (b + 255) // 256 * 256  # noqa: E731
    head = align(align(cells * nw * 4) + (cells * 2 if trunc else 0))
    got = fn(C.byref(w), H)
    assert head < got <= head + 100 * 4, (got, head)


def test_workspace_partials_cover_cluster_ctas(lib):
    """Envs above 1024 agents run one env per cluster of several CTAs, each of which writes
    one partial sum: the workspace holds one per CTA (E x 4 for 2048 agents)."""
    fn = lib.swarp_rollout_workspace_bytes
    fn.restype = C.c_size_t
    fn.argtypes = [C.POINTER(_lib.WorldC), C.c_int32]
    w = _world(2048, 8)
    cells = 6 * 2 * 100 * 2048
    head = (cells * 2 + 255) // 256 * 256  # cutoffs only (no masks above 256 agents)
    assert fn(C.byref(w), 6) >= head + 100 * 4 * 4
