"""The allocation-free rollout entry point against the allocating ones (GPU).

``swarp_rollout_noalloc`` exists for callers that cannot allocate device memory: code
running under another runtime's memory manager (an XLA/JAX custom call, another
framework's operator) must not allocate behind that manager's back, and a real-time
control loop cannot wait on cudaMalloc, which may synchronize the device. It keeps the
forward/adjoint workspace (per-substep contact masks, plus list cutoffs when the neighbor
cap truncates) in a static device array owned by the library.

Here it is called through the C ABI twice in a row per case, on different inputs, so the
second call starts from the first call's leftovers in that array. Both calls run the
same kernels on the same inputs as ``swarp_rollout_fwd`` + ``swarp_rollout_bwd`` with a
caller-allocated workspace, so every output must equal theirs bit for bit. Around the
second call neither torch's allocator nor the driver's free-memory count may move. This
file is collected last on purpose.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
E, A, T = 300, 16, 12


def _inputs(seed, dtype):
    g = torch.Generator(device=DEV).manual_seed(seed)
    pos = (torch.rand(E, A, 2, generator=g, device=DEV) - 0.5).to(dtype)  # dense: contacts
    z = torch.zeros(E, A, device=DEV, dtype=dtype)
    state5 = (pos, z.clone(), (torch.randn(E, A, 2, generator=g, device=DEV) * 0.2).to(dtype),
              z.clone(), z.clone())
    acts = (torch.rand(T, E, A, 2, generator=g, device=DEV) * 2 - 1).to(dtype)
    gfin = (torch.randn(E, A, 2, generator=g, device=DEV).to(dtype), None,
            torch.randn(E, A, 2, generator=g, device=DEV).to(dtype), None, None)
    return state5, acts, gfin


# (dtype, max_neighbors): K=16 checkpoints contact masks, K=8 truncates the lists and
# checkpoints their cutoffs beside the masks
CASES = [(torch.float32, 16), (torch.float32, 8), (torch.float64, 16)]


@pytest.mark.parametrize("dtype,K", CASES, ids=["f32-masks", "f32-cutoffs", "f64-masks"])
def test_noalloc_matches_allocating_entry_points_twice(dtype, K):
    from swarp_b200 import _lib
    from swarp_b200.core.config import WorldConfig
    from swarp_b200.core.stepper import Stepper
    from swarp_b200.dynamics.base import AgentConfig

    lib = _lib.load()
    world = WorldConfig(collision_k=100.0, collision_c=1.0, collision_margin=0.025,
                        bounds=(-1.0, 1.0, -1.0, 1.0), neighbor_radius=0.125, max_neighbors=K)
    st = Stepper([AgentConfig(radius=0.05, max_speed=1.0, max_accel=2.0) for _ in range(A)],
                 dt=0.05, device=DEV, dtype=dtype, world=world)
    wc = st.world_c(E, 2)
    need = lib.swarp_rollout_workspace_bytes(C.byref(wc), T)
    assert 0 < need <= 16 << 20  # this rollout does use scratch, and it fits the static array
    stream = _lib.stream_ptr(torch.device(DEV))

    for seed in (1, 2):
        state5, acts, gfin = _inputs(seed + K, dtype)
        traj_r, fin_r, _, ws = st.rollout_forward(state5, acts, final=True)
        gact_r, ginit_r = st.rollout_backward(state5, acts, traj_r, (None,) * 5, gfin, ws)

        traj = tuple(torch.empty_like(x) for x in traj_r)
        fin = tuple(torch.empty_like(x) for x in fin_r)
        gact = torch.empty_like(acts)
        ginit = tuple(torch.empty_like(x) for x in state5)
        torch.cuda.synchronize()
        torch_before = torch.cuda.memory_allocated(DEV)
        free_before = torch.cuda.mem_get_info(DEV)[0]
        rc = lib.swarp_rollout_noalloc(C.byref(wc), T, _lib.state_c(state5), acts.data_ptr(),
                                       _lib.state_c(traj), _lib.state_c(fin),
                                       _lib.state_c((None,) * 5), _lib.state_c(gfin),
                                       gact.data_ptr(), _lib.state_c(ginit), stream)
        assert rc == 0, lib.swarp_error_string(rc)
        torch.cuda.synchronize()
        if seed == 2:  # every kernel and the array's module are loaded by now
            assert torch.cuda.memory_allocated(DEV) == torch_before
            assert torch.cuda.mem_get_info(DEV)[0] == free_before
        for got, ref in zip(traj + fin + (gact,) + ginit, traj_r + fin_r + (gact_r,) + ginit_r,
                            strict=True):
            assert torch.equal(got, ref)


def test_noalloc_rejects_rollouts_above_the_static_scratch():
    from swarp_b200 import _lib
    from swarp_b200.core.config import WorldConfig
    from swarp_b200.core.stepper import Stepper
    from swarp_b200.dynamics.base import AgentConfig

    lib = _lib.load()
    st = Stepper([AgentConfig(radius=0.05) for _ in range(A)], dt=0.05, device=DEV,
                 dtype=torch.float32,
                 world=WorldConfig(neighbor_radius=0.125, max_neighbors=16))
    wc = st.world_c(16000, 2)
    assert lib.swarp_rollout_workspace_bytes(C.byref(wc), 64) > 16 << 20
    # The size check comes before any pointer is used or kernel launched.
    rc = lib.swarp_rollout_noalloc(C.byref(wc), 64, _lib.State(), None, _lib.State(),
                                   _lib.State(), _lib.State(), _lib.State(), None, _lib.State(),
                                   None)
    assert rc == -6
    assert b"static scratch" in lib.swarp_error_string(rc)
