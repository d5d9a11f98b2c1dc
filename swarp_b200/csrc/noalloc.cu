// Allocation-free BPTT rollout (swarp_rollout_noalloc, declared in include/swarp_b200.h).
//
// Some callers cannot allocate device memory: a plugin running under another runtime's
// memory manager (an XLA/JAX custom call, another framework's operator) must not create
// allocations behind that manager's back, and a real-time control loop cannot wait on
// cudaMalloc, which may synchronize the device.
// For them this entry point runs the forward rollout and its adjoint back to back with
// the workspace they share (per-substep contact masks or list cutoffs) placed in a
// static device array that the library owns, instead of a buffer the caller allocates.
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds
// its own SWARP_NOALLOC_SCRATCH_BYTES copy until the process exits. Host code cannot use
// the array's name as a device address (on the host it names a host-side shadow), so the
// device address is resolved with cudaGetSymbolAddress, once per device, with that
// device current, on the first call there (which should therefore come before any stream
// capture), and cached for the life of the process: a cudaDeviceReset destroys the array
// with the context, after which this entry point must not be called on that device. The forward writes every workspace cell the adjoint reads,
// so nothing in the array has to start at zero. All calls share the one array: calls
// whose work overlaps on a GPU (different streams, or different host threads on one
// device) race on it and must be serialized by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/swarp_b200.h"

static __device__ __align__(256) unsigned char g_noalloc_scratch[SWARP_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

// Device address of this device's copy of the scratch array (resolved on first use).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SWARP_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return SWARP_ERR_CUDA;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return SWARP_OK;
}

}  // namespace

extern "C" int swarp_rollout_noalloc(const swarp_world_t* w, int32_t horizon, swarp_state_t init,
                                     const void* actions, swarp_state_t traj,
                                     swarp_state_t final_out, swarp_state_t adj_traj,
                                     swarp_state_t adj_final, void* adj_actions,
                                     swarp_state_t adj_init, void* stream) {
  if (!w) return SWARP_ERR_INVALID_ARG;
  if (w->obstacles.n_obstacles > 0 && w->obstacles.any_movable && w->obstacles.bodies_move)
    return SWARP_ERR_UNSUPPORTED;  // movable-body state needs caller buffers
  const size_t need = swarp_rollout_workspace_bytes(w, horizon);
  if (need > SWARP_NOALLOC_SCRATCH_BYTES) return SWARP_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = scratch_address(&scratch);
    if (rc != SWARP_OK) return rc;
  }
  const swarp_bodies_t none = {nullptr, nullptr, nullptr, nullptr};
  const swarp_goal_loss_t no_goal = {nullptr, nullptr, nullptr};
  int rc = swarp_rollout_fwd(w, horizon, init, actions, traj, final_out, nullptr, none, none,
                             no_goal, scratch, need, stream);
  if (rc != SWARP_OK) return rc;
  return swarp_rollout_bwd(w, horizon, init, actions, traj, adj_traj, adj_final, none, none, none,
                           adj_actions, adj_init, nullptr, no_goal, scratch, need, stream);
}
