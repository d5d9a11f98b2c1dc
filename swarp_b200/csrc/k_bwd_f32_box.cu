// Kernel instances: bwd rollout, float, box agents, both integrators.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd_part<float, F_BOXES>(const RolloutArgs<float>&, int, cudaStream_t);
template int launch_bwd_part<float, F_BOXES | F_RK4>(const RolloutArgs<float>&, int, cudaStream_t);
}  // namespace swarp
