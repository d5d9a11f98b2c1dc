// Kernel instances: bwd rollout, double, box agents, both integrators.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd_part<double, F_BOXES>(const RolloutArgs<double>&, int, cudaStream_t);
template int launch_bwd_part<double, F_BOXES | F_RK4>(const RolloutArgs<double>&, int, cudaStream_t);
}  // namespace swarp
