// Kernel instances: bwd rollout, float, 6-DOF drone fleets, both integrators.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd_part<float, F_DRONE>(const RolloutArgs<float>&, int, cudaStream_t);
template int launch_bwd_part<float, F_DRONE | F_RK4>(const RolloutArgs<float>&, int, cudaStream_t);
}  // namespace swarp
