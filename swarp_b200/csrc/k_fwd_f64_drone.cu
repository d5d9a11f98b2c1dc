// Kernel instances: fwd rollout, double, 6-DOF drone fleets, both integrators.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_fwd_part<double, F_DRONE>(const RolloutArgs<double>&, int, cudaStream_t);
template int launch_fwd_part<double, F_DRONE | F_RK4>(const RolloutArgs<double>&, int, cudaStream_t);
}  // namespace swarp
