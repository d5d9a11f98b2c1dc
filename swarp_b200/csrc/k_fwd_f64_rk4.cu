// Kernel instances: fwd rollout, double, RK4 integrator.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_fwd_part<double, F_RK4>(const RolloutArgs<double>&, int, cudaStream_t);
}  // namespace swarp
