// Kernel instances: bwd rollout, double, semi-implicit Euler integrator.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd_part<double, 0>(const RolloutArgs<double>&, int, cudaStream_t);
}  // namespace swarp
