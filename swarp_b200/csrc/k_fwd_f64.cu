// Kernel instances: fwd rollout, double, semi-implicit Euler integrator.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_fwd_part<double, 0>(const RolloutArgs<double>&, int, cudaStream_t);
template int launch_neighbors<double>(int, int, int, int, double, double, const double*, int*, int*, int*, cudaStream_t);
}  // namespace swarp
