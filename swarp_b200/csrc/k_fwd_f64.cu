// Kernel instances: fwd rollout, double.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_fwd<double>(const RolloutArgs<double>&, int, cudaStream_t);
template int launch_neighbors<double>(int, int, int, int, double, const double*, int*, int*, int*, cudaStream_t);
}  // namespace swarp
