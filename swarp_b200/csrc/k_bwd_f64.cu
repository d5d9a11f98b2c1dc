// Kernel instances: bwd rollout, double.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd<double>(const RolloutArgs<double>&, int, cudaStream_t);
}  // namespace swarp
