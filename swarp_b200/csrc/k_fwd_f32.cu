// Kernel instances: fwd rollout, float, semi-implicit Euler integrator.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_fwd_part<float, 0>(const RolloutArgs<float>&, int, cudaStream_t);
template int launch_neighbors<float>(int, int, int, int, float, float, const float*, int*, int*, int*, cudaStream_t);
}  // namespace swarp
