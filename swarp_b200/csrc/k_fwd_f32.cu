// Kernel instances: fwd rollout, float.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_fwd<float>(const RolloutArgs<float>&, int, cudaStream_t);
template int launch_neighbors<float>(int, int, int, int, float, const float*, int*, int*, int*, cudaStream_t);
}  // namespace swarp
