// Kernel instances: bwd rollout, float.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd<float>(const RolloutArgs<float>&, int, cudaStream_t);
}  // namespace swarp
