// Kernel instances: bwd rollout, float, semi-implicit Euler integrator.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd_part<float, 0>(const RolloutArgs<float>&, int, cudaStream_t);
}  // namespace swarp
