// Kernel instances: bwd rollout, float, RK4 integrator.
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
namespace swarp {
template int launch_bwd_part<float, F_RK4>(const RolloutArgs<float>&, int, cudaStream_t);
}  // namespace swarp
