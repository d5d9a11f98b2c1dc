// Kernel instances: cluster adjoint rollout (float).
#include "k_cl.cuh"
namespace swarp {
template int launch_bwd_cl<float>(const RolloutArgs<float>&, int, int, cudaStream_t);
}  // namespace swarp
