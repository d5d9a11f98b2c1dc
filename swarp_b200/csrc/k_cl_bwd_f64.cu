// Kernel instances: cluster adjoint rollout (double).
#include "k_cl.cuh"
namespace swarp {
template int launch_bwd_cl<double>(const RolloutArgs<double>&, int, int, cudaStream_t);
}  // namespace swarp
