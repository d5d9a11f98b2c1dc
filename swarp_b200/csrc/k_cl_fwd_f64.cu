// Kernel instances: cluster forward rollout (double) and the wide-env neighbor lists.
#include "k_cl.cuh"
namespace swarp {
template int launch_fwd_cl<double>(const RolloutArgs<double>&, int, int, cudaStream_t);
template int launch_neighbors_wide<double>(int, int, int, int, int, double, double, const double*, int*, int*, int*, cudaStream_t);
}  // namespace swarp
