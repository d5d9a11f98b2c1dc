// Kernel instances: cluster forward rollout (float) and the wide-env neighbor lists.
#include "k_cl.cuh"
namespace swarp {
template int launch_fwd_cl<float>(const RolloutArgs<float>&, int, int, cudaStream_t);
template int launch_neighbors_wide<float>(int, int, int, int, int, float, float, const float*, int*, int*, int*, cudaStream_t);
}  // namespace swarp
