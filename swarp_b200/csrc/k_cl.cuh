// Launchers of the cluster kernels (rollout_cluster.cuh), instantiated per (direction,
// dtype) in k_cl_*.cu.
#pragma once
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
#include "rollout_cluster.cuh"

namespace swarp {

// One launch with a cluster of `cs` CTAs along x (grid a multiple of cs).
template <typename K>
inline int launch_cluster(K kernel, int grid, int block, int cs, size_t smem, cudaStream_t st,
                          const void* arg) {
  if (!ensure_smem_limit(kernel, smem)) return kErrCuda;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<void*>(arg)};
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), args) == cudaSuccess
             ? 0
             : kErrCuda;
}

template <typename T, int FL>
int run_fwd_cl(const RolloutArgs<T>& R, int block, cudaStream_t st) {
  const ClusterLayout<T> L(R.A, block, R.N, R.S, false);
  const int grid = R.E * R.CS;
  const int rc = launch_cluster(rollout_fwd_cl_kernel<T, FL>, grid, block, R.CS, L.total, st, &R);
  if (rc != 0 || !R.goal) return rc;
  sum_partials_kernel<T><<<1, 256, 0, st>>>(R.loss_partial, grid, R.loss_out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}
template <typename T, int FL>
int run_bwd_cl(const RolloutArgs<T>& R, int block, cudaStream_t st) {
  const ClusterLayout<T> L(R.A, block, R.N, R.S, true);
  const int grid = R.E * R.CS;
  const int rc = launch_cluster(rollout_bwd_cl_kernel<T, FL>, grid, block, R.CS, L.total, st, &R);
  if (rc != 0 || !R.gsq_partial) return rc;
  sum_partials_kernel<T><<<1, 256, 0, st>>>(R.gsq_partial, grid, R.gsq_out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

// Disc fleets: no contacts, contacts, truncating contacts; each with/without obstacles and
// the holonomic-velocity fleet; Euler (R = 0) or RK4 (R = F_RK4).
#define SWARP_CL_CASES(X, R) \
  X(R + 0) X(R + 4) X(R + 8) X(R + 12) X(R + 1) X(R + 5) X(R + 9) X(R + 13) X(R + 3) X(R + 7) \
  X(R + 11) X(R + 15)

template <typename T> int launch_fwd_cl(const RolloutArgs<T>& R, int fl, int block, cudaStream_t st) {
  switch (fl) {
#define SWARP_X(F) \
  case F:          \
    return run_fwd_cl<T, F>(R, block, st);
    SWARP_CL_CASES(SWARP_X, 0)
    SWARP_CL_CASES(SWARP_X, F_RK4)
#undef SWARP_X
  }
  return kErrUnsupported;
}

template <typename T> int launch_bwd_cl(const RolloutArgs<T>& R, int fl, int block, cudaStream_t st) {
  switch (fl) {
#define SWARP_X(F) \
  case F:          \
    return run_bwd_cl<T, F>(R, block, st);
    SWARP_CL_CASES(SWARP_X, 0)
    SWARP_CL_CASES(SWARP_X, F_RK4)
#undef SWARP_X
  }
  return kErrUnsupported;
}

template <typename T>
int launch_neighbors_wide(int E, int A, int slices, int block, int K, T r2_scan, T r2, const T* pos,
                          int* idx, int* cnt, int* tru, cudaStream_t st) {
  const size_t smem = size_t((A + 1) / 2) * 4 * sizeof(T);
  auto k = neighbors_wide_kernel<T>;
  if (!ensure_smem_limit(k, smem)) return kErrCuda;
  k<<<E * slices, block, smem, st>>>(E, A, slices, K, r2_scan, r2, pos, idx, cnt, tru);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace swarp
