// Kernel-instance selection. The launchers are defined in one translation unit per
// (direction, dtype) (k_*.cu) so the instances compile in parallel; capi.cu only
// declares them.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "rollout.cuh"

namespace swarp {

constexpr int kErrUnsupported = -2;
constexpr int kErrCuda = -4;

// The instances are split by integrator (RB = 0: Euler cases, RB = F_RK4: the same cases
// with RK4) and, for the forward, by whether box agents are present (RB | F_BOXES) so that
// each part compiles in a translation unit of its own (k_*.cu).
template <typename T, int RB> int launch_fwd_part(const RolloutArgs<T>& R, int fl, cudaStream_t st);
template <typename T, int RB> int launch_bwd_part(const RolloutArgs<T>& R, int fl, cudaStream_t st);
// Two agents per thread (float, A == 16, contact masks, no moving bodies; rollout_x2.cuh).
// R.G counts envs per CTA of 8 threads each.
int launch_fwd_x2(const RolloutArgs<float>& R, int fl, cudaStream_t st);
int launch_bwd_x2(const RolloutArgs<float>& R, int fl, cudaStream_t st);

template <typename T> inline int launch_fwd(const RolloutArgs<T>& R, int fl, cudaStream_t st) {
  if (fl & F_DRONE)
    return (fl & F_RK4) ? launch_fwd_part<T, F_DRONE | F_RK4>(R, fl, st)
                        : launch_fwd_part<T, F_DRONE>(R, fl, st);
  if (fl & F_BOXES)
    return (fl & F_RK4) ? launch_fwd_part<T, F_BOXES | F_RK4>(R, fl, st)
                        : launch_fwd_part<T, F_BOXES>(R, fl, st);
  return (fl & F_RK4) ? launch_fwd_part<T, F_RK4>(R, fl, st) : launch_fwd_part<T, 0>(R, fl, st);
}
template <typename T> inline int launch_bwd(const RolloutArgs<T>& R, int fl, cudaStream_t st) {
  if (fl & F_DRONE)
    return (fl & F_RK4) ? launch_bwd_part<T, F_DRONE | F_RK4>(R, fl, st)
                        : launch_bwd_part<T, F_DRONE>(R, fl, st);
  if (fl & F_BOXES)
    return (fl & F_RK4) ? launch_bwd_part<T, F_BOXES | F_RK4>(R, fl, st)
                        : launch_bwd_part<T, F_BOXES>(R, fl, st);
  return (fl & F_RK4) ? launch_bwd_part<T, F_RK4>(R, fl, st) : launch_bwd_part<T, 0>(R, fl, st);
}
template <typename T>
int launch_neighbors(int E, int A, int G, int K, T r2_scan, T r2, const T* pos, int* idx, int* cnt,
                     int* tru, cudaStream_t st);
// Envs wider than one CTA (rollout_cluster.cuh): one env per cluster of R.CS CTAs of
// `block` threads each; lists of such envs from `slices` CTAs per env.
template <typename T> int launch_fwd_cl(const RolloutArgs<T>& R, int fl, int block, cudaStream_t st);
template <typename T> int launch_bwd_cl(const RolloutArgs<T>& R, int fl, int block, cudaStream_t st);
template <typename T>
int launch_neighbors_wide(int E, int A, int slices, int block, int K, T r2_scan, T r2, const T* pos,
                          int* idx, int* cnt, int* tru, cudaStream_t st);

#ifdef SWARP_DEFINE_LAUNCHERS

// Raise a kernel's dynamic shared-memory limit once per size (per device): the attribute
// call is not stream-ordered, so keeping it off the common launch path also keeps launches
// inside CUDA-graph capture free of it after the first (uncaptured) call of a shape. The
// default limit (48 KB) covers static and dynamic shared memory together, and these kernels
// also hold a little static shared memory (the block reductions' warp sums), so sizes from
// kSmemNoRaise up are raised explicitly.
constexpr size_t kSmemNoRaise = 40 * 1024;
template <typename K>
inline bool ensure_smem_limit(K kernel, size_t smem) {
  if (smem <= kSmemNoRaise) return true;
  static std::mutex mu;
  static std::unordered_map<long long, size_t> raised;  // (device, kernel) -> limit set
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const long long key = (static_cast<long long>(dev) << 56) ^
                        static_cast<long long>(reinterpret_cast<uintptr_t>(kernel));
  std::lock_guard<std::mutex> lock(mu);
  auto it = raised.find(key);
  if (it != raised.end() && it->second >= smem) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return false;
  raised[key] = smem;
  return true;
}

template <typename K>
inline int launch_kernel(K kernel, int grid, int block, size_t smem, cudaStream_t st,
                         const void* arg) {
  if (!ensure_smem_limit(kernel, smem)) return kErrCuda;
  void* args[] = {const_cast<void*>(arg)};
  return cudaLaunchKernel(reinterpret_cast<const void*>(kernel), dim3(grid), dim3(block), args, smem,
                          st) == cudaSuccess
             ? 0
             : kErrCuda;
}

template <typename T, int FL, int AS, int LB = 1024>
int run_fwd(const RolloutArgs<T>& R, cudaStream_t st) {
  const Layout<T> L(R.G, R.A, R.N, R.S, false, (FL & F_BODIES) != 0,
                    (FL & F_BOXES) != 0 && (FL & (F_COLL | F_BODIES)) != 0);
  const int grid = (R.E + R.G - 1) / R.G;
  const int rc = launch_kernel(rollout_fwd_kernel<T, FL, AS, LB>, grid, R.G * R.A, L.total, st, &R);
  if (rc != 0 || !R.goal) return rc;
  sum_partials_kernel<T><<<1, 256, 0, st>>>(R.loss_partial, grid, R.loss_out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}
template <typename T, int FL, int AS, int LB = 1024>
int run_bwd(const RolloutArgs<T>& R, cudaStream_t st) {
  const Layout<T> L(R.G, R.A, R.N, R.S, true, (FL & F_BODIES) != 0,
                    (FL & F_BOXES) != 0 && (FL & F_COLL) != 0, (FL & F_DRONE) != 0);
  const int grid = (R.E + R.G - 1) / R.G;
  const int rc = launch_kernel(rollout_bwd_kernel<T, FL, AS, LB>, grid, R.G * R.A, L.total, st, &R);
  if (rc != 0 || !R.gsq_partial) return rc;
  sum_partials_kernel<T><<<1, 256, 0, st>>>(R.gsq_partial, grid, R.gsq_out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

// Every valid flag combination: no contacts, contacts, truncating contacts, checkpointed
// contacts, truncating checkpointed contacts; each with/without obstacles and with/without
// the holonomic-velocity fleet; moving bodies (always with obstacles) with each contact
// mode and fleet kind.
#define SWARP_FLAG_CASES_EULER(X, R)                                                           \
  X(R + 0) X(R + 4) X(R + 8) X(R + 12) X(R + 1) X(R + 5) X(R + 9) X(R + 13) X(R + 3) X(R + 7) \
  X(R + 11) X(R + 15) X(R + 17) X(R + 21) X(R + 25) X(R + 29) X(R + 36) X(R + 37) X(R + 39)   \
  X(R + 53) X(R + 44) X(R + 45) X(R + 47) X(R + 61) X(R + 19) X(R + 23) X(R + 27) X(R + 31)   \
  X(R + 55) X(R + 63)
// (each instantiated once with R = 0 and once with R = F_RK4)

// Drone worlds: the contact and obstacle cases, and movable bodies (always with obstacles)
// with each contact mode (R = F_DRONE, F_DRONE | F_RK4); a drone fleet is never a
// holonomic-velocity fleet.
#define SWARP_FLAG_CASES_DRONE(X, R)                                                       \
  X(R + 0) X(R + 4) X(R + 1) X(R + 5) X(R + 3) X(R + 7) X(R + 17) X(R + 21) X(R + 36) X(R + 37) \
  X(R + 39) X(R + 53)

// Box-agent worlds: the cases without moving bodies (R = F_BOXES, F_BOXES | F_RK4); the
// forward also runs box agents pushing movable bodies (their adjoint is not built).
#define SWARP_FLAG_CASES_BOXES(X, R)                                                           \
  X(R + 0) X(R + 4) X(R + 8) X(R + 12) X(R + 1) X(R + 5) X(R + 9) X(R + 13) X(R + 3) X(R + 7) \
  X(R + 11) X(R + 15) X(R + 17) X(R + 21) X(R + 25) X(R + 29)
#define SWARP_FLAG_CASES_BOXES_BODIES(X, R) \
  X(R + 36) X(R + 37) X(R + 39) X(R + 53) X(R + 44) X(R + 45) X(R + 47) X(R + 61)

template <typename T, int RB> int launch_fwd_part(const RolloutArgs<T>& R, int fl, cudaStream_t st) {
  const bool a16 = std::is_same<T, float>::value && R.A == 16;
#define SWARP_X(F)                                                          \
  case F:                                                                   \
    if constexpr (std::is_same<T, float>::value && ((F) & F_COLL))          \
      if (a16) return run_fwd<T, F, 16>(R, st);                             \
    if constexpr (((F) & F_BODIES) != 0)                                    \
      if (R.G * R.A <= kSmallCTA) return run_fwd<T, F, 0, kSmallCTA>(R, st); \
    return run_fwd<T, F, 0>(R, st);
  if constexpr ((RB & F_DRONE) != 0) {
    switch (fl) { SWARP_FLAG_CASES_DRONE(SWARP_X, RB) }
  } else if constexpr ((RB & F_BOXES) != 0) {
    switch (fl) { SWARP_FLAG_CASES_BOXES(SWARP_X, RB) SWARP_FLAG_CASES_BOXES_BODIES(SWARP_X, RB) }
  } else {
    switch (fl) { SWARP_FLAG_CASES_EULER(SWARP_X, RB) }
  }
#undef SWARP_X
  return kErrUnsupported;
}

template <typename T, int RB> int launch_bwd_part(const RolloutArgs<T>& R, int fl, cudaStream_t st) {
  const bool a16 = std::is_same<T, float>::value && R.A == 16;
#define SWARP_X(F)                                                          \
  case F:                                                                   \
    if constexpr (std::is_same<T, float>::value && ((F) & F_COLL))          \
      if (a16) return run_bwd<T, F, 16>(R, st);                             \
    if constexpr (((F) & F_BODIES) != 0)                                    \
      if (R.G * R.A <= kSmallCTA) return run_bwd<T, F, 0, kSmallCTA>(R, st); \
    return run_bwd<T, F, 0>(R, st);
  if constexpr ((RB & F_DRONE) != 0) {
    switch (fl) { SWARP_FLAG_CASES_DRONE(SWARP_X, RB) }
  } else if constexpr ((RB & F_BOXES) != 0) {
    switch (fl) { SWARP_FLAG_CASES_BOXES(SWARP_X, RB) }
  } else {
    switch (fl) { SWARP_FLAG_CASES_EULER(SWARP_X, RB) }
  }
#undef SWARP_X
  return kErrUnsupported;
}

template <typename T>
int launch_neighbors(int E, int A, int G, int K, T r2_scan, T r2, const T* pos, int* idx, int* cnt,
                     int* tru, cudaStream_t st) {
  const size_t smem = ((size_t(G) * ((A + 1) / 2) * 4 * sizeof(T) + 15) & ~size_t(15)) +
                      size_t(G) * A * 4 * sizeof(T);
  auto k = neighbors_kernel<T>;
  if (!ensure_smem_limit(k, smem)) return kErrCuda;
  k<<<(E + G - 1) / G, G * A, smem, st>>>(E, A, G, K, r2_scan, r2, pos, idx, cnt, tru);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

#endif  // SWARP_DEFINE_LAUNCHERS

}  // namespace swarp
