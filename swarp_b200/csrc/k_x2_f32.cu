// Kernel instances: the two-agents-per-thread forward and adjoint (float, 16 agents).
#define SWARP_DEFINE_LAUNCHERS
#include "launch.cuh"
#include "rollout_x2.cuh"

namespace swarp {

namespace {
template <int FL>
int run_fwd_x2(const RolloutArgs<float>& R, cudaStream_t st) {
  const Layout<float> L(R.G, kX2Agents, R.N, R.S, false, false);
  const int grid = (R.E + R.G - 1) / R.G;
  const int rc = launch_kernel(rollout_fwd_x2_kernel<FL>, grid, R.G * kX2Threads, L.total, st, &R);
  if (rc != 0 || !R.goal) return rc;
  sum_partials_kernel<float><<<1, 256, 0, st>>>(R.loss_partial, grid, R.loss_out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}
template <int FL>
int run_bwd_x2(const RolloutArgs<float>& R, cudaStream_t st) {
  const Layout<float> L(R.G, kX2Agents, R.N, 1, true, false);
  const int grid = (R.E + R.G - 1) / R.G;
  const int rc = launch_kernel(rollout_bwd_x2_kernel<FL>, grid, R.G * kX2Threads, L.total, st, &R);
  if (rc != 0 || !R.gsq_partial) return rc;
  sum_partials_kernel<float><<<1, 256, 0, st>>>(R.gsq_partial, grid, R.gsq_out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}
}  // namespace

// Contact-mask worlds without moving bodies: with/without obstacles, any or the
// holonomic-velocity fleet, each with either integrator.
#define SWARP_X2_CASES(X) X(17) X(21) X(25) X(29) X(81) X(85) X(89) X(93)

int launch_fwd_x2(const RolloutArgs<float>& R, int fl, cudaStream_t st) {
  switch (fl) {
#define SWARP_X(F) \
  case F:          \
    return run_fwd_x2<F>(R, st);
    SWARP_X2_CASES(SWARP_X)
#undef SWARP_X
  }
  return kErrUnsupported;
}

int launch_bwd_x2(const RolloutArgs<float>& R, int fl, cudaStream_t st) {
  switch (fl) {
#define SWARP_X(F) \
  case F:          \
    return run_bwd_x2<F>(R, st);
    SWARP_X2_CASES(SWARP_X)
#undef SWARP_X
  }
  return kErrUnsupported;
}

}  // namespace swarp
