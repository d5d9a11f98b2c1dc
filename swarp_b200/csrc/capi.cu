// C ABI of the rollout kernels: argument validation, kernel-instance selection and
// launch on the caller's stream. Declarations and contracts: include/swarp_b200.h.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <type_traits>

#include "../../include/swarp_b200.h"
#include "launch.cuh"
#include "rollout_cluster.cuh"

using namespace swarp;

namespace {

constexpr int kAbiVersion = 7;

int threads_target() {
  static int v = [] {
    const char* s = std::getenv("SWARP_CTA_THREADS");
    int t = s ? std::atoi(s) : 64;
    return (t >= 32 && t <= 1024) ? t : 64;
  }();
  return v;
}

// The two-agents-per-thread kernels (rollout_x2.cuh): on unless SWARP_X2=0.
bool x2_enabled() {
  static bool v = [] {
    const char* s = std::getenv("SWARP_X2");
    return !(s && s[0] == '0');
  }();
  return v;
}
bool aligned(const void* p, unsigned n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

// Whether a float world can take the two-agents-per-thread kernels (their preconditions:
// 16 agents, 2 action slots, checkpointed contact masks, no moving bodies, vector-aligned
// fields; the adjoint also one substep per step).
bool x2_ok(const RolloutArgs<float>& R, int fl, bool bwd) {
  if (!x2_enabled() || R.A != 16 || R.act_dim != 2) return false;
  if (!(fl & F_MASK) || (fl & (F_BODIES | F_TRUNC | F_BOXES | F_DRONE))) return false;
  if (bwd && R.S != 1) return false;
  const void* v16[] = {R.t_pos, R.t_vel, R.i_pos, R.i_vel, R.act, R.f_pos, R.f_vel, R.g_act};
  for (const void* p : v16)
    if (p && !aligned(p, 16)) return false;
  const void* v8[] = {R.t_th, R.t_s, R.t_w, R.i_th, R.i_s, R.i_w, R.f_th, R.f_s, R.f_w,
                      R.cmask, R.true_max};
  for (const void* p : v8)
    if (p && !aligned(p, 8)) return false;
  return true;
}
int x2_envs_per_cta(int E) { return E < 8 ? E : 8; }  // 64 threads: the kernels' launch bound

// Envs per CTA: whole envs, about threads_target() threads.
int envs_per_cta(int A, int E) {
  int target = threads_target();
  if (A == 16 && target > kMaxThreadsAS16) target = kMaxThreadsAS16;  // see rollout_bwd_kernel
  int G = A >= target ? 1 : target / A;
  if (G > E) G = E;
  return G < 1 ? 1 : G;
}

// Envs of more than one CTA's agents run one env per thread-block cluster
// (rollout_cluster.cuh). SWARP_CLUSTER_MIN_AGENTS (default 1025) and
// SWARP_CLUSTER_CTA_THREADS (default 512, at most kClusterMaxThreads) are read on every call,
// so a test can run small envs through the cluster kernels as well.
int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  return (s && *s) ? std::atoi(s) : dflt;
}
int cluster_min_agents() {
  const int v = env_int("SWARP_CLUSTER_MIN_AGENTS", SWARP_MAX_CTA_AGENTS + 1);
  return v < 2 ? 2 : v;
}
bool use_cluster(int A, int fl) {
  return A >= cluster_min_agents() && !(fl & F_MASK);
}
// CTAs per env (CS <= kClusterMaxCTAs) and threads per CTA (a multiple of 32): the fewest
// CTAs of at most SWARP_CLUSTER_CTA_THREADS threads that hold the env. False if none does.
bool cluster_shape(int A, int& CS, int& BT) {
  int bt_max = env_int("SWARP_CLUSTER_CTA_THREADS", kClusterMaxThreads);
  bt_max = std::max(32, std::min(kClusterMaxThreads, bt_max / 32 * 32));
  CS = (A + bt_max - 1) / bt_max;
  if (CS < 1) CS = 1;
  BT = ((A + CS - 1) / CS + 31) / 32 * 32;
  return CS <= kClusterMaxCTAs;
}
int max_smem_optin() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return 0;
  return v;
}
// Checks and sets up a cluster launch of R (fl its flags): 0, or the error code.
template <typename T> int cluster_setup(RolloutArgs<T>& R, int fl, bool bwd, int& BT) {
  if (fl & (F_BODIES | F_BOXES | F_DRONE | F_MASK)) return SWARP_ERR_UNSUPPORTED;
  int CS = 0;
  if (!cluster_shape(R.A, CS, BT)) return SWARP_ERR_TOO_MANY_AGENTS;
  const ClusterLayout<T> L(R.A, BT, R.N, R.S, bwd);
  if (L.total > (size_t)max_smem_optin()) return SWARP_ERR_TOO_MANY_AGENTS;
  R.CS = CS;
  R.G = 1;
  return SWARP_OK;
}

// Largest value x of type T with sqrt(x) <= R (both rounded in T): the exact set test
// sqrt(d2) <= R of the reference, evaluated without a square root.
template <typename T> T radius_sq_threshold(double Rd) {
  const T R = static_cast<T>(Rd);
  if (!(R > T(0))) return T(-1);
  T x = R * R;
  const T inf = std::numeric_limits<T>::infinity();
  while (std::sqrt(std::nextafter(x, inf)) <= R) x = std::nextafter(x, inf);
  while (std::sqrt(x) > R) x = std::nextafter(x, -inf);
  return x;
}

// The packed scan's threshold: r2_thr widened by 2^-19 (float) / 2^-48 (double) relative,
// i.e. >= 30 ulps, plus a tiny absolute term that covers underflow of dx^2 + dy^2 when
// r2_thr is subnormal. Every in-radius pair tests negative against it (the scan's two
// fused roundings err by < 3 ulps of the threshold), so the scan's set is a superset of
// the exact one; the kernels filter it with the exact test.
template <typename T> T radius_sq_scan_threshold(T thr) {
  if (!(thr > T(0))) return thr;
  const bool f = std::is_same<T, float>::value;
  const T rel = f ? T(0x1p-19) : T(0x1p-48);
  const T tiny = f ? T(0x1p-120) : T(0x1p-1000);
  return std::nextafter(thr * (T(1) + rel) + tiny, std::numeric_limits<T>::infinity());
}

int validate_world(const swarp_world_t* w, int horizon) {
  if (!w || horizon < 1) return SWARP_ERR_INVALID_ARG;
  if (w->dtype != SWARP_F32 && w->dtype != SWARP_F64) return SWARP_ERR_INVALID_ARG;
  if (w->n_envs < 1 || w->n_agents < 1 || w->substeps < 1 || w->act_dim < 2) return SWARP_ERR_INVALID_ARG;
  if (w->n_agents > SWARP_MAX_AGENTS) return SWARP_ERR_TOO_MANY_AGENTS;
  if (!(w->dt > 0.0)) return SWARP_ERR_INVALID_ARG;
  if (!w->params || !w->model_tag || !w->ctrl_mode) return SWARP_ERR_INVALID_ARG;
  if (w->fleet_models & ~0xF) return SWARP_ERR_UNSUPPORTED;  // unknown tags
  if (w->fleet_models == 0 || w->fleet_modes == 0 || (w->fleet_modes & ~0x7)) return SWARP_ERR_INVALID_ARG;
  // drones together with box agents (exclusive in the reference): not built
  if ((w->fleet_models & 0x8) && w->box_agents) return SWARP_ERR_UNSUPPORTED;
  if (w->bounds_mode < 0 || w->bounds_mode > 2) return SWARP_ERR_INVALID_ARG;
  if (w->integrator < 0 || w->integrator > 1) return SWARP_ERR_INVALID_ARG;
  if (w->box_agents < 0 || w->box_agents > 1) return SWARP_ERR_INVALID_ARG;
  if (w->collisions) {
    if (w->max_neighbors < 1 || !(w->neighbor_radius > 0.0)) return SWARP_ERR_INVALID_ARG;
    if (w->n_agents > 32767) return SWARP_ERR_TOO_MANY_AGENTS;
  }
  const swarp_obstacles_t& o = w->obstacles;
  if (o.n_obstacles < 0) return SWARP_ERR_INVALID_ARG;
  if (o.n_obstacles > 0) {
    if (!o.pos || !o.angle || !o.vel || !o.ang_vel || !o.radius || !o.half || !o.shape)
      return SWARP_ERR_INVALID_ARG;
    if (o.any_movable && o.bodies_move && (!o.kind || !o.mass || !o.inertia || !o.body || !o.body_off))
      return SWARP_ERR_INVALID_ARG;
  }
  return SWARP_OK;
}

bool state_complete(const swarp_state_t& s) {
  return s.pos && s.theta && s.vel && s.speed && s.ang_vel;
}
bool drone_complete(const swarp_state_t& s) { return s.z && s.vz && s.attitude && s.body_rates; }

// Contact masks checkpointed by the forward (F_MASK) so that the adjoint gathers its pairs
// without rescanning the env: for envs of up to 32 agents without list truncation (every
// world kind), and for 2-D disc fleets of up to kMaskMaxAgents agents with or without
// truncation (ceil(A / 32) words per agent and substep). SWARP_CONTACT_MASKS=0 (read on
// every call) keeps the larger worlds on the rescan path, for comparisons.
constexpr int kMaskMaxAgents = 256;
bool wide_masks_enabled() {
  const char* s = std::getenv("SWARP_CONTACT_MASKS");
  return !(s && s[0] == '0');
}

int flags_of(const swarp_world_t* w) {
  int fl = 0;
  if (w->collisions) {
    fl |= F_COLL;
    const bool trunc = w->n_agents - 1 > w->max_neighbors;
    if (trunc) fl |= F_TRUNC;
    if (!trunc && w->n_agents <= 32)
      fl |= F_MASK;
    else if (w->n_agents <= kMaskMaxAgents && !w->box_agents && !(w->fleet_models & 0x8) &&
             wide_masks_enabled())
      fl |= F_MASK;
  }
  if (w->obstacles.n_obstacles > 0) {
    fl |= F_OBS;
    if (w->obstacles.any_movable && w->obstacles.bodies_move) fl |= F_BODIES;
  }
  if (w->integrator == 1) fl |= F_RK4;
  if (w->box_agents) fl |= F_BOXES;
  if (w->fleet_models & 0x8) fl |= F_DRONE;
  if (w->fleet_models == 1 && w->fleet_modes == 1) fl |= F_HOLOVEL;
  return fl;
}

template <typename T>
void fill_common(const swarp_world_t* w, int horizon, RolloutArgs<T>& R) {
  std::memset(&R, 0, sizeof(R));
  R.E = w->n_envs;
  R.A = w->n_agents;
  R.G = envs_per_cta(R.A, R.E);
  R.H = horizon;
  R.S = w->substeps;
  R.act_dim = w->act_dim;
  R.N = w->obstacles.n_obstacles;
  WorldC<T>& W = R.W;
  W.dt = static_cast<T>(w->dt / w->substeps);
  W.k = static_cast<T>(w->k);
  W.c = static_cast<T>(w->c);
  W.margin = static_cast<T>(w->margin);
  W.max_overlap = static_cast<T>(w->max_overlap);
  W.r2_thr = w->collisions ? radius_sq_threshold<T>(w->neighbor_radius) : T(-1);
  W.r2_scan = radius_sq_scan_threshold(W.r2_thr);
  W.bx0 = static_cast<T>(w->bounds[0]);
  W.bx1 = static_cast<T>(w->bounds[1]);
  W.by0 = static_cast<T>(w->bounds[2]);
  W.by1 = static_cast<T>(w->bounds[3]);
  W.lin_decay = static_cast<T>(1.0 - w->lin_damping * (w->dt / w->substeps));
  W.ang_decay = static_cast<T>(1.0 - w->ang_damping * (w->dt / w->substeps));
  W.K = w->max_neighbors;
  W.bounds_mode = w->bounds_mode;
  R.params = static_cast<const T*>(w->params);
  R.params_env_stride = w->params_env_stride;
  R.model_tag = w->model_tag;
  R.ctrl_mode = w->ctrl_mode;
  const swarp_obstacles_t& o = w->obstacles;
  if (R.N > 0) {
    R.o_pos = static_cast<const T*>(o.pos);
    R.o_angle = static_cast<const T*>(o.angle);
    R.o_vel = static_cast<const T*>(o.vel);
    R.o_ang_vel = static_cast<const T*>(o.ang_vel);
    R.o_radius = static_cast<const T*>(o.radius);
    R.o_half = static_cast<const T*>(o.half);
    R.o_shape = o.shape;
    R.o_kind = o.kind;
    R.o_body = o.body;
    R.o_mass = static_cast<const T*>(o.mass);
    R.o_inertia = static_cast<const T*>(o.inertia);
    R.o_body_off = static_cast<const T*>(o.body_off);
  }
  R.body_clamp = w->bounds_mode != SWARP_BOUNDS_NONE;
  R.poses_from_bodies = o.poses_from_bodies;
}

bool bodies_complete(const swarp_bodies_t& b) { return b.pos && b.angle && b.vel && b.ang_vel; }

template <typename T>
void set_bodies(const swarp_bodies_t& b, const T*& p, const T*& a, const T*& v, const T*& w) {
  p = static_cast<const T*>(b.pos);
  a = static_cast<const T*>(b.angle);
  v = static_cast<const T*>(b.vel);
  w = static_cast<const T*>(b.ang_vel);
}

template <typename T>
void set_state(const swarp_state_t& s, const T*& p, const T*& th, const T*& v, const T*& sp,
               const T*& w) {
  p = static_cast<const T*>(s.pos);
  th = static_cast<const T*>(s.theta);
  v = static_cast<const T*>(s.vel);
  sp = static_cast<const T*>(s.speed);
  w = static_cast<const T*>(s.ang_vel);
}
template <typename T>
void set_state_out(const swarp_state_t& s, T*& p, T*& th, T*& v, T*& sp, T*& w) {
  p = static_cast<T*>(s.pos);
  th = static_cast<T*>(s.theta);
  v = static_cast<T*>(s.vel);
  sp = static_cast<T*>(s.speed);
  w = static_cast<T*>(s.ang_vel);
}
template <typename Q> DroneF<Q> drone_of(const swarp_state_t& s) {
  return DroneF<Q>{static_cast<Q*>(s.z), static_cast<Q*>(s.vz), static_cast<Q*>(s.attitude),
                   static_cast<Q*>(s.body_rates)};
}

// Workspace: [contact masks (F_MASK): cells x ceil(A/32) words] then, 256-byte aligned,
// [list cutoffs (F_TRUNC): cells int16] then, 256-byte aligned, one partial sum per CTA
// for the fused goal-loss and ||grad_actions||^2 epilogues.
size_t align256(size_t b) { return (b + 255) & ~size_t(255); }
size_t cutoff_offset(const swarp_world_t* w, int horizon) {
  const size_t cells = (size_t)horizon * w->substeps * (size_t)w->n_envs * w->n_agents;
  const size_t nw = (size_t)(w->n_agents + 31) / 32;
  return (flags_of(w) & F_MASK) ? align256(cells * nw * sizeof(uint32_t)) : 0;
}
size_t partials_offset(const swarp_world_t* w, int horizon) {
  const size_t cells = (size_t)horizon * w->substeps * (size_t)w->n_envs * w->n_agents;
  const size_t b = (flags_of(w) & F_TRUNC) ? cells * sizeof(int16_t) : 0;
  return align256(cutoff_offset(w, horizon) + b);
}
size_t partials_bytes(const swarp_world_t* w) {
  // the CTA count of the generic or the two-agents-per-thread kernels, whichever is larger,
  // or of the cluster kernels (CS CTAs per env)
  const int G = std::min(envs_per_cta(w->n_agents, w->n_envs), x2_envs_per_cta(w->n_envs));
  size_t n = (size_t)(w->n_envs + G - 1) / G;
  int CS = 1, BT = 0;
  if (use_cluster(w->n_agents, flags_of(w)) && cluster_shape(w->n_agents, CS, BT))
    n = std::max(n, (size_t)w->n_envs * CS);
  return n * (w->dtype == SWARP_F32 ? sizeof(float) : sizeof(double));
}

template <typename T>
int fwd_typed(const swarp_world_t* w, int horizon, swarp_state_t init, const void* actions,
              swarp_state_t traj, swarp_state_t fin, int32_t* true_max, swarp_bodies_t bi,
              swarp_bodies_t bt, swarp_goal_loss_t gl, void* ws, cudaStream_t st) {
  RolloutArgs<T> R;
  fill_common<T>(w, horizon, R);
  R.goal = static_cast<const T*>(gl.goal);
  R.loss_out = static_cast<T*>(gl.loss);
  R.loss_partial = gl.goal ? reinterpret_cast<T*>(static_cast<unsigned char*>(ws) +
                                                  partials_offset(w, horizon))
                           : nullptr;
  set_bodies<T>(bi, R.bi_pos, R.bi_ang, R.bi_vel, R.bi_om);
  R.bt_pos = static_cast<T*>(bt.pos);
  R.bt_ang = static_cast<T*>(bt.angle);
  R.bt_vel = static_cast<T*>(bt.vel);
  R.bt_om = static_cast<T*>(bt.ang_vel);
  set_state<T>(init, R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w);
  R.act = static_cast<const T*>(actions);
  set_state_out<T>(traj, R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w);
  set_state_out<T>(fin, R.f_pos, R.f_th, R.f_vel, R.f_s, R.f_w);
  R.i_d = drone_of<const T>(init);
  R.t_d = drone_of<T>(traj);
  R.f_d = drone_of<T>(fin);
  R.true_max = true_max;
  const int fl = flags_of(w);
  R.cutoff = (fl & F_TRUNC) ? reinterpret_cast<int16_t*>(static_cast<unsigned char*>(ws) +
                                                         cutoff_offset(w, horizon))
                            : nullptr;
  R.cmask = (fl & F_MASK) ? static_cast<uint32_t*>(ws) : nullptr;
  if (use_cluster(R.A, fl)) {
    int BT = 0;
    const int rc = cluster_setup(R, fl, false, BT);
    return rc != SWARP_OK ? rc : launch_fwd_cl<T>(R, fl, BT, st);
  }
  if constexpr (std::is_same<T, float>::value) {
    if (x2_ok(R, fl, false)) {
      R.G = x2_envs_per_cta(R.E);
      return launch_fwd_x2(R, fl, st);
    }
  }
  return launch_fwd<T>(R, fl, st);
}

template <typename T>
int bwd_typed(const swarp_world_t* w, int horizon, swarp_state_t init, const void* actions,
              swarp_state_t traj, swarp_state_t gtraj, swarp_state_t gfin, swarp_bodies_t bi,
              swarp_bodies_t bt, swarp_bodies_t gbf, void* gact, swarp_state_t ginit,
              void* gsq, swarp_goal_loss_t gl, void* ws, cudaStream_t st) {
  RolloutArgs<T> R;
  fill_common<T>(w, horizon, R);
  R.goal = static_cast<const T*>(gl.goal);
  R.loss_grad = static_cast<const T*>(gl.loss_grad);
  set_bodies<T>(bi, R.bi_pos, R.bi_ang, R.bi_vel, R.bi_om);
  R.bt_pos = static_cast<T*>(bt.pos);
  R.bt_ang = static_cast<T*>(bt.angle);
  R.bt_vel = static_cast<T*>(bt.vel);
  R.bt_om = static_cast<T*>(bt.ang_vel);
  set_bodies<T>(gbf, R.gb_pos, R.gb_ang, R.gb_vel, R.gb_om);
  set_state<T>(init, R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w);
  R.act = static_cast<const T*>(actions);
  set_state_out<T>(traj, R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w);
  set_state<T>(gtraj, R.gt_pos, R.gt_th, R.gt_vel, R.gt_s, R.gt_w);
  set_state<T>(gfin, R.gf_pos, R.gf_th, R.gf_vel, R.gf_s, R.gf_w);
  R.g_act = static_cast<T*>(gact);
  set_state_out<T>(ginit, R.gi_pos, R.gi_th, R.gi_vel, R.gi_s, R.gi_w);
  R.i_d = drone_of<const T>(init);
  R.t_d = drone_of<T>(traj);
  R.gt_d = drone_of<const T>(gtraj);
  R.gf_d = drone_of<const T>(gfin);
  R.gi_d = drone_of<T>(ginit);
  const int fl = flags_of(w);
  R.cutoff = (fl & F_TRUNC) ? reinterpret_cast<int16_t*>(static_cast<unsigned char*>(ws) +
                                                         cutoff_offset(w, horizon))
                            : nullptr;
  R.cmask = (fl & F_MASK) ? static_cast<uint32_t*>(ws) : nullptr;
  R.gsq_out = static_cast<T*>(gsq);
  R.gsq_partial = gsq ? reinterpret_cast<T*>(static_cast<unsigned char*>(ws) +
                                             partials_offset(w, horizon))
                      : nullptr;
  if (use_cluster(R.A, fl)) {
    int BT = 0;
    const int rc = cluster_setup(R, fl, true, BT);
    return rc != SWARP_OK ? rc : launch_bwd_cl<T>(R, fl, BT, st);
  }
  if constexpr (std::is_same<T, float>::value) {
    if (x2_ok(R, fl, true)) {
      R.G = x2_envs_per_cta(R.E);  // fewer CTAs than the partials buffer is sized for
      return launch_bwd_x2(R, fl, st);
    }
  }
  return launch_bwd<T>(R, fl, st);
}

template <typename T>
int nbr_typed(const swarp_world_t* w, const void* pos, int32_t* idx, int32_t* count,
              int32_t* true_count, cudaStream_t st) {
  const int E = w->n_envs, A = w->n_agents;
  const T thr = radius_sq_threshold<T>(w->neighbor_radius);
  if (A >= cluster_min_agents()) {  // several CTAs per env, each stages the whole env
    const int slices = (A + SWARP_MAX_CTA_AGENTS - 1) / SWARP_MAX_CTA_AGENTS;
    const int block = ((A + slices - 1) / slices + 31) / 32 * 32;
    if (size_t((A + 1) / 2) * 4 * sizeof(T) > (size_t)max_smem_optin())
      return SWARP_ERR_TOO_MANY_AGENTS;
    return launch_neighbors_wide<T>(E, A, slices, block, w->max_neighbors,
                                    radius_sq_scan_threshold(thr), thr,
                                    static_cast<const T*>(pos), idx, count, true_count, st);
  }
  const int G = envs_per_cta(A, E);
  return launch_neighbors<T>(E, A, G, w->max_neighbors, radius_sq_scan_threshold(thr), thr,
                             static_cast<const T*>(pos), idx, count, true_count, st);
}

}  // namespace

extern "C" {

size_t swarp_rollout_workspace_bytes(const swarp_world_t* w, int32_t horizon) {
  if (validate_world(w, horizon) != SWARP_OK) return 0;
  return partials_offset(w, horizon) + partials_bytes(w);
}

int swarp_rollout_fwd(const swarp_world_t* w, int32_t horizon, swarp_state_t init,
                      const void* actions, swarp_state_t traj, swarp_state_t final_out,
                      int32_t* true_count_max, swarp_bodies_t bodies_init,
                      swarp_bodies_t bodies_traj, swarp_goal_loss_t goal_loss, void* workspace,
                      size_t workspace_bytes, void* stream) {
  int rc = validate_world(w, horizon);
  if (rc != SWARP_OK) return rc;
  if (goal_loss.goal && !goal_loss.loss) return SWARP_ERR_INVALID_ARG;
  if (!state_complete(init) || !state_complete(traj) || !actions) return SWARP_ERR_INVALID_ARG;
  if ((flags_of(w) & F_BODIES) && (!bodies_complete(bodies_init) || !bodies_complete(bodies_traj)))
    return SWARP_ERR_INVALID_ARG;
  const bool any_fin = final_out.pos || final_out.theta || final_out.vel || final_out.speed || final_out.ang_vel;
  if (any_fin && !state_complete(final_out)) return SWARP_ERR_INVALID_ARG;
  if (flags_of(w) & F_DRONE) {
    if (!drone_complete(init) || !drone_complete(traj)) return SWARP_ERR_INVALID_ARG;
    if (any_fin && !drone_complete(final_out)) return SWARP_ERR_INVALID_ARG;
  }
  const size_t need = swarp_rollout_workspace_bytes(w, horizon);
  if (need > 0 && (!workspace || workspace_bytes < need)) return SWARP_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w->dtype == SWARP_F32)
    return fwd_typed<float>(w, horizon, init, actions, traj, final_out, true_count_max, bodies_init,
                            bodies_traj, goal_loss, workspace, st);
  return fwd_typed<double>(w, horizon, init, actions, traj, final_out, true_count_max, bodies_init,
                           bodies_traj, goal_loss, workspace, st);
}

int swarp_rollout_bwd(const swarp_world_t* w, int32_t horizon, swarp_state_t init,
                      const void* actions, swarp_state_t traj, swarp_state_t adj_traj,
                      swarp_state_t adj_final, swarp_bodies_t bodies_init,
                      swarp_bodies_t bodies_traj, swarp_bodies_t adj_bodies_final,
                      void* adj_actions, swarp_state_t adj_init, void* adj_actions_sqnorm,
                      swarp_goal_loss_t goal_loss, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc = validate_world(w, horizon);
  if (rc != SWARP_OK) return rc;
  if (goal_loss.goal && !goal_loss.loss_grad) return SWARP_ERR_INVALID_ARG;
  if ((flags_of(w) & F_BOXES) && (flags_of(w) & F_BODIES)) return SWARP_ERR_UNSUPPORTED;
  if (flags_of(w) & F_DRONE) {
    if (!drone_complete(init) || !drone_complete(traj) || !drone_complete(adj_init))
      return SWARP_ERR_INVALID_ARG;
  }
  if (flags_of(w) & F_BODIES) {
    if (!bodies_complete(bodies_init) || !bodies_complete(bodies_traj)) return SWARP_ERR_INVALID_ARG;
    if (w->obstacles.movable_shapes & ~(1 << SHAPE_CIRCLE)) return SWARP_ERR_UNSUPPORTED;
  }
  if (!state_complete(init) || !state_complete(traj) || !state_complete(adj_init) || !actions ||
      !adj_actions)
    return SWARP_ERR_INVALID_ARG;
  // the checkpoint cells are read; the partials (only with adj_actions_sqnorm) are written
  const size_t need = adj_actions_sqnorm ? swarp_rollout_workspace_bytes(w, horizon)
                                         : partials_offset(w, horizon);
  if (need > 0 && (!workspace || workspace_bytes < need)) return SWARP_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w->dtype == SWARP_F32)
    return bwd_typed<float>(w, horizon, init, actions, traj, adj_traj, adj_final, bodies_init,
                            bodies_traj, adj_bodies_final, adj_actions, adj_init,
                            adj_actions_sqnorm, goal_loss, workspace, st);
  return bwd_typed<double>(w, horizon, init, actions, traj, adj_traj, adj_final, bodies_init,
                           bodies_traj, adj_bodies_final, adj_actions, adj_init,
                           adj_actions_sqnorm, goal_loss, workspace, st);
}

int swarp_neighbors(const swarp_world_t* w, const void* pos, int32_t* idx, int32_t* count,
                    int32_t* true_count, void* stream) {
  if (!w || !pos || !idx || !count || !true_count) return SWARP_ERR_INVALID_ARG;
  if (w->n_envs < 1 || w->n_agents < 1 || w->max_neighbors < 1 || !(w->neighbor_radius > 0.0))
    return SWARP_ERR_INVALID_ARG;
  if (w->n_agents > SWARP_MAX_AGENTS) return SWARP_ERR_TOO_MANY_AGENTS;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w->dtype == SWARP_F32) return nbr_typed<float>(w, pos, idx, count, true_count, st);
  if (w->dtype == SWARP_F64) return nbr_typed<double>(w, pos, idx, count, true_count, st);
  return SWARP_ERR_INVALID_ARG;
}

const char* swarp_error_string(int code) {
  switch (code) {
    case SWARP_OK: return "ok";
    case SWARP_ERR_INVALID_ARG: return "invalid argument (null pointer, size or configuration)";
    case SWARP_ERR_UNSUPPORTED: return "unsupported model or option in this build";
    case SWARP_ERR_TOO_MANY_AGENTS: return "n_agents above SWARP_MAX_AGENTS";
    case SWARP_ERR_CUDA: return "CUDA launch or attribute call failed";
    case SWARP_ERR_WORKSPACE: return "workspace missing or too small";
    case SWARP_ERR_SCRATCH_LIMIT:
      return "rollout needs more workspace than the allocation-free entry point's static "
             "scratch (SWARP_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown error code";
  }
}

int swarp_copy_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch,
                    size_t row_bytes, size_t rows, void* stream) {
  if (rows == 0 || row_bytes == 0) return SWARP_OK;
  if (!dst || !src || dst_pitch < row_bytes || src_pitch < row_bytes) return SWARP_ERR_INVALID_ARG;
  return cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, row_bytes, rows, cudaMemcpyDefault,
                           static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? SWARP_OK
             : SWARP_ERR_CUDA;
}

int32_t swarp_abi_version(void) { return kAbiVersion; }

}  // extern "C"
