// Two agents per thread for float envs of exactly 16 agents (the benchmark shape).
//
// Thread j of an env owns agents 2j and 2j+1. Everything that is per agent (scan
// arithmetic, contact law, walls, integrator and their adjoints) is the same device code
// as the one-agent-per-thread kernels in rollout.cuh, evaluated twice in the same order,
// so results are bitwise those of those kernels; what the pairing saves is the work that
// was per thread: the pair's position row of the scan table is one 16-byte shared store,
// each 16-byte table load serves both agents' candidate tests, actions, trajectory
// fields, contact masks and action gradients move as 8/16-byte vectors for the two
// adjacent agents, and loop, barrier and address overhead is paid once per two agents.
// The two agents' independent chains also double the instruction-level parallelism.
//
// Preconditions (checked by the host): A == 16, act_dim == 2, contact masks checkpointed
// (no list truncation), no moving bodies, every pointer 16-byte aligned; the adjoint
// additionally one substep per step. Other worlds take the one-agent kernels.
#pragma once
#include "rollout.cuh"

namespace swarp {

constexpr int kX2Agents = 16;     // agents per env
constexpr int kX2Threads = 8;     // threads per env

// Register budgets, as resident 64-thread CTAs per SM. A 16,000-env batch is 4,000 warps:
// 14 CTAs (28 warps) per SM hold it in one wave on 148 SMs.
#ifndef SWARP_X2_FWD_MINB
#define SWARP_X2_FWD_MINB 14
#endif
#ifndef SWARP_X2_BWD_MINB
#define SWARP_X2_BWD_MINB 10
#endif

// Both agents' candidate masks over the env (self bits included; a superset of the
// in-radius sets at thr = W.r2_scan): one 16-byte table load per pair of candidates,
// shared by the two agents.
__device__ __forceinline__ void scan_pair16(const float* xy_env, const Agent<float>& x0,
                                            const Agent<float>& x1, float thr, unsigned& m0,
                                            unsigned& m1) {
  const float4* P = reinterpret_cast<const float4*>(xy_env);
  const float2 M1 = make_float2(-1.f, -1.f), NT = make_float2(-thr, -thr);
  const float2 PX0 = make_float2(x0.px, x0.px), PY0 = make_float2(x0.py, x0.py);
  const float2 PX1 = make_float2(x1.px, x1.px), PY1 = make_float2(x1.py, x1.py);
  m0 = 0u;
  m1 = 0u;
#pragma unroll
  for (int p = kX2Agents / 2 - 1; p >= 0; --p) {
    const float4 q = P[p];
    const float2 qx = make_float2(q.x, q.y), qy = make_float2(q.z, q.w);
    const float2 dx0 = __ffma2_rn(qx, M1, PX0), dy0 = __ffma2_rn(qy, M1, PY0);
    const float2 dx1 = __ffma2_rn(qx, M1, PX1), dy1 = __ffma2_rn(qy, M1, PY1);
    const float2 d0 = __ffma2_rn(dx0, dx0, __ffma2_rn(dy0, dy0, NT));
    const float2 d1 = __ffma2_rn(dx1, dx1, __ffma2_rn(dy1, dy1, NT));
    m0 = __funnelshift_l(__float_as_uint(d0.y), m0, 1);
    m0 = __funnelshift_l(__float_as_uint(d0.x), m0, 1);
    m1 = __funnelshift_l(__float_as_uint(d1.y), m1, 1);
    m1 = __funnelshift_l(__float_as_uint(d1.x), m1, 1);
  }
}

// Contact force on agent a from the members of its candidate mask m (self removed,
// ascending index; candidates outside the exact radius skipped); returns the contact mask
// and adds the member count to cnt.
__device__ __forceinline__ unsigned contacts_of(const float4* rec_env, const float* rad_env,
                                                unsigned m, const Agent<float>& x,
                                                const AgentP<float>& P, const WorldC<float>& W,
                                                float& fx, float& fy, int& cnt) {
  unsigned cm = 0u;
  while (m) {
    const int b = __ffs(m) - 1;
    m &= m - 1u;
    const float4 q = rec_env[b];
    const float dx = x.px - q.x, dy = x.py - q.y;
    if (!in_radius(dx, dy, W.r2_thr)) continue;
    ++cnt;
    if (pair_force_add(dx, dy, dot2(dx, dy, dx, dy), x.vx - q.z, x.vy - q.w,
                       P.radius + rad_env[b] + W.margin, P.inv_denom, W, fx, fy))
      cm |= 1u << b;
  }
  return cm;
}

// Both agents' contacts side by side (no depth saturation): each round takes the next
// candidate of each agent's mask (ascending index, as contacts_of) and evaluates the two
// pairs in one branch-free block, so the two independent chains interleave; the rounds
// are as many as the larger of the two counts instead of their sum. Results are bitwise
// contacts_of's.
__device__ __forceinline__ void contacts_of_both(const float4* rec_env, const float* rad_env,
                                                 unsigned m0, unsigned m1, const Agent<float>& x0,
                                                 const Agent<float>& x1, const AgentP<float>& P0,
                                                 const AgentP<float>& P1, const WorldC<float>& W,
                                                 float& fx0, float& fy0, float& fx1, float& fy1,
                                                 unsigned& c0, unsigned& c1, int& n0, int& n1) {
  c0 = 0u;
  c1 = 0u;
  while (m0 | m1) {
    const bool h0 = m0 != 0u, h1 = m1 != 0u;
    const int b0 = h0 ? __ffs(m0) - 1 : 0, b1 = h1 ? __ffs(m1) - 1 : 0;
    m0 &= m0 - 1u;
    m1 &= m1 - 1u;
    const float4 q0 = rec_env[b0], q1 = rec_env[b1];
    const float r0 = rad_env[b0], r1 = rad_env[b1];
    const float dx0 = x0.px - q0.x, dy0 = x0.py - q0.y;
    const float dx1 = x1.px - q1.x, dy1 = x1.py - q1.y;
    const bool in0 = h0 && in_radius(dx0, dy0, W.r2_thr);
    const bool in1 = h1 && in_radius(dx1, dy1, W.r2_thr);
    n0 += in0 ? 1 : 0;
    n1 += in1 ? 1 : 0;
    if (pair_force_add_nb(in0, dx0, dy0, x0.vx - q0.z, x0.vy - q0.w, P0.radius + r0 + W.margin,
                          P0.inv_denom, W, fx0, fy0))
      c0 |= 1u << b0;
    if (pair_force_add_nb(in1, dx1, dy1, x1.vx - q1.z, x1.vy - q1.w, P1.radius + r1 + W.margin,
                          P1.inv_denom, W, fx1, fy1))
      c1 |= 1u << b1;
  }
}

// The adjoint's counterpart over the two checkpointed contact masks (no depth
// saturation): the terms of pair_vjp_sym for the next contact of each agent per round,
// added to each agent's gradient in ascending partner order as force_vjp adds them.
__device__ __forceinline__ void contact_vjp_both(const float4* rec_env, const float2* fb_env,
                                                 const float* rad_env, const float* iden_env,
                                                 unsigned m0, unsigned m1, const Agent<float>& x0,
                                                 const Agent<float>& x1, const AgentP<float>& P0,
                                                 const AgentP<float>& P1, const WorldC<float>& W,
                                                 float gfx0, float gfy0, float gfx1, float gfy1,
                                                 Agent<float>& g0, Agent<float>& g1) {
  while (m0 | m1) {
    const bool h0 = m0 != 0u, h1 = m1 != 0u;
    const int b0 = h0 ? __ffs(m0) - 1 : 0, b1 = h1 ? __ffs(m1) - 1 : 0;
    m0 &= m0 - 1u;
    m1 &= m1 - 1u;
    const float4 q0 = rec_env[b0], q1 = rec_env[b1];
    const float2 f0 = fb_env[b0], f1 = fb_env[b1];
    PairTerms<float> t0, t1;
    const bool on0 = pair_vjp_terms_nb(h0, x0.px - q0.x, x0.py - q0.y, x0.vx - q0.z, x0.vy - q0.w,
                                       P0.radius + rad_env[b0] + W.margin, P0.inv_denom, gfx0,
                                       gfy0, iden_env[b0], f0.x, f0.y, W, t0);
    const bool on1 = pair_vjp_terms_nb(h1, x1.px - q1.x, x1.py - q1.y, x1.vx - q1.z, x1.vy - q1.w,
                                       P1.radius + rad_env[b1] + W.margin, P1.inv_denom, gfx1,
                                       gfy1, iden_env[b1], f1.x, f1.y, W, t1);
    g0.vx = on0 ? g0.vx + t0.vx : g0.vx;
    g0.vy = on0 ? g0.vy + t0.vy : g0.vy;
    g0.px = on0 ? g0.px + t0.px : g0.px;
    g0.py = on0 ? g0.py + t0.py : g0.py;
    g1.vx = on1 ? g1.vx + t1.vx : g1.vx;
    g1.vy = on1 ? g1.vy + t1.vy : g1.vy;
    g1.px = on1 ? g1.px + t1.px : g1.px;
    g1.py = on1 ? g1.py + t1.py : g1.py;
  }
}

// Static forces (obstacles, then walls) of both agents as static_force sums them, in one
// block: they depend on the agents' own states only, so the kernels evaluate them where
// their arithmetic can overlap the neighbor work.
template <int FL>
__device__ __forceinline__ void static_forces_both(const Obs<float>* obs, int N,
                                                   const Agent<float>& x0, const Agent<float>& x1,
                                                   const AgentP<float>& P0, const AgentP<float>& P1,
                                                   const WorldC<float>& W, float& sx0, float& sy0,
                                                   float& sx1, float& sy1) {
  sx0 = sy0 = sx1 = sy1 = 0.f;
  if (FL & F_OBS) {
    for (int o = 0; o < N; ++o) {
      float gx, gy;
      obstacle_force(x0.px, x0.py, x0.vx, x0.vy, P0.radius, P0.inv_denom, obs[o], W, gx, gy);
      sx0 = sx0 + gx;
      sy0 = sy0 + gy;
      obstacle_force(x1.px, x1.py, x1.vx, x1.vy, P1.radius, P1.inv_denom, obs[o], W, gx, gy);
      sx1 = sx1 + gx;
      sy1 = sy1 + gy;
    }
  }
  if (W.bounds_mode == BOUNDS_SOFT) {
    float wx0, wy0, wx1, wy1;
    if (W.max_overlap > 0.f) {
      wall_force(x0.px, x0.py, x0.vx, x0.vy, P0.radius, P0.inv_denom, W, wx0, wy0);
      wall_force(x1.px, x1.py, x1.vx, x1.vy, P1.radius, P1.inv_denom, W, wx1, wy1);
    } else {
      wall_force_lin(x0.px, x0.py, x0.vx, x0.vy, P0.radius, P0.inv_denom, W, wx0, wy0);
      wall_force_lin(x1.px, x1.py, x1.vx, x1.vy, P1.radius, P1.inv_denom, W, wx1, wy1);
    }
    sx0 = sx0 + wx0;
    sy0 = sy0 + wy0;
    sx1 = sx1 + wx1;
    sy1 = sy1 + wy1;
  }
}

__device__ __forceinline__ void load_pair(const float* pos, const float* th, const float* vel,
                                          const float* s, const float* w, long long i,
                                          Agent<float>& x0, Agent<float>& x1) {
  const float4 p = reinterpret_cast<const float4*>(pos)[i >> 1];
  const float4 v = reinterpret_cast<const float4*>(vel)[i >> 1];
  const float2 t = reinterpret_cast<const float2*>(th)[i >> 1];
  const float2 sp = reinterpret_cast<const float2*>(s)[i >> 1];
  const float2 om = reinterpret_cast<const float2*>(w)[i >> 1];
  x0 = Agent<float>{p.x, p.y, t.x, v.x, v.y, sp.x, om.x};
  x1 = Agent<float>{p.z, p.w, t.y, v.z, v.w, sp.y, om.y};
}
__device__ __forceinline__ void load_pair_pv(const float* pos, const float* vel, long long i,
                                             Agent<float>& x0, Agent<float>& x1) {
  const float4 p = reinterpret_cast<const float4*>(pos)[i >> 1];
  const float4 v = reinterpret_cast<const float4*>(vel)[i >> 1];
  x0 = Agent<float>{p.x, p.y, 0.f, v.x, v.y, 0.f, 0.f};
  x1 = Agent<float>{p.z, p.w, 0.f, v.z, v.w, 0.f, 0.f};
}
__device__ __forceinline__ void store_pair(float* pos, float* th, float* vel, float* s, float* w,
                                           long long i, const Agent<float>& x0,
                                           const Agent<float>& x1) {
  reinterpret_cast<float4*>(pos)[i >> 1] = make_float4(x0.px, x0.py, x1.px, x1.py);
  reinterpret_cast<float4*>(vel)[i >> 1] = make_float4(x0.vx, x0.vy, x1.vx, x1.vy);
  reinterpret_cast<float2*>(th)[i >> 1] = make_float2(x0.th, x1.th);
  reinterpret_cast<float2*>(s)[i >> 1] = make_float2(x0.s, x1.s);
  reinterpret_cast<float2*>(w)[i >> 1] = make_float2(x0.w, x1.w);
}
__device__ __forceinline__ void add_cotangent_pair(const float* pos, const float* th,
                                                   const float* vel, const float* s,
                                                   const float* w, long long i, Agent<float>& g0,
                                                   Agent<float>& g1) {
  add_cotangent(pos, th, vel, s, w, i, g0);
  add_cotangent(pos, th, vel, s, w, i + 1, g1);
}

// ------------------------------------------------------------------- forward
template <int FL>
__global__ void __launch_bounds__(64, SWARP_X2_FWD_MINB) rollout_fwd_x2_kernel(const RolloutArgs<float> R) {
  constexpr int A = kX2Agents;
  extern __shared__ __align__(16) unsigned char smem[];
  const int G = R.G, GA = G * A, N = R.N;
  const int tid = threadIdx.x;
  const int le = tid / kX2Threads, j = tid - le * kX2Threads;
  const int a0 = 2 * j;
  const int e0 = blockIdx.x * G;
  const int e = e0 + le;
  const bool valid = e < R.E;
  const int ec = valid ? e : R.E - 1;
  const Layout<float> L(G, A, N, R.S, false, false);
  const int NP4 = L.NP * 4;
  float* sxy = reinterpret_cast<float*>(smem + L.xy);
  float4* srec = reinterpret_cast<float4*>(smem + L.rec);
  float* srad = reinterpret_cast<float*>(smem + L.rad);
  float* siden = reinterpret_cast<float*>(smem + L.iden);
  Obs<float>* sobs = reinterpret_cast<Obs<float>*>(smem + L.obs);

  AgentP<float> P0, P1;
  load_params(R, ec, a0, P0);
  load_params(R, ec, a0 + 1, P1);
  const WorldC<float> W = R.W;
  srad[le * A + a0] = P0.radius;
  srad[le * A + a0 + 1] = P1.radius;
  siden[le * A + a0] = P0.inv_denom;
  siden[le * A + a0 + 1] = P1.inv_denom;
  if (FL & F_OBS) load_obstacles(R, sobs, e0);
  __syncthreads();

  const long long ia = (long long)ec * A + a0;  // the pair's first agent (even)
  const long long EA = (long long)R.E * A;
  Agent<float> x0, x1;
  load_pair(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, x0, x1);
  int tmax0 = 0, tmax1 = 0;
  int buf = 0;
  float4 act = reinterpret_cast<const float4*>(R.act)[ia >> 1];
  float4 nact = act;
  const float* rad_env = srad + le * A;
  const Obs<float>* obs_env = sobs + le * N;
#pragma unroll 2
  for (int t = 0; t < R.H; ++t) {
    if (t + 1 < R.H) nact = reinterpret_cast<const float4*>(R.act)[((long long)(t + 1) * EA + ia) >> 1];
    for (int k = 0; k < R.S; ++k) {
      float* xy_env = sxy + (buf * G + le) * NP4;
      float4* rec_env = srec + buf * GA + le * A;
      reinterpret_cast<float4*>(xy_env)[j] = make_float4(x0.px, x1.px, x0.py, x1.py);
      rec_env[a0] = make_float4(x0.px, x0.py, x0.vx, x0.vy);
      rec_env[a0 + 1] = make_float4(x1.px, x1.py, x1.vx, x1.vy);
      float sx0, sy0, sx1, sy1;
      static_forces_both<FL>(obs_env, N, x0, x1, P0, P1, W, sx0, sy0, sx1, sy1);
      __syncthreads();
      unsigned m0, m1;
      scan_pair16(xy_env, x0, x1, W.r2_scan, m0, m1);
      m0 &= ~(1u << a0);
      m1 &= ~(1u << (a0 + 1));
      float fx0 = 0.f, fy0 = 0.f, fx1 = 0.f, fy1 = 0.f;
      int n0 = 0, n1 = 0;
      unsigned c0, c1;
      if (W.max_overlap > 0.f) {
        c0 = contacts_of(rec_env, rad_env, m0, x0, P0, W, fx0, fy0, n0);
        c1 = contacts_of(rec_env, rad_env, m1, x1, P1, W, fx1, fy1, n1);
      } else {
        contacts_of_both(rec_env, rad_env, m0, m1, x0, x1, P0, P1, W, fx0, fy0, fx1, fy1, c0, c1,
                         n0, n1);
      }
      tmax0 = max(tmax0, n0);
      tmax1 = max(tmax1, n1);
      if (valid)
        reinterpret_cast<uint2*>(R.cmask)[(((long long)t * R.S + k) * EA + ia) >> 1] =
            make_uint2(c0, c1);
      fx0 = fx0 + sx0;
      fy0 = fy0 + sy0;
      fx1 = fx1 + sx1;
      fy1 = fy1 + sy1;
      buf ^= 1;
      Agent<float> y0, y1;
      integrate_sel<float, FL>(x0, act.x, act.y, fx0, fy0, P0, W, y0);
      integrate_sel<float, FL>(x1, act.z, act.w, fx1, fy1, P1, W, y1);
      x0 = y0;
      x1 = y1;
    }
    if (valid)
      store_pair(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, (long long)t * EA + ia, x0, x1);
    act = nact;
  }
  if (valid) {
    if (R.f_pos) store_pair(R.f_pos, R.f_th, R.f_vel, R.f_s, R.f_w, ia, x0, x1);
    if (R.true_max) reinterpret_cast<int2*>(R.true_max)[ia >> 1] = make_int2(tmax0, tmax1);
  }
  if (R.goal)
    block_sum_store(valid ? goal_dist2(R.goal, ia, x0.px, x0.py) +
                                goal_dist2(R.goal, ia + 1, x1.px, x1.py)
                          : 0.f,
                    R.loss_partial + blockIdx.x);
}

// ------------------------------------------------------------------- adjoint
// One substep per step, contacts from the checkpointed masks.
template <int FL>
__global__ void __launch_bounds__(64, SWARP_X2_BWD_MINB) rollout_bwd_x2_kernel(const RolloutArgs<float> R) {
  constexpr int A = kX2Agents;
  extern __shared__ __align__(16) unsigned char smem[];
  const int G = R.G, GA = G * A, N = R.N;
  const int tid = threadIdx.x;
  const int le = tid / kX2Threads, j = tid - le * kX2Threads;
  const int a0 = 2 * j;
  const int e0 = blockIdx.x * G;
  const int e = e0 + le;
  const bool valid = e < R.E;
  const int ec = valid ? e : R.E - 1;
  const Layout<float> L(G, A, N, 1, true, false);
  float4* srec = reinterpret_cast<float4*>(smem + L.rec);  // [2][GA]
  float2* sfb = reinterpret_cast<float2*>(smem + L.fb);    // [2][GA]
  float* srad = reinterpret_cast<float*>(smem + L.rad);
  float* siden = reinterpret_cast<float*>(smem + L.iden);
  Obs<float>* sobs = reinterpret_cast<Obs<float>*>(smem + L.obs);

  AgentP<float> P0, P1;
  load_params(R, ec, a0, P0);
  load_params(R, ec, a0 + 1, P1);
  const WorldC<float> W = R.W;
  srad[le * A + a0] = P0.radius;
  srad[le * A + a0 + 1] = P1.radius;
  siden[le * A + a0] = P0.inv_denom;
  siden[le * A + a0 + 1] = P1.inv_denom;
  if (FL & F_OBS) load_obstacles(R, sobs, e0);
  __syncthreads();

  const long long ia = (long long)ec * A + a0;
  const long long EA = (long long)R.E * A;
  const int H = R.H;
  const float* rad_env = srad + le * A;
  const float* iden_env = siden + le * A;
  const Obs<float>* obs_env = sobs + le * N;
  const bool has_gt = R.gt_pos || R.gt_th || R.gt_vel || R.gt_s || R.gt_w;
  constexpr bool kPV = (FL & F_HOLOVEL) != 0;  // only positions/velocities enter the adjoint
  auto load_traj = [&](long long i, Agent<float>& u0, Agent<float>& u1) {
    if (kPV)
      load_pair_pv(R.t_pos, R.t_vel, i, u0, u1);
    else
      load_pair(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, i, u0, u1);
  };
  auto load_init = [&](Agent<float>& u0, Agent<float>& u1) {
    if (kPV)
      load_pair_pv(R.i_pos, R.i_vel, ia, u0, u1);
    else
      load_pair(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, u0, u1);
  };

  Agent<float> g0{}, g1{};
  add_cotangent_pair(R.gf_pos, R.gf_th, R.gf_vel, R.gf_s, R.gf_w, ia, g0, g1);
  if (R.goal) {  // the fused goal loss's seed, from the final positions
    const float4 pH = reinterpret_cast<const float4*>(R.t_pos)[((long long)(H - 1) * EA + ia) >> 1];
    seed_goal_loss(R, ia, pH.x, pH.y, g0);
    seed_goal_loss(R, ia + 1, pH.z, pH.w, g1);
  }
  Agent<float> n0, n1, c0, c1;  // output and input states of step t
  load_traj((long long)(H - 1) * EA + ia, n0, n1);

  if (H > 1)
    load_traj((long long)(H - 2) * EA + ia, c0, c1);
  else
    load_init(c0, c1);
  float4 act = reinterpret_cast<const float4*>(R.act)[((long long)(H - 1) * EA + ia) >> 1];
  uint2 cm = reinterpret_cast<const uint2*>(R.cmask)[((long long)(H - 1) * EA + ia) >> 1];
  int fbuf = 0;
  float gsq = 0.f;
  for (int t = H - 1; t >= 0; --t) {
    if (has_gt) add_cotangent_pair(R.gt_pos, R.gt_th, R.gt_vel, R.gt_s, R.gt_w, (long long)t * EA + ia, g0, g1);
    Agent<float> p0{}, p1{};
    float4 pact = make_float4(0.f, 0.f, 0.f, 0.f);
    uint2 pcm = make_uint2(0u, 0u);
    if (t > 0) {
      if (t > 1)
        load_traj((long long)(t - 2) * EA + ia, p0, p1);
      else
        load_init(p0, p1);
      pact = reinterpret_cast<const float4*>(R.act)[((long long)(t - 1) * EA + ia) >> 1];
      pcm = reinterpret_cast<const uint2*>(R.cmask)[((long long)(t - 1) * EA + ia) >> 1];
    }
    float ga00 = 0.f, ga01 = 0.f, ga10 = 0.f, ga11 = 0.f;
    Agent<float> gi0, gi1;
    float gfx0, gfy0, gfx1, gfy1;
    integrate_vjp_sel<float, FL>(c0, act.x, act.y, n0, g0, P0, W, gi0, gfx0, gfy0, ga00, ga01);
    integrate_vjp_sel<float, FL>(c1, act.z, act.w, n1, g1, P1, W, gi1, gfx1, gfy1, ga10, ga11);
    float4* rec_env = srec + fbuf * GA + le * A;
    float2* fb_env = sfb + fbuf * GA + le * A;
    rec_env[a0] = make_float4(c0.px, c0.py, c0.vx, c0.vy);
    rec_env[a0 + 1] = make_float4(c1.px, c1.py, c1.vx, c1.vy);
    reinterpret_cast<float4*>(fb_env)[j] = make_float4(gfx0, gfy0, gfx1, gfy1);
    // the walls' VJP factors need only the agents' own states and force cotangents
    const bool lin_walls = W.bounds_mode == BOUNDS_SOFT && !(W.max_overlap > 0.f);
    float wdx0 = 0.f, wdy0 = 0.f, wdx1 = 0.f, wdy1 = 0.f;
    if (lin_walls) {
      wall_lin_vjp_factors(c0.px, c0.py, c0.vx, c0.vy, P0.radius, P0.inv_denom, gfx0, gfy0, W,
                           wdx0, wdy0);
      wall_lin_vjp_factors(c1.px, c1.py, c1.vx, c1.vy, P1.radius, P1.inv_denom, gfx1, gfy1, W,
                           wdx1, wdy1);
    }
    __syncthreads();
    if (W.max_overlap > 0.f) {
      force_vjp<float, FL, A>(nullptr, rec_env, fb_env, nullptr, rad_env, iden_env, obs_env,
                              nullptr, nullptr, N, A, a0, cm.x, c0, P0, W, gfx0, gfy0, gi0);
      force_vjp<float, FL, A>(nullptr, rec_env, fb_env, nullptr, rad_env, iden_env, obs_env,
                              nullptr, nullptr, N, A, a0 + 1, cm.y, c1, P1, W, gfx1, gfy1, gi1);
    } else {
      contact_vjp_both(rec_env, fb_env, rad_env, iden_env, cm.x, cm.y, c0, c1, P0, P1, W, gfx0,
                       gfy0, gfx1, gfy1, gi0, gi1);
      if (FL & F_OBS) {
        for (int o = 0; o < N; ++o) {
          obstacle_force_vjp(c0.px, c0.py, c0.vx, c0.vy, P0.radius, P0.inv_denom, obs_env[o],
                             gfx0, gfy0, W, gi0.px, gi0.py, gi0.vx, gi0.vy);
          obstacle_force_vjp(c1.px, c1.py, c1.vx, c1.vy, P1.radius, P1.inv_denom, obs_env[o],
                             gfx1, gfy1, W, gi1.px, gi1.py, gi1.vx, gi1.vy);
        }
      }
      if (lin_walls) {
        wall_lin_vjp_apply(wdx0, wdy0, W, gi0.px, gi0.py, gi0.vx, gi0.vy);
        wall_lin_vjp_apply(wdx1, wdy1, W, gi1.px, gi1.py, gi1.vx, gi1.vy);
      }
    }
    g0 = gi0;
    g1 = gi1;
    fbuf ^= 1;
    if (valid) {
      reinterpret_cast<float4*>(R.g_act)[((long long)t * EA + ia) >> 1] =
          make_float4(ga00, ga01, ga10, ga11);
      gsq = Num<float>::fma_(ga00, ga00, Num<float>::fma_(ga01, ga01, gsq));
      gsq = Num<float>::fma_(ga10, ga10, Num<float>::fma_(ga11, ga11, gsq));
    }
    n0 = c0;
    n1 = c1;
    c0 = p0;
    c1 = p1;
    act = pact;
    cm = pcm;
  }
  if (valid) {
    store_state(R.gi_pos, R.gi_th, R.gi_vel, R.gi_s, R.gi_w, ia, g0);
    store_state(R.gi_pos, R.gi_th, R.gi_vel, R.gi_s, R.gi_w, ia + 1, g1);
  }
  if (R.gsq_partial) block_sum_store(gsq, R.gsq_partial + blockIdx.x);
}

}  // namespace swarp
