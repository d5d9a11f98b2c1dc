// Fused multi-step rollout kernels (forward and adjoint) for sm_100a.
//
// Layout: one thread per agent, the agents of G whole envs per CTA (G * A threads),
// so the O(A^2) neighbor pass of an env reads its agents' positions from shared
// memory. Each CTA runs its envs through the whole horizon: the forward kernel keeps
// the state in registers and streams actions in / trajectory out (structure of arrays,
// consecutive threads -> consecutive (env, agent) -> coalesced); the adjoint kernel
// walks the horizon backwards, re-reading each step's input state from the trajectory
// (the checkpoint) and recomputing contacts instead of storing them. Accumulation is
// a gather in fixed (ascending agent index) order: no atomics, bitwise deterministic.
#pragma once
#include "physics.cuh"

namespace swarp {

template <typename T> struct V2;
template <> struct V2<float> { using t = float2; };
template <> struct V2<double> { using t = double2; };
template <typename T> struct V4;
template <> struct V4<float> { using t = float4; };
template <> struct V4<double> { using t = double4; };

// Compile-time feature switches of one kernel instance.
enum : int {
  F_COLL = 1,      // agent-agent contacts
  F_TRUNC = 2,     // list cap can truncate (A - 1 > K): store/read per-substep cutoffs
  F_OBS = 4,       // obstacles present
  F_HOLOVEL = 8,   // every agent is holonomic / VELOCITY
  F_BODIES = 16,   // movable bodies integrated in the substep loop
};

template <typename T> struct RolloutArgs {
  int E, A, G, H, S, act_dim, N;
  WorldC<T> W;
  const T* params;
  long long params_env_stride;
  const int* model_tag;
  const int* ctrl_mode;
  // obstacles
  const T *o_pos, *o_angle, *o_vel, *o_ang_vel, *o_radius, *o_half;
  const int* o_shape;
  // init / actions / trajectory / final
  const T *i_pos, *i_th, *i_vel, *i_s, *i_w;
  const T* act;
  T *t_pos, *t_th, *t_vel, *t_s, *t_w;
  T *f_pos, *f_th, *f_vel, *f_s, *f_w;
  int* true_max;
  int16_t* cutoff;  // workspace [H*S, E, A] (F_TRUNC)
  // adjoint
  const T *gt_pos, *gt_th, *gt_vel, *gt_s, *gt_w;  // cotangent of trajectory (nullable)
  const T *gf_pos, *gf_th, *gf_vel, *gf_s, *gf_w;  // cotangent of final (nullable)
  T* g_act;
  T *gi_pos, *gi_th, *gi_vel, *gi_s, *gi_w;
};

// ------------------------------------------------------------------ loaders
template <typename T>
__device__ __forceinline__ void load_params(const RolloutArgs<T>& R, int e, int a, AgentP<T>& P) {
  const T* row = R.params + (long long)e * R.params_env_stride + (long long)a * 22;
  P.radius = row[0];
  P.mass = row[1];
  P.max_speed = row[2];
  P.max_accel = row[3];
  P.max_ang_vel = row[4];
  P.max_ang_accel = row[5];
  P.l_f = row[6];
  P.l_r = row[7];
  P.max_steer = row[8];
  P.min_speed = row[16];
  P.gain_v = row[20];
  P.gain_w = row[21];
  P.tag = R.model_tag[a];
  P.mode = R.ctrl_mode[a];
  P.dt_over_m = R.W.dt / P.mass;
  P.denom = T(1) + R.W.c * R.W.dt / P.mass;
}

template <typename T>
__device__ __forceinline__ void load_state(const T* pos, const T* th, const T* vel, const T* s,
                                           const T* w, long long i, Agent<T>& x) {
  using T2 = typename V2<T>::t;
  T2 p = reinterpret_cast<const T2*>(pos)[i];
  T2 v = reinterpret_cast<const T2*>(vel)[i];
  x.px = p.x;
  x.py = p.y;
  x.vx = v.x;
  x.vy = v.y;
  x.th = th[i];
  x.s = s[i];
  x.w = w[i];
}

template <typename T>
__device__ __forceinline__ void store_state(T* pos, T* th, T* vel, T* s, T* w, long long i,
                                            const Agent<T>& x) {
  using T2 = typename V2<T>::t;
  reinterpret_cast<T2*>(pos)[i] = T2{x.px, x.py};
  reinterpret_cast<T2*>(vel)[i] = T2{x.vx, x.vy};
  th[i] = x.th;
  s[i] = x.s;
  w[i] = x.w;
}

// Cotangent fields may be absent (NULL = zero).
template <typename T>
__device__ __forceinline__ void add_cotangent(const T* pos, const T* th, const T* vel, const T* s,
                                              const T* w, long long i, Agent<T>& g) {
  using T2 = typename V2<T>::t;
  if (pos) {
    T2 p = reinterpret_cast<const T2*>(pos)[i];
    g.px += p.x;
    g.py += p.y;
  }
  if (vel) {
    T2 v = reinterpret_cast<const T2*>(vel)[i];
    g.vx += v.x;
    g.vy += v.y;
  }
  if (th) g.th += th[i];
  if (s) g.s += s[i];
  if (w) g.w += w[i];
}

template <typename T>
__device__ __forceinline__ void load_action(const RolloutArgs<T>& R, long long i, T& a0, T& a1) {
  using T2 = typename V2<T>::t;
  if (R.act_dim == 2) {
    T2 v = reinterpret_cast<const T2*>(R.act)[i];
    a0 = v.x;
    a1 = v.y;
  } else {
    a0 = R.act[i * R.act_dim];
    a1 = R.act[i * R.act_dim + 1];
  }
}

// Obstacles of this CTA's envs into shared memory (the agent pass re-reads them every
// substep). Angle -> (cos, sin) once.
template <typename T>
__device__ __forceinline__ void load_obstacles(const RolloutArgs<T>& R, Obs<T>* sobs, int e0) {
  const int total = R.G * R.N;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int le = i / R.N, o = i - le * R.N;
    int e = e0 + le;
    if (e >= R.E) e = R.E - 1;
    const long long eo = (long long)e * R.N + o;
    Obs<T> ob;
    ob.cx = R.o_pos[2 * eo];
    ob.cy = R.o_pos[2 * eo + 1];
    T ang = R.o_angle[eo];
    ob.ca = Num<T>::cos_(ang);
    ob.sa = Num<T>::sin_(ang);
    ob.vx = R.o_vel[2 * eo];
    ob.vy = R.o_vel[2 * eo + 1];
    ob.om = R.o_ang_vel[eo];
    ob.r = R.o_radius[o];
    ob.hx = R.o_half[2 * o];
    ob.hy = R.o_half[2 * o + 1];
    ob.type = R.o_shape[o];
    if (ob.type == SHAPE_BOX)
      ob.bound = len2(ob.hx, ob.hy);
    else if (ob.type == SHAPE_SEGMENT)
      ob.bound = ob.hx + ob.r;
    else
      ob.bound = ob.r;
    sobs[i] = ob;
  }
}

// ------------------------------------------------------------- neighbor scan
// Calls fn(b, dx, dy, d2) for every agent b != a of this env with sqrt(d2) <= R, in
// ascending b. Positions come from spv (x, y in the first two lanes).
template <typename T, typename Fn>
__device__ __forceinline__ int scan_radius(const typename V4<T>::t* spv, int base, int A, int a,
                                           T px, T py, T r2_thr, Fn&& fn) {
  int total = 0;
  for (int c0 = 0; c0 < A; c0 += 32) {
    const int n = min(32, A - c0);
    unsigned m = 0u;
#pragma unroll 8
    for (int jj = 0; jj < n; ++jj) {
      const auto q = spv[base + c0 + jj];
      const T dx = px - q.x, dy = py - q.y;
      const T d2 = dot2(dx, dy, dx, dy);
      m |= (d2 <= r2_thr) ? (1u << jj) : 0u;
    }
    const int rel = a - c0;
    if (rel >= 0 && rel < 32) m &= ~(1u << rel);
    total += __popc(m);
    while (m) {
      const int jj = __ffs(m) - 1;
      m &= m - 1u;
      const int b = c0 + jj;
      const auto q = spv[base + b];
      const T dx = px - q.x, dy = py - q.y;
      fn(b, dx, dy, dot2(dx, dy, dx, dy), q);
    }
  }
  return total;
}

// Contact force on agent a from its capped neighbor list (the first K within R by index).
// Returns the uncapped count; cutoff = index of the K-th listed neighbor if truncated, else A.
template <typename T, int FL>
__device__ __forceinline__ int neighbor_force(const typename V4<T>::t* spv, const T* srad, int base,
                                              int A, int a, const Agent<T>& x, const AgentP<T>& P,
                                              const WorldC<T>& W, T& fx, T& fy, int& cutoff) {
  int listed = 0;
  cutoff = A;
  const int total = scan_radius<T>(spv, base, A, a, x.px, x.py, W.r2_thr,
                                   [&](int b, T dx, T dy, T d2, const typename V4<T>::t& q) {
    if (FL & F_TRUNC) {
      if (listed >= W.K) return;
      ++listed;
      if (listed == W.K) cutoff = b;
    }
    pair_force_add(dx, dy, d2, x.vx - q.z, x.vy - q.w, P.radius + srad[base + b] + W.margin,
                   P.denom, W, fx, fy);
  });
  if ((FL & F_TRUNC) && total <= W.K) cutoff = A;
  return total;
}

template <typename T, int FL>
__device__ __forceinline__ void static_force(const Obs<T>* sobs, int N, const Agent<T>& x,
                                             const AgentP<T>& P, const WorldC<T>& W, T& fx, T& fy) {
  T sx = T(0), sy = T(0);
  if (FL & F_OBS) {
    for (int o = 0; o < N; ++o) {
      T gx, gy;
      obstacle_force(x.px, x.py, x.vx, x.vy, P.radius, P.denom, sobs[o], W, gx, gy);
      sx = sx + gx;
      sy = sy + gy;
    }
  }
  if (W.bounds_mode == BOUNDS_SOFT) {
    T wx, wy;
    wall_force(x.px, x.py, x.vx, x.vy, P.radius, P.denom, W, wx, wy);
    sx = sx + wx;
    sy = sy + wy;
  }
  fx = fx + sx;
  fy = fy + sy;
}

template <typename T, int FL>
__device__ __forceinline__ void integrate_sel(const Agent<T>& in, T a0, T a1, T fx, T fy,
                                              const AgentP<T>& P, const WorldC<T>& W, Agent<T>& out) {
  if (FL & F_HOLOVEL) {
    AgentP<T> Q = P;
    Q.tag = TAG_HOLONOMIC;
    Q.mode = MODE_VELOCITY;
    integrate_fwd(in, a0, a1, fx, fy, Q, W, out);
  } else {
    integrate_fwd(in, a0, a1, fx, fy, P, W, out);
  }
}

// Shared-memory footprint.
template <typename T> struct Smem {
  static size_t fwd(int GA, int GN) {
    return 2 * GA * sizeof(typename V4<T>::t) + GA * sizeof(T) + GN * sizeof(Obs<T>) + 64;
  }
  static size_t bwd(int GA, int GN, int S) {
    const int nb = S > 2 ? S : 2;
    return nb * GA * sizeof(typename V4<T>::t)      // pos/vel per substep
           + S * GA * sizeof(typename V4<T>::t)     // own th/s/w per substep
           + 2 * GA * sizeof(typename V2<T>::t)     // force cotangent, double buffered
           + 2 * GA * sizeof(int)                   // cutoffs, double buffered
           + 2 * GA * sizeof(T)                     // radius, denominator
           + GN * sizeof(Obs<T>) + 128;
  }
};

// ================================================================== forward
template <typename T, int FL>
__global__ void __launch_bounds__(1024) rollout_fwd_kernel(const RolloutArgs<T> R) {
  using T4 = typename V4<T>::t;
  extern __shared__ __align__(16) unsigned char smem[];
  const int A = R.A, G = R.G, GA = G * A;
  const int tid = threadIdx.x;
  const int le = tid / A, a = tid - le * A;
  const int e0 = blockIdx.x * G;
  const int e = e0 + le;
  const bool valid = e < R.E;
  const int ec = valid ? e : R.E - 1;
  const int base = le * A;

  T4* spv = reinterpret_cast<T4*>(smem);            // [2][GA]
  T* srad = reinterpret_cast<T*>(spv + 2 * GA);     // [GA]
  Obs<T>* sobs = reinterpret_cast<Obs<T>*>(
      (reinterpret_cast<uintptr_t>(srad + GA) + 15) & ~uintptr_t(15));  // [G][N]

  AgentP<T> P;
  load_params(R, ec, a, P);
  const WorldC<T> W = R.W;
  srad[tid] = P.radius;
  if (FL & F_OBS) load_obstacles(R, sobs, e0);

  const long long ia = (long long)ec * A + a;  // (env, agent) linear index
  const long long EA = (long long)R.E * A;
  Agent<T> x;
  load_state(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, x);
  int tmax = 0;
  int buf = 0;
  T a0, a1, n0, n1;
  load_action(R, ia, a0, a1);
  for (int t = 0; t < R.H; ++t) {
    if (t + 1 < R.H) load_action(R, (long long)(t + 1) * EA + ia, n0, n1);
    for (int k = 0; k < R.S; ++k) {
      T fx = T(0), fy = T(0);
      if (FL & F_COLL) {
        spv[buf * GA + tid] = T4{x.px, x.py, x.vx, x.vy};
        __syncthreads();
        int cutoff;
        const int tc = neighbor_force<T, FL>(spv + buf * GA, srad, base, A, a, x, P, W, fx, fy, cutoff);
        tmax = max(tmax, tc);
        if ((FL & F_TRUNC) && valid) R.cutoff[((long long)t * R.S + k) * EA + ia] = (int16_t)cutoff;
        buf ^= 1;
      } else if (t == 0 && k == 0) {
        __syncthreads();  // obstacles / radii visible
      }
      static_force<T, FL>(sobs + le * R.N, R.N, x, P, W, fx, fy);
      Agent<T> y;
      integrate_sel<T, FL>(x, a0, a1, fx, fy, P, W, y);
      x = y;
    }
    if (valid)
      store_state(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, (long long)t * EA + ia, x);
    a0 = n0;
    a1 = n1;
  }
  if (valid) {
    if (R.f_pos) store_state(R.f_pos, R.f_th, R.f_vel, R.f_s, R.f_w, ia, x);
    if (R.true_max) R.true_max[ia] = tmax;
  }
}

// ================================================================== adjoint
// Adjoint of the neighbor + static force pass of agent a at one substep: given the
// force cotangents of every agent of the env (sfb), adds d(loss)/d(pos, vel) of agent a.
template <typename T, int FL>
__device__ __forceinline__ void force_vjp(const typename V4<T>::t* spv,
                                          const typename V2<T>::t* sfb, const int* scut,
                                          const T* srad, const T* sden, const Obs<T>* sobs,
                                          int N, int base, int A, int a, const Agent<T>& x,
                                          const AgentP<T>& P, const WorldC<T>& W, T gfx, T gfy,
                                          Agent<T>& gin) {
  if (FL & F_COLL) {
    const int cut_a = (FL & F_TRUNC) ? scut[base + a] : A;
    scan_radius<T>(spv, base, A, a, x.px, x.py, W.r2_thr,
                   [&](int b, T dx, T dy, T d2, const typename V4<T>::t& q) {
      const T rb = srad[base + b];
      const T min_dist = P.radius + rb + W.margin;
      const T dist = Num<T>::sqrt_(wmax(d2, Eps2<T>::v));
      if (!(min_dist - dist > T(0))) return;  // not in contact: zero force both ways
      const T rvx = x.vx - q.z, rvy = x.vy - q.w;
      const bool own = !(FL & F_TRUNC) || b <= cut_a;
      const bool cross = !(FL & F_TRUNC) || a <= scut[base + b];
      if (own) {
        pair_force_vjp(dx, dy, rvx, rvy, min_dist, P.denom, gfx, gfy, W, gin.px, gin.py, gin.vx,
                       gin.vy);
      }
      if (cross) {
        const auto gb = sfb[base + b];
        T gdx = T(0), gdy = T(0), grx = T(0), gry = T(0);
        pair_force_vjp(-dx, -dy, -rvx, -rvy, rb + P.radius + W.margin, sden[base + b], gb.x, gb.y,
                       W, gdx, gdy, grx, gry);
        gin.px -= gdx;
        gin.py -= gdy;
        gin.vx -= grx;
        gin.vy -= gry;
      }
    });
  }
  if (FL & F_OBS) {
    for (int o = 0; o < N; ++o)
      obstacle_force_vjp(x.px, x.py, x.vx, x.vy, P.radius, P.denom, sobs[o], gfx, gfy, W, gin.px,
                         gin.py, gin.vx, gin.vy);
  }
  if (W.bounds_mode == BOUNDS_SOFT)
    wall_force_vjp(x.px, x.py, x.vx, x.vy, P.radius, P.denom, gfx, gfy, W, gin.px, gin.py, gin.vx,
                   gin.vy);
}

template <typename T, int FL>
__device__ __forceinline__ void integrate_vjp_sel(const Agent<T>& in, T a0, T a1, const Agent<T>& out,
                                                  const Agent<T>& g, const AgentP<T>& P,
                                                  const WorldC<T>& W, Agent<T>& gin, T& gfx, T& gfy,
                                                  T& ga0, T& ga1) {
  if (FL & F_HOLOVEL) {
    AgentP<T> Q = P;
    Q.tag = TAG_HOLONOMIC;
    Q.mode = MODE_VELOCITY;
    integrate_vjp(in, a0, a1, out, g, Q, W, gin, gfx, gfy, ga0, ga1);
  } else {
    integrate_vjp(in, a0, a1, out, g, P, W, gin, gfx, gfy, ga0, ga1);
  }
}

template <typename T, int FL>
__global__ void __launch_bounds__(1024) rollout_bwd_kernel(const RolloutArgs<T> R) {
  using T2 = typename V2<T>::t;
  using T4 = typename V4<T>::t;
  extern __shared__ __align__(16) unsigned char smem[];
  const int A = R.A, G = R.G, GA = G * A, S = R.S;
  const int tid = threadIdx.x;
  const int le = tid / A, a = tid - le * A;
  const int e0 = blockIdx.x * G;
  const int e = e0 + le;
  const bool valid = e < R.E;
  const int ec = valid ? e : R.E - 1;
  const int base = le * A;
  const int nb = S > 2 ? S : 2;

  T4* spv = reinterpret_cast<T4*>(smem);           // [nb][GA] pos/vel of substep inputs
  T4* sown = spv + nb * GA;                         // [S][GA]  th/s/w of substep inputs
  T2* sfb = reinterpret_cast<T2*>(sown + S * GA);   // [2][GA]  force cotangents
  int* scut = reinterpret_cast<int*>(sfb + 2 * GA); // [2][GA]  cutoffs
  T* srad = reinterpret_cast<T*>(
      (reinterpret_cast<uintptr_t>(scut + 2 * GA) + 15) & ~uintptr_t(15));  // [GA]
  T* sden = srad + GA;                                                     // [GA]
  Obs<T>* sobs = reinterpret_cast<Obs<T>*>(
      (reinterpret_cast<uintptr_t>(sden + GA) + 15) & ~uintptr_t(15));

  AgentP<T> P;
  load_params(R, ec, a, P);
  const WorldC<T> W = R.W;
  srad[tid] = P.radius;
  sden[tid] = P.denom;
  if (FL & F_OBS) load_obstacles(R, sobs, e0);
  __syncthreads();

  const long long ia = (long long)ec * A + a;
  const long long EA = (long long)R.E * A;
  const int H = R.H;

  Agent<T> g{};
  add_cotangent(R.gf_pos, R.gf_th, R.gf_vel, R.gf_s, R.gf_w, ia, g);
  Agent<T> nxt;  // output state of step t
  load_state(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, (long long)(H - 1) * EA + ia, nxt);
  int fbuf = 0;
  for (int t = H - 1; t >= 0; --t) {
    if (R.gt_pos || R.gt_th || R.gt_vel || R.gt_s || R.gt_w)
      add_cotangent(R.gt_pos, R.gt_th, R.gt_vel, R.gt_s, R.gt_w, (long long)t * EA + ia, g);
    Agent<T> cur;
    if (t > 0)
      load_state(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, (long long)(t - 1) * EA + ia, cur);
    else
      load_state(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, cur);
    T a0, a1;
    load_action(R, (long long)t * EA + ia, a0, a1);
    T ga0 = T(0), ga1 = T(0);

    if (S == 1) {
      Agent<T> gin;
      T gfx, gfy;
      integrate_vjp_sel<T, FL>(cur, a0, a1, nxt, g, P, W, gin, gfx, gfy, ga0, ga1);
      spv[fbuf * GA + tid] = T4{cur.px, cur.py, cur.vx, cur.vy};
      sfb[fbuf * GA + tid] = T2{gfx, gfy};
      if (FL & F_TRUNC) scut[fbuf * GA + tid] = R.cutoff[(long long)t * EA + ia];
      __syncthreads();
      force_vjp<T, FL>(spv + fbuf * GA, sfb + fbuf * GA, scut + fbuf * GA, srad, sden,
                       sobs + le * R.N, R.N, base, A, a, cur, P, W, gfx, gfy, gin);
      g = gin;
      fbuf ^= 1;
    } else {
      // recompute the substep chain from the checkpointed step input
      __syncthreads();  // every thread is done reading last step's stash
      Agent<T> x = cur;
      for (int k = 0; k < S; ++k) {
        spv[k * GA + tid] = T4{x.px, x.py, x.vx, x.vy};
        sown[k * GA + tid] = T4{x.th, x.s, x.w, T(0)};
        if (k == S - 1) break;
        T fx = T(0), fy = T(0);
        if (FL & F_COLL) {
          __syncthreads();
          int cutoff;
          neighbor_force<T, FL>(spv + k * GA, srad, base, A, a, x, P, W, fx, fy, cutoff);
        }
        static_force<T, FL>(sobs + le * R.N, R.N, x, P, W, fx, fy);
        Agent<T> y;
        integrate_sel<T, FL>(x, a0, a1, fx, fy, P, W, y);
        x = y;
      }
      Agent<T> out = nxt;
      for (int k = S - 1; k >= 0; --k) {
        const T4 pv = spv[k * GA + tid];
        const T4 ow = sown[k * GA + tid];
        Agent<T> in{pv.x, pv.y, ow.x, pv.z, pv.w, ow.y, ow.z};
        Agent<T> gin;
        T gfx, gfy;
        integrate_vjp_sel<T, FL>(in, a0, a1, out, g, P, W, gin, gfx, gfy, ga0, ga1);
        sfb[fbuf * GA + tid] = T2{gfx, gfy};
        if (FL & F_TRUNC) scut[fbuf * GA + tid] = R.cutoff[((long long)t * S + k) * EA + ia];
        __syncthreads();
        force_vjp<T, FL>(spv + k * GA, sfb + fbuf * GA, scut + fbuf * GA, srad, sden,
                         sobs + le * R.N, R.N, base, A, a, in, P, W, gfx, gfy, gin);
        g = gin;
        out = in;
        fbuf ^= 1;
      }
    }
    if (valid) {
      const long long ja = (long long)t * EA + ia;
      if (R.act_dim == 2) {
        reinterpret_cast<T2*>(R.g_act)[ja] = T2{ga0, ga1};
      } else {
        R.g_act[ja * R.act_dim] = ga0;
        R.g_act[ja * R.act_dim + 1] = ga1;
        for (int j = 2; j < R.act_dim; ++j) R.g_act[ja * R.act_dim + j] = T(0);
      }
    }
    nxt = cur;
  }
  if (valid) store_state(R.gi_pos, R.gi_th, R.gi_vel, R.gi_s, R.gi_w, ia, g);
}

// ============================================================ neighbor lists
template <typename T>
__global__ void __launch_bounds__(1024) neighbors_kernel(int E, int A, int G, int K, T r2_thr,
                                                         const T* pos, int* idx, int* count,
                                                         int* true_count) {
  using T2 = typename V2<T>::t;
  using T4 = typename V4<T>::t;
  extern __shared__ __align__(16) unsigned char smem[];
  T4* spv = reinterpret_cast<T4*>(smem);
  const int tid = threadIdx.x;
  const int le = tid / A, a = tid - le * A;
  const int e = blockIdx.x * G + le;
  const bool valid = e < E;
  const int ec = valid ? e : E - 1;
  const long long ia = (long long)ec * A + a;
  const T2 p = reinterpret_cast<const T2*>(pos)[ia];
  spv[tid] = T4{p.x, p.y, T(0), T(0)};
  __syncthreads();
  int listed = 0;
  const int total = scan_radius<T>(spv, le * A, A, a, p.x, p.y, r2_thr,
                                   [&](int b, T, T, T, const T4&) {
    if (listed < K) {
      if (valid) idx[ia * K + listed] = b;
      ++listed;
    }
  });
  if (valid) {
    count[ia] = listed;
    true_count[ia] = total;
  }
}

}  // namespace swarp
