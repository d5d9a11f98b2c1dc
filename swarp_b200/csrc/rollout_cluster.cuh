// Rollout kernels for envs larger than one CTA (n_agents > 1024): one env per thread-block
// cluster of CS CTAs (CS <= 8, the portable cluster size), BT threads per CTA, one thread
// per agent (agent a = cluster rank * BT + thread).
//
// Shared memory across the cluster (distributed shared memory, DSMEM):
//  - the env's pair-packed scan table (x, y of every agent, the layout of rollout.cuh) is
//    REPLICATED: each agent stores its position into every CTA's copy (CS remote stores),
//    so the O(A) candidate scan of every agent reads only its own CTA's shared memory;
//  - each agent's record (vx, vy, radius, damping denominator) and, in the adjoint, its
//    (force cotangent, list cutoff) record stay in its OWN CTA; a thread reads them from
//    the owning CTA (mapa + ld.shared::cluster, one 16-byte load each) only for the
//    neighbors it actually lists, and takes their positions from its local scan table.
// A cluster barrier (barrier.cluster arrive.release / wait.acquire) replaces the CTA
// barrier of the single-CTA kernels wherever an env's agents exchange data, and a last one
// keeps every CTA resident until no peer can still read its shared memory.
//
// The arithmetic is the single-CTA kernels' device code in the same order (scan in
// ascending index, the first K members listed, forces summed in list order, the merged
// symmetric pair VJP gathered by the owner), so an env gives bitwise the same trajectory
// and gradients whichever kernel runs it (tested by forcing this path on small envs).
// Scope: 2-D disc fleets (every model and control mode), contacts with or without list
// truncation, static obstacles, walls, substeps, Euler or RK4, per-env parameters, the
// fused goal loss and gradient-norm partials. Movable bodies, box agents and drones in
// envs above 1024 agents are rejected on the host (SWARP_ERR_UNSUPPORTED).
#pragma once
#include <cooperative_groups.h>

#include "rollout.cuh"

namespace swarp {

namespace cg = cooperative_groups;

constexpr int kClusterMaxThreads = 512;  // launch bound of the cluster kernels' CTAs
constexpr int kClusterMaxCTAs = 8;       // portable cluster size

// Shared-memory carve-up of one cluster CTA (host: sizes; device: offsets).
template <typename T> struct ClusterLayout {
  int NP, nbuf;
  size_t xy, rec, own, fbc, obs, total;
  __host__ __device__ ClusterLayout(int A, int BT, int N, int S, bool bwd) {
    NP = (A + 1) / 2;
    nbuf = bwd ? (S > 2 ? S : 2) : 2;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = (off + bytes + 15) & ~size_t(15); return o; };
    xy = take(size_t(nbuf) * NP * 4 * sizeof(T));        // whole env, replicated
    rec = take(size_t(nbuf) * BT * 4 * sizeof(T));  // own agents' (vx, vy, radius, 1/denom)
    own = bwd ? take(size_t(S) * BT * 5 * sizeof(T)) : 0;  // own (th, s, w, x, y) per substep
    fbc = bwd ? take(size_t(2) * BT * 4 * sizeof(T)) : 0;  // own (force cot. x, y, cutoff, -)
    obs = take(size_t(N > 0 ? N : 0) * sizeof(Obs<T>));
    total = off;
  }
};

// Where agent b of the env lives: cluster rank b / BT, slot b % BT.
struct Owner {
  int BT;
  __device__ __forceinline__ unsigned rank(int b) const { return unsigned(b) / unsigned(BT); }
  __device__ __forceinline__ int slot(int b) const { return b - int(rank(b)) * BT; }
};

template <typename Q>
__device__ __forceinline__ Q peer_load(const cg::cluster_group& cl, const Q* base, const Owner& o,
                                       int b) {
  return *cl.map_shared_rank(base + o.slot(b), o.rank(b));
}

// Agent a's position into the scan table of every CTA of the cluster.
template <typename T>
__device__ __forceinline__ void put_xy_all(const cg::cluster_group& cl, T* xy_env, int CS, int a,
                                           T x, T y) {
  for (int r = 0; r < CS; ++r) put_xy(cl.map_shared_rank(xy_env, r), a, x, y);
}

// for_each_in_radius with the exact test on the scan table's coordinates: calls
// fn(b, x_b, y_b) for every member b != a in ascending order; returns the count.
template <typename T, typename Fn>
__device__ __forceinline__ int for_each_in_radius_xy(const T* xy_env, int A, int a, T px, T py,
                                                     T thr_scan, T thr, Fn&& fn) {
  const int NP = (A + 1) / 2;
  int total = 0;
  const int nchunk = (A + 31) / 32;
  for (int c = 0; c < nchunk; ++c) {
    const int npairs = min(16, NP - c * 16);
    unsigned m = scan_chunk<0>(xy_env, c, npairs, px, py, thr_scan);
    const int rel = a - 32 * c;
    if (rel >= 0 && rel < 32) m &= ~(1u << rel);
    while (m) {
      const int jj = __ffs(m) - 1;
      m &= m - 1u;
      const int b = 32 * c + jj;
      T qx, qy;
      get_xy(xy_env, b, qx, qy);
      if (!in_radius(px - qx, py - qy, thr)) continue;
      ++total;
      fn(b, qx, qy);
    }
  }
  return total;
}

// neighbor_force of the single-CTA kernels, the listed neighbors' records (vx, vy,
// radius, 1/denom) read from the CTA that owns them.
template <typename T, int FL>
__device__ __forceinline__ int neighbor_force_cl(const cg::cluster_group& cl, const Owner& own,
                                                 const T* xy_env, const typename V4<T>::t* rec,
                                                 int A, int a, const Agent<T>& x,
                                                 const AgentP<T>& P, const WorldC<T>& W, T& fx,
                                                 T& fy, int& cutoff) {
  int listed = 0;
  cutoff = A;
  const int total = for_each_in_radius_xy<T>(xy_env, A, a, x.px, x.py, W.r2_scan, W.r2_thr,
                                             [&](int b, T qx, T qy) {
    if (FL & F_TRUNC) {
      if (listed >= W.K) return;
      ++listed;
      if (listed == W.K) cutoff = b;
    }
    const auto q = peer_load(cl, rec, own, b);
    const T dx = x.px - qx, dy = x.py - qy;
    pair_force_add(dx, dy, dot2(dx, dy, dx, dy), x.vx - q.x, x.vy - q.y, P.radius + q.z + W.margin,
                   P.inv_denom, W, fx, fy);
  });
  if ((FL & F_TRUNC) && total <= W.K) cutoff = A;
  return total;
}

// force_vjp of the single-CTA kernels (rescan path), remote reads of the members' records
// and (force cotangent, cutoff) records.
template <typename T, int FL>
__device__ __forceinline__ void force_vjp_cl(const cg::cluster_group& cl, const Owner& own,
                                             const T* xy_env, const typename V4<T>::t* rec,
                                             const typename V4<T>::t* fbc, const Obs<T>* sobs,
                                             int N, int A, int a, int cut_a, const Agent<T>& x,
                                             const AgentP<T>& P, const WorldC<T>& W, T gfx, T gfy,
                                             Agent<T>& gin) {
  if (FL & F_COLL) {
    for_each_in_radius_xy<T>(xy_env, A, a, x.px, x.py, W.r2_scan, W.r2_thr,
                             [&](int b, T qx, T qy) {
      const auto q = peer_load(cl, rec, own, b);
      const auto gb = peer_load(cl, fbc, own, b);
      const bool mine = !(FL & F_TRUNC) || b <= cut_a;
      const bool cross = !(FL & F_TRUNC) || T(a) <= gb.z;
      pair_vjp_sym(x.px - qx, x.py - qy, x.vx - q.x, x.vy - q.y, P.radius + q.z + W.margin,
                   P.inv_denom, mine ? gfx : T(0), mine ? gfy : T(0), q.w, cross ? gb.x : T(0),
                   cross ? gb.y : T(0), W, gin.px, gin.py, gin.vx, gin.vy);
    });
  }
  static_force_vjp<T, FL>(sobs, nullptr, nullptr, N, x, P, W, gfx, gfy, gin);
}

// ================================================================== forward
template <typename T, int FL>
__global__ void __launch_bounds__(kClusterMaxThreads, 1) rollout_fwd_cl_kernel(const RolloutArgs<T> R) {
  using T4 = typename V4<T>::t;
  constexpr bool kColl = (FL & F_COLL) != 0;
  extern __shared__ __align__(16) unsigned char smem[];
  const cg::cluster_group cl = cg::this_cluster();
  const int CS = R.CS, BT = blockDim.x, A = R.A, N = R.N;
  const int tid = threadIdx.x;
  const int rank = (int)cl.block_rank();
  const int e = blockIdx.x / CS;
  const int a = rank * BT + tid;
  const bool live = a < A;  // the last CTA's threads past the env's agents only take barriers
  const int ac = live ? a : A - 1;
  const Owner own{BT};
  const ClusterLayout<T> L(A, BT, N, R.S, false);
  const int NP4 = L.NP * 4;
  T* sxy = reinterpret_cast<T*>(smem + L.xy);
  T4* srec = reinterpret_cast<T4*>(smem + L.rec);
  Obs<T>* sobs = reinterpret_cast<Obs<T>*>(smem + L.obs);

  AgentP<T> P;
  load_params(R, e, ac, P);
  const WorldC<T> W = R.W;
  if (FL & F_OBS) load_obstacles(R, sobs, e);
  if (kColl) init_pads(sxy, 2, 1, A);
  cl.sync();  // every CTA of the cluster has started and set up its shared memory

  const long long ia = (long long)e * A + ac;
  const long long EA = (long long)R.E * A;
  Agent<T> x;
  load_state(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, x);
  int tmax = 0;
  int buf = 0;
  T a0, a1, n0 = T(0), n1 = T(0);
  load_action(R, ia, a0, a1);
  for (int t = 0; t < R.H; ++t) {
    if (t + 1 < R.H) load_action(R, (long long)(t + 1) * EA + ia, n0, n1);
    for (int k = 0; k < R.S; ++k) {
      T fx = T(0), fy = T(0);
      if (kColl) {
        T* xy_env = sxy + buf * NP4;
        T4* rec = srec + buf * BT;
        if (live) put_xy_all(cl, xy_env, CS, a, x.px, x.py);
        rec[tid] = T4{x.vx, x.vy, P.radius, P.inv_denom};
        cl.sync();
        if (live) {
          int cutoff;
          const int tc = neighbor_force_cl<T, FL>(cl, own, xy_env, rec, A, a, x, P, W, fx, fy,
                                                  cutoff);
          tmax = max(tmax, tc);
          if (FL & F_TRUNC) R.cutoff[((long long)t * R.S + k) * EA + ia] = (int16_t)cutoff;
        }
        buf ^= 1;
      }
      static_force<T, FL>(sobs, N, x, P, W, fx, fy);
      Agent<T> y;
      integrate_sel<T, FL>(x, a0, a1, fx, fy, P, W, y);
      x = y;
    }
    if (live) store_state(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, (long long)t * EA + ia, x);
    a0 = n0;
    a1 = n1;
  }
  if (live) {
    if (R.f_pos) store_state(R.f_pos, R.f_th, R.f_vel, R.f_s, R.f_w, ia, x);
    if (R.true_max) R.true_max[ia] = tmax;
  }
  if (R.goal) block_sum_store(live ? goal_dist2(R.goal, ia, x.px, x.py) : T(0),
                              R.loss_partial + blockIdx.x);
  cl.sync();  // no CTA leaves while a peer may still read its records
}

// ================================================================== adjoint
template <typename T, int FL>
__global__ void __launch_bounds__(kClusterMaxThreads, 1) rollout_bwd_cl_kernel(const RolloutArgs<T> R) {
  using T2 = typename V2<T>::t;
  using T4 = typename V4<T>::t;
  constexpr bool kColl = (FL & F_COLL) != 0;
  extern __shared__ __align__(16) unsigned char smem[];
  const cg::cluster_group cl = cg::this_cluster();
  const int CS = R.CS, BT = blockDim.x, A = R.A, S = R.S, N = R.N;
  const int tid = threadIdx.x;
  const int rank = (int)cl.block_rank();
  const int e = blockIdx.x / CS;
  const int a = rank * BT + tid;
  const bool live = a < A;
  const int ac = live ? a : A - 1;
  const Owner own{BT};
  const ClusterLayout<T> L(A, BT, N, S, true);
  const int NP4 = L.NP * 4;
  T* sxy = reinterpret_cast<T*>(smem + L.xy);      // [nbuf][NP*4] whole env
  T4* srec = reinterpret_cast<T4*>(smem + L.rec);  // [nbuf][BT]
  T* sown = reinterpret_cast<T*>(smem + L.own);    // [S][BT][5] th, s, w, x, y
  T4* sfbc = reinterpret_cast<T4*>(smem + L.fbc);  // [2][BT] force cotangent, cutoff
  Obs<T>* sobs = reinterpret_cast<Obs<T>*>(smem + L.obs);

  AgentP<T> P;
  load_params(R, e, ac, P);
  const WorldC<T> W = R.W;
  if (FL & F_OBS) load_obstacles(R, sobs, e);
  if (kColl) init_pads(sxy, L.nbuf, 1, A);
  cl.sync();

  const long long ia = (long long)e * A + ac;
  const long long EA = (long long)R.E * A;
  const int H = R.H;
  const bool has_gt = R.gt_pos || R.gt_th || R.gt_vel || R.gt_s || R.gt_w;
  Agent<T> g{};
  add_cotangent(R.gf_pos, R.gf_th, R.gf_vel, R.gf_s, R.gf_w, ia, g);
  if (R.goal) {
    const T2 pH = reinterpret_cast<const T2*>(R.t_pos)[(long long)(R.H - 1) * R.E * A + ia];
    seed_goal_loss(R, ia, pH.x, pH.y, g);
  }
  const bool pv_only = (FL & F_HOLOVEL) && S == 1;
  auto load_traj = [&](long long i, Agent<T>& x) {
    if (pv_only)
      load_state_pv(R.t_pos, R.t_vel, i, x);
    else
      load_state(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, i, x);
  };
  auto load_init = [&](Agent<T>& x) {
    if (pv_only)
      load_state_pv(R.i_pos, R.i_vel, ia, x);
    else
      load_state(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, x);
  };
  Agent<T> nxt;
  load_traj((long long)(H - 1) * EA + ia, nxt);
  Agent<T> cur;
  T a0, a1;
  if (H > 1)
    load_traj((long long)(H - 2) * EA + ia, cur);
  else
    load_init(cur);
  load_action(R, (long long)(H - 1) * EA + ia, a0, a1);
  int fbuf = 0;
  T gsq = T(0);
  for (int t = H - 1; t >= 0; --t) {
    if (has_gt) add_cotangent(R.gt_pos, R.gt_th, R.gt_vel, R.gt_s, R.gt_w, (long long)t * EA + ia, g);
    Agent<T> pcur{};
    T pa0 = T(0), pa1 = T(0);
    if (t > 0) {
      if (t > 1)
        load_traj((long long)(t - 2) * EA + ia, pcur);
      else
        load_init(pcur);
      load_action(R, (long long)(t - 1) * EA + ia, pa0, pa1);
    }
    T ga0 = T(0), ga1 = T(0);
    if (S == 1) {
      Agent<T> gin;
      T gfx, gfy;
      integrate_vjp_sel<T, FL>(cur, a0, a1, nxt, g, P, W, gin, gfx, gfy, ga0, ga1);
      T* xy_env = sxy + fbuf * NP4;
      T4* rec = srec + fbuf * BT;
      T4* fbc = sfbc + fbuf * BT;
      int cut_a = A;
      if (kColl) {
        if (live) put_xy_all(cl, xy_env, CS, a, cur.px, cur.py);
        rec[tid] = T4{cur.vx, cur.vy, P.radius, P.inv_denom};
        if (FL & F_TRUNC) cut_a = R.cutoff[(long long)t * EA + ia];
        fbc[tid] = T4{gfx, gfy, T(cut_a), T(0)};
        cl.sync();
      }
      if (live)
        force_vjp_cl<T, FL>(cl, own, xy_env, rec, fbc, sobs, N, A, a, cut_a, cur, P, W, gfx, gfy,
                            gin);
      g = gin;
      fbuf ^= 1;
    } else {
      // recompute the substep chain from the checkpointed step input
      if (kColl) cl.sync();  // every peer is done with last step's records
      Agent<T> x = cur;
      for (int k = 0; k < S; ++k) {
        T* xy_env = sxy + k * NP4;
        T4* rec = srec + k * BT;
        if (kColl && live) put_xy_all(cl, xy_env, CS, a, x.px, x.py);
        rec[tid] = T4{x.vx, x.vy, P.radius, P.inv_denom};
        T* ow = sown + (size_t(k) * BT + tid) * 5;
        ow[0] = x.th;
        ow[1] = x.s;
        ow[2] = x.w;
        ow[3] = x.px;
        ow[4] = x.py;
        if (k == S - 1) break;
        T fx = T(0), fy = T(0);
        if (kColl) {
          cl.sync();
          if (live) {
            int cutoff;
            neighbor_force_cl<T, FL>(cl, own, xy_env, rec, A, a, x, P, W, fx, fy, cutoff);
          }
        }
        static_force<T, FL>(sobs, N, x, P, W, fx, fy);
        Agent<T> y;
        integrate_sel<T, FL>(x, a0, a1, fx, fy, P, W, y);
        x = y;
      }
      Agent<T> out = nxt;
      for (int k = S - 1; k >= 0; --k) {
        T* xy_env = sxy + k * NP4;
        T4* rec = srec + k * BT;
        const T* ow = sown + (size_t(k) * BT + tid) * 5;
        const T4 rr = rec[tid];
        const Agent<T> in{ow[3], ow[4], ow[0], rr.x, rr.y, ow[1], ow[2]};
        Agent<T> gin;
        T gfx, gfy;
        integrate_vjp_sel<T, FL>(in, a0, a1, out, g, P, W, gin, gfx, gfy, ga0, ga1);
        T4* fbc = sfbc + fbuf * BT;
        int cut_a = A;
        if (kColl) {
          if (FL & F_TRUNC) cut_a = R.cutoff[((long long)t * S + k) * EA + ia];
          fbc[tid] = T4{gfx, gfy, T(cut_a), T(0)};
          cl.sync();
        }
        if (live)
          force_vjp_cl<T, FL>(cl, own, xy_env, rec, fbc, sobs, N, A, a, cut_a, in, P, W, gfx, gfy,
                              gin);
        g = gin;
        out = in;
        fbuf ^= 1;
      }
    }
    if (live) {
      const long long ja = (long long)t * EA + ia;
      gsq = Num<T>::fma_(ga0, ga0, Num<T>::fma_(ga1, ga1, gsq));
      if (R.act_dim == 2) {
        reinterpret_cast<T2*>(R.g_act)[ja] = T2{ga0, ga1};
      } else {
        R.g_act[ja * R.act_dim] = ga0;
        R.g_act[ja * R.act_dim + 1] = ga1;
        for (int j = 2; j < R.act_dim; ++j) R.g_act[ja * R.act_dim + j] = T(0);
      }
    }
    nxt = cur;
    cur = pcur;
    a0 = pa0;
    a1 = pa1;
  }
  if (live) store_state(R.gi_pos, R.gi_th, R.gi_vel, R.gi_s, R.gi_w, ia, g);
  if (R.gsq_partial) block_sum_store(gsq, R.gsq_partial + blockIdx.x);
  cl.sync();  // no CTA leaves while a peer may still read its records
}

// ============================================================ neighbor lists
// Padded lists of envs wider than one CTA: grid (E x slices); each CTA stages the whole
// env's positions in its shared memory and lists the agents of its slice (no exchange
// between CTAs, so no cluster).
template <typename T>
__global__ void __launch_bounds__(1024) neighbors_wide_kernel(int E, int A, int slices, int K,
                                                              T r2_scan, T r2_thr, const T* pos,
                                                              int* idx, int* count,
                                                              int* true_count) {
  using T2 = typename V2<T>::t;
  extern __shared__ __align__(16) unsigned char smem[];
  T* xy_env = reinterpret_cast<T*>(smem);
  const int e = blockIdx.x / slices, sl = blockIdx.x - e * slices;
  const T2* P = reinterpret_cast<const T2*>(pos) + (long long)e * A;
  for (int j = threadIdx.x; j < A; j += blockDim.x) {
    const T2 p = P[j];
    put_xy(xy_env, j, p.x, p.y);
  }
  if ((A & 1) && threadIdx.x == 0) put_xy(xy_env, A, T(1e30), T(1e30));
  __syncthreads();
  const int a = sl * blockDim.x + threadIdx.x;
  if (a >= A) return;
  const long long ia = (long long)e * A + a;
  T px, py;
  get_xy(xy_env, a, px, py);
  int listed = 0;
  const int total = for_each_in_radius_xy<T>(xy_env, A, a, px, py, r2_scan, r2_thr,
                                             [&](int b, T, T) {
    if (listed < K) idx[ia * K + listed++] = b;
  });
  count[ia] = listed;
  true_count[ia] = total;
}

}  // namespace swarp
