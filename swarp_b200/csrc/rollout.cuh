// Fused multi-step rollout kernels (forward and adjoint) for sm_100a.
//
// Layout: one thread per agent, the agents of G whole envs per CTA (G * A threads),
// so the O(A^2) neighbor pass of an env reads its agents' positions from shared
// memory. Each CTA runs its envs through the whole horizon: the forward kernel keeps
// the state in registers and streams actions in / trajectory out (structure of arrays,
// consecutive threads -> consecutive (env, agent) -> coalesced); the adjoint kernel
// walks the horizon backwards, re-reading each step's input state from the trajectory
// (the checkpoint). Accumulation is a gather in fixed (ascending agent index) order:
// no atomics, bitwise deterministic.
//
// Neighbor pass: positions sit in shared memory packed by agent pairs
// (x_2p, x_2p+1, y_2p, y_2p+1), so one 16-byte load feeds one packed fp32x2
// (FFMA2/FMUL2, sm_100) distance test of two neighbors. The test builds a 32-bit
// membership mask per chunk of 32 agents; only set bits run the contact law.
//
// Contact checkpoint (F_MASK: envs of up to 32 agents, and 2-D disc fleets of up to 256
// agents with or without list truncation): the forward stores per agent and substep the
// mask of the in-radius agents it is in contact with, listed or not, one 32-bit word per
// 32 agents (word-major, [H*S][words][E*A]). Contact is symmetric, so the adjoint runs the
// pair VJPs over exactly those bits, in the rescan's ascending order, and never repeats
// the neighbor scan; with a truncating cap the forward also stores each list's cutoff
// index, which gates each pair's own and cross terms. Otherwise (larger envs, box agents
// or drones beyond one word or with truncation) the adjoint rescans with the cutoffs.
#pragma once
#include "bodies.cuh"
#include "boxes.cuh"
#include "boxes_vjp.cuh"
#include "drone.cuh"
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
  F_COLL = 1,     // agent-agent contacts
  F_TRUNC = 2,    // list cap can truncate (A - 1 > K): cutoffs checkpointed
  F_OBS = 4,      // obstacles present
  F_HOLOVEL = 8,  // every agent is holonomic / VELOCITY
  F_MASK = 16,    // contact masks checkpointed (A <= 32, no truncation)
  F_BODIES = 32,  // movable bodies integrated in the substep loop (with F_OBS)
  F_RK4 = 64,     // classic RK4 integrator instead of semi-implicit Euler
  F_BOXES = 128,  // some agents are oriented boxes (boxes.cuh)
  F_DRONE = 256,  // some agents are 6-DOF drones (drone.cuh)
};

// Largest CTA the 16-agent specializations are launched with (host: envs_per_cta).
constexpr int kMaxThreadsAS16 = 256;
// Launch bound of the small-CTA instances of movable-body worlds (CTAs of at most this many
// threads): their kernels then keep their state in up to 255 registers instead of 64.
// Body worlds are latency-bound (one body thread per env, a few agents), where spilled
// registers cost more than the occupancy the 1024-thread bound buys (measured at
// 4096 envs x 4 agents + one 3-circle body: 2.09 -> 1.84 ms per BPTT step).
constexpr int kSmallCTA = 256;

// The four drone field arrays of one state (null when the world has no drones).
template <typename P> struct DroneF {
  P *z, *vz, *att, *br;
};

template <typename T> struct RolloutArgs {
  int E, A, G, H, S, act_dim, N;
  int CS;  // CTAs per env (cluster kernels, rollout_cluster.cuh); 0 or 1 otherwise
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
  int16_t* cutoff;   // workspace [H*S, E, A] (F_TRUNC)
  uint32_t* cmask;   // workspace [H*S, NW, E*A], NW = ceil(A / 32) (F_MASK)
  // adjoint
  const T *gt_pos, *gt_th, *gt_vel, *gt_s, *gt_w;  // cotangent of trajectory (nullable)
  const T *gf_pos, *gf_th, *gf_vel, *gf_s, *gf_w;  // cotangent of final (nullable)
  T* g_act;
  T *gi_pos, *gi_th, *gi_vel, *gi_s, *gi_w;
  // optional fused epilogue: per-CTA partial sums of g_act^2 (workspace [gridDim.x]) and
  // the reduced total (one scalar); both null when the norm is not requested
  T* gsq_partial;
  T* gsq_out;
  // optional fused goal loss: goal [E, A, 2]; forward: per-CTA partials (workspace) and the
  // reduced scalar; adjoint: the scalar cotangent of the loss (all null without a goal)
  const T* goal;
  T* loss_partial;
  T* loss_out;
  const T* loss_grad;
  // movable bodies (F_BODIES): per-shape constants, state per shape slot [E, N] at t = 0
  // and after every step [H, E, N], cotangent of the final body state (nullable)
  const int *o_kind, *o_body;
  const T *o_mass, *o_inertia, *o_body_off;
  const T *bi_pos, *bi_ang, *bi_vel, *bi_om;
  T *bt_pos, *bt_ang, *bt_vel, *bt_om;
  const T *gb_pos, *gb_ang, *gb_vel, *gb_om;
  int body_clamp;
  int poses_from_bodies;
  // drone fields (F_DRONE): z, vz [.., E, A], attitude [.., E, A, 4], body rates [.., E, A, 3]
  // of the init, trajectory, final, their cotangents and the init cotangent
  DroneF<const T> i_d;
  DroneF<T> t_d, f_d;
  DroneF<const T> gt_d, gf_d;
  DroneF<T> gi_d;
};

// Shared-memory carve-up, identical on host (sizes) and device (pointers).
template <typename T> struct Layout {
  int G, A, NP, nbuf, S;
  size_t xy, rec, own, fb, cut, rad, iden, obs, bc, bst, gpose, gag, gbody, gbnew, gshape, thw, shp,
      dro, total;
  __host__ __device__ Layout(int G_, int A_, int N, int S_, bool bwd, bool bodies = false,
                             bool boxes = false, bool drone = false)
      : G(G_), A(A_), S(S_) {
    NP = (A + 1) / 2;
    nbuf = bwd ? (S > 2 ? S : 2) : 2;
    const int GA = G * A;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = (off + bytes + 15) & ~size_t(15); return o; };
    xy = take(size_t(nbuf) * G * NP * 4 * sizeof(T));   // scan table (pair-packed x, y)
    rec = take(size_t(nbuf) * GA * 4 * sizeof(T));      // per-agent (x, y, vx, vy) records
    own = bwd ? take(size_t(S) * GA * 4 * sizeof(T)) : 0;
    fb = bwd ? take(size_t(2) * GA * 2 * sizeof(T)) : 0;
    cut = bwd ? take(size_t(2) * GA * sizeof(int)) : 0;
    rad = take(size_t(GA) * sizeof(T));
    iden = take(size_t(GA) * sizeof(T));
    obs = take(size_t(G) * (N > 0 ? N : 0) * sizeof(Obs<T>));
    const int NB = bodies ? N : 0;
    bc = take(size_t(NB) * sizeof(BodyC<T>));
    bst = take(size_t(bwd ? S : 1) * G * NB * sizeof(BodyS<T>));  // body states (per substep)
    gpose = bwd ? take(size_t(GA) * NB * 4 * sizeof(T)) : 0;       // agent -> shape pose cot.
    gag = bwd ? take(size_t(bodies ? GA : 0) * 4 * sizeof(T)) : 0;   // body -> agent cot.
    gbody = bwd ? take(size_t(G) * NB * sizeof(BodyG<T>)) : 0;
    gbnew = bwd ? take(size_t(G) * NB * sizeof(BodyG<T>)) : 0;
    gshape = bwd ? take(size_t(G) * NB * 4 * sizeof(T)) : 0;
    // box worlds: every agent's (heading, turn rate) per buffer and (box, hx, hy) once
    thw = boxes ? take(size_t(nbuf) * GA * 2 * sizeof(T)) : 0;
    shp = boxes ? take(size_t(GA) * 4 * sizeof(T)) : 0;
    // drone worlds, adjoint: every substep's drone state of the recomputed chain
    dro = (bwd && drone) ? take(size_t(S) * GA * sizeof(Drone<T>)) : 0;
    total = off;
  }
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
  P.inv_denom = T(1) / (T(1) + R.W.c * R.W.dt / P.mass);
  P.box = row[17] > T(0.5);
  P.hx = row[18];
  P.hy = row[19];
  P.tmax = row[9];
  P.arm = row[10];
  P.ixx = row[11];
  P.iyy = row[12];
  P.izz = row[13];
  P.kappa = row[14];
  P.grav = row[15];
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

// Position and velocity only (heading, speed and turn rate read as 0): what the adjoint of
// a holonomic velocity-controlled step reads of its input and output states.
template <typename T>
__device__ __forceinline__ void load_state_pv(const T* pos, const T* vel, long long i, Agent<T>& x) {
  using T2 = typename V2<T>::t;
  const T2 p = reinterpret_cast<const T2*>(pos)[i];
  const T2 v = reinterpret_cast<const T2*>(vel)[i];
  x = Agent<T>{p.x, p.y, T(0), v.x, v.y, T(0), T(0)};
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

// Action slots 2 and 3 (a drone's rotors 2, 3); zero past act_dim (kernels.py:797-810).
template <typename T>
__device__ __forceinline__ void load_action23(const RolloutArgs<T>& R, long long i, T& a2, T& a3) {
  a2 = R.act_dim > 2 ? R.act[i * R.act_dim + 2] : T(0);
  a3 = R.act_dim > 3 ? R.act[i * R.act_dim + 3] : T(0);
}

template <typename T>
__device__ __forceinline__ void load_drone(const DroneF<const T>& F, long long i, Drone<T>& d) {
  d.z = F.z[i];
  d.vz = F.vz[i];
  d.qx = F.att[4 * i];
  d.qy = F.att[4 * i + 1];
  d.qz = F.att[4 * i + 2];
  d.qw = F.att[4 * i + 3];
  d.bx = F.br[3 * i];
  d.by = F.br[3 * i + 1];
  d.bz = F.br[3 * i + 2];
}
template <typename T>
__device__ __forceinline__ void load_drone(const DroneF<T>& F, long long i, Drone<T>& d) {
  load_drone(DroneF<const T>{F.z, F.vz, F.att, F.br}, i, d);
}
template <typename T>
__device__ __forceinline__ void store_drone(const DroneF<T>& F, long long i, const Drone<T>& d) {
  F.z[i] = d.z;
  F.vz[i] = d.vz;
  F.att[4 * i] = d.qx;
  F.att[4 * i + 1] = d.qy;
  F.att[4 * i + 2] = d.qz;
  F.att[4 * i + 3] = d.qw;
  F.br[3 * i] = d.bx;
  F.br[3 * i + 1] = d.by;
  F.br[3 * i + 2] = d.bz;
}
// Cotangent fields may be absent (NULL = zero), each array on its own.
template <typename T>
__device__ __forceinline__ void add_drone_cotangent(const DroneF<const T>& F, long long i,
                                                    Drone<T>& g) {
  if (F.z) g.z += F.z[i];
  if (F.vz) g.vz += F.vz[i];
  if (F.att) {
    g.qx += F.att[4 * i];
    g.qy += F.att[4 * i + 1];
    g.qz += F.att[4 * i + 2];
    g.qw += F.att[4 * i + 3];
  }
  if (F.br) {
    g.bx += F.br[3 * i];
    g.by += F.br[3 * i + 1];
    g.bz += F.br[3 * i + 2];
  }
}

// One obstacle's installed pose and constants (angle -> cos, sin once).
template <typename T>
__device__ __forceinline__ Obs<T> make_obs(const RolloutArgs<T>& R, int e, int o) {
  const long long eo = (long long)e * R.N + o;
  Obs<T> ob;
  ob.cx = R.o_pos[2 * eo];
  ob.cy = R.o_pos[2 * eo + 1];
  const T ang = R.o_angle[eo];
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
  return ob;
}

// Obstacles of this CTA's envs into shared memory (the agent pass re-reads them every
// substep).
template <typename T>
__device__ __forceinline__ void load_obstacles(const RolloutArgs<T>& R, Obs<T>* sobs, int e0) {
  const int total = R.G * R.N;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int le = i / R.N, o = i - le * R.N;
    sobs[i] = make_obs(R, min(e0 + le, R.E - 1), o);
  }
}

// ------------------------------------------------------------- movable bodies
template <typename T>
__device__ __forceinline__ void load_body_consts(const RolloutArgs<T>& R, BodyC<T>* sbc) {
  for (int i = threadIdx.x; i < R.N; i += blockDim.x) {
    BodyC<T> c;
    c.offx = R.o_body_off[2 * i];
    c.offy = R.o_body_off[2 * i + 1];
    c.mass = R.o_mass[i];
    c.inertia = R.o_inertia[i];
    c.kind = R.o_kind[i];
    c.body = R.o_body[i];
    c.reach = shape_reach(R.o_shape[i], c.offx, c.offy, R.o_radius[i], R.o_half[2 * i],
                          R.o_half[2 * i + 1]);
    sbc[i] = c;
  }
}

template <typename T>
__device__ __forceinline__ bool moving_shape(const BodyC<T>* bc, int s) {
  return bc[bc[s].body].kind == 1;
}
template <typename T>
__device__ __forceinline__ bool moving_root(const BodyC<T>* bc, int o) {
  return bc[o].body == o && bc[o].kind == 1;
}

// Body state of one env's N shape slots from [.., E, N] arrays at element base (e*N).
template <typename T>
__device__ __forceinline__ void load_bodies(const T* pos, const T* ang, const T* vel, const T* om,
                                            long long base, int N, BodyS<T>* dst) {
  for (int o = 0; o < N; ++o) {
    const long long i = base + o;
    dst[o] = BodyS<T>{pos[2 * i], pos[2 * i + 1], ang[i], vel[2 * i], vel[2 * i + 1], om[i]};
  }
}
template <typename T>
__device__ __forceinline__ void store_bodies(T* pos, T* ang, T* vel, T* om, long long base, int N,
                                             const BodyS<T>* src) {
  for (int o = 0; o < N; ++o) {
    const long long i = base + o;
    const BodyS<T> b = src[o];
    pos[2 * i] = b.qx;
    pos[2 * i + 1] = b.qy;
    ang[i] = b.th;
    vel[2 * i] = b.vx;
    vel[2 * i + 1] = b.vy;
    om[i] = b.om;
  }
}

// One substep of every moving body of an env (one thread): reads states `in`, the
// shapes' current poses and the agents' records; writes states `out` (may alias `in`)
// and re-places the moving shapes in `obs`.
template <typename T, typename T4>
__device__ __forceinline__ void bodies_step(const BodyS<T>* in, BodyS<T>* out, const BodyC<T>* bc,
                                            Obs<T>* obs, int N, const T4* rec, const T* rad,
                                            const T* iden, int A, const WorldC<T>& W, bool clamp,
                                            const T* thw = nullptr, const T* shp = nullptr) {
  for (int o = 0; o < N; ++o) {
    if (!moving_root(bc, o)) {
      if (out != in) out[o] = in[o];
      continue;
    }
    BodyPassOut<T> P;
    body_pass_root(o, in[o], bc, obs, N, rec, rad, iden, A, W, clamp, P, thw, shp);
    out[o] = P.next;
  }
  for (int s = 0; s < N; ++s)
    if (moving_shape(bc, s)) place_shape(out[bc[s].body], bc[s], obs[s]);
}

// Shape poses of substep input states `st`: the installed poses at the very first
// substep of the rollout, else placed from the body states.
template <typename T>
__device__ __forceinline__ void set_body_poses(const RolloutArgs<T>& R, int e, bool installed,
                                               const BodyS<T>* st, const BodyC<T>* bc, Obs<T>* obs) {
  for (int s = 0; s < R.N; ++s) {
    if (!moving_shape(bc, s)) continue;
    if (installed)
      obs[s] = make_obs(R, e, s);
    else
      place_shape(st[bc[s].body], bc[s], obs[s]);
  }
}

// ------------------------------------------------------- packed position table
// Agent j of an env sits at xy[(j/2)*4 + j%2] (x) and xy[(j/2)*4 + 2 + j%2] (y).
template <typename T> __device__ __forceinline__ int xslot(int j) { return (j >> 1) * 4 + (j & 1); }

template <typename T>
__device__ __forceinline__ void put_xy(T* xy_env, int j, T x, T y) {
  xy_env[xslot<T>(j)] = x;
  xy_env[xslot<T>(j) + 2] = y;
}
template <typename T>
__device__ __forceinline__ void get_xy(const T* xy_env, int j, T& x, T& y) {
  x = xy_env[xslot<T>(j)];
  y = xy_env[xslot<T>(j) + 2];
}

// Candidate mask of agents [32c, 32c + 32) of one env near (px, py) (self not removed):
// bit j is the sign of dx^2 + (dy^2 - thr), two fused roundings, shifted in with one
// funnel shift per neighbor, neighbors visited in descending index. Called with the
// widened threshold W.r2_scan, the mask is a superset of the exact in-radius set (see
// in_radius); callers drop the few extra bits. AS > 0: the env has exactly AS agents
// (compile-time).
template <int AS>
__device__ __forceinline__ unsigned scan_chunk(const float* xy_env, int c, int npairs, float px,
                                               float py, float thr) {
  const float4* P = reinterpret_cast<const float4*>(xy_env) + c * 16;
  const float2 PX = make_float2(px, px), PY = make_float2(py, py), M1 = make_float2(-1.f, -1.f);
  const float2 NT = make_float2(-thr, -thr);
  unsigned m = 0u;
  auto visit = [&](int p) {
    const float4 q = P[p];
    const float2 dx = __ffma2_rn(make_float2(q.x, q.y), M1, PX);
    const float2 dy = __ffma2_rn(make_float2(q.z, q.w), M1, PY);
    const float2 d = __ffma2_rn(dx, dx, __ffma2_rn(dy, dy, NT));
    m = __funnelshift_l(__float_as_uint(d.y), m, 1);
    m = __funnelshift_l(__float_as_uint(d.x), m, 1);
  };
  if constexpr (AS > 0) {
    constexpr int NPC = (AS + 1) / 2 < 16 ? (AS + 1) / 2 : 16;
#pragma unroll
    for (int p = NPC - 1; p >= 0; --p) visit(p);
  } else {
    // only the chunk's real pairs (a predicated 16-pair unroll would issue all 16)
#pragma unroll 4
    for (int p = npairs - 1; p >= 0; --p) visit(p);
  }
  return m;
}
template <int AS>
__device__ __forceinline__ unsigned scan_chunk(const double* xy_env, int c, int npairs, double px,
                                               double py, double thr) {
  unsigned m = 0u;
  const int NPC = AS > 0 ? ((AS + 1) / 2 < 16 ? (AS + 1) / 2 : 16) : npairs;
#pragma unroll 4
  for (int p = NPC - 1; p >= 0; --p) {
    const double* q = xy_env + (c * 16 + p) * 4;
    const double dx1 = px - q[1], dy1 = py - q[3];
    const double dx0 = px - q[0], dy0 = py - q[2];
    m = (m << 1) | (__fma_rn(dx1, dx1, __fma_rn(dy1, dy1, -thr)) < 0.0 ? 1u : 0u);
    m = (m << 1) | (__fma_rn(dx0, dx0, __fma_rn(dy0, dy0, -thr)) < 0.0 ? 1u : 0u);
  }
  return m;
}

// Calls fn(b, q) for every agent b != a of the env within the neighbor radius, ascending
// b, with q = b's (x, y, vx, vy) record. Returns the count of such agents. thr_scan is
// the scan's widened threshold, thr the exact one (in_radius).
struct NoChunkEnd {
  __device__ __forceinline__ void operator()(int) const {}
};
template <typename T, int AS, typename Fn, typename EndFn = NoChunkEnd>
__device__ __forceinline__ int for_each_in_radius(const T* xy_env, const typename V4<T>::t* rec_env,
                                                  int A, int a, T px, T py, T thr_scan, T thr,
                                                  Fn&& fn, EndFn&& chunk_end = EndFn{}) {
  const int NP = (A + 1) / 2;
  int total = 0;
  const int nchunk = AS > 0 ? (AS + 31) / 32 : (A + 31) / 32;
  for (int c = 0; c < nchunk; ++c) {
    const int npairs = min(16, NP - c * 16);
    unsigned m = scan_chunk<AS>(xy_env, c, npairs, px, py, thr_scan);
    const int rel = a - 32 * c;
    if (rel >= 0 && rel < 32) m &= ~(1u << rel);
    while (m) {
      const int jj = __ffs(m) - 1;
      m &= m - 1u;
      const int b = 32 * c + jj;
      const auto q = rec_env[b];
      if (!in_radius(px - q.x, py - q.y, thr)) continue;
      ++total;
      fn(b, q);
    }
    chunk_end(c);  // after the chunk's members (every thread of the env reaches it)
  }
  return total;
}

// Contact force on agent a from its capped neighbor list (the first K within R by index).
// Returns the uncapped count; cutoff = index of the K-th listed neighbor if truncated,
// else A. With contact masks (F_MASK; mout non-null) it also writes the env's contact mask
// of agent a, one 32-bit word per 32 agents (word c at mout[c * mstride]): bit b for every
// agent b within the radius that a is in contact with, listed or not (pair contact is
// symmetric, so the adjoint can gather each pair from either side without a rescan).
template <typename T, int FL, int AS>
__device__ __forceinline__ int neighbor_force(const T* xy_env, const typename V4<T>::t* rec_env,
                                              const T* rad_env, int A, int a, const Agent<T>& x,
                                              const AgentP<T>& P, const WorldC<T>& W, T& fx, T& fy,
                                              int& cutoff, uint32_t* mout = nullptr,
                                              long long mstride = 0) {
  int listed = 0;
  cutoff = A;
  unsigned word = 0u;  // contacts of the current chunk of 32 agents
  const int total = for_each_in_radius<T, AS>(
      xy_env, rec_env, A, a, x.px, x.py, W.r2_scan, W.r2_thr,
      [&](int b, const typename V4<T>::t& q) {
        bool listed_b = true;
        if (FL & F_TRUNC) {
          if (listed >= W.K) {
            listed_b = false;
          } else {
            ++listed;
            if (listed == W.K) cutoff = b;
          }
        }
        if (!(FL & F_MASK) && !listed_b) return;
        const T dx = x.px - q.x, dy = x.py - q.y;
        const T md = P.radius + rad_env[b] + W.margin;
        const bool contact = listed_b ? pair_force_add(dx, dy, dot2(dx, dy, dx, dy), x.vx - q.z,
                                                       x.vy - q.w, md, P.inv_denom, W, fx, fy)
                                      : pair_in_contact(dx, dy, md);
        if ((FL & F_MASK) && contact) word |= 1u << (b & 31);
      },
      [&](int c) {
        if (FL & F_MASK) {
          if (mout) mout[c * mstride] = word;
          word = 0u;
        }
      });
  if ((FL & F_TRUNC) && total <= W.K) cutoff = A;
  return total;
}

// Box worlds: the agent's pose as an oriented box (heading th, turn rate w).
template <typename T>
__device__ __forceinline__ Ob<T> ob_of(T px, T py, T th, T vx, T vy, T w, T hx, T hy) {
  return Ob<T>{px, py, Num<T>::cos_(th), Num<T>::sin_(th), hx, hy, vx, vy, w};
}

// neighbor_force for worlds with box agents: the same capped list, each pair through the
// shape dispatch (disc-disc, disc-box, box-box). thw_env holds every agent's (th, w) of
// the substep, shp_env its (box, hx, hy).
template <typename T, int FL, int AS>
__device__ __forceinline__ int neighbor_force_box(const T* xy_env, const typename V4<T>::t* rec_env,
                                                  const typename V2<T>::t* thw_env,
                                                  const typename V4<T>::t* shp_env,
                                                  const T* rad_env, int A, int a, const Agent<T>& x,
                                                  const AgentP<T>& P, const WorldC<T>& W, T& fx,
                                                  T& fy, int& cutoff, unsigned& cmask) {
  int listed = 0;
  cutoff = A;
  cmask = 0u;
  const Ob<T> oa = ob_of(x.px, x.py, x.th, x.vx, x.vy, x.w, P.hx, P.hy);
  const bool box_a = P.box != 0;
  const int total = for_each_in_radius<T, AS>(xy_env, rec_env, A, a, x.px, x.py, W.r2_scan, W.r2_thr,
                                              [&](int b, const typename V4<T>::t& q) {
    if (FL & F_TRUNC) {
      if (listed >= W.K) return;
      ++listed;
      if (listed == W.K) cutoff = b;
    }
    const auto tw = thw_env[b];
    const auto sh = shp_env[b];
    const Ob<T> ob = ob_of(q.x, q.y, tw.x, q.z, q.w, tw.y, sh.y, sh.z);
    if (pair_force_shaped(a, b, box_a, oa, P.radius, sh.x > T(0.5), ob, rad_env[b], P.inv_denom,
                          W, fx, fy))
      cmask |= 1u << (b & 31);
  });
  if ((FL & F_TRUNC) && total <= W.K) cutoff = A;
  return total;
}

// Contact force from the checkpointed contact mask words mw[c * mstride] (c < NW), the
// forward's sum: ascending b, only neighbors on the agent's list (b <= cut_a with list
// truncation).
template <typename T, int FL>
__device__ __forceinline__ void mask_force_w(const typename V4<T>::t* rec_env, const T* rad_env,
                                             const uint32_t* mw, long long mstride, int NW,
                                             int cut_a, const Agent<T>& x, const AgentP<T>& P,
                                             const WorldC<T>& W, T& fx, T& fy) {
  for (int c = 0; c < NW; ++c) {
    unsigned m = mw[c * mstride];
    while (m) {
      const int b = 32 * c + __ffs(m) - 1;
      m &= m - 1u;
      if ((FL & F_TRUNC) && b > cut_a) {  // ascending: the rest are past the list
        c = NW;
        break;
      }
      const auto q = rec_env[b];
      const T dx = x.px - q.x, dy = x.py - q.y;
      pair_force_add(dx, dy, dot2(dx, dy, dx, dy), x.vx - q.z, x.vy - q.w,
                     P.radius + rad_env[b] + W.margin, P.inv_denom, W, fx, fy);
    }
  }
}

// Contact force from a checkpointed contact mask (ascending b, the forward's order).
template <typename T>
__device__ __forceinline__ void mask_force(const typename V4<T>::t* rec_env, const T* rad_env,
                                           unsigned m, const Agent<T>& x, const AgentP<T>& P,
                                           const WorldC<T>& W, T& fx, T& fy) {
  while (m) {
    const int b = __ffs(m) - 1;
    m &= m - 1u;
    const auto q = rec_env[b];
    const T dx = x.px - q.x, dy = x.py - q.y;
    pair_force_add(dx, dy, dot2(dx, dy, dx, dy), x.vx - q.z, x.vy - q.w,
                   P.radius + rad_env[b] + W.margin, P.inv_denom, W, fx, fy);
  }
}

// mask_force for worlds with box agents (pair_force_shaped on every listed contact).
template <typename T>
__device__ __forceinline__ void mask_force_box(const typename V4<T>::t* rec_env,
                                               const typename V2<T>::t* thw_env,
                                               const typename V4<T>::t* shp_env, const T* rad_env,
                                               unsigned m, int a, const Agent<T>& x,
                                               const AgentP<T>& P, const WorldC<T>& W, T& fx,
                                               T& fy) {
  const Ob<T> oa = ob_of(x.px, x.py, x.th, x.vx, x.vy, x.w, P.hx, P.hy);
  while (m) {
    const int b = __ffs(m) - 1;
    m &= m - 1u;
    const auto q = rec_env[b];
    const auto tw = thw_env[b];
    const auto sh = shp_env[b];
    const Ob<T> ob = ob_of(q.x, q.y, tw.x, q.z, q.w, tw.y, sh.y, sh.z);
    pair_force_shaped(a, b, P.box != 0, oa, P.radius, sh.x > T(0.5), ob, rad_env[b], P.inv_denom,
                      W, fx, fy);
  }
}

template <typename T, int FL>
__device__ __forceinline__ void static_force(const Obs<T>* sobs, int N, const Agent<T>& x,
                                             const AgentP<T>& P, const WorldC<T>& W, T& fx, T& fy) {
  if ((FL & F_BOXES) && P.box) {  // collisions.py:951-994: the oriented static forces
    box_static_force((FL & F_OBS) ? sobs : nullptr, (FL & F_OBS) ? N : 0,
                     W.bounds_mode == BOUNDS_SOFT,
                     ob_of(x.px, x.py, x.th, x.vx, x.vy, x.w, P.hx, P.hy), P.inv_denom, W, fx, fy);
    return;
  }
  T sx = T(0), sy = T(0);
  if (FL & F_OBS) {
    for (int o = 0; o < N; ++o) {
      T gx, gy;
      obstacle_force(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, sobs[o], W, gx, gy);
      sx = sx + gx;
      sy = sy + gy;
    }
  }
  if (W.bounds_mode == BOUNDS_SOFT) {
    T wx, wy;
    wall_force(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, W, wx, wy);
    sx = sx + wx;
    sy = sy + wy;
  }
  fx = fx + sx;
  fy = fy + sy;
}

template <typename T, int FL>
__device__ __forceinline__ void integrate_sel(const Agent<T>& in, T a0, T a1, T fx, T fy,
                                              const AgentP<T>& P, const WorldC<T>& W, Agent<T>& out) {
  AgentP<T> Q = P;
  if (FL & F_HOLOVEL) {
    Q.tag = TAG_HOLONOMIC;
    Q.mode = MODE_VELOCITY;
  }
  constexpr bool kBox = (FL & F_BOXES) != 0;
  if (FL & F_RK4)
    integrate_rk4_fwd<T, kBox>(in, a0, a1, fx, fy, Q, W, out);
  else
    integrate_fwd<T, kBox>(in, a0, a1, fx, fy, Q, W, out);
}

template <typename T, int FL>
__device__ __forceinline__ void integrate_vjp_sel(const Agent<T>& in, T a0, T a1, const Agent<T>& out,
                                                  const Agent<T>& g, const AgentP<T>& P,
                                                  const WorldC<T>& W, Agent<T>& gin, T& gfx, T& gfy,
                                                  T& ga0, T& ga1) {
  AgentP<T> Q = P;
  if (FL & F_HOLOVEL) {
    Q.tag = TAG_HOLONOMIC;
    Q.mode = MODE_VELOCITY;
  }
  constexpr bool kBox = (FL & F_BOXES) != 0;
  if (FL & F_RK4)
    integrate_rk4_vjp<T, kBox>(in, a0, a1, out, g, Q, W, gin, gfx, gfy, ga0, ga1);
  else
    integrate_vjp<T, kBox>(in, a0, a1, out, g, Q, W, gin, gfx, gfy, ga0, ga1);
}

// Drone worlds: a drone agent takes the 6-DOF substep (rotor slots a0..a3, the servo
// rewrite of slots 0/1 first, as the reference's kernels apply it to every SERVO agent),
// every other agent its 2-D model with the drone fields passed through.
template <typename T, int FL>
__device__ __forceinline__ void integrate_drone_sel(const Agent<T>& in, const Drone<T>& d, T a0,
                                                    T a1, T a2, T a3, T fx, T fy,
                                                    const AgentP<T>& P, const WorldC<T>& W,
                                                    Agent<T>& out, Drone<T>& dout) {
  if (P.tag != TAG_DRONE) {
    integrate_sel<T, FL>(in, a0, a1, fx, fy, P, W, out);
    dout = d;
    return;
  }
  T a[4] = {a0, a1, a2, a3};
  if (P.mode == MODE_SERVO) servo_cmd(a0, a1, in.s, in.w, P, W.dt, a[0], a[1]);
  if (FL & F_RK4)
    drone_rk4_fwd(in, d, a, fx, fy, P, W, out, dout);
  else
    drone_euler_fwd(in, d, a, fx, fy, P, W, out, dout);
}

// Adjoint of integrate_drone_sel; same contract as integrate_vjp_sel, plus the drone
// fields' cotangents (gd in, gdin out) and the action slots 2, 3 (ga2, ga3 added).
template <typename T, int FL>
__device__ __forceinline__ void integrate_vjp_drone_sel(const Agent<T>& in, const Drone<T>& d,
                                                        T a0, T a1, T a2, T a3,
                                                        const Agent<T>& out, const Agent<T>& g,
                                                        const Drone<T>& gd, const AgentP<T>& P,
                                                        const WorldC<T>& W, Agent<T>& gin,
                                                        Drone<T>& gdin, T& gfx, T& gfy, T& ga0,
                                                        T& ga1, T& ga2, T& ga3) {
  if (P.tag != TAG_DRONE) {
    integrate_vjp_sel<T, FL>(in, a0, a1, out, g, P, W, gin, gfx, gfy, ga0, ga1);
    gdin = gd;
    return;
  }
  T ac[4] = {a0, a1, a2, a3};
  const bool servo = P.mode == MODE_SERVO;
  if (servo) servo_cmd(a0, a1, in.s, in.w, P, W.dt, ac[0], ac[1]);
  T gac[4] = {T(0), T(0), T(0), T(0)};
  gfx = T(0);
  gfy = T(0);
  if (FL & F_RK4)
    drone_rk4_vjp(in, d, ac, out, g, gd, P, W, gin, gdin, gfx, gfy, gac);
  else
    drone_euler_vjp(in, d, ac, out, g, gd, P, W, gin, gdin, gfx, gfy, gac);
  if (servo) {
    servo_cmd_vjp(a0, a1, in.s, in.w, P, W.dt, gac[0], gac[1], ga0, ga1, gin.s, gin.w);
  } else {
    ga0 += gac[0];
    ga1 += gac[1];
  }
  ga2 += gac[2];
  ga3 += gac[3];
}

// Pad slot of an odd-sized env: never within any radius.
template <typename T>
__device__ __forceinline__ void init_pads(T* xy, int nbuf, int G, int A) {
  if ((A & 1) == 0) return;
  const int NP = (A + 1) / 2;
  for (int i = threadIdx.x; i < nbuf * G; i += blockDim.x) {
    T* env = xy + size_t(i) * NP * 4;
    put_xy(env, A, T(1e30), T(1e30));
  }
}

// Deterministic CTA sum (fixed shuffle tree, then warp sums in warp order) stored by
// thread 0. Every thread of the block must call it. A partial warp (a CTA size that is
// not a multiple of 32) may not shuffle over its missing lanes: it gathers its lanes' values
// in lane order instead.
template <typename T>
__device__ __forceinline__ void block_sum_store(T v, T* out) {
  __shared__ T warp_sums[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int in_warp = min(32, (int)blockDim.x - wid * 32);  // this warp's threads
  if (in_warp < 32) {
    const unsigned mask = (1u << in_warp) - 1u;
    __syncwarp(mask);
    T s = T(0);
    for (int i = 0; i < in_warp; ++i) s += __shfl_sync(mask, v, i);
    v = s;
  } else {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  if (lane == 0) warp_sums[wid] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    T s = T(0);
    const int nw = (blockDim.x + 31) >> 5;
    for (int i = 0; i < nw; ++i) s += warp_sums[i];
    *out = s;
  }
}

// The fused goal loss (swarp_goal_loss_t): one agent's |pos_T - goal|^2, and the seed of
// its cotangent, loss_grad * 2 (pos_T - goal), added to the final-position cotangent.
template <typename T>
__device__ __forceinline__ T goal_dist2(const T* goal, long long i, T px, T py) {
  const T dx = px - goal[2 * i], dy = py - goal[2 * i + 1];
  return Num<T>::fma_(dx, dx, dy * dy);
}
template <typename T>
__device__ __forceinline__ void seed_goal_loss(const RolloutArgs<T>& R, long long i, T px, T py,
                                               Agent<T>& g) {
  const T s = T(2) * R.loss_grad[0];
  g.px = Num<T>::fma_(s, px - R.goal[2 * i], g.px);
  g.py = Num<T>::fma_(s, py - R.goal[2 * i + 1], g.py);
}

// ================================================================== forward
template <typename T, int FL, int AS, int LB = 1024>
__global__ void __launch_bounds__(LB) rollout_fwd_kernel(const RolloutArgs<T> R) {
  using T4 = typename V4<T>::t;
  constexpr bool kBodies = (FL & F_BODIES) != 0;
  constexpr bool kShare = (FL & (F_COLL | F_BODIES)) != 0;  // agent records in smem each substep
  constexpr bool kBoxes = (FL & F_BOXES) != 0 && (FL & F_COLL) != 0;  // shapes meet in pairs
  // box agents' (heading, turn rate) and (box, hx, hy) tables: for agent pairs, and for the
  // reactions of box agents on movable bodies
  constexpr bool kBoxTab = (FL & F_BOXES) != 0 && (FL & (F_COLL | F_BODIES)) != 0;
  using T2 = typename V2<T>::t;
  extern __shared__ __align__(16) unsigned char smem[];
  const int A = AS > 0 ? AS : R.A;
  const int G = R.G, GA = G * A, N = R.N;
  const int tid = threadIdx.x;
  const int le = tid / A, a = tid - le * A;
  const int e0 = blockIdx.x * G;
  const int e = e0 + le;
  const bool valid = e < R.E;
  const int ec = valid ? e : R.E - 1;
  const Layout<T> L(G, A, N, R.S, false, kBodies, kBoxTab);
  const int NP4 = L.NP * 4;
  T2* sthw = reinterpret_cast<T2*>(smem + L.thw);  // [2][G*A] (th, w), box worlds
  T4* sshp = reinterpret_cast<T4*>(smem + L.shp);  // [G*A] (box, hx, hy, -)
  T* sxy = reinterpret_cast<T*>(smem + L.xy);
  T4* srec = reinterpret_cast<T4*>(smem + L.rec);
  T* srad = reinterpret_cast<T*>(smem + L.rad);
  T* siden = reinterpret_cast<T*>(smem + L.iden);
  Obs<T>* sobs = reinterpret_cast<Obs<T>*>(smem + L.obs);
  BodyC<T>* sbc = reinterpret_cast<BodyC<T>*>(smem + L.bc);
  BodyS<T>* sbst = reinterpret_cast<BodyS<T>*>(smem + L.bst);  // [G][N]

  AgentP<T> P;
  load_params(R, ec, a, P);
  const WorldC<T> W = R.W;
  srad[tid] = P.radius;
  siden[tid] = P.inv_denom;
  if (kBoxTab) sshp[tid] = T4{P.box ? T(1) : T(0), P.hx, P.hy, T(0)};
  if (FL & F_OBS) load_obstacles(R, sobs, e0);
  if (FL & F_COLL) init_pads(sxy, 2, G, A);
  if (kBodies) {
    load_body_consts(R, sbc);
    if (a == 0) load_bodies(R.bi_pos, R.bi_ang, R.bi_vel, R.bi_om, (long long)ec * N, N, sbst + le * N);
  }
  __syncthreads();
  if (kBodies && R.poses_from_bodies && a == 0)
    set_body_poses(R, ec, false, sbst + le * N, sbc, sobs + le * N);
  __syncthreads();

  const T2* thw_env0 = sthw + le * A;
  const T4* shp_env = sshp + le * A;
  const long long ia = (long long)ec * A + a;
  const long long EA = (long long)R.E * A;
  const int NW = (A + 31) >> 5;  // contact-mask words per agent and substep
  Agent<T> x;
  load_state(R.i_pos, R.i_th, R.i_vel, R.i_s, R.i_w, ia, x);
  constexpr bool kDrone = (FL & F_DRONE) != 0;
  Drone<T> xd{};
  if (kDrone) load_drone(R.i_d, ia, xd);
  int tmax = 0;
  int buf = 0;
  T a0, a1, n0 = T(0), n1 = T(0);
  T a2 = T(0), a3 = T(0), n2 = T(0), n3 = T(0);  // drone rotor slots
  load_action(R, ia, a0, a1);
  if (kDrone) load_action23(R, ia, a2, a3);
  const T* rad_env = srad + le * A;
  const T* iden_env = siden + le * A;
  Obs<T>* obs_env = sobs + le * N;
  // unrolled: the step's state and prefetched action rotate through registers instead of
  // being copied at the end of each step (measured: 223.6 -> 203.1 us at 16000 x 16 x 64);
  // not for box and drone worlds, whose larger step body would then thrash the
  // instruction cache (measured: ~77% of issue slots lost to instruction fetch)
  constexpr int kUnrollT = (FL & (F_BOXES | F_DRONE)) ? 1 : 4;
#pragma unroll kUnrollT
  for (int t = 0; t < R.H; ++t) {
    if (t + 1 < R.H) load_action(R, (long long)(t + 1) * EA + ia, n0, n1);
    if (kDrone && t + 1 < R.H) load_action23(R, (long long)(t + 1) * EA + ia, n2, n3);
    for (int k = 0; k < R.S; ++k) {
      T fx = T(0), fy = T(0);
      T* xy_env = sxy + (buf * G + le) * NP4;
      T4* rec_env = srec + buf * GA + le * A;
      if (kShare) {
        if (FL & F_COLL) put_xy(xy_env, a, x.px, x.py);
        rec_env[a] = T4{x.px, x.py, x.vx, x.vy};
        if (kBoxTab) sthw[buf * GA + le * A + a] = T2{x.th, x.w};
        __syncthreads();
      }
      if (FL & F_COLL) {
        int cutoff;
        int tc;
        const long long ws = ((long long)t * R.S + k) * EA + ia;
        if (kBoxes) {
          unsigned cm;
          tc = neighbor_force_box<T, FL, AS>(xy_env, rec_env, thw_env0 + buf * GA, shp_env, rad_env,
                                             A, a, x, P, W, fx, fy, cutoff, cm);
          if ((FL & F_MASK) && valid) R.cmask[ws] = cm;  // box worlds: one word (A <= 32)
        } else {
          // contact-mask words of this substep: word-major [H*S][NW][E*A]
          uint32_t* mout = ((FL & F_MASK) && valid)
                               ? R.cmask + ((long long)t * R.S + k) * NW * EA + ia
                               : nullptr;
          tc = neighbor_force<T, FL, AS>(xy_env, rec_env, rad_env, A, a, x, P, W, fx, fy, cutoff,
                                         mout, EA);
        }
        tmax = max(tmax, tc);
        if ((FL & F_TRUNC) && valid) R.cutoff[ws] = (int16_t)cutoff;
      }
      static_force<T, FL>(obs_env, N, x, P, W, fx, fy);
      if (kBodies) {
        __syncthreads();  // every agent has read this substep's shape poses
        if (a == 0)
          bodies_step(sbst + le * N, sbst + le * N, sbc, obs_env, N, rec_env, rad_env, iden_env, A,
                      W, R.body_clamp != 0,
                      kBoxTab ? reinterpret_cast<const T*>(sthw + buf * GA + le * A) : nullptr,
                      kBoxTab ? reinterpret_cast<const T*>(shp_env) : nullptr);
      }
      if (kShare) buf ^= 1;
      Agent<T> y;
      if (kDrone) {
        Drone<T> yd;
        integrate_drone_sel<T, FL>(x, xd, a0, a1, a2, a3, fx, fy, P, W, y, yd);
        xd = yd;
      } else {
        integrate_sel<T, FL>(x, a0, a1, fx, fy, P, W, y);
      }
      x = y;
    }
    if (valid) store_state(R.t_pos, R.t_th, R.t_vel, R.t_s, R.t_w, (long long)t * EA + ia, x);
    if (kDrone && valid) store_drone(R.t_d, (long long)t * EA + ia, xd);
    if (kBodies && a == 0 && valid)
      store_bodies(R.bt_pos, R.bt_ang, R.bt_vel, R.bt_om, ((long long)t * R.E + e) * N, N,
                   sbst + le * N);
    a0 = n0;
    a1 = n1;
    a2 = n2;
    a3 = n3;
  }
  if (valid) {
    if (R.f_pos) store_state(R.f_pos, R.f_th, R.f_vel, R.f_s, R.f_w, ia, x);
    if (kDrone && R.f_d.z) store_drone(R.f_d, ia, xd);
    if (R.true_max) R.true_max[ia] = tmax;
  }
  if (R.goal) block_sum_store(valid ? goal_dist2(R.goal, ia, x.px, x.py) : T(0),
                              R.loss_partial + blockIdx.x);
}

// ================================================================== adjoint
template <typename T, int FL>
__device__ __forceinline__ void static_force_vjp(const Obs<T>* sobs, const BodyC<T>* sbc,
                                                 typename V4<T>::t* gpose, int N,
                                                 const Agent<T>& x, const AgentP<T>& P,
                                                 const WorldC<T>& W, T gfx, T gfy, Agent<T>& gin);

// Force VJP of agent a at one substep: given every env agent's (x, y, vx, vy) record and
// force cotangent, adds d(loss)/d(pos, vel) of agent a through its own force and
// through the forces its contacts feel from it. With moving bodies, also writes the
// cotangent of each moving (circle) shape's centre and velocity through this agent's
// force into gpose[s] (x, y, vx, vy).
template <typename T, int FL, int AS>
__device__ __forceinline__ void force_vjp(const T* xy_env, const typename V4<T>::t* rec_env,
                                          const typename V2<T>::t* fb_env, const int* cut_env,
                                          const T* rad_env, const T* iden_env, const Obs<T>* sobs,
                                          const BodyC<T>* sbc, typename V4<T>::t* gpose, int N,
                                          int A, int a, unsigned cmask, const Agent<T>& x,
                                          const AgentP<T>& P, const WorldC<T>& W, T gfx, T gfy,
                                          Agent<T>& gin, const uint32_t* mw = nullptr,
                                          long long mstride = 0) {
  using T4 = typename V4<T>::t;
  if (FL & F_MASK) {
    // the checkpointed contacts (word 0 in cmask, words c >= 1 at mw[c * mstride]): every
    // in-radius contact of agent a in ascending order, the pairs the rescan below finds in
    // contact; with list truncation the own and cross terms are gated by the cutoffs
    const int cut_a = (FL & F_TRUNC) ? cut_env[a] : A;
    auto visit = [&](int b) {
      const auto q = rec_env[b];
      const auto gb = fb_env[b];
      if (FL & F_TRUNC) {
        const bool own = b <= cut_a;
        const bool cross = a <= cut_env[b];
        pair_vjp_sym(x.px - q.x, x.py - q.y, x.vx - q.z, x.vy - q.w,
                     P.radius + rad_env[b] + W.margin, P.inv_denom, own ? gfx : T(0),
                     own ? gfy : T(0), iden_env[b], cross ? gb.x : T(0), cross ? gb.y : T(0), W,
                     gin.px, gin.py, gin.vx, gin.vy);
      } else {
        pair_vjp_sym(x.px - q.x, x.py - q.y, x.vx - q.z, x.vy - q.w,
                     P.radius + rad_env[b] + W.margin, P.inv_denom, gfx, gfy, iden_env[b], gb.x,
                     gb.y, W, gin.px, gin.py, gin.vx, gin.vy);
      }
    };
    unsigned m = cmask;
    if (A <= 32) {
      while (m) {
        const int b = __ffs(m) - 1;
        m &= m - 1u;
        visit(b);
      }
    } else {
      const int NW = (A + 31) >> 5;
      for (int c = 0; c < NW; ++c) {
        const unsigned next = (c + 1 < NW) ? mw[(c + 1) * mstride] : 0u;  // load ahead
        while (m) {
          const int b = 32 * c + __ffs(m) - 1;
          m &= m - 1u;
          visit(b);
        }
        m = next;
      }
    }
  } else if (FL & F_COLL) {
    const int cut_a = (FL & F_TRUNC) ? cut_env[a] : A;
    for_each_in_radius<T, AS>(xy_env, rec_env, A, a, x.px, x.py, W.r2_scan, W.r2_thr,
                              [&](int b, const T4& q) {
      const bool own = !(FL & F_TRUNC) || b <= cut_a;
      const bool cross = !(FL & F_TRUNC) || a <= cut_env[b];
      const auto gb = fb_env[b];
      pair_vjp_sym(x.px - q.x, x.py - q.y, x.vx - q.z, x.vy - q.w,
                   P.radius + rad_env[b] + W.margin, P.inv_denom, own ? gfx : T(0),
                   own ? gfy : T(0), iden_env[b], cross ? gb.x : T(0), cross ? gb.y : T(0), W,
                   gin.px, gin.py, gin.vx, gin.vy);
    });
  }
  static_force_vjp<T, FL>(sobs, sbc, gpose, N, x, P, W, gfx, gfy, gin);
}

// The obstacle and wall part of force_vjp (after the contacts, the forward's order).
template <typename T, int FL>
__device__ __forceinline__ void static_force_vjp(const Obs<T>* sobs, const BodyC<T>* sbc,
                                                 typename V4<T>::t* gpose, int N,
                                                 const Agent<T>& x, const AgentP<T>& P,
                                                 const WorldC<T>& W, T gfx, T gfy, Agent<T>& gin) {
  using T4 = typename V4<T>::t;
  if (FL & F_OBS) {
    for (int o = 0; o < N; ++o) {
      obstacle_force_vjp(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, sobs[o], gfx, gfy, W,
                         gin.px, gin.py, gin.vx, gin.vy);
      if ((FL & F_BODIES) && moving_shape(sbc, o)) {
        T gcx = T(0), gcy = T(0), gvx = T(0), gvy = T(0);
        circle_obstacle_vjp_pose(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, sobs[o], gfx, gfy,
                                 W, gcx, gcy, gvx, gvy);
        gpose[o] = T4{gcx, gcy, gvx, gvy};
      }
    }
  }
  if (W.bounds_mode == BOUNDS_SOFT)
    wall_force_vjp(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, gfx, gfy, W, gin.px, gin.py,
                   gin.vx, gin.vy);
}

// force_vjp for worlds with box agents (no moving bodies): every contact through the
// shape dispatch's VJP (boxes_vjp.cuh), into all six state gradients of agent a.
template <typename T, int FL, int AS>
__device__ __forceinline__ void force_vjp_box(const T* xy_env, const typename V4<T>::t* rec_env,
                                              const typename V2<T>::t* thw_env,
                                              const typename V4<T>::t* shp_env,
                                              const typename V2<T>::t* fb_env, const int* cut_env,
                                              const T* rad_env, const T* iden_env,
                                              const Obs<T>* sobs, int N, int A, int a,
                                              unsigned cmask, const Agent<T>& x,
                                              const AgentP<T>& P, const WorldC<T>& W, T gfx, T gfy,
                                              Agent<T>& gin) {
  using T4 = typename V4<T>::t;
  const Ob<T> oa = ob_of(x.px, x.py, x.th, x.vx, x.vy, x.w, P.hx, P.hy);
  const bool box_a = P.box != 0;
  auto pair = [&](int b, const T4& q, bool own, bool cross) {
    const auto tw = thw_env[b];
    const auto sh = shp_env[b];
    const auto gb = fb_env[b];
    const Ob<T> ob = ob_of(q.x, q.y, tw.x, q.z, q.w, tw.y, sh.y, sh.z);
    pair_shaped_vjp(a, b, box_a, oa, x.th, P.radius, P.inv_denom, own ? gfx : T(0),
                    own ? gfy : T(0), sh.x > T(0.5), ob, tw.x, rad_env[b], iden_env[b],
                    cross ? gb.x : T(0), cross ? gb.y : T(0), W, gin);
  };
  if (FL & F_MASK) {
    unsigned m = cmask;
    while (m) {
      const int b = __ffs(m) - 1;
      m &= m - 1u;
      pair(b, rec_env[b], true, true);
    }
  } else if (FL & F_COLL) {
    const int cut_a = (FL & F_TRUNC) ? cut_env[a] : A;
    for_each_in_radius<T, AS>(xy_env, rec_env, A, a, x.px, x.py, W.r2_scan, W.r2_thr,
                              [&](int b, const T4& q) {
      pair(b, q, !(FL & F_TRUNC) || b <= cut_a, !(FL & F_TRUNC) || a <= cut_env[b]);
    });
  }
  if (box_a) {
    box_static_vjp((FL & F_OBS) ? sobs : nullptr, (FL & F_OBS) ? N : 0,
                   W.bounds_mode == BOUNDS_SOFT, oa, x.th, P.inv_denom, gfx, gfy, W, gin);
    return;
  }
  if (FL & F_OBS)
    for (int o = 0; o < N; ++o)
      obstacle_force_vjp(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, sobs[o], gfx, gfy, W,
                         gin.px, gin.py, gin.vx, gin.vy);
  if (W.bounds_mode == BOUNDS_SOFT)
    wall_force_vjp(x.px, x.py, x.vx, x.vy, P.radius, P.inv_denom, gfx, gfy, W, gin.px, gin.py,
                   gin.vx, gin.vy);
}

// Adjoint of one env's body substep (one thread): consumes the cotangent of the bodies'
// output states (gbody) and the agents' shape-pose cotangents (gpose [A][N]); writes the
// cotangent of the input states back to gbody and the agents' (pos, vel) cotangents
// through the reactions to gag [A].
template <typename T, typename T4>
__device__ __forceinline__ void bodies_step_vjp(const BodyS<T>* st, const BodyC<T>* bc,
                                                const Obs<T>* obs, int N, const T4* rec,
                                                const T* rad, const T* iden, int A,
                                                const WorldC<T>& W, bool clamp, bool placed,
                                                const T4* gpose, T4* gag, T4* gshape,
                                                BodyG<T>* gbody, BodyG<T>* gbnew) {
  for (int s = 0; s < N; ++s) {
    T4 acc = T4{T(0), T(0), T(0), T(0)};
    if (moving_shape(bc, s)) {
      for (int a = 0; a < A; ++a) {
        const T4 g = gpose[a * N + s];
        acc.x += g.x;
        acc.y += g.y;
        acc.z += g.z;
        acc.w += g.w;
      }
    }
    gshape[s] = acc;
  }
  for (int a = 0; a < A; ++a) gag[a] = T4{T(0), T(0), T(0), T(0)};
  for (int o = 0; o < N; ++o) {
    gbnew[o] = BodyG<T>{T(0), T(0), T(0), T(0), T(0), T(0)};
    if (!moving_root(bc, o)) continue;
    body_pass_root_vjp(o, st[o], bc, obs, N, rec, rad, iden, A, W, clamp, gbody[o], gag, gshape,
                       gbnew[o]);
  }
  if (placed) {
    for (int s = 0; s < N; ++s) {
      if (!moving_shape(bc, s)) continue;
      const T4 g = gshape[s];
      place_vjp(st[bc[s].body], bc[s], g.x, g.y, g.z, g.w, gbnew[bc[s].body]);
    }
  }
  for (int o = 0; o < N; ++o) gbody[o] = gbnew[o];
}

// Sum of the per-CTA partials in a fixed order (one block), accumulated in double.
template <typename T>
__global__ void __launch_bounds__(256) sum_partials_kernel(const T* partial, int n, T* out) {
  __shared__ double acc[256];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += 256) s += static_cast<double>(partial[i]);
  acc[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) acc[threadIdx.x] += acc[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = static_cast<T>(acc[0]);
}

// The compile-time 16-agent instances run in CTAs of at most kMaxThreadsAS16 threads:
// their adjoint then has up to 255 registers instead of 64 (measured 230 -> 224 us).
template <typename T, int FL, int AS, int LB = 1024>
__global__ void __launch_bounds__(AS == 16 ? kMaxThreadsAS16 : LB)
    rollout_bwd_kernel(const RolloutArgs<T> R) {
  using T2 = typename V2<T>::t;
  using T4 = typename V4<T>::t;
  constexpr bool kBodies = (FL & F_BODIES) != 0;
  constexpr bool kBoxes = (FL & F_BOXES) != 0 && (FL & F_COLL) != 0;  // shapes meet in pairs
  extern __shared__ __align__(16) unsigned char smem[];
  const int A = AS > 0 ? AS : R.A;
  const int G = R.G, GA = G * A, S = R.S, N = R.N;
  const int tid = threadIdx.x;
  const int le = tid / A, a = tid - le * A;
  const int e0 = blockIdx.x * G;
  const int e = e0 + le;
  const bool valid = e < R.E;
  const int ec = valid ? e : R.E - 1;
  constexpr bool kDrone = (FL & F_DRONE) != 0;
  const Layout<T> L(G, A, N, S, true, kBodies, kBoxes, kDrone);
  T2* sthw = reinterpret_cast<T2*>(smem + L.thw);  // [nbuf][GA] (th, w), box worlds
  T4* sshp = reinterpret_cast<T4*>(smem + L.shp);  // [GA] (box, hx, hy, -)
  Drone<T>* sdro = reinterpret_cast<Drone<T>*>(smem + L.dro);  // [S][GA], drone worlds
  const int NP4 = L.NP * 4;
  T* sxy = reinterpret_cast<T*>(smem + L.xy);       // [nbuf][G][NP*4] scan tables
  T4* srec = reinterpret_cast<T4*>(smem + L.rec);   // [nbuf][GA] (x, y, vx, vy)
  T* sown = reinterpret_cast<T*>(smem + L.own);     // [S][GA][4] th, s, w
  T2* sfb = reinterpret_cast<T2*>(smem + L.fb);     // [2][GA] force cotangents
  int* scut = reinterpret_cast<int*>(smem + L.cut); // [2][GA] list cutoffs
  T* srad = reinterpret_cast<T*>(smem + L.rad);
  T* siden = reinterpret_cast<T*>(smem + L.iden);
  Obs<T>* sobs = reinterpret_cast<Obs<T>*>(smem + L.obs);
  BodyC<T>* sbc = reinterpret_cast<BodyC<T>*>(smem + L.bc);
  BodyS<T>* sbst = reinterpret_cast<BodyS<T>*>(smem + L.bst);  // [S][G][N]
  T4* sgpose = reinterpret_cast<T4*>(smem + L.gpose);          // [GA][N]
  T4* sgag = reinterpret_cast<T4*>(smem + L.gag);              // [GA]
  BodyG<T>* sgbody = reinterpret_cast<BodyG<T>*>(smem + L.gbody);  // [G][N]
  BodyG<T>* sgbnew = reinterpret_cast<BodyG<T>*>(smem + L.gbnew);  // [G][N]
  T4* sgshape = reinterpret_cast<T4*>(smem + L.gshape);        // [G][N]
  // A rescan is needed unless contacts come from checkpointed masks.
  constexpr bool kScan = (FL & F_COLL) && !(FL & F_MASK);
  constexpr bool kShare = (FL & (F_COLL | F_BODIES)) != 0;

  AgentP<T> P;
  load_params(R, ec, a, P);
  const WorldC<T> W = R.W;
  srad[tid] = P.radius;
  siden[tid] = P.inv_denom;
  if (kBoxes) sshp[tid] = T4{P.box ? T(1) : T(0), P.hx, P.hy, T(0)};
  if (FL & F_OBS) load_obstacles(R, sobs, e0);
  if (kScan) init_pads(sxy, L.nbuf, G, A);
  if (kBodies) {
    load_body_consts(R, sbc);
    if (a == 0) {
      for (int o = 0; o < N; ++o) {
        const long long i = (long long)ec * N + o;
        BodyG<T> gb{T(0), T(0), T(0), T(0), T(0), T(0)};
        if (R.gb_pos) { gb.qx = R.gb_pos[2 * i]; gb.qy = R.gb_pos[2 * i + 1]; }
        if (R.gb_ang) gb.th = R.gb_ang[i];
        if (R.gb_vel) { gb.vx = R.gb_vel[2 * i]; gb.vy = R.gb_vel[2 * i + 1]; }
        if (R.gb_om) gb.om = R.gb_om[i];
        sgbody[le * N + o] = gb;
      }
    }
  }
  __syncthreads();

  const long long ia = (long long)ec * A + a;
  const long long EA = (long long)R.E * A;
  const int H = R.H;
  const T* rad_env = srad + le * A;
  const T* iden_env = siden + le * A;
  Obs<T>* obs_env = sobs + le * N;
  const T4* shp_env = sshp + le * A;
  const bool has_gt = R.gt_pos || R.gt_th || R.gt_vel || R.gt_s || R.gt_w;
  const bool has_gtd = kDrone && (R.gt_d.z || R.gt_d.vz || R.gt_d.att || R.gt_d.br);

  Agent<T> g{};
  add_cotangent(R.gf_pos, R.gf_th, R.gf_vel, R.gf_s, R.gf_w, ia, g);
  if (R.goal) {  // the fused goal loss's seed, from the final positions
    const T2 pH = reinterpret_cast<const T2*>(R.t_pos)[(long long)(R.H - 1) * R.E * A + ia];
    seed_goal_loss(R, ia, pH.x, pH.y, g);
  }
  Drone<T> gd{};  // cotangent of the drone fields
  if (kDrone) add_drone_cotangent(R.gf_d, ia, gd);
  // One-substep holonomic velocity fleets without bodies: the step's adjoint reads only the
  // positions and velocities of its input and output states (heading passes through,
  // speed is recomputed from the velocity), so the other three fields are not loaded.
  const bool pv_only = (FL & F_HOLOVEL) && S == 1 && !kBodies;
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
  Agent<T> nxt;  // output state of step t
  load_traj((long long)(H - 1) * EA + ia, nxt);
  // software pipeline: the inputs of step t are loaded during step t+1
  Agent<T> cur;
  T a0, a1;
  unsigned cm0 = 0u;
  if (H > 1)
    load_traj((long long)(H - 2) * EA + ia, cur);
  else
    load_init(cur);
  load_action(R, (long long)(H - 1) * EA + ia, a0, a1);
  Drone<T> curd{};
  T a2 = T(0), a3 = T(0);
  if (kDrone) {
    if (H > 1)
      load_drone(R.t_d, (long long)(H - 2) * EA + ia, curd);
    else
      load_drone(R.i_d, ia, curd);
    load_action23(R, (long long)(H - 1) * EA + ia, a2, a3);
  }
  // contact-mask words, word-major [H*S][NW][E*A]; word 0 of each step is loaded ahead
  const int NW = (A + 31) >> 5;
  if ((FL & F_MASK) && S == 1) cm0 = R.cmask[(long long)(H - 1) * NW * EA + ia];
  int fbuf = 0;
  T gsq = T(0);  // this agent's sum over the horizon of ||d loss / d action||^2
  for (int t = H - 1; t >= 0; --t) {
    if (has_gt) add_cotangent(R.gt_pos, R.gt_th, R.gt_vel, R.gt_s, R.gt_w, (long long)t * EA + ia, g);
    if (has_gtd) add_drone_cotangent(R.gt_d, (long long)t * EA + ia, gd);
    Agent<T> pcur{};
    Drone<T> pcurd{};
    T pa0 = T(0), pa1 = T(0), pa2 = T(0), pa3 = T(0);
    unsigned pcm = 0u;
    if (t > 0) {
      if (t > 1)
        load_traj((long long)(t - 2) * EA + ia, pcur);
      else
        load_init(pcur);
      load_action(R, (long long)(t - 1) * EA + ia, pa0, pa1);
      if (kDrone) {
        if (t > 1)
          load_drone(R.t_d, (long long)(t - 2) * EA + ia, pcurd);
        else
          load_drone(R.i_d, ia, pcurd);
        load_action23(R, (long long)(t - 1) * EA + ia, pa2, pa3);
      }
      if ((FL & F_MASK) && S == 1) pcm = R.cmask[(long long)(t - 1) * NW * EA + ia];
    }
    T ga0 = T(0), ga1 = T(0), ga2 = T(0), ga3 = T(0);

    if (S == 1 && !kBodies) {
      Agent<T> gin;
      T gfx, gfy;
      if (kDrone) {
        Drone<T> gdin;
        integrate_vjp_drone_sel<T, FL>(cur, curd, a0, a1, a2, a3, nxt, g, gd, P, W, gin, gdin, gfx,
                                       gfy, ga0, ga1, ga2, ga3);
        gd = gdin;
      } else {
        integrate_vjp_sel<T, FL>(cur, a0, a1, nxt, g, P, W, gin, gfx, gfy, ga0, ga1);
      }
      T* xy_env = sxy + (fbuf * G + le) * NP4;
      T4* rec_env = srec + fbuf * GA + le * A;
      T2* fb_env = sfb + fbuf * GA + le * A;
      int* cut_env = scut + fbuf * GA + le * A;
      if (FL & F_COLL) {
        if (kScan) put_xy(xy_env, a, cur.px, cur.py);
        rec_env[a] = T4{cur.px, cur.py, cur.vx, cur.vy};
        if (kBoxes) sthw[fbuf * GA + le * A + a] = T2{cur.th, cur.w};
        fb_env[a] = T2{gfx, gfy};
        if (FL & F_TRUNC) cut_env[a] = R.cutoff[(long long)t * EA + ia];
        __syncthreads();
      }
      if (FL & F_BOXES)
        force_vjp_box<T, FL, AS>(xy_env, rec_env, sthw + fbuf * GA + le * A, shp_env, fb_env,
                                 cut_env, rad_env, iden_env, obs_env, N, A, a, cm0, cur, P, W, gfx,
                                 gfy, gin);
      else
        force_vjp<T, FL, AS>(xy_env, rec_env, fb_env, cut_env, rad_env, iden_env, obs_env, sbc,
                             nullptr, N, A, a, cm0, cur, P, W, gfx, gfy, gin,
                             (FL & F_MASK) ? R.cmask + (long long)t * NW * EA + ia : nullptr, EA);
      g = gin;
      fbuf ^= 1;
    } else {
      // recompute the substep chain (agents and bodies) from the checkpointed step input
      __syncthreads();  // every thread is done with last step's stash and shape poses
      if (kBodies && a == 0) {
        BodyS<T>* b0 = sbst + le * N;
        if (t > 0)
          load_bodies(R.bt_pos, R.bt_ang, R.bt_vel, R.bt_om, ((long long)(t - 1) * R.E + ec) * N, N, b0);
        else
          load_bodies(R.bi_pos, R.bi_ang, R.bi_vel, R.bi_om, (long long)ec * N, N, b0);
        set_body_poses(R, ec, t == 0 && !R.poses_from_bodies, b0, sbc, obs_env);
      }
      Agent<T> x = cur;
      Drone<T> xd = curd;
      for (int k = 0; k < S; ++k) {
        T* xy_env = sxy + (k * G + le) * NP4;
        T4* rec_env = srec + k * GA + le * A;
        if (kScan) put_xy(xy_env, a, x.px, x.py);
        rec_env[a] = T4{x.px, x.py, x.vx, x.vy};
        if (kDrone) sdro[size_t(k) * GA + tid] = xd;
        if (kBoxes) sthw[k * GA + le * A + a] = T2{x.th, x.w};
        T* ow = sown + (size_t(k) * GA + tid) * 4;
        ow[0] = x.th;
        ow[1] = x.s;
        ow[2] = x.w;
        if (k == S - 1) break;
        T fx = T(0), fy = T(0);
        if (kShare) __syncthreads();
        if (FL & F_COLL) {
          const T2* thw_env = sthw + k * GA + le * A;
          if (FL & F_MASK) {
            const uint32_t* mw = R.cmask + ((long long)t * S + k) * NW * EA + ia;
            if (kBoxes) {
              mask_force_box(rec_env, thw_env, shp_env, rad_env, mw[0], a, x, P, W, fx, fy);
            } else {
              const int cut_a =
                  (FL & F_TRUNC) ? R.cutoff[((long long)t * S + k) * EA + ia] : A;
              mask_force_w<T, FL>(rec_env, rad_env, mw, EA, NW, cut_a, x, P, W, fx, fy);
            }
          } else {
            int cutoff;
            unsigned cm;
            if (kBoxes)
              neighbor_force_box<T, FL, AS>(xy_env, rec_env, thw_env, shp_env, rad_env, A, a, x, P,
                                            W, fx, fy, cutoff, cm);
            else
              neighbor_force<T, FL, AS>(xy_env, rec_env, rad_env, A, a, x, P, W, fx, fy, cutoff);
          }
        }
        static_force<T, FL>(obs_env, N, x, P, W, fx, fy);
        if (kBodies) {
          __syncthreads();  // every agent has read this substep's shape poses
          if (a == 0)
            bodies_step(sbst + (k * G + le) * N, sbst + ((k + 1) * G + le) * N, sbc, obs_env, N,
                        rec_env, rad_env, iden_env, A, W, R.body_clamp != 0);
        }
        Agent<T> y;
        if (kDrone) {
          Drone<T> yd;
          integrate_drone_sel<T, FL>(x, xd, a0, a1, a2, a3, fx, fy, P, W, y, yd);
          xd = yd;
        } else {
          integrate_sel<T, FL>(x, a0, a1, fx, fy, P, W, y);
        }
        x = y;
      }
      Agent<T> out = nxt;
      for (int k = S - 1; k >= 0; --k) {
        T* xy_env = sxy + (k * G + le) * NP4;
        T4* rec_env = srec + k * GA + le * A;
        const BodyS<T>* bk = sbst + (k * G + le) * N;
        if (kBodies && a == 0 && k < S - 1)
          set_body_poses(R, ec, t == 0 && k == 0 && !R.poses_from_bodies, bk, sbc, obs_env);
        const T* ow = sown + (size_t(k) * GA + tid) * 4;
        const T4 rr = rec_env[a];
        Agent<T> in{rr.x, rr.y, ow[0], rr.z, rr.w, ow[1], ow[2]};
        Agent<T> gin;
        T gfx, gfy;
        if (kDrone) {
          Drone<T> gdin;
          integrate_vjp_drone_sel<T, FL>(in, sdro[size_t(k) * GA + tid], a0, a1, a2, a3, out, g, gd,
                                         P, W, gin, gdin, gfx, gfy, ga0, ga1, ga2, ga3);
          gd = gdin;
        } else {
          integrate_vjp_sel<T, FL>(in, a0, a1, out, g, P, W, gin, gfx, gfy, ga0, ga1);
        }
        T2* fb_env = sfb + fbuf * GA + le * A;
        int* cut_env = scut + fbuf * GA + le * A;
        fb_env[a] = T2{gfx, gfy};
        const long long ws = ((long long)t * S + k) * EA + ia;
        if (FL & F_TRUNC) cut_env[a] = R.cutoff[ws];
        const uint32_t* mw =
            (FL & F_MASK) ? R.cmask + ((long long)t * S + k) * NW * EA + ia : nullptr;
        const unsigned cm = (FL & F_MASK) ? mw[0] : 0u;
        __syncthreads();
        if (FL & F_BOXES)
          force_vjp_box<T, FL, AS>(xy_env, rec_env, sthw + k * GA + le * A, shp_env, fb_env,
                                   cut_env, rad_env, iden_env, obs_env, N, A, a, cm, in, P, W, gfx,
                                   gfy, gin);
        else
          force_vjp<T, FL, AS>(xy_env, rec_env, fb_env, cut_env, rad_env, iden_env, obs_env, sbc,
                               sgpose + size_t(tid) * N, N, A, a, cm, in, P, W, gfx, gfy, gin,
                               mw, EA);
        if (kBodies) {
          __syncthreads();  // shape-pose cotangents of every agent are in
          if (a == 0)
            bodies_step_vjp(bk, sbc, obs_env, N, rec_env, rad_env, iden_env, A, W,
                            R.body_clamp != 0, !(t == 0 && k == 0 && !R.poses_from_bodies),
                            sgpose + size_t(le) * A * N,
                            sgag + le * A, sgshape + le * N, sgbody + le * N, sgbnew + le * N);
          __syncthreads();  // reaction cotangents of every agent are in
          const T4 gr = sgag[tid];
          gin.px += gr.x;
          gin.py += gr.y;
          gin.vx += gr.z;
          gin.vy += gr.w;
        }
        g = gin;
        out = in;
        fbuf ^= 1;
      }
    }
    if (valid) {
      const long long ja = (long long)t * EA + ia;
      gsq = Num<T>::fma_(ga0, ga0, Num<T>::fma_(ga1, ga1, gsq));
      if (kDrone) gsq = Num<T>::fma_(ga2, ga2, Num<T>::fma_(ga3, ga3, gsq));
      if (R.act_dim == 2) {
        reinterpret_cast<T2*>(R.g_act)[ja] = T2{ga0, ga1};
      } else {
        R.g_act[ja * R.act_dim] = ga0;
        R.g_act[ja * R.act_dim + 1] = ga1;
        for (int j = 2; j < R.act_dim; ++j)
          R.g_act[ja * R.act_dim + j] = (kDrone && j == 2) ? ga2 : ((kDrone && j == 3) ? ga3 : T(0));
      }
    }
    nxt = cur;
    cur = pcur;
    a0 = pa0;
    a1 = pa1;
    if (kDrone) {
      curd = pcurd;
      a2 = pa2;
      a3 = pa3;
    }
    cm0 = pcm;
  }
  if (valid) store_state(R.gi_pos, R.gi_th, R.gi_vel, R.gi_s, R.gi_w, ia, g);
  if (kDrone && valid) store_drone(R.gi_d, ia, gd);
  if (R.gsq_partial) block_sum_store(gsq, R.gsq_partial + blockIdx.x);
}

// ============================================================ neighbor lists
template <typename T>
__global__ void __launch_bounds__(1024) neighbors_kernel(int E, int A, int G, int K, T r2_scan, T r2_thr,
                                                         const T* pos, int* idx, int* count,
                                                         int* true_count) {
  using T2 = typename V2<T>::t;
  using T4 = typename V4<T>::t;
  extern __shared__ __align__(16) unsigned char smem[];
  const int NP4 = ((A + 1) / 2) * 4;
  T* sxy = reinterpret_cast<T*>(smem);
  T4* srec = reinterpret_cast<T4*>(smem + ((size_t(G) * NP4 * sizeof(T) + 15) & ~size_t(15)));
  const int tid = threadIdx.x;
  const int le = tid / A, a = tid - le * A;
  const int e = blockIdx.x * G + le;
  const bool valid = e < E;
  const int ec = valid ? e : E - 1;
  const long long ia = (long long)ec * A + a;
  init_pads(sxy, 1, G, A);
  const T2 p = reinterpret_cast<const T2*>(pos)[ia];
  T* xy_env = sxy + le * NP4;
  put_xy(xy_env, a, p.x, p.y);
  srec[tid] = T4{p.x, p.y, T(0), T(0)};
  __syncthreads();
  int listed = 0;
  const int total = for_each_in_radius<T, 0>(xy_env, srec + le * A, A, a, p.x, p.y, r2_scan, r2_thr,
                                             [&](int b, const T4&) {
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
