// Device math of one agent substep: contact law, obstacles, walls and the three 2-D
// motion models, each as a forward function and its hand-derived vector-Jacobian
// product (VJP). Shared by the rollout forward and adjoint kernels.
//
// Reference semantics (ddebenedittis/swarp):
//   contact law          swarp/core/collisions.py:87-143  (_normal_coeff, pair_force)
//   segment / box        swarp/core/collisions.py:156-260 (closest_on_segment, box_force)
//   broad phase          swarp/core/collisions.py:61-84   (shape_bound, bounds_apart)
//   walls                swarp/core/collisions.py:745-780 (_wall_forces)
//   motion models        swarp/dynamics/kernels.py:68-71, 166-275 (clamp_norm, servo, _step_2d)
//   disc bounds clamp    swarp/dynamics/kernels.py:395-403
// The reference differentiates these with Warp's generated adjoints; the VJPs here
// follow the same branch conventions at kinks: max(a, b) sends the gradient to b on a
// tie, clamp passes it on the closed interval, length() has zero gradient at the zero
// vector, abs() has +1 at zero.
//
// The whole translation unit is compiled with -fmad=false: every multiply-add below
// rounds exactly as written, so a quantity recomputed in the adjoint kernel (contact
// activity, clamp activity, neighbor membership) is bitwise the value the forward
// kernel saw. Fused multiply-adds are placed explicitly with fma().
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace swarp {

// ------------------------------------------------------------------ scalar helpers
template <typename T> struct Num;
template <> struct Num<float> {
  static __device__ __forceinline__ float sqrt_(float x) { return ::sqrtf(x); }
  static __device__ __forceinline__ float fma_(float a, float b, float c) { return __fmaf_rn(a, b, c); }
  static __device__ __forceinline__ float sin_(float x) { return ::sinf(x); }
  static __device__ __forceinline__ float cos_(float x) { return ::cosf(x); }
  static __device__ __forceinline__ float tan_(float x) { return ::tanf(x); }
  static __device__ __forceinline__ float atan_(float x) { return ::atanf(x); }
  static __device__ __forceinline__ float tanh_(float x) { return ::tanhf(x); }
  static __device__ __forceinline__ float rsqrt_(float x) { return ::rsqrtf(x); }
};
template <> struct Num<double> {
  static __device__ __forceinline__ double sqrt_(double x) { return ::sqrt(x); }
  static __device__ __forceinline__ double fma_(double a, double b, double c) { return __fma_rn(a, b, c); }
  static __device__ __forceinline__ double sin_(double x) { return ::sin(x); }
  static __device__ __forceinline__ double cos_(double x) { return ::cos(x); }
  static __device__ __forceinline__ double tan_(double x) { return ::tan(x); }
  static __device__ __forceinline__ double atan_(double x) { return ::atan(x); }
  static __device__ __forceinline__ double tanh_(double x) { return ::tanh(x); }
  static __device__ __forceinline__ double rsqrt_(double x) { return ::rsqrt(x); }
};

template <typename T> __device__ __forceinline__ T wmax(T a, T b) { return a > b ? a : b; }
template <typename T> __device__ __forceinline__ T wmin(T a, T b) { return a < b ? a : b; }
// Warp clamp: min(max(lo, x), hi)
template <typename T> __device__ __forceinline__ T wclamp(T x, T lo, T hi) { return wmin(wmax(lo, x), hi); }
// wmax(x, c) for a constant c >= +0 in one min/max instruction: the same value for every x
// (a NaN x gives c in both forms; -0 against +0 gives +0 in both).
template <typename T> __device__ __forceinline__ T wmax_c(T x, T c) { return fmax(x, c); }
// gradient gate of Warp's clamp adjoint (closed interval)
template <typename T> __device__ __forceinline__ bool clamp_pass(T x, T lo, T hi) { return !(x < lo) && !(x > hi); }
template <typename T> __device__ __forceinline__ T dot2(T ax, T ay, T bx, T by) { return Num<T>::fma_(ax, bx, ay * by); }
template <typename T> __device__ __forceinline__ T len2(T x, T y) { return Num<T>::sqrt_(dot2(x, y, x, y)); }

template <typename T> struct Eps2 { static constexpr T v = T(1.0e-10); };

// Neighbor membership, the reference's wp.length(p_b - p_a) <= radius
// (swarp/core/neighbors.py:91), as IEEE arithmetic rounds the expression without
// contraction: sqrt(fl(fl(dx*dx) + fl(dy*dy))) <= R. The square root is correctly rounded
// and monotone, so with thr = the largest T whose square root is <= R (computed on the
// host) the test is fl(fl(dx*dx) + fl(dy*dy)) <= thr, bit for bit, with no square root.
// The kernels' packed scan evaluates dx^2 + (dy^2 - thr') with two fused roundings, which
// can differ from this sum within an ulp of the threshold; it runs with thr' = thr widened
// by at least 8 ulps, so its set contains every member (the fused error is below
// 3 ulps of thr), and this exact test then drops the extra candidates.
__device__ __forceinline__ bool in_radius(float dx, float dy, float thr) {
  return __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)) <= thr;
}
__device__ __forceinline__ bool in_radius(double dx, double dy, double thr) {
  return __dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)) <= thr;
}

// Model / mode / shape tags (values of the reference enums).
enum : int { TAG_HOLONOMIC = 0, TAG_DIFF_DRIVE = 1, TAG_BICYCLE = 2, TAG_DRONE = 3 };
enum : int { MODE_VELOCITY = 0, MODE_ACCELERATION = 1, MODE_SERVO = 2 };
enum : int { SHAPE_CIRCLE = 0, SHAPE_BOX = 1, SHAPE_SEGMENT = 2 };
enum : int { BOUNDS_NONE = 0, BOUNDS_SOFT = 1, BOUNDS_CLAMP = 2 };

// Per-agent state (the five live 2-D fields).
template <typename T> struct Agent {
  T px, py, th, vx, vy, s, w;
};

// Per-agent constants, loaded once per launch.
template <typename T> struct AgentP {
  T radius, mass, max_speed, min_speed, max_accel, max_ang_vel, max_ang_accel;
  T l_f, l_r, max_steer, gain_v, gain_w;
  T dt_over_m;  // sub_dt / mass  (the reference's force * (dt / mass))
  T inv_denom;  // 1 / (1 + c * sub_dt / mass): implicit damping denominator, inverted once
  int tag, mode;
  int box;     // shape BOX (else disc)
  T hx, hy;    // box half extents
  T tmax, arm, ixx, iyy, izz, kappa, grav;  // drone: rotor thrust limit, geometry, gravity
};

// World constants of one launch.
template <typename T> struct WorldC {
  T dt;  // sub-step
  T k, c, margin, max_overlap;
  T r2_thr;   // largest d2 with sqrt(d2) <= neighbor_radius (exact membership test)
  T r2_scan;  // r2_thr widened by >= 8 ulps: the fused scan's superset threshold
  T bx0, bx1, by0, by1;
  T lin_decay, ang_decay;  // movable bodies: 1 - damping * dt
  int K;                   // max_neighbors
  int bounds_mode;
};

// ------------------------------------------------------------------- contact law
// Division and square root are formulated with one reciprocal square root and
// multiplications by reciprocals precomputed per agent (the reference divides); the
// forward and adjoint kernels use the same formulation, so every recomputed branch
// decision is bitwise the forward's.
//
// Depth saturation mo * tanh(ov / mo) (contact_max_overlap > 0 only): a cold call, so the
// common unsaturated contact stays a handful of instructions.
template <typename T> __device__ __noinline__ T tanh_ratio(T ov, T mo) { return Num<T>::tanh_(ov / mo); }

// Numerator of the contact coefficient, k*ov' - c*vn, with one rounding less than the
// reference's (an explicit fma). Every kernel that decides a branch on its sign (the
// forward's max(x, 0) and the adjoints recomputing that activity) takes it from here, so
// the decisions agree bit for bit.
template <typename T> __device__ __forceinline__ T nc_num(T ovs, T vn, const WorldC<T>& W) {
  return Num<T>::fma_(W.k, ovs, -(W.c * vn));
}
// Overlap of a disc pair, min_dist - |d| with |d| = m * rsqrt(m) (one fma); shared by the
// forward and every adjoint that recomputes whether the pair is in contact.
template <typename T> __device__ __forceinline__ T pair_overlap(T min_dist, T m, T inv) {
  return Num<T>::fma_(-m, inv, min_dist);
}

// f = max(0, (k*ov' - c*vn) / denom), ov' = mo*tanh(ov/mo) when mo > 0
template <typename T>
__device__ __forceinline__ T normal_coeff(T ov, T vn, T inv_denom, const WorldC<T>& W) {
  T ovs = ov;
  if (W.max_overlap > T(0)) ovs = W.max_overlap * tanh_ratio(ov, W.max_overlap);
  T x = nc_num(ovs, vn, W) * inv_denom;
  return wmax_c(x, T(0));
}
// VJP of normal_coeff: cotangent g on its value -> (d ov, d vn)
template <typename T>
__device__ __forceinline__ void normal_coeff_vjp(T ov, T vn, T inv_denom, T g, const WorldC<T>& W,
                                                 T& gov, T& gvn) {
  T ovs = ov, th = T(0);
  if (W.max_overlap > T(0)) {
    th = tanh_ratio(ov, W.max_overlap);
    ovs = W.max_overlap * th;
  }
  T x = nc_num(ovs, vn, W) * inv_denom;
  if (x > T(0)) {
    T gnum = g * inv_denom;
    T govs = W.k * gnum;
    gvn = -W.c * gnum;
    gov = (W.max_overlap > T(0)) ? govs * (T(1) - th * th) : govs;
  } else {
    gov = T(0);
    gvn = T(0);
  }
}

// Disc-disc contact: force on self, d = p_self - p_other, rv = v_self - v_other.
// d2 is dot(d, d) as computed by the caller (the membership test reuses it).
// Returns whether the pair is in contact (overlap > 0).
template <typename T>
__device__ __forceinline__ bool pair_force_add(T dx, T dy, T d2, T rvx, T rvy, T min_dist,
                                               T inv_denom, const WorldC<T>& W, T& fx, T& fy) {
  const T m = wmax_c(d2, Eps2<T>::v);
  const T inv = Num<T>::rsqrt_(m);
  const T ov = pair_overlap(min_dist, m, inv);
  if (ov > T(0)) {
    T nx = dx * inv, ny = dy * inv;
    T vn = dot2(rvx, rvy, nx, ny);
    T cf = normal_coeff(ov, vn, inv_denom, W);
    fx = Num<T>::fma_(cf, nx, fx);
    fy = Num<T>::fma_(cf, ny, fy);
    return true;
  }
  return false;
}
// Whether two discs at d = p_self - p_other with min_dist are in contact, the decision of
// pair_force_add and pair_vjp_terms (the same arithmetic).
template <typename T>
__device__ __forceinline__ bool pair_in_contact(T dx, T dy, T min_dist) {
  const T m = wmax_c(dot2(dx, dy, dx, dy), Eps2<T>::v);
  const T inv = Num<T>::rsqrt_(m);
  return pair_overlap(min_dist, m, inv) > T(0);
}

// Force value (no accumulation), used where the result is negated/levered.
template <typename T>
__device__ __forceinline__ void pair_force(T dx, T dy, T rvx, T rvy, T min_dist, T inv_denom,
                                           const WorldC<T>& W, T& fx, T& fy) {
  fx = T(0);
  fy = T(0);
  pair_force_add(dx, dy, dot2(dx, dy, dx, dy), rvx, rvy, min_dist, inv_denom, W, fx, fy);
}

// VJP of pair_force: cotangent (gx, gy) on f -> adds to (gdx, gdy) and (grvx, grvy).
template <typename T>
__device__ __forceinline__ void pair_force_vjp(T dx, T dy, T rvx, T rvy, T min_dist, T inv_denom,
                                               T gx, T gy, const WorldC<T>& W, T& gdx, T& gdy,
                                               T& grvx, T& grvy) {
  const T d2 = dot2(dx, dy, dx, dy);
  const T m = wmax_c(d2, Eps2<T>::v);
  const T inv = Num<T>::rsqrt_(m);
  const T ov = pair_overlap(min_dist, m, inv);
  if (!(ov > T(0))) return;
  T nx = dx * inv, ny = dy * inv;
  T vn = dot2(rvx, rvy, nx, ny);
  T cf = normal_coeff(ov, vn, inv_denom, W);
  T gcf = dot2(gx, gy, nx, ny);
  T gnx = cf * gx, gny = cf * gy;
  T gov, gvn;
  normal_coeff_vjp(ov, vn, inv_denom, gcf, W, gov, gvn);
  grvx += gvn * nx;
  grvy += gvn * ny;
  gnx += gvn * rvx;
  gny += gvn * rvy;
  // n = d / dist, dist = sqrt(max(d2, eps)), ov = min_dist - dist
  T gdist = -gov - dot2(gnx, gny, nx, ny) * inv;
  T ddx = gnx * inv, ddy = gny * inv;
  if (d2 > Eps2<T>::v) {
    T gd2 = gdist * T(0.5) * inv;
    ddx += T(2) * dx * gd2;
    ddy += T(2) * dy * gd2;
  }
  gdx += ddx;
  gdy += ddy;
}

// Both directions of one disc-disc contact in a single VJP. With d = p_a - p_b and
// rv = v_a - v_b, the force on a is cf_a n and on b is -cf_b n (cf_x uses x's implicit
// denominator); ga and gb are their cotangents (zero to exclude a side, e.g. a truncated
// list). L = cf_a (ga.n) - cf_b (gb.n). pair_vjp_terms returns dL/dd and dL/drv
// (= dL/dp_a, dL/dv_a) as four separate values, false when the pair is not in contact;
// agent b's own call with the roles swapped gives their exact negatives. The owner adds
// each value once, so where the terms are computed (by the owner or another lane) does
// not change the sums.
template <typename T> struct PairTerms {
  T px, py, vx, vy;
};
template <typename T>
__device__ __forceinline__ bool pair_vjp_terms(T dx, T dy, T rvx, T rvy, T min_dist, T ida, T gax,
                                               T gay, T idb, T gbx, T gby, const WorldC<T>& W,
                                               PairTerms<T>& r) {
  const T d2 = dot2(dx, dy, dx, dy);
  const T m = wmax_c(d2, Eps2<T>::v);
  const T inv = Num<T>::rsqrt_(m);
  const T ov = pair_overlap(min_dist, m, inv);
  if (!(ov > T(0))) return false;
  const T nx = dx * inv, ny = dy * inv;
  const T vn = dot2(rvx, rvy, nx, ny);
  T ovs = ov, th = T(0);
  if (W.max_overlap > T(0)) {
    th = tanh_ratio(ov, W.max_overlap);
    ovs = W.max_overlap * th;
  }
  const T num = nc_num(ovs, vn, W);
  const T xa = num * ida, xb = num * idb;
  const T cfa = wmax_c(xa, T(0)), cfb = wmax_c(xb, T(0));
  const T q = (xa > T(0) ? ida * dot2(gax, gay, nx, ny) : T(0)) -
              (xb > T(0) ? idb * dot2(gbx, gby, nx, ny) : T(0));  // dL/dnum
  const T gvn = -W.c * q;
  const T govs = W.k * q;
  const T gov = (W.max_overlap > T(0)) ? govs * (T(1) - th * th) : govs;
  r.vx = gvn * nx;
  r.vy = gvn * ny;
  // dL/dn: at fixed num, then through vn = rv.n
  const T gnx = Num<T>::fma_(gvn, rvx, Num<T>::fma_(cfa, gax, -(cfb * gbx)));
  const T gny = Num<T>::fma_(gvn, rvy, Num<T>::fma_(cfa, gay, -(cfb * gby)));
  // n = d / dist, dist = sqrt(max(d2, eps)), ov = min_dist - dist
  const T gdist = Num<T>::fma_(-dot2(gnx, gny, nx, ny), inv, -gov);
  r.px = gnx * inv;
  r.py = gny * inv;
  if (d2 > Eps2<T>::v) {
    const T gd2 = gdist * T(0.5) * inv;
    r.px = Num<T>::fma_(T(2) * dx, gd2, r.px);
    r.py = Num<T>::fma_(T(2) * dy, gd2, r.py);
  }
  return true;
}
template <typename T>
__device__ __forceinline__ void pair_vjp_sym(T dx, T dy, T rvx, T rvy, T min_dist, T ida, T gax,
                                             T gay, T idb, T gbx, T gby, const WorldC<T>& W,
                                             T& gdx, T& gdy, T& grvx, T& grvy) {
  PairTerms<T> t;
  if (!pair_vjp_terms(dx, dy, rvx, rvy, min_dist, ida, gax, gay, idb, gbx, gby, W, t)) return;
  grvx += t.vx;
  grvy += t.vy;
  gdx += t.px;
  gdy += t.py;
}

// Branch-free forms of the disc-disc contact without depth saturation (max_overlap == 0),
// for loops that evaluate two agents' contacts side by side: every operation of
// pair_force_add / pair_vjp_terms in the same order, the branches turned into selects, so
// the results are bitwise theirs. `have` false (no pair this round) leaves everything as it
// was; a pair out of contact adds nothing.
template <typename T>
__device__ __forceinline__ bool pair_force_add_nb(bool have, T dx, T dy, T rvx, T rvy, T min_dist,
                                                  T inv_denom, const WorldC<T>& W, T& fx, T& fy) {
  const T d2 = dot2(dx, dy, dx, dy);
  const T m = wmax_c(d2, Eps2<T>::v);
  const T inv = Num<T>::rsqrt_(m);
  const T ov = pair_overlap(min_dist, m, inv);
  const bool on = have && ov > T(0);
  const T nx = dx * inv, ny = dy * inv;
  const T vn = dot2(rvx, rvy, nx, ny);
  const T cf = wmax_c(nc_num(ov, vn, W) * inv_denom, T(0));
  fx = on ? Num<T>::fma_(cf, nx, fx) : fx;
  fy = on ? Num<T>::fma_(cf, ny, fy) : fy;
  return on;
}
template <typename T>
__device__ __forceinline__ bool pair_vjp_terms_nb(bool have, T dx, T dy, T rvx, T rvy, T min_dist,
                                                  T ida, T gax, T gay, T idb, T gbx, T gby,
                                                  const WorldC<T>& W, PairTerms<T>& r) {
  const T d2 = dot2(dx, dy, dx, dy);
  const T m = wmax_c(d2, Eps2<T>::v);
  const T inv = Num<T>::rsqrt_(m);
  const T ov = pair_overlap(min_dist, m, inv);
  const T nx = dx * inv, ny = dy * inv;
  const T vn = dot2(rvx, rvy, nx, ny);
  const T num = nc_num(ov, vn, W);
  const T xa = num * ida, xb = num * idb;
  const T cfa = wmax_c(xa, T(0)), cfb = wmax_c(xb, T(0));
  const T q = (xa > T(0) ? ida * dot2(gax, gay, nx, ny) : T(0)) -
              (xb > T(0) ? idb * dot2(gbx, gby, nx, ny) : T(0));
  const T gvn = -W.c * q;
  const T gov = W.k * q;
  r.vx = gvn * nx;
  r.vy = gvn * ny;
  const T gnx = Num<T>::fma_(gvn, rvx, Num<T>::fma_(cfa, gax, -(cfb * gbx)));
  const T gny = Num<T>::fma_(gvn, rvy, Num<T>::fma_(cfa, gay, -(cfb * gby)));
  const T gdist = Num<T>::fma_(-dot2(gnx, gny, nx, ny), inv, -gov);
  const T bx = gnx * inv, by = gny * inv;
  const T gd2 = gdist * T(0.5) * inv;
  const bool far = d2 > Eps2<T>::v;
  r.px = far ? Num<T>::fma_(T(2) * dx, gd2, bx) : bx;
  r.py = far ? Num<T>::fma_(T(2) * dy, gd2, by) : by;
  return have && ov > T(0);
}

// ------------------------------------------------------------- static obstacles
// One obstacle as seen by the agent pass. Position/velocity are per env; the cos/sin
// of the angle are precomputed (the reference evaluates cos(angle), sin(angle) in place;
// same values).
template <typename T> struct Obs {
  T cx, cy, ca, sa, vx, vy, om;  // pose and motion
  T r, hx, hy, bound;            // shape constants; bound = shape_bound()
  int type;
};

template <typename T>
__device__ __forceinline__ bool bounds_apart(T dx, T dy, T reach) {
  T lim = reach * T(1.0001) + T(1.0e-6);
  return dot2(dx, dy, dx, dy) > lim * lim;
}

// Box SDF contact (collisions.py:174-260): force on an agent at p with velocity v.
template <typename T>
__device__ __forceinline__ bool box_force(T px, T py, T vx, T vy, const Obs<T>& o, T reach, T inv_denom,
                                          const WorldC<T>& W, T& fx, T& fy) {
  fx = T(0);
  fy = T(0);
  const T ca = o.ca, sa = o.sa;
  T dx = px - o.cx, dy = py - o.cy;
  T lx = ca * dx + sa * dy;
  T ly = -sa * dx + ca * dy;
  T qx = fabs(lx) - o.hx;
  T qy = fabs(ly) - o.hy;
  T cx = wclamp(lx, -o.hx, o.hx), cy = wclamp(ly, -o.hy, o.hy);
  T ox = lx - cx, oy = ly - cy;
  T od2 = ox * ox + oy * oy;
  T s, nlx, nly;
  if (od2 > Eps2<T>::v) {
    const T is = Num<T>::rsqrt_(od2);
    s = od2 * is;
    nlx = ox * is;
    nly = oy * is;
  } else if (qx > qy) {
    s = qx;
    nlx = lx >= T(0) ? T(1) : T(-1);
    nly = T(0);
  } else {
    s = qy;
    nlx = T(0);
    nly = ly >= T(0) ? T(1) : T(-1);
  }
  T overlap = reach - s;
  if (overlap > T(0)) {
    T nx = ca * nlx - sa * nly, ny = sa * nlx + ca * nly;
    T spx = lx - s * nlx, spy = ly - s * nly;
    T rx = ca * spx - sa * spy, ry = sa * spx + ca * spy;
    T vsx = o.vx + (-o.om * ry), vsy = o.vy + o.om * rx;
    T vn = dot2(vx - vsx, vy - vsy, nx, ny);
    T cf = normal_coeff(overlap, vn, inv_denom, W);
    fx = cf * nx;
    fy = cf * ny;
    return true;
  }
  return false;
}

template <typename T>
__device__ __forceinline__ void box_force_vjp(T px, T py, T vx, T vy, const Obs<T>& o, T reach,
                                              T inv_denom, T gx, T gy, const WorldC<T>& W, T& gpx,
                                              T& gpy, T& gvx, T& gvy) {
  const T ca = o.ca, sa = o.sa;
  T dx = px - o.cx, dy = py - o.cy;
  T lx = ca * dx + sa * dy;
  T ly = -sa * dx + ca * dy;
  T qx = fabs(lx) - o.hx;
  T qy = fabs(ly) - o.hy;
  T cx = wclamp(lx, -o.hx, o.hx), cy = wclamp(ly, -o.hy, o.hy);
  T ox = lx - cx, oy = ly - cy;
  T od2 = ox * ox + oy * oy;
  T s, nlx, nly;
  const bool ext = od2 > Eps2<T>::v;
  const bool use_x = qx > qy;
  T is = T(0);
  if (ext) {
    is = Num<T>::rsqrt_(od2);
    s = od2 * is;
    nlx = ox * is;
    nly = oy * is;
  } else if (use_x) {
    s = qx;
    nlx = lx >= T(0) ? T(1) : T(-1);
    nly = T(0);
  } else {
    s = qy;
    nlx = T(0);
    nly = ly >= T(0) ? T(1) : T(-1);
  }
  T overlap = reach - s;
  if (!(overlap > T(0))) return;
  T nx = ca * nlx - sa * nly, ny = sa * nlx + ca * nly;
  T spx = lx - s * nlx, spy = ly - s * nly;
  T rx = ca * spx - sa * spy, ry = sa * spx + ca * spy;
  T vsx = o.vx + (-o.om * ry), vsy = o.vy + o.om * rx;
  T relx = vx - vsx, rely = vy - vsy;
  T vn = dot2(relx, rely, nx, ny);
  T cf = normal_coeff(overlap, vn, inv_denom, W);
  // f = cf * n
  T gcf = dot2(gx, gy, nx, ny);
  T gnx = cf * gx, gny = cf * gy;
  T gov, gvn;
  normal_coeff_vjp(overlap, vn, inv_denom, gcf, W, gov, gvn);
  // vn = rel . n
  T grelx = gvn * nx, grely = gvn * ny;
  gnx += gvn * relx;
  gny += gvn * rely;
  gvx += grelx;
  gvy += grely;
  // vs = vo + om x r ; rel = v - vs
  T grx = o.om * (-grely);   // vsy = vy_o + om*rx, gvs = -grel
  T gry = -o.om * (-grelx);  // vsx = vx_o - om*ry
  // r = R sp
  T gspx = ca * grx + sa * gry;
  T gspy = -sa * grx + ca * gry;
  // sp = l - s*nl
  T glx = gspx, gly = gspy;
  T gs = -(nlx * gspx + nly * gspy) - gov;  // overlap = reach - s
  T gnlx = -s * gspx + (ca * gnx + sa * gny);
  T gnly = -s * gspy + (-sa * gnx + ca * gny);
  if (ext) {
    // nl = o / s, s = sqrt(od2), o = l - clamp(l)
    T gox = gnlx * is, goy = gnly * is;
    gs -= (gnlx * nlx + gnly * nly) * is;
    T god2 = gs * T(0.5) * is;
    gox += T(2) * ox * god2;
    goy += T(2) * oy * god2;
    glx += gox - (clamp_pass(lx, -o.hx, o.hx) ? gox : T(0));
    gly += goy - (clamp_pass(ly, -o.hy, o.hy) ? goy : T(0));
  } else if (use_x) {
    glx += (lx < T(0) ? -gs : gs);  // s = |lx| - hx
  } else {
    gly += (ly < T(0) ? -gs : gs);
  }
  // l = R^T d
  gpx += ca * glx - sa * gly;
  gpy += sa * glx + ca * gly;
}

// Force on an agent (radius ra, inverse implicit denominator) from one obstacle.
template <typename T>
__device__ __forceinline__ void obstacle_force(T px, T py, T vx, T vy, T ra, T inv_denom, const Obs<T>& o,
                                               const WorldC<T>& W, T& fx, T& fy) {
  fx = T(0);
  fy = T(0);
  if (bounds_apart(px - o.cx, py - o.cy, ra + W.margin + o.bound)) return;
  if (o.type == SHAPE_BOX) {
    box_force(px, py, vx, vy, o, ra + W.margin, inv_denom, W, fx, fy);
  } else if (o.type == SHAPE_SEGMENT) {
    T t = wclamp(dot2(px - o.cx, py - o.cy, o.ca, o.sa), -o.hx, o.hx);
    T qx = o.cx + t * o.ca, qy = o.cy + t * o.sa;
    T rx = qx - o.cx, ry = qy - o.cy;
    T vsx = o.vx + (-o.om * ry), vsy = o.vy + o.om * rx;
    pair_force(px - qx, py - qy, vx - vsx, vy - vsy, ra + o.r + W.margin, inv_denom, W, fx, fy);
  } else {
    pair_force(px - o.cx, py - o.cy, vx - o.vx, vy - o.vy, ra + o.r + W.margin, inv_denom, W, fx, fy);
  }
}

template <typename T>
__device__ __forceinline__ void obstacle_force_vjp(T px, T py, T vx, T vy, T ra, T inv_denom,
                                                   const Obs<T>& o, T gx, T gy, const WorldC<T>& W,
                                                   T& gpx, T& gpy, T& gvx, T& gvy) {
  if (bounds_apart(px - o.cx, py - o.cy, ra + W.margin + o.bound)) return;
  if (o.type == SHAPE_BOX) {
    box_force_vjp(px, py, vx, vy, o, ra + W.margin, inv_denom, gx, gy, W, gpx, gpy, gvx, gvy);
  } else if (o.type == SHAPE_SEGMENT) {
    T sproj = dot2(px - o.cx, py - o.cy, o.ca, o.sa);
    T t = wclamp(sproj, -o.hx, o.hx);
    T qx = o.cx + t * o.ca, qy = o.cy + t * o.sa;
    T rx = qx - o.cx, ry = qy - o.cy;
    T vsx = o.vx + (-o.om * ry), vsy = o.vy + o.om * rx;
    T gdx = T(0), gdy = T(0), grvx = T(0), grvy = T(0);
    pair_force_vjp(px - qx, py - qy, vx - vsx, vy - vsy, ra + o.r + W.margin, inv_denom, gx, gy, W,
                   gdx, gdy, grvx, grvy);
    gpx += gdx;
    gpy += gdy;
    gvx += grvx;
    gvy += grvy;
    // q enters through d = p - q and vs (via r = q - c)
    T gqx = -gdx, gqy = -gdy;
    T gvsx = -grvx, gvsy = -grvy;
    gqx += o.om * gvsy;    // vsy = vo_y + om*rx
    gqy += -o.om * gvsx;   // vsx = vo_x - om*ry
    T gt = dot2(gqx, gqy, o.ca, o.sa);
    if (clamp_pass(sproj, -o.hx, o.hx)) {
      gpx += gt * o.ca;
      gpy += gt * o.sa;
    }
  } else {
    T gdx = T(0), gdy = T(0), grvx = T(0), grvy = T(0);
    pair_force_vjp(px - o.cx, py - o.cy, vx - o.vx, vy - o.vy, ra + o.r + W.margin, inv_denom, gx, gy,
                   W, gdx, gdy, grvx, grvy);
    gpx += gdx;
    gpy += gdy;
    gvx += grvx;
    gvy += grvy;
  }
}

// ------------------------------------------------------------------------ walls
// Penetrations of the four walls (left, right, bottom, top); inward normals +x, -x, +y, -y.
template <typename T>
__device__ __forceinline__ void wall_pens(T px, T py, T reach, const WorldC<T>& W, T& pl, T& pr,
                                          T& pb, T& pt) {
  pl = reach - (px - W.bx0);
  pr = reach - (W.bx1 - px);
  pb = reach - (py - W.by0);
  pt = reach - (W.by1 - py);
}

// Four soft walls. Most warps have some lane at a wall on most steps, so a branch per
// wall would be taken anyway: without depth saturation every wall's coefficient is
// computed and masked by its penetration sign (no divergence). The accumulation order
// matches the reference (left, right into fx; bottom, top into fy).
// The four walls without depth saturation (max_overlap == 0), branch-free.
template <typename T>
__device__ __forceinline__ void wall_force_lin(T px, T py, T vx, T vy, T ra, T inv_denom,
                                               const WorldC<T>& W, T& fx, T& fy) {
  T pl, pr, pb, pt;
  wall_pens(px, py, ra + W.margin, W, pl, pr, pb, pt);
  const T cl = wmax_c(nc_num(pl, vx, W) * inv_denom, T(0));
  const T cr = wmax_c(nc_num(pr, (-vx), W) * inv_denom, T(0));
  const T cb = wmax_c(nc_num(pb, vy, W) * inv_denom, T(0));
  const T ct = wmax_c(nc_num(pt, (-vy), W) * inv_denom, T(0));
  fx = (pl > T(0) ? cl : T(0)) + (pr > T(0) ? -cr : T(0));
  fy = (pb > T(0) ? cb : T(0)) + (pt > T(0) ? -ct : T(0));
}
// The VJP of wall_force_lin in two parts: the factors dx = dL/d(numerators) of the x
// walls (right minus left) and dy, which need only the agent's own state and force
// cotangent, and their application to the state gradient (wall_lin_vjp_apply).
template <typename T>
__device__ __forceinline__ void wall_lin_vjp_factors(T px, T py, T vx, T vy, T ra, T inv_denom,
                                                     T gx, T gy, const WorldC<T>& W, T& dx,
                                                     T& dy) {
  T pl, pr, pb, pt;
  wall_pens(px, py, ra + W.margin, W, pl, pr, pb, pt);
  // d(coefficient)/d(numerator) = inv_denom on the active side of max(x, 0)
  const bool al = pl > T(0) && nc_num(pl, vx, W) * inv_denom > T(0);
  const bool ar = pr > T(0) && nc_num(pr, (-vx), W) * inv_denom > T(0);
  const bool ab = pb > T(0) && nc_num(pb, vy, W) * inv_denom > T(0);
  const bool at = pt > T(0) && nc_num(pt, (-vy), W) * inv_denom > T(0);
  const T nl = al ? gx * inv_denom : T(0);   // left:   f_x += c_l
  const T nr = ar ? -gx * inv_denom : T(0);  // right:  f_x -= c_r
  const T nb = ab ? gy * inv_denom : T(0);
  const T nt = at ? -gy * inv_denom : T(0);
  dx = nr - nl;
  dy = nt - nb;
}
// numerator k*pen - c*vn; pen_l = reach - px + x0 (d/dpx = -1), pen_r (+1); vn = +-v
template <typename T>
__device__ __forceinline__ void wall_lin_vjp_apply(T dx, T dy, const WorldC<T>& W, T& gpx, T& gpy,
                                                   T& gvx, T& gvy) {
  gpx = Num<T>::fma_(W.k, dx, gpx);
  gvx = Num<T>::fma_(W.c, dx, gvx);
  gpy = Num<T>::fma_(W.k, dy, gpy);
  gvy = Num<T>::fma_(W.c, dy, gvy);
}

template <typename T>
__device__ __forceinline__ void wall_force(T px, T py, T vx, T vy, T ra, T inv_denom,
                                           const WorldC<T>& W, T& fx, T& fy) {
  T pl, pr, pb, pt;
  wall_pens(px, py, ra + W.margin, W, pl, pr, pb, pt);
  if (W.max_overlap > T(0)) {
    fx = T(0);
    fy = T(0);
    if (pl > T(0)) fx = fx + normal_coeff(pl, vx, inv_denom, W);
    if (pr > T(0)) fx = fx + (-normal_coeff(pr, -vx, inv_denom, W));
    if (pb > T(0)) fy = fy + normal_coeff(pb, vy, inv_denom, W);
    if (pt > T(0)) fy = fy + (-normal_coeff(pt, -vy, inv_denom, W));
    return;
  }
  wall_force_lin(px, py, vx, vy, ra, inv_denom, W, fx, fy);
}

template <typename T>
__device__ __forceinline__ void wall_force_vjp(T px, T py, T vx, T vy, T ra, T inv_denom, T gx, T gy,
                                               const WorldC<T>& W, T& gpx, T& gpy, T& gvx, T& gvy) {
  T pl, pr, pb, pt;
  wall_pens(px, py, ra + W.margin, W, pl, pr, pb, pt);
  if (W.max_overlap > T(0)) {
    T gov, gvn;
    if (pl > T(0)) {
      normal_coeff_vjp(pl, vx, inv_denom, gx, W, gov, gvn);
      gpx -= gov;
      gvx += gvn;
    }
    if (pr > T(0)) {
      normal_coeff_vjp(pr, -vx, inv_denom, -gx, W, gov, gvn);
      gpx += gov;
      gvx -= gvn;
    }
    if (pb > T(0)) {
      normal_coeff_vjp(pb, vy, inv_denom, gy, W, gov, gvn);
      gpy -= gov;
      gvy += gvn;
    }
    if (pt > T(0)) {
      normal_coeff_vjp(pt, -vy, inv_denom, -gy, W, gov, gvn);
      gpy += gov;
      gvy -= gvn;
    }
    return;
  }
  T dx, dy;
  wall_lin_vjp_factors(px, py, vx, vy, ra, inv_denom, gx, gy, W, dx, dy);
  wall_lin_vjp_apply(dx, dy, W, gpx, gpy, gvx, gvy);
}

// ------------------------------------------------------------------- integrate
// clamp_norm(v, L) = v * (L / max(|v|, L)): the scale is exactly 1 while |v|^2 <= L^2,
// else L * rsqrt(|v|^2).
template <typename T>
__device__ __forceinline__ void clamp_norm(T x, T y, T L, T& ox, T& oy) {
  const T n2 = dot2(x, y, x, y);
  const T sc = (n2 > L * L) ? L * Num<T>::rsqrt_(n2) : T(1);
  ox = x * sc;
  oy = y * sc;
}
template <typename T>
__device__ __forceinline__ void clamp_norm_vjp(T x, T y, T L, T gx, T gy, T& rx, T& ry) {
  const T n2 = dot2(x, y, x, y);
  if (n2 > L * L) {
    const T inv = Num<T>::rsqrt_(n2);
    const T sc = L * inv;
    const T gn = -dot2(gx, gy, x, y) * sc * inv * inv;  // d/dn of L/n times (g . v) / n
    rx = Num<T>::fma_(x, gn, gx * sc);
    ry = Num<T>::fma_(y, gn, gy * sc);
  } else {
    rx = gx;
    ry = gy;
  }
}

// |v| with Warp's adjoint convention (zero gradient at the zero vector).
template <typename T> __device__ __forceinline__ T norm2(T x, T y) {
  const T n2 = dot2(x, y, x, y);
  return n2 > T(0) ? n2 * Num<T>::rsqrt_(n2) : T(0);
}

// SERVO (diff-drive): the VELOCITY command the rate-limited servo delivers this substep.
template <typename T>
__device__ __forceinline__ void servo_cmd(T a0, T a1, T s, T w, const AgentP<T>& P, T dt, T& c0, T& c1) {
  T tv = wclamp(a0, -P.max_speed, P.max_speed) * P.gain_v;
  T tw = wclamp(a1, -P.max_ang_vel, P.max_ang_vel) * P.gain_w;
  T dv = P.max_accel * dt, dw = P.max_ang_accel * dt;
  c0 = s + wclamp(tv - s, -dv, dv);
  c1 = w + wclamp(tw - w, -dw, dw);
}
template <typename T>
__device__ __forceinline__ void servo_cmd_vjp(T a0, T a1, T s, T w, const AgentP<T>& P, T dt, T gc0,
                                              T gc1, T& ga0, T& ga1, T& gs, T& gw) {
  T tv = wclamp(a0, -P.max_speed, P.max_speed) * P.gain_v;
  T tw = wclamp(a1, -P.max_ang_vel, P.max_ang_vel) * P.gain_w;
  T dv = P.max_accel * dt, dw = P.max_ang_accel * dt;
  gs += gc0;
  gw += gc1;
  T gd0 = clamp_pass(tv - s, -dv, dv) ? gc0 : T(0);
  T gd1 = clamp_pass(tw - w, -dw, dw) ? gc1 : T(0);
  gs -= gd0;
  gw -= gd1;
  ga0 += clamp_pass(a0, -P.max_speed, P.max_speed) ? gd0 * P.gain_v : T(0);
  ga1 += clamp_pass(a1, -P.max_ang_vel, P.max_ang_vel) ? gd1 * P.gain_w : T(0);
}

// One semi-implicit Euler substep of a 2-D agent under force (fx, fy).
// p_new = p + v_new * dt is an explicit fma in both directions, so the adjoint
// reconstructs the pre-clamp position bit for bit from the stored output velocity.
// Hard clamp of the new position (dynamics/kernels.py:80-99, clamp_footprint): a disc is
// inset by its radius, a box (kBox worlds) by its support extents at the new heading.
template <typename T, bool kBox>
__device__ __forceinline__ void footprint_extents(T th, const AgentP<T>& P, T& ex, T& ey);
template <typename T, bool kBox>
__device__ __forceinline__ void clamp_footprint(Agent<T>& out, const AgentP<T>& P, const WorldC<T>& W) {
  T ex, ey;
  footprint_extents<T, kBox>(out.th, P, ex, ey);
  out.px = wclamp(out.px, W.bx0 + ex, W.bx1 - ex);
  out.py = wclamp(out.py, W.by0 + ey, W.by1 - ey);
}

// Adjoint of the box footprint clamp beyond the position gate: Warp's clamp adjoint sends
// a clamped coordinate's gradient to its active bound (lo = b0 + e, hi = b1 - e), and the
// support extents e = hx|cos| + hy|sin| (x), hx|sin| + hy|cos| (y) carry it into the new
// heading th (abs with slope +1 at zero).
template <typename T>
__device__ __forceinline__ void box_clamp_vjp(int sidex, int sidey, T th, const AgentP<T>& P, T gpx,
                                              T gpy, T& gth) {
  const T gex = sidex < 0 ? gpx : (sidex > 0 ? -gpx : T(0));
  const T gey = sidey < 0 ? gpy : (sidey > 0 ? -gpy : T(0));
  const T c = Num<T>::cos_(th), s = Num<T>::sin_(th);
  const T sc = c < T(0) ? T(-1) : T(1), ss = s < T(0) ? T(-1) : T(1);
  const T dex = P.hx * (sc * -s) + P.hy * (ss * c);
  const T dey = P.hx * (ss * c) + P.hy * (sc * -s);
  gth += gex * dex + gey * dey;
}
// Support extents of the footprint at heading th (a disc: its radius).
template <typename T, bool kBox>
__device__ __forceinline__ void footprint_extents(T th, const AgentP<T>& P, T& ex, T& ey) {
  ex = P.radius;
  ey = P.radius;
  if (kBox && P.box) {
    const T ca = fabs(Num<T>::cos_(th)), sa = fabs(Num<T>::sin_(th));
    ex = P.hx * ca + P.hy * sa;
    ey = P.hx * sa + P.hy * ca;
  }
}

template <typename T, bool kBox = false>
__device__ __forceinline__ void integrate_fwd(const Agent<T>& in, T a0, T a1, T fx, T fy,
                                              const AgentP<T>& P, const WorldC<T>& W, Agent<T>& out) {
  const T dt = W.dt;
  int mode = P.mode;
  if (mode == MODE_SERVO) {
    servo_cmd(a0, a1, in.s, in.w, P, dt, a0, a1);
    mode = MODE_VELOCITY;
  }
  const T dvx = fx * P.dt_over_m, dvy = fy * P.dt_over_m;
  if (P.tag == TAG_HOLONOMIC) {
    T vx, vy;
    if (mode == MODE_VELOCITY) {
      clamp_norm(a0, a1, P.max_speed, vx, vy);
    } else {
      T ax, ay;
      clamp_norm(a0, a1, P.max_accel, ax, ay);
      clamp_norm(Num<T>::fma_(ax, dt, in.vx), Num<T>::fma_(ay, dt, in.vy), P.max_speed, vx, vy);
    }
    vx = Num<T>::fma_(fx, P.dt_over_m, vx);
    vy = Num<T>::fma_(fy, P.dt_over_m, vy);
    out.px = Num<T>::fma_(vx, dt, in.px);
    out.py = Num<T>::fma_(vy, dt, in.py);
    out.th = in.th;
    out.vx = vx;
    out.vy = vy;
    out.s = norm2(vx, vy);
    out.w = T(0);
  } else if (P.tag == TAG_DIFF_DRIVE) {
    T sn, wn;
    if (mode == MODE_VELOCITY) {
      sn = wclamp(a0, -P.max_speed, P.max_speed);
      wn = wclamp(a1, -P.max_ang_vel, P.max_ang_vel);
    } else {
      T acc = wclamp(a0, -P.max_accel, P.max_accel);
      T alp = wclamp(a1, -P.max_ang_accel, P.max_ang_accel);
      sn = wclamp(Num<T>::fma_(acc, dt, in.s), -P.max_speed, P.max_speed);
      wn = wclamp(Num<T>::fma_(alp, dt, in.w), -P.max_ang_vel, P.max_ang_vel);
    }
    T c = Num<T>::cos_(in.th), sn_ = Num<T>::sin_(in.th);
    T vx = sn * c + dvx, vy = sn * sn_ + dvy;
    out.px = Num<T>::fma_(vx, dt, in.px);
    out.py = Num<T>::fma_(vy, dt, in.py);
    out.th = Num<T>::fma_(wn, dt, in.th);
    out.vx = vx;
    out.vy = vy;
    out.s = sn;
    out.w = wn;
  } else {  // TAG_BICYCLE (host rejects other tags)
    T acc = wclamp(a0, -P.max_accel, P.max_accel);
    T delta = wclamp(a1, -P.max_steer, P.max_steer);
    T sn = wclamp(Num<T>::fma_(acc, dt, in.s), P.min_speed, P.max_speed);
    T wb = P.l_f + P.l_r;
    T td = Num<T>::tan_(delta);
    T beta = Num<T>::atan_(td * P.l_r / wb);
    T ang = in.th + beta;
    T vx = sn * Num<T>::cos_(ang) + dvx, vy = sn * Num<T>::sin_(ang) + dvy;
    T wn = sn / wb * Num<T>::cos_(beta) * td;
    out.px = Num<T>::fma_(vx, dt, in.px);
    out.py = Num<T>::fma_(vy, dt, in.py);
    out.th = Num<T>::fma_(wn, dt, in.th);
    out.vx = vx;
    out.vy = vy;
    out.s = sn;
    out.w = wn;
  }
  if (W.bounds_mode == BOUNDS_CLAMP) clamp_footprint<T, kBox>(out, P, W);
}

// Adjoint of integrate_fwd. `out` is the substep's stored output (only its velocity
// and speed are read). Writes the gradients that flow straight to the substep input
// into gin (overwriting), the force cotangent into (gfx, gfy) and adds the action
// cotangent into (ga0, ga1).
template <typename T, bool kBox = false>
__device__ __forceinline__ void integrate_vjp(const Agent<T>& in, T a0, T a1, const Agent<T>& out,
                                              const Agent<T>& g_out, const AgentP<T>& P,
                                              const WorldC<T>& W, Agent<T>& gin, T& gfx, T& gfy,
                                              T& ga0, T& ga1) {
  const T dt = W.dt;
  Agent<T> g = g_out;
  gin.px = gin.py = gin.th = gin.vx = gin.vy = gin.s = gin.w = T(0);
  // bounds clamp on the new position
  T gpx = g.px, gpy = g.py;
  if (W.bounds_mode == BOUNDS_CLAMP) {
    T pxn = Num<T>::fma_(out.vx, dt, in.px), pyn = Num<T>::fma_(out.vy, dt, in.py);
    T ex, ey;
    footprint_extents<T, kBox>(out.th, P, ex, ey);
    const T lox = W.bx0 + ex, hix = W.bx1 - ex, loy = W.by0 + ey, hiy = W.by1 - ey;
    if (!clamp_pass(pxn, lox, hix)) gpx = T(0);
    if (!clamp_pass(pyn, loy, hiy)) gpy = T(0);
    if (kBox && P.box)
      box_clamp_vjp(pxn < lox ? -1 : (pxn > hix ? 1 : 0), pyn < loy ? -1 : (pyn > hiy ? 1 : 0),
                    out.th, P, g.px, g.py, g.th);
  }
  int mode = P.mode;
  T c0 = a0, c1 = a1;
  if (mode == MODE_SERVO) {
    servo_cmd(a0, a1, in.s, in.w, P, dt, c0, c1);
    mode = MODE_VELOCITY;
  }
  T gc0 = T(0), gc1 = T(0);
  // p_new = p + v_out*dt, v_out = vel-level + F*dt/m
  gin.px = gpx;
  gin.py = gpy;
  T gvx = Num<T>::fma_(gpx, dt, g.vx), gvy = Num<T>::fma_(gpy, dt, g.vy);
  if (P.tag == TAG_HOLONOMIC) {
    // s_out = |v_new|
    const T n2 = dot2(out.vx, out.vy, out.vx, out.vy);
    if (n2 > T(0)) {
      const T q = g.s * Num<T>::rsqrt_(n2);
      gvx = Num<T>::fma_(out.vx, q, gvx);
      gvy = Num<T>::fma_(out.vy, q, gvy);
    }
    gin.th = g.th;
    gfx = gvx * P.dt_over_m;
    gfy = gvy * P.dt_over_m;
    if (mode == MODE_VELOCITY) {
      clamp_norm_vjp(c0, c1, P.max_speed, gvx, gvy, gc0, gc1);
    } else {
      T ax, ay;
      clamp_norm(c0, c1, P.max_accel, ax, ay);
      T ux = Num<T>::fma_(ax, dt, in.vx), uy = Num<T>::fma_(ay, dt, in.vy);
      T gux, guy;
      clamp_norm_vjp(ux, uy, P.max_speed, gvx, gvy, gux, guy);
      gin.vx = gux;
      gin.vy = guy;
      clamp_norm_vjp(c0, c1, P.max_accel, gux * dt, guy * dt, gc0, gc1);
    }
  } else if (P.tag == TAG_DIFF_DRIVE) {
    T c = Num<T>::cos_(in.th), sn_ = Num<T>::sin_(in.th);
    T sn = out.s;
    gfx = gvx * P.dt_over_m;
    gfy = gvy * P.dt_over_m;
    T gsn = g.s + dot2(gvx, gvy, c, sn_);
    gin.th = g.th + sn * (c * gvy - sn_ * gvx);
    T gwn = g.w + g.th * dt;
    if (mode == MODE_VELOCITY) {
      gc0 = clamp_pass(c0, -P.max_speed, P.max_speed) ? gsn : T(0);
      gc1 = clamp_pass(c1, -P.max_ang_vel, P.max_ang_vel) ? gwn : T(0);
    } else {
      T acc = wclamp(c0, -P.max_accel, P.max_accel);
      T alp = wclamp(c1, -P.max_ang_accel, P.max_ang_accel);
      T us = Num<T>::fma_(acc, dt, in.s), uw = Num<T>::fma_(alp, dt, in.w);
      T gus = clamp_pass(us, -P.max_speed, P.max_speed) ? gsn : T(0);
      T guw = clamp_pass(uw, -P.max_ang_vel, P.max_ang_vel) ? gwn : T(0);
      gin.s = gus;
      gin.w = guw;
      gc0 = clamp_pass(c0, -P.max_accel, P.max_accel) ? gus * dt : T(0);
      gc1 = clamp_pass(c1, -P.max_ang_accel, P.max_ang_accel) ? guw * dt : T(0);
    }
  } else {  // bicycle
    T acc = wclamp(c0, -P.max_accel, P.max_accel);
    T delta = wclamp(c1, -P.max_steer, P.max_steer);
    T us = Num<T>::fma_(acc, dt, in.s);
    T sn = out.s;
    T wb = P.l_f + P.l_r;
    T td = Num<T>::tan_(delta);
    T z = td * P.l_r / wb;
    T beta = Num<T>::atan_(z);
    T ang = in.th + beta;
    T ca = Num<T>::cos_(ang), sa = Num<T>::sin_(ang);
    T cb = Num<T>::cos_(beta), sb = Num<T>::sin_(beta);
    gfx = gvx * P.dt_over_m;
    gfy = gvy * P.dt_over_m;
    T gwn = g.w + g.th * dt;
    T gsn = g.s + dot2(gvx, gvy, ca, sa);
    T gang = sn * (ca * gvy - sa * gvx);
    gin.th = g.th + gang;
    T gbeta = gang;
    // wn = ((sn / wb) * cos(beta)) * tan(delta)
    T q = sn / wb;
    gsn += gwn * td * cb / wb;
    gbeta += -gwn * td * q * sb;
    T sec2 = T(1) + td * td;
    T gdelta = gwn * q * cb * sec2;
    // beta = atan(z), z = tan(delta) * l_r / wb
    T gz = gbeta / (T(1) + z * z);
    gdelta += gz * P.l_r / wb * sec2;
    T gus = clamp_pass(us, P.min_speed, P.max_speed) ? gsn : T(0);
    gin.s = gus;
    gc0 = clamp_pass(c0, -P.max_accel, P.max_accel) ? gus * dt : T(0);
    gc1 = clamp_pass(c1, -P.max_steer, P.max_steer) ? gdelta : T(0);
  }
  if (P.mode == MODE_SERVO) {
    T gs = T(0), gw = T(0);
    servo_cmd_vjp(a0, a1, in.s, in.w, P, dt, gc0, gc1, ga0, ga1, gs, gw);
    gin.s += gs;
    gin.w += gw;
  } else {
    ga0 += gc0;
    ga1 += gc1;
  }
}

// ------------------------------------------------------------------- RK4
// Classic RK4 over the 2-D models' independent states (swarp/dynamics/kernels.py:420-793):
// the derivative holds the actions; velocity-mode commands first set the velocity-level
// state; the limits apply to the combined result; the contact force enters as the Euler
// path's F/m dt on the velocity (and F/m dt^2 on the pose). The adjoint recomputes the
// four stages from the substep input and walks them backwards.
template <typename T>
__device__ __forceinline__ Agent<T> rk4_axpy(const Agent<T>& x, const Agent<T>& k, T h) {
  return Agent<T>{x.px + k.px * h, x.py + k.py * h, x.th + k.th * h, x.vx + k.vx * h,
                  x.vy + k.vy * h, x.s + k.s * h, x.w + k.w * h};
}

// Steering terms of the bicycle (constant over a step): tan(delta), beta, wheelbase.
template <typename T> struct Steer {
  T td, beta, cb, sb, wb;
};
template <typename T>
__device__ __forceinline__ Steer<T> steer_of(T c1, const AgentP<T>& P) {
  Steer<T> q;
  q.wb = P.l_f + P.l_r;
  q.td = Num<T>::tan_(wclamp(c1, -P.max_steer, P.max_steer));
  q.beta = Num<T>::atan_(q.td * P.l_r / q.wb);
  q.cb = Num<T>::cos_(q.beta);
  q.sb = Num<T>::sin_(q.beta);
  return q;
}

template <typename T>
__device__ __forceinline__ Agent<T> rk4_deriv(const Agent<T>& x, T c0, T c1, int mode,
                                               const AgentP<T>& P, const Steer<T>& q) {
  Agent<T> d{T(0), T(0), T(0), T(0), T(0), T(0), T(0)};
  if (P.tag == TAG_HOLONOMIC) {
    d.px = x.vx;
    d.py = x.vy;
    if (mode != MODE_VELOCITY) clamp_norm(c0, c1, P.max_accel, d.vx, d.vy);
  } else if (P.tag == TAG_DIFF_DRIVE) {
    d.px = x.s * Num<T>::cos_(x.th);
    d.py = x.s * Num<T>::sin_(x.th);
    d.th = x.w;
    if (mode != MODE_VELOCITY) {
      d.s = wclamp(c0, -P.max_accel, P.max_accel);
      d.w = wclamp(c1, -P.max_ang_accel, P.max_ang_accel);
    }
  } else {
    const T ang = x.th + q.beta;
    d.px = x.s * Num<T>::cos_(ang);
    d.py = x.s * Num<T>::sin_(ang);
    d.th = x.s / q.wb * q.cb * q.td;
    d.s = wclamp(c0, -P.max_accel, P.max_accel);
  }
  return d;
}

// Adjoint of rk4_deriv at x for the cotangent gk: adds into gx, the command cotangents
// (gc0, gc1) and, for the bicycle, the cotangents of beta and tan(delta).
template <typename T>
__device__ __forceinline__ void rk4_deriv_vjp(const Agent<T>& x, const Agent<T>& gk, T c0, T c1,
                                              int mode, const AgentP<T>& P, const Steer<T>& q,
                                              Agent<T>& gx, T& gc0, T& gc1, T& gbeta, T& gtd) {
  if (P.tag == TAG_HOLONOMIC) {
    gx.vx += gk.px;
    gx.vy += gk.py;
    if (mode != MODE_VELOCITY) {
      T r0, r1;
      clamp_norm_vjp(c0, c1, P.max_accel, gk.vx, gk.vy, r0, r1);
      gc0 += r0;
      gc1 += r1;
    }
  } else if (P.tag == TAG_DIFF_DRIVE) {
    const T c = Num<T>::cos_(x.th), sn = Num<T>::sin_(x.th);
    gx.s += gk.px * c + gk.py * sn;
    gx.th += x.s * (c * gk.py - sn * gk.px);
    gx.w += gk.th;
    if (mode != MODE_VELOCITY) {
      if (clamp_pass(c0, -P.max_accel, P.max_accel)) gc0 += gk.s;
      if (clamp_pass(c1, -P.max_ang_accel, P.max_ang_accel)) gc1 += gk.w;
    }
  } else {
    const T ang = x.th + q.beta;
    const T ca = Num<T>::cos_(ang), sa = Num<T>::sin_(ang);
    // dth = ((s / wb) * cos(beta)) * tan(delta)
    gx.s += gk.px * ca + gk.py * sa + gk.th * q.td * q.cb / q.wb;
    const T gang = x.s * (ca * gk.py - sa * gk.px);
    gx.th += gang;
    gbeta += gang - gk.th * q.td * (x.s / q.wb) * q.sb;
    gtd += gk.th * (x.s / q.wb) * q.cb;
    if (clamp_pass(c0, -P.max_accel, P.max_accel)) gc0 += gk.s;
  }
}

// The four stages from the substep input: x (after the velocity-mode command), the
// stage states x2..x4, the slopes k1..k4 and the combined independent state xi.
template <typename T> struct Rk4Stages {
  Agent<T> x, x2, x3, x4, k1, k2, k3, k4, xi;
  T c0, c1;
  int mode;
  Steer<T> q;
};
template <typename T>
__device__ __forceinline__ void rk4_stages(const Agent<T>& in, T a0, T a1, const AgentP<T>& P,
                                           T dt, Rk4Stages<T>& R) {
  R.mode = P.mode;
  R.c0 = a0;
  R.c1 = a1;
  if (R.mode == MODE_SERVO) {
    servo_cmd(a0, a1, in.s, in.w, P, dt, R.c0, R.c1);
    R.mode = MODE_VELOCITY;
  }
  R.q = steer_of(R.c1, P);
  R.x = in;
  if (R.mode == MODE_VELOCITY) {
    if (P.tag == TAG_HOLONOMIC) {
      clamp_norm(R.c0, R.c1, P.max_speed, R.x.vx, R.x.vy);
    } else if (P.tag == TAG_DIFF_DRIVE) {
      R.x.s = wclamp(R.c0, -P.max_speed, P.max_speed);
      R.x.w = wclamp(R.c1, -P.max_ang_vel, P.max_ang_vel);
    }
  }
  const T h = dt * T(0.5), sixth = dt / T(6);
  R.k1 = rk4_deriv(R.x, R.c0, R.c1, R.mode, P, R.q);
  R.x2 = rk4_axpy(R.x, R.k1, h);
  R.k2 = rk4_deriv(R.x2, R.c0, R.c1, R.mode, P, R.q);
  R.x3 = rk4_axpy(R.x, R.k2, h);
  R.k3 = rk4_deriv(R.x3, R.c0, R.c1, R.mode, P, R.q);
  R.x4 = rk4_axpy(R.x, R.k3, dt);
  R.k4 = rk4_deriv(R.x4, R.c0, R.c1, R.mode, P, R.q);
  auto comb = [&](T x, T a, T b, T c, T d) { return x + (a + b * T(2) + c * T(2) + d) * sixth; };
  R.xi = Agent<T>{comb(R.x.px, R.k1.px, R.k2.px, R.k3.px, R.k4.px),
                  comb(R.x.py, R.k1.py, R.k2.py, R.k3.py, R.k4.py),
                  comb(R.x.th, R.k1.th, R.k2.th, R.k3.th, R.k4.th),
                  comb(R.x.vx, R.k1.vx, R.k2.vx, R.k3.vx, R.k4.vx),
                  comb(R.x.vy, R.k1.vy, R.k2.vy, R.k3.vy, R.k4.vy),
                  comb(R.x.s, R.k1.s, R.k2.s, R.k3.s, R.k4.s),
                  comb(R.x.w, R.k1.w, R.k2.w, R.k3.w, R.k4.w)};
}

template <typename T, bool kBox = false>
__device__ __forceinline__ void integrate_rk4_fwd(const Agent<T>& in, T a0, T a1, T fx, T fy,
                                                  const AgentP<T>& P, const WorldC<T>& W,
                                                  Agent<T>& out) {
  const T dt = W.dt;
  Rk4Stages<T> R;
  rk4_stages(in, a0, a1, P, dt, R);
  const Agent<T>& xi = R.xi;
  const T dvx = fx * P.dt_over_m, dvy = fy * P.dt_over_m;
  out.px = xi.px + dvx * dt;
  out.py = xi.py + dvy * dt;
  if (P.tag == TAG_HOLONOMIC) {
    T vx, vy;
    clamp_norm(xi.vx, xi.vy, P.max_speed, vx, vy);
    vx = vx + dvx;
    vy = vy + dvy;
    out.th = in.th;
    out.vx = vx;
    out.vy = vy;
    out.s = norm2(vx, vy);
    out.w = T(0);
  } else if (P.tag == TAG_DIFF_DRIVE) {
    const T so = wclamp(xi.s, -P.max_speed, P.max_speed);
    out.w = wclamp(xi.w, -P.max_ang_vel, P.max_ang_vel);
    out.th = xi.th;
    out.vx = so * Num<T>::cos_(xi.th) + dvx;
    out.vy = so * Num<T>::sin_(xi.th) + dvy;
    out.s = so;
  } else {
    const T so = wclamp(xi.s, P.min_speed, P.max_speed);
    const Steer<T>& q = R.q;
    out.th = xi.th;
    out.w = so / q.wb * q.cb * q.td;
    out.vx = so * Num<T>::cos_(xi.th + q.beta) + dvx;
    out.vy = so * Num<T>::sin_(xi.th + q.beta) + dvy;
    out.s = so;
  }
  if (W.bounds_mode == BOUNDS_CLAMP) clamp_footprint<T, kBox>(out, P, W);
}

// Adjoint of integrate_rk4_fwd (same contract as integrate_vjp: gin overwritten, force
// cotangent written, action cotangent added). `out` is the substep's stored output: the
// position clamp's side test uses it (strictly inside the interval: not clamped; on its
// boundary: the pre-clamp position rebuilt from the stored velocity decides).
template <typename T, bool kBox = false>
__device__ __forceinline__ void integrate_rk4_vjp(const Agent<T>& in, T a0, T a1, const Agent<T>& out,
                                                  const Agent<T>& g_out, const AgentP<T>& P,
                                                  const WorldC<T>& W, Agent<T>& gin, T& gfx, T& gfy,
                                                  T& ga0, T& ga1) {
  const T dt = W.dt;
  Agent<T> g = g_out;
  Rk4Stages<T> R;
  rk4_stages(in, a0, a1, P, dt, R);
  const Agent<T>& xi = R.xi;
  const Steer<T>& q = R.q;
  // ---- output map: cotangent of xi, of the force term and of the steering
  Agent<T> gxi{T(0), T(0), T(0), T(0), T(0), T(0), T(0)};
  T gc0 = T(0), gc1 = T(0), gbeta = T(0), gtd = T(0);
  T gpx = g.px, gpy = g.py;
  T vbx, vby;  // velocity without the force term
  if (P.tag == TAG_HOLONOMIC) {
    clamp_norm(xi.vx, xi.vy, P.max_speed, vbx, vby);
  } else if (P.tag == TAG_DIFF_DRIVE) {
    const T so = wclamp(xi.s, -P.max_speed, P.max_speed);
    vbx = so * Num<T>::cos_(xi.th);
    vby = so * Num<T>::sin_(xi.th);
  } else {
    const T so = wclamp(xi.s, P.min_speed, P.max_speed);
    vbx = so * Num<T>::cos_(xi.th + q.beta);
    vby = so * Num<T>::sin_(xi.th + q.beta);
  }
  if (W.bounds_mode == BOUNDS_CLAMP) {
    T ex, ey;
    footprint_extents<T, kBox>(out.th, P, ex, ey);
    const T lox = W.bx0 + ex, hix = W.bx1 - ex;
    const T loy = W.by0 + ey, hiy = W.by1 - ey;
    const T prex = xi.px + (out.vx - vbx) * dt, prey = xi.py + (out.vy - vby) * dt;
    const bool px_in = (out.px > lox && out.px < hix) || clamp_pass(prex, lox, hix);
    const bool py_in = (out.py > loy && out.py < hiy) || clamp_pass(prey, loy, hiy);
    if (!px_in) gpx = T(0);
    if (!py_in) gpy = T(0);
    // a clamped coordinate sits on its bound: below the upper one it is the lower one
    if (kBox && P.box)
      box_clamp_vjp(px_in ? 0 : (out.px < hix ? -1 : 1), py_in ? 0 : (out.py < hiy ? -1 : 1),
                    out.th, P, g.px, g.py, g.th);
  }
  gxi.px = gpx;
  gxi.py = gpy;
  // p = xi.p + dv * dt, v = vb + dv, dv = F * dt / m
  T gvx = g.vx, gvy = g.vy;
  if (P.tag == TAG_HOLONOMIC) {
    const T n2 = dot2(out.vx, out.vy, out.vx, out.vy);  // s = |v|
    if (n2 > T(0)) {
      const T qq = g.s * Num<T>::rsqrt_(n2);
      gvx += out.vx * qq;
      gvy += out.vy * qq;
    }
  }
  gfx = (gvx + gpx * dt) * P.dt_over_m;
  gfy = (gvy + gpy * dt) * P.dt_over_m;
  if (P.tag == TAG_HOLONOMIC) {
    clamp_norm_vjp(xi.vx, xi.vy, P.max_speed, gvx, gvy, gxi.vx, gxi.vy);
    gxi.th = g.th;  // heading passes through
  } else if (P.tag == TAG_DIFF_DRIVE) {
    const T so = wclamp(xi.s, -P.max_speed, P.max_speed);
    const T c = Num<T>::cos_(xi.th), sn = Num<T>::sin_(xi.th);
    const T gso = g.s + gvx * c + gvy * sn;
    gxi.th = g.th + so * (c * gvy - sn * gvx);
    gxi.s = clamp_pass(xi.s, -P.max_speed, P.max_speed) ? gso : T(0);
    gxi.w = clamp_pass(xi.w, -P.max_ang_vel, P.max_ang_vel) ? g.w : T(0);
  } else {
    const T so = wclamp(xi.s, P.min_speed, P.max_speed);
    const T ang = xi.th + q.beta;
    const T ca = Num<T>::cos_(ang), sa = Num<T>::sin_(ang);
    // w = ((so / wb) * cos(beta)) * tan(delta)
    const T gso = g.s + gvx * ca + gvy * sa + g.w * q.td * q.cb / q.wb;
    const T gang = so * (ca * gvy - sa * gvx);
    gxi.th = g.th + gang;
    gbeta += gang - g.w * q.td * (so / q.wb) * q.sb;
    gtd += g.w * (so / q.wb) * q.cb;
    gxi.s = clamp_pass(xi.s, P.min_speed, P.max_speed) ? gso : T(0);
  }
  // ---- combine: xi = x + (k1 + 2 k2 + 2 k3 + k4) * dt / 6
  const T h = dt * T(0.5), sixth = dt / T(6);
  auto scale = [](const Agent<T>& v, T c) {
    return Agent<T>{v.px * c, v.py * c, v.th * c, v.vx * c, v.vy * c, v.s * c, v.w * c};
  };
  auto add = [](Agent<T>& a, const Agent<T>& b) {
    a.px += b.px; a.py += b.py; a.th += b.th; a.vx += b.vx; a.vy += b.vy; a.s += b.s; a.w += b.w;
  };
  const Agent<T> gS = scale(gxi, sixth);
  Agent<T> gx = gxi;
  Agent<T> gk1 = gS, gk2 = scale(gS, T(2)), gk3 = scale(gS, T(2));
  const Agent<T> gk4 = gS;
  Agent<T> gst{T(0), T(0), T(0), T(0), T(0), T(0), T(0)};
  rk4_deriv_vjp(R.x4, gk4, R.c0, R.c1, R.mode, P, q, gst, gc0, gc1, gbeta, gtd);
  add(gx, gst);
  add(gk3, scale(gst, dt));
  gst = Agent<T>{T(0), T(0), T(0), T(0), T(0), T(0), T(0)};
  rk4_deriv_vjp(R.x3, gk3, R.c0, R.c1, R.mode, P, q, gst, gc0, gc1, gbeta, gtd);
  add(gx, gst);
  add(gk2, scale(gst, h));
  gst = Agent<T>{T(0), T(0), T(0), T(0), T(0), T(0), T(0)};
  rk4_deriv_vjp(R.x2, gk2, R.c0, R.c1, R.mode, P, q, gst, gc0, gc1, gbeta, gtd);
  add(gx, gst);
  add(gk1, scale(gst, h));
  gst = Agent<T>{T(0), T(0), T(0), T(0), T(0), T(0), T(0)};
  rk4_deriv_vjp(R.x, gk1, R.c0, R.c1, R.mode, P, q, gst, gc0, gc1, gbeta, gtd);
  add(gx, gst);
  // ---- velocity-mode command: it replaced the velocity-level input state
  gin = gx;
  if (R.mode == MODE_VELOCITY) {
    if (P.tag == TAG_HOLONOMIC) {
      T r0, r1;
      clamp_norm_vjp(R.c0, R.c1, P.max_speed, gx.vx, gx.vy, r0, r1);
      gc0 += r0;
      gc1 += r1;
      gin.vx = gin.vy = T(0);
    } else if (P.tag == TAG_DIFF_DRIVE) {
      if (clamp_pass(R.c0, -P.max_speed, P.max_speed)) gc0 += gx.s;
      if (clamp_pass(R.c1, -P.max_ang_vel, P.max_ang_vel)) gc1 += gx.w;
      gin.s = gin.w = T(0);
    }
  }
  // ---- steering: beta = atan(tan(delta) * l_r / wb), tan(delta) with delta = clamp(c1)
  if (P.tag == TAG_BICYCLE) {
    const T z = q.td * P.l_r / q.wb;
    gtd += gbeta / (T(1) + z * z) * P.l_r / q.wb;
    const T gdelta = gtd * (T(1) + q.td * q.td);
    if (clamp_pass(R.c1, -P.max_steer, P.max_steer)) gc1 += gdelta;
  }
  if (P.mode == MODE_SERVO) {
    T gs = T(0), gw = T(0);
    servo_cmd_vjp(a0, a1, in.s, in.w, P, dt, gc0, gc1, ga0, ga1, gs, gw);
    gin.s += gs;
    gin.w += gw;
  } else {
    ga0 += gc0;
    ga1 += gc1;
  }
}

}  // namespace swarp
