// The 6-DOF quadrotor drone (DynamicsModel.DRONE): forward substep and hand-derived VJP,
// semi-implicit Euler and classic RK4.
//
// Reference semantics (ddebenedittis/swarp):
//   rotor model, rates      swarp/dynamics/kernels.py:102-163 (_quat_rotate_vec, _quat_deriv,
//                           _drone_rates)
//   Euler branch            swarp/dynamics/kernels.py:349-369
//   RK4 branch              swarp/dynamics/kernels.py:494-508 (_deriv), 758-768 (combine)
// A "+" quadrotor: the four action slots are rotor thrusts clamped to [0, thrust_max];
// total thrust acts along body +z, roll/pitch torques come from opposing rotor pairs over
// the arm, yaw from the rotor reactions; attitude is an (x, y, z, w) unit quaternion
// (body to world) and the body rates follow Euler's equation with diagonal inertia. The
// drone contacts the 2-D world as a disc: the contact force enters its horizontal
// velocity as the 2-D models' F dt / m term; heading, speed and turn rate pass through.
#pragma once
#include "physics.cuh"

namespace swarp {

template <typename T> struct Drone {
  T z, vz, qx, qy, qz, qw, bx, by, bz;
};

// Rotor thrusts: the action slots clamped to [0, thrust_max].
template <typename T>
__device__ __forceinline__ void drone_thrusts(const T a[4], const AgentP<T>& P, T f[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = wclamp(a[i], T(0), P.tmax);
}

// World acceleration and body angular acceleration. The rotation of (0, 0, F) by q
// is v + w t + u x t with t = 2 u x v (u = (qx, qy, qz)), written out with its zero terms
// removed (each removed term is an exact zero in the reference's evaluation).
template <typename T>
__device__ __forceinline__ void drone_rates(const T f[4], T qx, T qy, T qz, T qw, T bx, T by, T bz,
                                            const AgentP<T>& P, T acc[3], T ang[3]) {
  const T F = f[0] + f[1] + f[2] + f[3];
  const T tx = T(2) * (qy * F), ty = T(2) * (-(qx * F));
  const T fwx = qw * tx - qz * ty;
  const T fwy = qw * ty + qz * tx;
  const T fwz = F + (qx * ty - qy * tx);
  acc[0] = fwx / P.mass;
  acc[1] = fwy / P.mass;
  acc[2] = fwz / P.mass - P.grav;
  const T taux = P.arm * (f[1] - f[3]);
  const T tauy = P.arm * (f[2] - f[0]);
  const T tauz = P.kappa * (f[0] - f[1] + f[2] - f[3]);
  ang[0] = (taux - (P.izz - P.iyy) * by * bz) / P.ixx;
  ang[1] = (tauy - (P.ixx - P.izz) * bz * bx) / P.iyy;
  ang[2] = (tauz - (P.iyy - P.ixx) * bx * by) / P.izz;
}

// VJP of drone_rates: cotangents (gacc, gang) -> adds into gf (thrusts), gq, gb.
template <typename T>
__device__ __forceinline__ void drone_rates_vjp(const T f[4], T qx, T qy, T qz, T qw, T bx, T by,
                                                T bz, const AgentP<T>& P, const T gacc[3],
                                                const T gang[3], T gf[4], T gq[4], T gb[3]) {
  const T F = f[0] + f[1] + f[2] + f[3];
  // fw = F (2(qw qy + qx qz), 2(qy qz - qw qx), 1 - 2(qx^2 + qy^2)), each a polynomial in q
  const T gx = gacc[0] / P.mass, gy = gacc[1] / P.mass, gz = gacc[2] / P.mass;
  const T F2 = T(2) * F;
  gq[0] += F2 * (gx * qz - gy * qw) - T(2) * F2 * gz * qx;
  gq[1] += F2 * (gx * qw + gy * qz) - T(2) * F2 * gz * qy;
  gq[2] += F2 * (gx * qx + gy * qy);
  gq[3] += F2 * (gx * qy - gy * qx);
  const T gF = T(2) * (gx * (qw * qy + qx * qz) + gy * (qy * qz - qw * qx)) +
               gz * (T(1) - T(2) * (qx * qx + qy * qy));
  // body rates
  const T hx = gang[0] / P.ixx, hy = gang[1] / P.iyy, hz = gang[2] / P.izz;
  const T cx = P.izz - P.iyy, cy = P.ixx - P.izz, cz = P.iyy - P.ixx;
  gb[0] += -(hy * cy * bz) - hz * cz * by;
  gb[1] += -(hx * cx * bz) - hz * cz * bx;
  gb[2] += -(hx * cx * by) - hy * cy * bx;
  const T gtx = P.arm * hx, gty = P.arm * hy, gtz = P.kappa * hz;
  gf[0] += gF - gty + gtz;
  gf[1] += gF + gtx - gtz;
  gf[2] += gF + gty + gtz;
  gf[3] += gF - gtx - gtz;
}

// qd = 0.5 q (x) (w, 0)
template <typename T>
__device__ __forceinline__ void quat_deriv(T qx, T qy, T qz, T qw, T wx, T wy, T wz, T d[4]) {
  d[0] = T(0.5) * (qw * wx + qy * wz - qz * wy);
  d[1] = T(0.5) * (qw * wy - qx * wz + qz * wx);
  d[2] = T(0.5) * (qw * wz + qx * wy - qy * wx);
  d[3] = T(0.5) * (-qx * wx - qy * wy - qz * wz);
}
template <typename T>
__device__ __forceinline__ void quat_deriv_vjp(T qx, T qy, T qz, T qw, T wx, T wy, T wz,
                                               const T gd[4], T gq[4], T gw[3]) {
  const T hx = T(0.5) * gd[0], hy = T(0.5) * gd[1], hz = T(0.5) * gd[2], hw = T(0.5) * gd[3];
  gq[0] += -hy * wz + hz * wy - hw * wx;
  gq[1] += hx * wz - hz * wx - hw * wy;
  gq[2] += -hx * wy + hy * wx - hw * wz;
  gq[3] += hx * wx + hy * wy + hz * wz;
  gw[0] += hx * qw + hy * qz - hz * qy - hw * qx;
  gw[1] += -hx * qz + hy * qw + hz * qx - hw * qy;
  gw[2] += hx * qy - hy * qx + hz * qw - hw * qz;
}

// Warp normalize of a 4-vector (zero for the zero vector) and its VJP.
template <typename T> __device__ __forceinline__ void normalize4(const T q[4], T n[4]) {
  const T n2 = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
  if (n2 > T(0)) {
    const T l = Num<T>::sqrt_(n2);
#pragma unroll
    for (int i = 0; i < 4; ++i) n[i] = q[i] / l;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) n[i] = T(0);
  }
}
template <typename T>
__device__ __forceinline__ void normalize4_vjp(const T q[4], const T g[4], T gq[4]) {
  const T n2 = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
  if (!(n2 > T(0))) return;
  const T l = Num<T>::sqrt_(n2);
  T n[4], dn = T(0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    n[i] = q[i] / l;
    dn += n[i] * g[i];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) gq[i] += (g[i] - n[i] * dn) / l;
}

template <typename T>
__device__ __forceinline__ void drone_clamp(T& px, T& py, const AgentP<T>& P, const WorldC<T>& W) {
  if (W.bounds_mode != BOUNDS_CLAMP) return;
  px = wclamp(px, W.bx0 + P.radius, W.bx1 - P.radius);
  py = wclamp(py, W.by0 + P.radius, W.by1 - P.radius);
}

// ------------------------------------------------------------------ Euler
// Rates and velocities first, then the attitude with the new rates and the position with
// the new velocities. `a` are the four action slots (after the servo rewrite of 0/1).
template <typename T>
__device__ __forceinline__ void drone_euler_fwd(const Agent<T>& in, const Drone<T>& d,
                                                const T a[4], T fx, T fy, const AgentP<T>& P,
                                                const WorldC<T>& W, Agent<T>& out,
                                                Drone<T>& dout) {
  const T dt = W.dt;
  T f[4], acc[3], ang[3];
  drone_thrusts(a, P, f);
  drone_rates(f, d.qx, d.qy, d.qz, d.qw, d.bx, d.by, d.bz, P, acc, ang);
  dout.bx = d.bx + ang[0] * dt;
  dout.by = d.by + ang[1] * dt;
  dout.bz = d.bz + ang[2] * dt;
  dout.vz = d.vz + acc[2] * dt;
  const T vx = in.vx + acc[0] * dt + fx * P.dt_over_m;
  const T vy = in.vy + acc[1] * dt + fy * P.dt_over_m;
  T qd[4];
  quat_deriv(d.qx, d.qy, d.qz, d.qw, dout.bx, dout.by, dout.bz, qd);
  const T qu[4] = {d.qx + qd[0] * dt, d.qy + qd[1] * dt, d.qz + qd[2] * dt, d.qw + qd[3] * dt};
  T qn[4];
  normalize4(qu, qn);
  dout.qx = qn[0];
  dout.qy = qn[1];
  dout.qz = qn[2];
  dout.qw = qn[3];
  out.px = in.px + vx * dt;
  out.py = in.py + vy * dt;
  dout.z = d.z + dout.vz * dt;
  out.th = in.th;
  out.vx = vx;
  out.vy = vy;
  out.s = in.s;
  out.w = in.w;
  drone_clamp(out.px, out.py, P, W);
}

// Adjoint of drone_euler_fwd (recomputes its intermediates). `out` is the substep's stored
// output (its velocity rebuilds the pre-clamp position exactly); g/gd: cotangents of the
// outputs. Writes the input cotangents into gin/gdin (overwriting) and adds the force and
// action cotangents into gfx, gfy, ga.
template <typename T>
__device__ __forceinline__ void drone_euler_vjp(const Agent<T>& in, const Drone<T>& d,
                                                const T a[4], const Agent<T>& out,
                                                const Agent<T>& g, const Drone<T>& gd,
                                                const AgentP<T>& P, const WorldC<T>& W,
                                                Agent<T>& gin, Drone<T>& gdin, T& gfx, T& gfy,
                                                T ga[4]) {
  const T dt = W.dt;
  T f[4], acc[3], ang[3];
  drone_thrusts(a, P, f);
  drone_rates(f, d.qx, d.qy, d.qz, d.qw, d.bx, d.by, d.bz, P, acc, ang);
  const T nb[3] = {d.bx + ang[0] * dt, d.by + ang[1] * dt, d.bz + ang[2] * dt};
  T qd[4];
  quat_deriv(d.qx, d.qy, d.qz, d.qw, nb[0], nb[1], nb[2], qd);
  const T qu[4] = {d.qx + qd[0] * dt, d.qy + qd[1] * dt, d.qz + qd[2] * dt, d.qw + qd[3] * dt};
  T gpx = g.px, gpy = g.py;
  if (W.bounds_mode == BOUNDS_CLAMP) {
    if (!clamp_pass(in.px + out.vx * dt, W.bx0 + P.radius, W.bx1 - P.radius)) gpx = T(0);
    if (!clamp_pass(in.py + out.vy * dt, W.by0 + P.radius, W.by1 - P.radius)) gpy = T(0);
  }
  // p = p_in + v dt, z = z_in + vz dt; v = v_in + acc dt + F dt / m, vz = vz_in + acc_z dt
  const T gvx = g.vx + gpx * dt, gvy = g.vy + gpy * dt, gvz = gd.vz + gd.z * dt;
  gin = Agent<T>{gpx, gpy, g.th, gvx, gvy, g.s, g.w};
  gfx += gvx * P.dt_over_m;
  gfy += gvy * P.dt_over_m;
  const T gacc[3] = {gvx * dt, gvy * dt, gvz * dt};
  // q = normalize(qu), qu = q + qd(q, nb) dt
  T gq[4] = {T(0), T(0), T(0), T(0)};
  const T gqo[4] = {gd.qx, gd.qy, gd.qz, gd.qw};
  normalize4_vjp(qu, gqo, gq);
  const T gqd[4] = {gq[0] * dt, gq[1] * dt, gq[2] * dt, gq[3] * dt};
  T gnb[3] = {gd.bx, gd.by, gd.bz};
  quat_deriv_vjp(d.qx, d.qy, d.qz, d.qw, nb[0], nb[1], nb[2], gqd, gq, gnb);
  // nb = b + ang dt
  T gb[3] = {gnb[0], gnb[1], gnb[2]};
  const T gang[3] = {gnb[0] * dt, gnb[1] * dt, gnb[2] * dt};
  T gf[4] = {T(0), T(0), T(0), T(0)};
  drone_rates_vjp(f, d.qx, d.qy, d.qz, d.qw, d.bx, d.by, d.bz, P, gacc, gang, gf, gq, gb);
#pragma unroll
  for (int i = 0; i < 4; ++i) ga[i] += clamp_pass(a[i], T(0), P.tmax) ? gf[i] : T(0);
  gdin = Drone<T>{gd.z, gvz, gq[0], gq[1], gq[2], gq[3], gb[0], gb[1], gb[2]};
}

// -------------------------------------------------------------------- RK4
// Stage state (px, py, vx, vy, z, vz, qx, qy, qz, qw, bx, by, bz) and its derivative.
template <typename T>
__device__ __forceinline__ void drone_deriv(const T x[13], const T f[4], const AgentP<T>& P,
                                            T k[13]) {
  T acc[3], ang[3];
  drone_rates(f, x[6], x[7], x[8], x[9], x[10], x[11], x[12], P, acc, ang);
  k[0] = x[2];
  k[1] = x[3];
  k[2] = acc[0];
  k[3] = acc[1];
  k[4] = x[5];
  k[5] = acc[2];
  quat_deriv(x[6], x[7], x[8], x[9], x[10], x[11], x[12], k + 6);
  k[10] = ang[0];
  k[11] = ang[1];
  k[12] = ang[2];
}
template <typename T>
__device__ __forceinline__ void drone_deriv_vjp(const T x[13], const T f[4], const AgentP<T>& P,
                                                const T gk[13], T gx[13], T gf[4]) {
  gx[2] += gk[0];
  gx[3] += gk[1];
  gx[5] += gk[4];
  const T gacc[3] = {gk[2], gk[3], gk[5]};
  const T gang[3] = {gk[10], gk[11], gk[12]};
  drone_rates_vjp(f, x[6], x[7], x[8], x[9], x[10], x[11], x[12], P, gacc, gang, gf, gx + 6,
                  gx + 10);
  quat_deriv_vjp(x[6], x[7], x[8], x[9], x[10], x[11], x[12], gk + 6, gx + 6, gx + 10);
}

template <typename T>
__device__ __forceinline__ void drone_x0(const Agent<T>& in, const Drone<T>& d, T x[13]) {
  x[0] = in.px; x[1] = in.py; x[2] = in.vx; x[3] = in.vy; x[4] = d.z; x[5] = d.vz;
  x[6] = d.qx; x[7] = d.qy; x[8] = d.qz; x[9] = d.qw; x[10] = d.bx; x[11] = d.by; x[12] = d.bz;
}

// The four stages and the combine (before the force term and the renormalization).
template <typename T>
__device__ __forceinline__ void drone_rk4_stages(const T x0[13], const T f[4], const AgentP<T>& P,
                                                 T dt, T k1[13], T k2[13], T k3[13], T k4[13],
                                                 T xi[13]) {
  const T dt2 = dt * T(0.5), sixth = dt / T(6);
  T xs[13];
  drone_deriv(x0, f, P, k1);
#pragma unroll
  for (int j = 0; j < 13; ++j) xs[j] = x0[j] + k1[j] * dt2;
  drone_deriv(xs, f, P, k2);
#pragma unroll
  for (int j = 0; j < 13; ++j) xs[j] = x0[j] + k2[j] * dt2;
  drone_deriv(xs, f, P, k3);
#pragma unroll
  for (int j = 0; j < 13; ++j) xs[j] = x0[j] + k3[j] * dt;
  drone_deriv(xs, f, P, k4);
#pragma unroll
  for (int j = 0; j < 13; ++j) xi[j] = x0[j] + (k1[j] + k2[j] * T(2) + k3[j] * T(2) + k4[j]) * sixth;
}

template <typename T>
__device__ __forceinline__ void drone_rk4_fwd(const Agent<T>& in, const Drone<T>& d, const T a[4],
                                              T fx, T fy, const AgentP<T>& P, const WorldC<T>& W,
                                              Agent<T>& out, Drone<T>& dout) {
  const T dt = W.dt;
  T f[4], x0[13], k1[13], k2[13], k3[13], k4[13], xi[13];
  drone_thrusts(a, P, f);
  drone_x0(in, d, x0);
  drone_rk4_stages(x0, f, P, dt, k1, k2, k3, k4, xi);
  const T dvx = fx * P.dt_over_m, dvy = fy * P.dt_over_m;
  out.px = xi[0] + dvx * dt;
  out.py = xi[1] + dvy * dt;
  out.th = in.th;
  out.vx = xi[2] + dvx;
  out.vy = xi[3] + dvy;
  out.s = in.s;
  out.w = in.w;
  T qn[4];
  normalize4(xi + 6, qn);
  dout = Drone<T>{xi[4], xi[5], qn[0], qn[1], qn[2], qn[3], xi[10], xi[11], xi[12]};
  drone_clamp(out.px, out.py, P, W);
}

// Adjoint of drone_rk4_fwd. The pre-clamp position is rebuilt from the stored output
// velocity (xi.p + (v_out - xi.v) dt); a coordinate strictly inside its bounds passed the
// clamp whatever the rebuild's rounding.
template <typename T>
__device__ __forceinline__ void drone_rk4_vjp(const Agent<T>& in, const Drone<T>& d, const T a[4],
                                              const Agent<T>& out, const Agent<T>& g,
                                              const Drone<T>& gd, const AgentP<T>& P,
                                              const WorldC<T>& W, Agent<T>& gin, Drone<T>& gdin,
                                              T& gfx, T& gfy, T ga[4]) {
  const T dt = W.dt;
  const T dt2 = dt * T(0.5), sixth = dt / T(6);
  T f[4], x0[13], k1[13], k2[13], k3[13], k4[13], xi[13];
  drone_thrusts(a, P, f);
  drone_x0(in, d, x0);
  drone_rk4_stages(x0, f, P, dt, k1, k2, k3, k4, xi);
  T gpx = g.px, gpy = g.py;
  if (W.bounds_mode == BOUNDS_CLAMP) {
    const T lox = W.bx0 + P.radius, hix = W.bx1 - P.radius;
    const T loy = W.by0 + P.radius, hiy = W.by1 - P.radius;
    const T prex = xi[0] + (out.vx - xi[2]) * dt, prey = xi[1] + (out.vy - xi[3]) * dt;
    if (!((out.px > lox && out.px < hix) || clamp_pass(prex, lox, hix))) gpx = T(0);
    if (!((out.py > loy && out.py < hiy) || clamp_pass(prey, loy, hiy))) gpy = T(0);
  }
  T gxi[13];
  gxi[0] = gpx;
  gxi[1] = gpy;
  gxi[2] = g.vx;
  gxi[3] = g.vy;
  const T gdvx = g.vx + gpx * dt, gdvy = g.vy + gpy * dt;
  gfx += gdvx * P.dt_over_m;
  gfy += gdvy * P.dt_over_m;
  gxi[4] = gd.z;
  gxi[5] = gd.vz;
#pragma unroll
  for (int j = 6; j < 10; ++j) gxi[j] = T(0);
  const T gqo[4] = {gd.qx, gd.qy, gd.qz, gd.qw};
  normalize4_vjp(xi + 6, gqo, gxi + 6);
  gxi[10] = gd.bx;
  gxi[11] = gd.by;
  gxi[12] = gd.bz;
  // xi = x0 + (k1 + 2 k2 + 2 k3 + k4) / 6 dt; stages x_{j+1} = x0 + k_j c_j
  T gx0[13], gk[13], gs[13], xs[13], gf[4] = {T(0), T(0), T(0), T(0)};
#pragma unroll
  for (int j = 0; j < 13; ++j) {
    gx0[j] = gxi[j];
    gk[j] = gxi[j] * sixth;  // k4
  }
  // k4 = deriv(x0 + k3 dt)
#pragma unroll
  for (int j = 0; j < 13; ++j) { xs[j] = x0[j] + k3[j] * dt; gs[j] = T(0); }
  drone_deriv_vjp(xs, f, P, gk, gs, gf);
#pragma unroll
  for (int j = 0; j < 13; ++j) { gx0[j] += gs[j]; gk[j] = gxi[j] * sixth * T(2) + gs[j] * dt; }
  // k3 = deriv(x0 + k2 dt/2)
#pragma unroll
  for (int j = 0; j < 13; ++j) { xs[j] = x0[j] + k2[j] * dt2; gs[j] = T(0); }
  drone_deriv_vjp(xs, f, P, gk, gs, gf);
#pragma unroll
  for (int j = 0; j < 13; ++j) { gx0[j] += gs[j]; gk[j] = gxi[j] * sixth * T(2) + gs[j] * dt2; }
  // k2 = deriv(x0 + k1 dt/2)
#pragma unroll
  for (int j = 0; j < 13; ++j) { xs[j] = x0[j] + k1[j] * dt2; gs[j] = T(0); }
  drone_deriv_vjp(xs, f, P, gk, gs, gf);
#pragma unroll
  for (int j = 0; j < 13; ++j) { gx0[j] += gs[j]; gk[j] = gxi[j] * sixth + gs[j] * dt2; }
  // k1 = deriv(x0)
#pragma unroll
  for (int j = 0; j < 13; ++j) gs[j] = T(0);
  drone_deriv_vjp(x0, f, P, gk, gs, gf);
#pragma unroll
  for (int j = 0; j < 13; ++j) gx0[j] += gs[j];
  (void)k4;
#pragma unroll
  for (int i = 0; i < 4; ++i) ga[i] += clamp_pass(a[i], T(0), P.tmax) ? gf[i] : T(0);
  gin = Agent<T>{gx0[0], gx0[1], g.th, gx0[2], gx0[3], g.s, g.w};
  gdin = Drone<T>{gx0[4], gx0[5], gx0[6], gx0[7], gx0[8], gx0[9], gx0[10], gx0[11], gx0[12]};
}

}  // namespace swarp
