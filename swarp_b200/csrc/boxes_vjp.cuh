// Adjoint of the box-agent contacts (boxes.cuh): the VJP of every force a box agent
// takes part in, with respect to the agent's own position, heading, velocity and turn
// rate.
//
// Each contact is first evaluated in plain arithmetic (the forward's own functions, so
// the winning branch, SAT axis or vertex and the contact activity are bitwise the
// forward's), then re-evaluated along that one branch in forward-mode dual numbers whose
// tangents are the own agent's state variables. The pair's contribution to the loss,
// L = gA.F_A + gB.F_B with the two agents' force cotangents, is formed in the same dual
// arithmetic; its tangents are dL/d(own state). The primal parts repeat the forward's
// operations in the forward's order, and the gradient at every kink follows the
// reference's (Warp's) adjoint conventions: max/min pass the gradient to the selected
// operand, clamp to the bound that is active (else to x), abs has slope +1 at zero, and
// sign() and the branch choices are locally constant.
#pragma once
#include "boxes.cuh"

namespace swarp {

// --------------------------------------------------------------- dual numbers
template <typename T, int N> struct Dual {
  T v;
  T d[N];
};

template <typename T, int N> __device__ __forceinline__ Dual<T, N> dconst(T v) {
  Dual<T, N> r;
  r.v = v;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = T(0);
  return r;
}
// Variable number j (unit tangent e_j).
template <int J, typename T, int N> __device__ __forceinline__ Dual<T, N> dvar(T v) {
  Dual<T, N> r;
  r.v = v;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = i == J ? T(1) : T(0);
  return r;
}
template <typename T> __device__ __forceinline__ Dual<T, 6> up6(const Dual<T, 3>& x) {
  Dual<T, 6> r;
  r.v = x.v;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    r.d[i] = x.d[i];
    r.d[i + 3] = T(0);
  }
  return r;
}

#define SWARP_DUAL_FOR _Pragma("unroll") for (int i = 0; i < N; ++i)
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator+(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r;
  r.v = a.v + b.v;
  SWARP_DUAL_FOR r.d[i] = a.d[i] + b.d[i];
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator+(const Dual<T, N>& a, T b) {
  Dual<T, N> r = a;
  r.v = a.v + b;
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator+(T a, const Dual<T, N>& b) {
  Dual<T, N> r = b;
  r.v = a + b.v;
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator-(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r;
  r.v = a.v - b.v;
  SWARP_DUAL_FOR r.d[i] = a.d[i] - b.d[i];
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator-(const Dual<T, N>& a, T b) {
  Dual<T, N> r = a;
  r.v = a.v - b;
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator-(T a, const Dual<T, N>& b) {
  Dual<T, N> r;
  r.v = a - b.v;
  SWARP_DUAL_FOR r.d[i] = -b.d[i];
  return r;
}
template <typename T, int N> __device__ __forceinline__ Dual<T, N> operator-(const Dual<T, N>& a) {
  Dual<T, N> r;
  r.v = -a.v;
  SWARP_DUAL_FOR r.d[i] = -a.d[i];
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator*(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r;
  r.v = a.v * b.v;
  SWARP_DUAL_FOR r.d[i] = a.d[i] * b.v + a.v * b.d[i];
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator*(const Dual<T, N>& a, T b) {
  Dual<T, N> r;
  r.v = a.v * b;
  SWARP_DUAL_FOR r.d[i] = a.d[i] * b;
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator*(T a, const Dual<T, N>& b) {
  Dual<T, N> r;
  r.v = a * b.v;
  SWARP_DUAL_FOR r.d[i] = a * b.d[i];
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> operator/(T a, const Dual<T, N>& b) {
  Dual<T, N> r;
  r.v = a / b.v;
  const T q = -r.v / b.v;
  SWARP_DUAL_FOR r.d[i] = q * b.d[i];
  return r;
}
// fma(a, b, c) rounded once, as Num<T>::fma_ in the forward
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> dfma(const Dual<T, N>& a, const Dual<T, N>& b,
                                           const Dual<T, N>& c) {
  Dual<T, N> r;
  r.v = Num<T>::fma_(a.v, b.v, c.v);
  SWARP_DUAL_FOR r.d[i] = a.d[i] * b.v + a.v * b.d[i] + c.d[i];
  return r;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> ddot2(const Dual<T, N>& ax, const Dual<T, N>& ay,
                                            const Dual<T, N>& bx, const Dual<T, N>& by) {
  return dfma(ax, bx, ay * by);
}
template <typename T, int N> __device__ __forceinline__ Dual<T, N> dabs(const Dual<T, N>& x) {
  return x.v < T(0) ? -x : x;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> dmax(const Dual<T, N>& a, const Dual<T, N>& b) {
  return a.v > b.v ? a : b;
}
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> dmin(const Dual<T, N>& a, const Dual<T, N>& b) {
  return a.v < b.v ? a : b;
}
// clamp to constant bounds: value min(max(lo, x), hi), tangent of x on the closed interval
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> dclamp(const Dual<T, N>& x, T lo, T hi) {
  Dual<T, N> r = clamp_pass(x.v, lo, hi) ? x : dconst<T, N>(T(0));
  r.v = wclamp(x.v, lo, hi);
  return r;
}
template <typename T, int N> __device__ __forceinline__ Dual<T, N> drsqrt(const Dual<T, N>& x) {
  Dual<T, N> r;
  r.v = Num<T>::rsqrt_(x.v);
  const T q = T(-0.5) * r.v * r.v * r.v;
  SWARP_DUAL_FOR r.d[i] = q * x.d[i];
  return r;
}
#undef SWARP_DUAL_FOR

// cos and sin of a heading that is variable J (else constant)
template <int J, typename T, int N>
__device__ __forceinline__ void dcossin(T th, bool var, Dual<T, N>& c, Dual<T, N>& s) {
  const T cv = Num<T>::cos_(th), sv = Num<T>::sin_(th);
  c = dconst<T, N>(cv);
  s = dconst<T, N>(sv);
  if (var) {
    c.d[J] = -sv;
    s.d[J] = cv;
  }
}

// normal_coeff in dual arithmetic (same primal operations)
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> dnormal_coeff(const Dual<T, N>& ov, const Dual<T, N>& vn,
                                                    T inv_denom, const WorldC<T>& W) {
  Dual<T, N> ovs = ov;
  if (W.max_overlap > T(0)) {
    const T t = tanh_ratio(ov.v, W.max_overlap);
    ovs = ov * (T(1) - t * t);
    ovs.v = W.max_overlap * t;
  }
  Dual<T, N> num = W.k * ovs - W.c * vn;
  num.v = nc_num(ovs.v, vn.v, W);  // the primal exactly as normal_coeff rounds it
  const Dual<T, N> x = num * inv_denom;
  return dmax(x, dconst<T, N>(T(0)));
}

// The loss of one contact, L = cf_A (gA.n) - cf_B (gB.n): the force on A is cf_A n and on
// B is -cf_B n (n points from B to A; cf_X carries X's implicit denominator).
template <typename T, int N>
__device__ __forceinline__ Dual<T, N> contact_loss(const Dual<T, N>& ov, const Dual<T, N>& vn,
                                                   const Dual<T, N>& nx, const Dual<T, N>& ny,
                                                   T idA, T gAx, T gAy, T idB, T gBx, T gBy,
                                                   const WorldC<T>& W) {
  Dual<T, N> L = dconst<T, N>(T(0));
  if (gAx != T(0) || gAy != T(0)) L = dnormal_coeff(ov, vn, idA, W) * (gAx * nx + gAy * ny);
  if (gBx != T(0) || gBy != T(0)) L = L - dnormal_coeff(ov, vn, idB, W) * (gBx * nx + gBy * ny);
  return L;
}

template <typename T>
__device__ __forceinline__ void add_state_grad(const Dual<T, 6>& L, Agent<T>& gin) {
  gin.px += L.d[0];
  gin.py += L.d[1];
  gin.th += L.d[2];
  gin.vx += L.d[3];
  gin.vy += L.d[4];
  gin.w += L.d[5];
}

// ------------------------------------------------------- box-box (obb) contacts
template <typename T> struct ObbD {
  Dual<T, 3> cx, cy, ca, sa;
  T hx, hy;
};
// A box's pose in duals: the own box's centre and heading are variables 0, 1, 2.
template <typename T>
__device__ __forceinline__ ObbD<T> obb_dual(const Ob<T>& b, T th, bool own) {
  ObbD<T> r;
  r.cx = own ? dvar<0, T, 3>(b.cx) : dconst<T, 3>(b.cx);
  r.cy = own ? dvar<1, T, 3>(b.cy) : dconst<T, 3>(b.cy);
  if (own) {
    dcossin<2, T, 3>(th, true, r.ca, r.sa);
  } else {
    r.ca = dconst<T, 3>(b.ca);
    r.sa = dconst<T, 3>(b.sa);
  }
  r.hx = b.hx;
  r.hy = b.hy;
  return r;
}

// obb_contact's geometry (s, n, contact point) along the branch c that the plain
// evaluation selected (boxes.cuh: obb_contact, point_box, box_vertex).
template <typename T>
__device__ __forceinline__ void obb_geom_dual(const ObbD<T>& A, const ObbD<T>& B,
                                              const ObbContact<T>& c, Dual<T, 3>& s,
                                              Dual<T, 3>& nx, Dual<T, 3>& ny, Dual<T, 3>& px,
                                              Dual<T, 3>& py) {
  using D = Dual<T, 3>;
  if (c.branch == 1) {
    const bool ownA = c.vert < 4;
    const ObbD<T> own = ownA ? A : B;  // values, not a run-time reference (local memory)
    const ObbD<T> oth = ownA ? B : A;
    const T flip = ownA ? T(1) : T(-1);
    const int v = c.vert & 3;
    const D e0x = own.ca * own.hx, e0y = own.sa * own.hx;
    const D e1x = (-own.sa) * own.hy, e1y = own.ca * own.hy;
    const bool p0 = (v == 0 || v == 3), p1 = (v < 2);
    D x = p0 ? own.cx + e0x : own.cx - e0x;
    D y = p0 ? own.cy + e0y : own.cy - e0y;
    x = p1 ? x + e1x : x - e1x;
    y = p1 ? y + e1y : y - e1y;
    // point_box(x, y, oth)
    const D dx = x - oth.cx, dy = y - oth.cy;
    const D lx = oth.ca * dx + oth.sa * dy;
    const D ly = (-oth.sa) * dx + oth.ca * dy;
    const D clx = dclamp(lx, -oth.hx, oth.hx), cly = dclamp(ly, -oth.hy, oth.hy);
    const D ox = lx - clx, oy = ly - cly;
    const D m = dmax(ox * ox + oy * oy, dconst<T, 3>(Eps2<T>::v));
    const D dist = m * drsqrt(m);
    const D qx = oth.cx + (oth.ca * clx - oth.sa * cly);
    const D qy = oth.cy + (oth.sa * clx + oth.ca * cly);
    const D f = flip / dist;
    nx = (x - qx) * f;
    ny = (y - qy) * f;
    px = (x + qx) * T(0.5);
    py = (y + qy) * T(0.5);
    s = dist;
    return;
  }
  // overlapping: the least-overlap SAT axis
  const D dx = A.cx - B.cx, dy = A.cy - B.cy;
  const D a00 = dabs(A.ca * B.ca + A.sa * B.sa);
  const D a01 = dabs(A.ca * (-B.sa) + A.sa * B.ca);
  const D a10 = dabs((-A.sa) * B.ca + A.ca * B.sa);
  const D a11 = dabs((-A.sa) * (-B.sa) + A.ca * B.ca);
  D ux, uy, tx, ty, dn, rt;
  T hn, ht;
  switch (c.axis) {
    case 0:
      ux = A.ca; uy = A.sa; tx = -A.sa; ty = A.ca;
      dn = dx * A.ca + dy * A.sa; hn = A.hx; ht = A.hy;
      rt = B.hx * a10 + B.hy * a11;
      s = dabs(dn) - A.hx - (B.hx * a00 + B.hy * a01);
      break;
    case 1:
      ux = -A.sa; uy = A.ca; tx = A.ca; ty = A.sa;
      dn = dx * (-A.sa) + dy * A.ca; hn = A.hy; ht = A.hx;
      rt = B.hx * a00 + B.hy * a01;
      s = dabs(dn) - A.hy - (B.hx * a10 + B.hy * a11);
      break;
    case 2:
      ux = B.ca; uy = B.sa; tx = -B.sa; ty = B.ca;
      dn = dx * B.ca + dy * B.sa; hn = B.hx; ht = B.hy;
      rt = A.hx * a01 + A.hy * a11;
      s = dabs(dn) - B.hx - (A.hx * a00 + A.hy * a10);
      break;
    default:
      ux = -B.sa; uy = B.ca; tx = B.ca; ty = B.sa;
      dn = dx * (-B.sa) + dy * B.ca; hn = B.hy; ht = B.hx;
      rt = A.hx * a00 + A.hy * a10;
      s = dabs(dn) - B.hy - (A.hx * a01 + A.hy * a11);
      break;
  }
  const T sgn = dn.v < T(0) ? T(-1) : T(1);
  nx = ux * sgn;
  ny = uy * sgn;
  const bool bref = c.axis >= 2;
  const D rcx = bref ? B.cx : A.cx, rcy = bref ? B.cy : A.cy;
  const D icx = bref ? A.cx : B.cx, icy = bref ? A.cy : B.cy;
  const D xn = bref ? (B.cx * nx + B.cy * ny) + hn : (A.cx * nx + A.cy * ny) - hn;
  const D ct_ref = rcx * tx + rcy * ty, ct_inc = icx * tx + icy * ty;
  const D lo = dmax(ct_ref - ht, ct_inc - rt), hi = dmin(ct_ref + ht, ct_inc + rt);
  const D mid = T(0.5) * (lo + hi);
  px = nx * xn + tx * mid;
  py = ny * xn + ty * mid;
}

// VJP of one obb_force contact between boxes A and B (A's force cf_A n, B's -cf_B n,
// gA/gB their cotangents) into the own box's state gradient (own = A or B; the other
// box's state is constant). thA/thB are the headings the Ob poses were built from.
template <typename T>
__device__ __noinline__ void obb_contact_vjp(const Ob<T>& A, T thA, const Ob<T>& B, T thB,
                                                bool ownA, T reach, T idA, T gAx, T gAy, T idB,
                                                T gBx, T gBy, const WorldC<T>& W,
                                                Agent<T>& gin) {
  const ObbContact<T> c = obb_contact(A, B, reach);
  if (!(reach - c.s > T(0))) return;
  const ObbD<T> AD = obb_dual(A, thA, ownA), BD = obb_dual(B, thB, !ownA);
  Dual<T, 3> s3, nx3, ny3, px3, py3;
  obb_geom_dual(AD, BD, c, s3, nx3, ny3, px3, py3);
  using D6 = Dual<T, 6>;
  const D6 nx = up6(nx3), ny = up6(ny3), px = up6(px3), py = up6(py3);
  const D6 ov = reach - up6(s3);
  const D6 rax = px - up6(AD.cx), ray = py - up6(AD.cy);
  const D6 rbx = px - up6(BD.cx), rby = py - up6(BD.cy);
  // the own box's velocity and turn rate are variables 3, 4, 5
  const D6 avx = ownA ? dvar<3, T, 6>(A.vx) : dconst<T, 6>(A.vx);
  const D6 avy = ownA ? dvar<4, T, 6>(A.vy) : dconst<T, 6>(A.vy);
  const D6 aom = ownA ? dvar<5, T, 6>(A.om) : dconst<T, 6>(A.om);
  const D6 bvx = ownA ? dconst<T, 6>(B.vx) : dvar<3, T, 6>(B.vx);
  const D6 bvy = ownA ? dconst<T, 6>(B.vy) : dvar<4, T, 6>(B.vy);
  const D6 bom = ownA ? dconst<T, 6>(B.om) : dvar<5, T, 6>(B.om);
  const D6 rvx = (avx + ((-aom) * ray)) - (bvx + ((-bom) * rby));
  const D6 rvy = (avy + aom * rax) - (bvy + bom * rbx);
  const D6 vn = rvx * nx + rvy * ny;
  add_state_grad(contact_loss(ov, vn, nx, ny, idA, gAx, gAy, idB, gBx, gBy, W), gin);
}

// ------------------------------------------------------ point-box (SDF) contacts
// VJP of one box_force contact of a point P (a disc agent's centre or a circle
// obstacle's) against box B (force cf_P n on the point, -cf_B n on the box); own = the
// point (its position and velocity are variables 0, 1, 3, 4) or the box (all six).
template <typename T>
__device__ __noinline__ void sdf_contact_vjp(T ppx, T ppy, T pvx, T pvy, const Ob<T>& B,
                                                T thB, bool ownP, T reach, T idP, T gPx, T gPy,
                                                T idB, T gBx, T gBy, const WorldC<T>& W,
                                                Agent<T>& gin) {
  using D = Dual<T, 6>;
  const D px = ownP ? dvar<0, T, 6>(ppx) : dconst<T, 6>(ppx);
  const D py = ownP ? dvar<1, T, 6>(ppy) : dconst<T, 6>(ppy);
  const D vx = ownP ? dvar<3, T, 6>(pvx) : dconst<T, 6>(pvx);
  const D vy = ownP ? dvar<4, T, 6>(pvy) : dconst<T, 6>(pvy);
  const D cx = ownP ? dconst<T, 6>(B.cx) : dvar<0, T, 6>(B.cx);
  const D cy = ownP ? dconst<T, 6>(B.cy) : dvar<1, T, 6>(B.cy);
  const D ovx = ownP ? dconst<T, 6>(B.vx) : dvar<3, T, 6>(B.vx);
  const D ovy = ownP ? dconst<T, 6>(B.vy) : dvar<4, T, 6>(B.vy);
  const D om = ownP ? dconst<T, 6>(B.om) : dvar<5, T, 6>(B.om);
  D ca, sa;
  if (ownP) {
    ca = dconst<T, 6>(B.ca);
    sa = dconst<T, 6>(B.sa);
  } else {
    dcossin<2, T, 6>(thB, true, ca, sa);
  }
  const T hx = B.hx, hy = B.hy;
  // box_force (physics.cuh), same operations
  const D dx = px - cx, dy = py - cy;
  const D lx = ca * dx + sa * dy;
  const D ly = (-sa) * dx + ca * dy;
  const D qx = dabs(lx) - hx;
  const D qy = dabs(ly) - hy;
  const D clx = dclamp(lx, -hx, hx), cly = dclamp(ly, -hy, hy);
  const D ox = lx - clx, oy = ly - cly;
  const D od2 = ox * ox + oy * oy;
  D s, nlx, nly;
  if (od2.v > Eps2<T>::v) {
    const D is = drsqrt(od2);
    s = od2 * is;
    nlx = ox * is;
    nly = oy * is;
  } else if (qx.v > qy.v) {
    s = qx;
    nlx = dconst<T, 6>(lx.v >= T(0) ? T(1) : T(-1));
    nly = dconst<T, 6>(T(0));
  } else {
    s = qy;
    nlx = dconst<T, 6>(T(0));
    nly = dconst<T, 6>(ly.v >= T(0) ? T(1) : T(-1));
  }
  const D overlap = reach - s;
  if (!(overlap.v > T(0))) return;
  const D nx = ca * nlx - sa * nly, ny = sa * nlx + ca * nly;
  const D spx = lx - s * nlx, spy = ly - s * nly;
  const D rx = ca * spx - sa * spy, ry = sa * spx + ca * spy;
  const D vsx = ovx + ((-om) * ry), vsy = ovy + om * rx;
  const D vn = ddot2(vx - vsx, vy - vsy, nx, ny);
  add_state_grad(contact_loss(overlap, vn, nx, ny, idP, gPx, gPy, idB, gBx, gBy, W), gin);
}

// ------------------------------------------------------------ dispatchers
// Both directions of one agent-agent contact of any two shapes (pair_force_shaped's
// dispatch), into agent a's state gradient. ga = cotangent of a's force (zero when b is
// not in a's list), gb = of b's force (zero when a is not in b's list).
template <typename T>
__device__ __forceinline__ void pair_shaped_vjp(int a, int b, bool box_a, const Ob<T>& oa, T tha,
                                                T ra, T ida, T gax, T gay, bool box_b,
                                                const Ob<T>& ob, T thb, T rb, T idb, T gbx,
                                                T gby, const WorldC<T>& W, Agent<T>& gin) {
  if (!box_a && !box_b) {
    pair_vjp_sym(oa.cx - ob.cx, oa.cy - ob.cy, oa.vx - ob.vx, oa.vy - ob.vy, ra + rb + W.margin,
                 ida, gax, gay, idb, gbx, gby, W, gin.px, gin.py, gin.vx, gin.vy);
    return;
  }
  // the forward's broad phase (pair_force_shaped): such pairs carry no force
  const T reach = box_a && box_b ? W.margin : (box_a ? rb : ra) + W.margin;
  if (bounds_apart(oa.cx - ob.cx, oa.cy - ob.cy, (box_a ? norm2(oa.hx, oa.hy) : T(0)) +
                                                     (box_b ? norm2(ob.hx, ob.hy) : T(0)) + reach))
    return;
  if (!box_a) {
    sdf_contact_vjp(oa.cx, oa.cy, oa.vx, oa.vy, ob, thb, true, ra + W.margin, ida, gax, gay, idb,
                    gbx, gby, W, gin);
  } else if (!box_b) {
    sdf_contact_vjp(ob.cx, ob.cy, ob.vx, ob.vy, oa, tha, false, rb + W.margin, idb, gbx, gby, ida,
                    gax, gay, W, gin);
  } else if (a < b) {
    obb_contact_vjp(oa, tha, ob, thb, true, W.margin, ida, gax, gay, idb, gbx, gby, W, gin);
  } else {
    obb_contact_vjp(ob, thb, oa, tha, false, W.margin, idb, gbx, gby, ida, gax, gay, W, gin);
  }
}

// VJP of box_static_force (obstacles, then the support-extent walls) of a box agent at
// heading th with force cotangent (gfx, gfy).
template <typename T>
__device__ __noinline__ void box_static_vjp(const Obs<T>* sobs, int N, bool walls,
                                               const Ob<T>& oa, T th, T inv_denom, T gfx, T gfy,
                                               const WorldC<T>& W, Agent<T>& gin) {
  const T ra = norm2(oa.hx, oa.hy);
  for (int o = 0; o < N; ++o) {
    const Obs<T>& ob = sobs[o];
    if (bounds_apart(oa.cx - ob.cx, oa.cy - ob.cy, ra + W.margin + ob.bound)) continue;
    if (ob.type == SHAPE_BOX || ob.type == SHAPE_SEGMENT) {
      const bool seg = ob.type == SHAPE_SEGMENT;
      const Ob<T> B{ob.cx, ob.cy, ob.ca, ob.sa, ob.hx, seg ? T(0) : ob.hy, ob.vx, ob.vy, ob.om};
      obb_contact_vjp(oa, th, B, T(0), true, seg ? ob.r + W.margin : W.margin, inv_denom, gfx, gfy,
                      T(1), T(0), T(0), W, gin);
    } else {
      sdf_contact_vjp(ob.cx, ob.cy, ob.vx, ob.vy, oa, th, false, ob.r + W.margin, T(1), T(0), T(0),
                      inv_denom, gfx, gfy, W, gin);
    }
  }
  if (!walls) return;
  using D = Dual<T, 6>;
  D ca, sa;
  dcossin<2, T, 6>(th, true, ca, sa);
  const D cx = dvar<0, T, 6>(oa.cx), cy = dvar<1, T, 6>(oa.cy);
  const D vx = dvar<3, T, 6>(oa.vx), vy = dvar<4, T, 6>(oa.vy), om = dvar<5, T, 6>(oa.om);
  const T hx = oa.hx, hy = oa.hy;
  const D ex = hx * dabs(ca) + hy * dabs(sa);
  const D ey = hx * dabs(sa) + hy * dabs(ca);
  const T sc = sgn0(ca.v), ss = sgn0(sa.v);
  const D rly = (-sc * hx) * sa + (ss * hy) * ca;
  const D rbx = (-ss * hx) * ca + (sc * hy) * sa;
  D L = dconst<T, 6>(T(0));
  D pen = ex + W.margin - (cx - W.bx0);
  if (pen.v > T(0)) L = L + gfx * dnormal_coeff(pen, vx - om * rly, inv_denom, W);
  pen = ex + W.margin - (W.bx1 - cx);
  if (pen.v > T(0)) L = L - gfx * dnormal_coeff(pen, -(vx + om * rly), inv_denom, W);
  pen = ey + W.margin - (cy - W.by0);
  if (pen.v > T(0)) L = L + gfy * dnormal_coeff(pen, vy + om * rbx, inv_denom, W);
  pen = ey + W.margin - (W.by1 - cy);
  if (pen.v > T(0)) L = L - gfy * dnormal_coeff(pen, -(vy - om * rbx), inv_denom, W);
  add_state_grad(L, gin);
}

}  // namespace swarp
