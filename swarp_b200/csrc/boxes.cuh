// Box agents: oriented-box contacts (swarp/core/collisions.py:262-690 restated).
//
// An agent with shape BOX carries half extents (hx, hy) in its own frame at heading th.
// Agent-agent pairs dispatch on the two shapes: disc-disc is the disc law, disc-box the
// oriented-box SDF law (negated on the box), box-box the separating-axis contact with the
// lower agent index as box A on both agents (so the pair's forces cancel). Against
// obstacles a box agent meets BOX obstacles with the same box-box contact, SEGMENT
// obstacles as the degenerate box (half_len, 0) with reach radius + margin (an exact
// capsule) and CIRCLE obstacles through the SDF law with the circle's centre as the point.
// Walls see the box's support extents and the velocity of its touching support vertex.
#pragma once
#include "physics.cuh"

namespace swarp {

// Sign with 0 at 0 (the support-vertex choice on a face flush with a wall).
template <typename T> __device__ __forceinline__ T sgn0(T x) {
  return x > T(0) ? T(1) : (x < T(0) ? T(-1) : T(0));
}

// An oriented box in motion: centre, cos/sin of its heading, half extents, velocity,
// angular velocity.
template <typename T> struct Ob {
  T cx, cy, ca, sa, hx, hy, vx, vy, om;
};

// Distance and closest point from a point outside an oriented box (distance floored).
template <typename T>
__device__ __forceinline__ T point_box(T vx, T vy, const Ob<T>& b, T& qx, T& qy) {
  const T dx = vx - b.cx, dy = vy - b.cy;
  const T lx = b.ca * dx + b.sa * dy;
  const T ly = -b.sa * dx + b.ca * dy;
  const T clx = wclamp(lx, -b.hx, b.hx), cly = wclamp(ly, -b.hy, b.hy);
  const T ox = lx - clx, oy = ly - cly;
  const T m = wmax(ox * ox + oy * oy, Eps2<T>::v);
  const T dist = m * Num<T>::rsqrt_(m);
  qx = b.cx + (b.ca * clx - b.sa * cly);
  qy = b.cy + (b.sa * clx + b.ca * cly);
  return dist;
}

// Contact geometry of boxes A and B: signed distance s, unit normal (B to A), contact
// point, and which branch produced them (0: beyond reach, 1: disjoint, winning vertex
// `vert` 0..7 (0-3 of A against B, 4-7 of B against A), 2: overlapping on SAT `axis`).
template <typename T> struct ObbContact {
  T s, nx, ny, px, py;
  int branch, axis, vert;
};

template <typename T>
__device__ __forceinline__ void box_vertex(const Ob<T>& b, int v, T& x, T& y) {
  // vertex order (+,+), (-,+), (-,-), (+,-) along the box's own axes
  const T e0x = b.ca * b.hx, e0y = b.sa * b.hx;
  const T e1x = -b.sa * b.hy, e1y = b.ca * b.hy;
  const bool p0 = (v == 0 || v == 3), p1 = (v < 2);
  x = (p0 ? b.cx + e0x : b.cx - e0x);
  y = (p0 ? b.cy + e0y : b.cy - e0y);
  x = p1 ? x + e1x : x - e1x;
  y = p1 ? y + e1y : y - e1y;
}

template <typename T>
__device__ __noinline__ ObbContact<T> obb_contact(const Ob<T>& A, const Ob<T>& B, T reach) {
  const T dx = A.cx - B.cx, dy = A.cy - B.cy;
  // unit axes: uA0 = (caA, saA), uA1 = (-saA, caA), likewise B
  const T a00 = fabs(A.ca * B.ca + A.sa * B.sa);
  const T a01 = fabs(A.ca * (-B.sa) + A.sa * B.ca);
  const T a10 = fabs((-A.sa) * B.ca + A.ca * B.sa);
  const T a11 = fabs((-A.sa) * (-B.sa) + A.ca * B.ca);
  const T dA0 = dx * A.ca + dy * A.sa, dA1 = dx * (-A.sa) + dy * A.ca;
  const T dB0 = dx * B.ca + dy * B.sa, dB1 = dx * (-B.sa) + dy * B.ca;
  ObbContact<T> r;
  r.s = fabs(dA0) - A.hx - (B.hx * a00 + B.hy * a01);
  r.axis = 0;
  T t = fabs(dA1) - A.hy - (B.hx * a10 + B.hy * a11);
  if (t > r.s) { r.s = t; r.axis = 1; }
  t = fabs(dB0) - B.hx - (A.hx * a00 + A.hy * a10);
  if (t > r.s) { r.s = t; r.axis = 2; }
  t = fabs(dB1) - B.hy - (A.hx * a01 + A.hy * a11);
  if (t > r.s) { r.s = t; r.axis = 3; }
  r.nx = T(0);
  r.ny = T(0);
  r.px = A.cx;
  r.py = A.cy;
  r.vert = -1;
  if (r.s > reach) {
    r.branch = 0;
  } else if (r.s > T(0)) {
    r.branch = 1;
    T best = T(1.0e30);
    // the vertices of A against B, then of B against A (two loops, so that which box
    // owns the vertex is known at compile time)
    auto scan = [&](const Ob<T>& own, const Ob<T>& other, T flip, int v0) {
#pragma unroll 1
      for (int v = 0; v < 4; ++v) {
        T vx, vy, qx, qy;
        box_vertex(own, v, vx, vy);
        const T dist = point_box(vx, vy, other, qx, qy);
        if (dist < best) {
          best = dist;
          r.nx = (vx - qx) * (flip / dist);
          r.ny = (vy - qy) * (flip / dist);
          r.px = (vx + qx) * T(0.5);
          r.py = (vy + qy) * T(0.5);
          r.vert = v0 + v;
        }
      }
    };
    scan(A, B, T(1), 0);
    scan(B, A, T(-1), 4);
    r.s = best;
  } else {
    r.branch = 2;
    T ux, uy, tx, ty, dn, hn, ht, rt;
    switch (r.axis) {
      case 0: ux = A.ca; uy = A.sa; tx = -A.sa; ty = A.ca; dn = dA0; hn = A.hx; ht = A.hy;
              rt = B.hx * a10 + B.hy * a11; break;
      case 1: ux = -A.sa; uy = A.ca; tx = A.ca; ty = A.sa; dn = dA1; hn = A.hy; ht = A.hx;
              rt = B.hx * a00 + B.hy * a01; break;
      case 2: ux = B.ca; uy = B.sa; tx = -B.sa; ty = B.ca; dn = dB0; hn = B.hx; ht = B.hy;
              rt = A.hx * a01 + A.hy * a11; break;
      default: ux = -B.sa; uy = B.ca; tx = B.ca; ty = B.sa; dn = dB1; hn = B.hy; ht = B.hx;
              rt = A.hx * a00 + A.hy * a10; break;
    }
    const T sgn = dn < T(0) ? T(-1) : T(1);
    r.nx = ux * sgn;
    r.ny = uy * sgn;
    const bool bref = r.axis >= 2;
    const T rcx = bref ? B.cx : A.cx, rcy = bref ? B.cy : A.cy;  // reference box centre
    const T icx = bref ? A.cx : B.cx, icy = bref ? A.cy : B.cy;  // incident box centre
    const T xn = bref ? (B.cx * r.nx + B.cy * r.ny) + hn : (A.cx * r.nx + A.cy * r.ny) - hn;
    const T ct_ref = rcx * tx + rcy * ty, ct_inc = icx * tx + icy * ty;
    const T lo = wmax(ct_ref - ht, ct_inc - rt), hi = wmin(ct_ref + ht, ct_inc + rt);
    const T mid = T(0.5) * (lo + hi);
    r.px = r.nx * xn + tx * mid;
    r.py = r.ny * xn + ty * mid;
  }
  return r;
}

// Force on box A from box B (spring-damper along the contact normal, damped by the two
// material points' closing velocity at the contact point). Returns whether in contact.
template <typename T>
__device__ __noinline__ bool obb_force_at(const Ob<T>& A, const Ob<T>& B, T reach, T inv_denom,
                                          const WorldC<T>& W, T& fx, T& fy, T& xx, T& xy) {
  const ObbContact<T> c = obb_contact(A, B, reach);
  fx = T(0);
  fy = T(0);
  xx = c.px;  // the contact point (collisions.py:447-486 returns it with the force)
  xy = c.py;
  const T ov = reach - c.s;
  if (!(ov > T(0))) return false;
  const T rax = c.px - A.cx, ray = c.py - A.cy, rbx = c.px - B.cx, rby = c.py - B.cy;
  const T rvx = (A.vx + (-A.om * ray)) - (B.vx + (-B.om * rby));
  const T rvy = (A.vy + A.om * rax) - (B.vy + B.om * rbx);
  const T cf = normal_coeff(ov, rvx * c.nx + rvy * c.ny, inv_denom, W);
  fx = cf * c.nx;
  fy = cf * c.ny;
  return true;
}
template <typename T>
__device__ __forceinline__ bool obb_force(const Ob<T>& A, const Ob<T>& B, T reach, T inv_denom,
                                          const WorldC<T>& W, T& fx, T& fy) {
  T xx, xy;
  return obb_force_at(A, B, reach, inv_denom, W, fx, fy, xx, xy);
}

// box_force for agent pairs, kept out of line: the box paths are the cold, large part of
// a box world's contact pass, and one copy of their code per kernel keeps the hot loop in
// the instruction cache.
template <typename T>
__device__ __noinline__ bool box_force_pair(T px, T py, T vx, T vy, const Obs<T>& o, T reach,
                                            T inv_denom, const WorldC<T>& W, T& fx, T& fy) {
  return box_force(px, py, vx, vy, o, reach, inv_denom, W, fx, fy);
}

// Obs (the SDF law's box description) of an agent box.
template <typename T>
__device__ __forceinline__ Obs<T> obs_of(const Ob<T>& b) {
  Obs<T> o;
  o.cx = b.cx; o.cy = b.cy; o.ca = b.ca; o.sa = b.sa; o.vx = b.vx; o.vy = b.vy; o.om = b.om;
  o.r = T(0); o.hx = b.hx; o.hy = b.hy; o.bound = T(0); o.type = SHAPE_BOX;
  return o;
}

// Agent-agent force on a from b for any two shapes (collisions.py:490-537): adds into
// (fx, fy) and returns whether the pair is in contact.
template <typename T>
__device__ __forceinline__ bool pair_force_shaped(int a, int b, bool box_a, const Ob<T>& oa, T ra,
                                                  bool box_b, const Ob<T>& ob, T rb, T inv_denom,
                                                  const WorldC<T>& W, T& fx, T& fy) {
  if (!box_a && !box_b) {
    const T dx = oa.cx - ob.cx, dy = oa.cy - ob.cy;
    return pair_force_add(dx, dy, dot2(dx, dy, dx, dy), oa.vx - ob.vx, oa.vy - ob.vy,
                          ra + rb + W.margin, inv_denom, W, fx, fy);
  }
  // Broad phase: a box lies within its circumradius of its centre, so centres farther apart
  // than the two bounds plus the contact reach cannot touch (the exact test below would find
  // no overlap; the same slack as bounds_apart keeps every borderline pair).
  const T bnd_a = box_a ? norm2(oa.hx, oa.hy) : ra, bnd_b = box_b ? norm2(ob.hx, ob.hy) : rb;
  const T reach = box_a && box_b ? W.margin : (box_a ? rb : ra) + W.margin;
  if (bounds_apart(oa.cx - ob.cx, oa.cy - ob.cy, (box_a ? bnd_a : T(0)) + (box_b ? bnd_b : T(0)) +
                                                     reach))
    return false;
  T gx, gy;
  bool on;
  if (!box_a) {
    on = box_force_pair(oa.cx, oa.cy, oa.vx, oa.vy, obs_of(ob), ra + W.margin, inv_denom, W, gx, gy);
  } else if (!box_b) {
    on = box_force_pair(ob.cx, ob.cy, ob.vx, ob.vy, obs_of(oa), rb + W.margin, inv_denom, W, gx, gy);
    gx = -gx;
    gy = -gy;
  } else if (a < b) {
    on = obb_force(oa, ob, W.margin, inv_denom, W, gx, gy);
  } else {
    on = obb_force(ob, oa, W.margin, inv_denom, W, gx, gy);
    gx = -gx;
    gy = -gy;
  }
  fx = fx + gx;
  fy = fy + gy;
  return on;
}

// Obstacles and walls on a box agent (collisions.py:540-690), obstacles first.
template <typename T>
__device__ __noinline__ void box_static_force(const Obs<T>* sobs, int N, bool walls,
                                                 const Ob<T>& oa, T inv_denom,
                                                 const WorldC<T>& W, T& fx, T& fy) {
  T sx = T(0), sy = T(0);
  const T ra = norm2(oa.hx, oa.hy);
  for (int o = 0; o < N; ++o) {
    const Obs<T>& ob = sobs[o];
    if (bounds_apart(oa.cx - ob.cx, oa.cy - ob.cy, ra + W.margin + ob.bound)) continue;
    T gx = T(0), gy = T(0);
    if (ob.type == SHAPE_BOX || ob.type == SHAPE_SEGMENT) {
      const bool seg = ob.type == SHAPE_SEGMENT;
      const Ob<T> B{ob.cx, ob.cy, ob.ca, ob.sa, ob.hx, seg ? T(0) : ob.hy, ob.vx, ob.vy, ob.om};
      obb_force(oa, B, seg ? ob.r + W.margin : W.margin, inv_denom, W, gx, gy);
    } else {
      Obs<T> me = obs_of(oa);
      box_force(ob.cx, ob.cy, ob.vx, ob.vy, me, ob.r + W.margin, inv_denom, W, gx, gy);
      gx = -gx;
      gy = -gy;
    }
    sx = sx + gx;
    sy = sy + gy;
  }
  if (walls) {
    const T ex = oa.hx * fabs(oa.ca) + oa.hy * fabs(oa.sa);
    const T ey = oa.hx * fabs(oa.sa) + oa.hy * fabs(oa.ca);
    const T sc = sgn0(oa.ca), ss = sgn0(oa.sa);
    const T rly = -sc * oa.hx * oa.sa + ss * oa.hy * oa.ca;
    const T rbx = -ss * oa.hx * oa.ca + sc * oa.hy * oa.sa;
    T wx = T(0), wy = T(0);
    T pen = ex + W.margin - (oa.cx - W.bx0);
    if (pen > T(0)) wx = wx + normal_coeff(pen, oa.vx - oa.om * rly, inv_denom, W);
    pen = ex + W.margin - (W.bx1 - oa.cx);
    if (pen > T(0)) wx = wx + (-normal_coeff(pen, -(oa.vx + oa.om * rly), inv_denom, W));
    pen = ey + W.margin - (oa.cy - W.by0);
    if (pen > T(0)) wy = wy + normal_coeff(pen, oa.vy + oa.om * rbx, inv_denom, W);
    pen = ey + W.margin - (W.by1 - oa.cy);
    if (pen > T(0)) wy = wy + (-normal_coeff(pen, -(oa.vy - oa.om * rbx), inv_denom, W));
    sx = sx + wx;
    sy = sy + wy;
  }
  fx = fx + sx;
  fy = fy + sy;
}

// Force on a box agent (pose oa, inverse implicit denominator ida) from one obstacle
// shape, and the point it acts at (collisions.py:544-582, _box_obstacle_force): a BOX is
// the box-box contact with reach = margin, a SEGMENT the degenerate box (half length, 0)
// with reach = radius + margin, a CIRCLE the negated SDF law of its centre, acting there.
// box_static_force sums these forces on the agent; the body pass negates the same values
// for the reaction on a movable shape (bodies.py:131-166), lever = point - shape centre.
template <typename T>
__device__ __noinline__ void box_agent_shape_force(const Ob<T>& oa, const Obs<T>& ob, T ida,
                                                   const WorldC<T>& W, T& fx, T& fy, T& xx,
                                                   T& xy) {
  if (ob.type == SHAPE_BOX || ob.type == SHAPE_SEGMENT) {
    const bool seg = ob.type == SHAPE_SEGMENT;
    const Ob<T> B{ob.cx, ob.cy, ob.ca, ob.sa, ob.hx, seg ? T(0) : ob.hy, ob.vx, ob.vy, ob.om};
    obb_force_at(oa, B, seg ? ob.r + W.margin : W.margin, ida, W, fx, fy, xx, xy);
  } else {
    Obs<T> me = obs_of(oa);
    T gx, gy;
    box_force(ob.cx, ob.cy, ob.vx, ob.vy, me, ob.r + W.margin, ida, W, gx, gy);
    fx = -gx;
    fy = -gy;
    xx = ob.cx;
    xy = ob.cy;
  }
}

}  // namespace swarp
