// Movable compound rigid bodies inside the fused substep loop: forward pass and adjoint.
//
// Reference semantics: swarp/core/bodies.py:367-569 (obstacle_dynamics_kernel), its
// helpers _reaction (:79-127), _closest_in_box (:167-180), _body_body (:182-255), and the
// placement at stepper.py/_body_seed. A body is a set of obstacle shapes sharing one
// pose; its state lives at the root shape's slot. Each substep: the agent force pass
// reads the shapes' current poses, then the body pass sums the reactions of every agent
// contact (the negated agent-side force, so action and reaction are one number) and
// contacts with shapes of other bodies, integrates the body with linear/angular drag,
// clamps it inside the world bounds (zeroing the clamped velocity component), and
// re-places its shapes for the next substep. All bodies of an env are advanced by one
// thread, reading the other bodies' pre-pass poses.
//
// The reference does not differentiate bodies (its body pass is untaped). The adjoint
// here differentiates the body pass and the shape placement for bodies made of CIRCLE
// shapes (agent reactions, lever arms through the body angle, contacts with any other
// shape, drag, the clamp); bodies with box or segment shapes run forward only.
#pragma once
#include "boxes.cuh"
#include "physics.cuh"

namespace swarp {

template <typename T> struct BodyS {
  T qx, qy, th, vx, vy, om;
};

// Per-shape body constants.
template <typename T> struct BodyC {
  T offx, offy, mass, inertia;
  T reach;  // farthest point of the shape from its body origin (for the bounds clamp)
  int kind, body;
};

template <typename T>
__device__ __forceinline__ T shape_reach(int st, T offx, T offy, T r, T hx, T hy) {
  const T ax = fabs(offx), ay = fabs(offy);
  if (st == SHAPE_BOX) return Num<T>::sqrt_((ax + hx) * (ax + hx) + (ay + hy) * (ay + hy));
  if (st == SHAPE_SEGMENT) return Num<T>::sqrt_((ax + hx) * (ax + hx) + ay * ay) + r;
  return Num<T>::sqrt_(ax * ax + ay * ay) + r;
}

// Offset of a shape in world axes at body angle (ca, sa).
template <typename T>
__device__ __forceinline__ void body_offset(T ca, T sa, T offx, T offy, T& owx, T& owy) {
  owx = ca * offx - sa * offy;
  owy = sa * offx + ca * offy;
}

// Agent-side pose of a shape of body b (how the reference re-places shapes after a pass).
template <typename T>
__device__ __forceinline__ void place_shape(const BodyS<T>& b, const BodyC<T>& c, Obs<T>& o) {
  const T ca = Num<T>::cos_(b.th), sa = Num<T>::sin_(b.th);
  T owx, owy;
  body_offset(ca, sa, c.offx, c.offy, owx, owy);
  o.cx = b.qx + owx;
  o.cy = b.qy + owy;
  o.ca = ca;
  o.sa = sa;
  o.vx = b.vx - b.om * owy;
  o.vy = b.vy + b.om * owx;
  o.om = b.om;
}

// Closest point of a box (centre-relative vector d, body angle (ca, sa)) in world axes.
template <typename T>
__device__ __forceinline__ void closest_in_box(T dx, T dy, T ca, T sa, T hx, T hy, T& rx, T& ry) {
  const T lx = ca * dx + sa * dy, ly = -sa * dx + ca * dy;
  const T cx = wclamp(lx, -hx, hx), cy = wclamp(ly, -hy, hy);
  rx = ca * cx - sa * cy;
  ry = sa * cx + ca * cy;
}

// Force on the body shape `self` (pose s: centre, angle, surface velocity of its centre,
// spin) from an agent (disc of radius ra, inverse implicit denominator ida), and the lever
// from the shape centre.
template <typename T>
__device__ __forceinline__ void reaction(T px, T py, T vx, T vy, T ra, T ida, const Obs<T>& s,
                                         const WorldC<T>& W, T& fx, T& fy, T& rx, T& ry) {
  if (s.type == SHAPE_BOX) {
    box_force(px, py, vx, vy, s, ra + W.margin, ida, W, fx, fy);
    rx = px - s.cx;
    ry = py - s.cy;
  } else if (s.type == SHAPE_SEGMENT) {
    const T t = wclamp(dot2(px - s.cx, py - s.cy, s.ca, s.sa), -s.hx, s.hx);
    const T qx = s.cx + t * s.ca, qy = s.cy + t * s.sa;
    const T rrx = qx - s.cx, rry = qy - s.cy;
    const T vsx = s.vx + (-s.om * rry), vsy = s.vy + s.om * rrx;
    pair_force(px - qx, py - qy, vx - vsx, vy - vsy, ra + s.r + W.margin, ida, W, fx, fy);
    rx = rrx;
    ry = rry;
  } else {
    pair_force(px - s.cx, py - s.cy, vx - s.vx, vy - s.vy, ra + s.r + W.margin, ida, W, fx, fy);
    rx = T(0);
    ry = T(0);
  }
  fx = -fx;
  fy = -fy;
}

// Contact force on body shape `self` from another shape o2 (bodies.py:182-255); lever
// from the shape centre. ids = inverse implicit denominator of the self body.
template <typename T>
__device__ __forceinline__ void body_body(const Obs<T>& s, const Obs<T>& o2, T ids, const WorldC<T>& W,
                                          T& fx, T& fy, T& rx, T& ry) {
  fx = fy = rx = ry = T(0);
  if (s.type == SHAPE_BOX) {
    if (o2.type == SHAPE_BOX) return;  // box-box not modelled (reference)
    T c2x = o2.cx, c2y = o2.cy, v2x = o2.vx, v2y = o2.vy;
    if (o2.type == SHAPE_SEGMENT) {
      const T t = wclamp(dot2(s.cx - o2.cx, s.cy - o2.cy, o2.ca, o2.sa), -o2.hx, o2.hx);
      c2x = o2.cx + t * o2.ca;
      c2y = o2.cy + t * o2.sa;
      const T rrx = c2x - o2.cx, rry = c2y - o2.cy;
      v2x = o2.vx + (-o2.om * rry);
      v2y = o2.vy + o2.om * rrx;
    }
    T gx, gy;
    box_force(c2x, c2y, v2x, v2y, s, o2.r + W.margin, ids, W, gx, gy);
    fx = -gx;
    fy = -gy;
    closest_in_box(c2x - s.cx, c2y - s.cy, s.ca, s.sa, s.hx, s.hy, rx, ry);
  } else if (o2.type == SHAPE_BOX) {
    box_force(s.cx, s.cy, s.vx, s.vy, o2, s.r + W.margin, ids, W, fx, fy);
  } else if (o2.type == SHAPE_SEGMENT) {
    const T t = wclamp(dot2(s.cx - o2.cx, s.cy - o2.cy, o2.ca, o2.sa), -o2.hx, o2.hx);
    const T cpx = o2.cx + t * o2.ca, cpy = o2.cy + t * o2.sa;
    const T rrx = cpx - o2.cx, rry = cpy - o2.cy;
    const T vsx = o2.vx + (-o2.om * rry), vsy = o2.vy + o2.om * rrx;
    pair_force(s.cx - cpx, s.cy - cpy, s.vx - vsx, s.vy - vsy, s.r + o2.r + W.margin, ids, W, fx,
               fy);
  } else {
    pair_force(s.cx - o2.cx, s.cy - o2.cy, s.vx - o2.vx, s.vy - o2.vy, s.r + o2.r + W.margin, ids,
               W, fx, fy);
  }
}

// Reaction/contact sums of one root and the integration inputs/outputs.
template <typename T> struct BodyPassOut {
  T fx, fy, tau;
  T nvx_pre, nvy_pre, nx_pre, ny_pre;  // before the bounds clamp
  BodyS<T> next;
  bool clamp_x, clamp_y;
};

// Reaction of a box agent (heading th, turn rate w, half extents hx, hy; its record q and
// inverse implicit denominator ida) on the body shape `sh`: the negated force the agent
// feels from that shape (box_agent_shape_force, the function its own static pass sums)
// and the lever from the shape centre to the contact point (bodies.py:131-166).
template <typename T, typename T4>
__device__ __forceinline__ void reaction_box(const T4& q, T th, T w, T hx, T hy, T ida,
                                             const Obs<T>& sh, const WorldC<T>& W, T& fx, T& fy,
                                             T& rx, T& ry) {
  const Ob<T> oa{q.x, q.y, Num<T>::cos_(th), Num<T>::sin_(th), hx, hy, q.z, q.w, w};
  T gx, gy, xx, xy;
  box_agent_shape_force(oa, sh, ida, W, gx, gy, xx, xy);
  fx = -gx;
  fy = -gy;
  rx = xx - sh.cx;
  ry = xy - sh.cy;
}

// Forward body pass of root o of one env. `obs` holds the env's current shape poses;
// agent records rec (x, y, vx, vy), radii and inverse denominators for the reactions.
// Worlds with box agents also pass every agent's (heading, turn rate) pairs thw and
// (box flag, hx, hy, -) rows shp (both null otherwise).
template <typename T, typename T4>
__device__ __forceinline__ void body_pass_root(int o, const BodyS<T>& b, const BodyC<T>* bc,
                                               const Obs<T>* obs, int N, const T4* rec,
                                               const T* rad, const T* iden, int A,
                                               const WorldC<T>& W, bool clamp, BodyPassOut<T>& out,
                                               const T* thw = nullptr, const T* shp = nullptr) {
  const T dt = W.dt;
  const T ca = Num<T>::cos_(b.th), sa = Num<T>::sin_(b.th);
  T fx = T(0), fy = T(0), tau = T(0), ext = T(0);
  const T ids = T(1) / (T(1) + W.c * dt / bc[o].mass);
  for (int s = 0; s < N; ++s) {
    if (bc[s].body != o) continue;
    T owx, owy;
    body_offset(ca, sa, bc[s].offx, bc[s].offy, owx, owy);
    Obs<T> sh = obs[s];  // shape constants; pose from the body state
    sh.cx = b.qx + owx;
    sh.cy = b.qy + owy;
    sh.ca = ca;
    sh.sa = sa;
    sh.vx = b.vx - b.om * owy;
    sh.vy = b.vy + b.om * owx;
    sh.om = b.om;
    ext = wmax(ext, bc[s].reach);
    for (int a = 0; a < A; ++a) {
      const T4 q = rec[a];
      const bool boxa = shp != nullptr && shp[4 * a] > T(0.5);
      T hx = T(0), hy = T(0), rb = rad[a];
      if (boxa) {  // the agent's bounding disc: max(radius, half-diagonal)
        hx = shp[4 * a + 1];
        hy = shp[4 * a + 2];
        rb = wmax(rb, Num<T>::sqrt_(hx * hx + hy * hy));
      }
      if (bounds_apart(q.x - sh.cx, q.y - sh.cy, rb + sh.bound + W.margin)) continue;
      T gx, gy, rx, ry;
      if (boxa)
        reaction_box(q, thw[2 * a], thw[2 * a + 1], hx, hy, iden[a], sh, W, gx, gy, rx, ry);
      else
        reaction(q.x, q.y, q.z, q.w, rad[a], iden[a], sh, W, gx, gy, rx, ry);
      const T lx = owx + rx, ly = owy + ry;
      fx = fx + gx;
      fy = fy + gy;
      tau = tau + (lx * gy - ly * gx);
    }
    for (int o2 = 0; o2 < N; ++o2) {
      if (bc[o2].body == o) continue;
      if (bounds_apart(obs[o2].cx - sh.cx, obs[o2].cy - sh.cy, sh.bound + obs[o2].bound + W.margin))
        continue;
      T gx, gy, rx, ry;
      body_body(sh, obs[o2], ids, W, gx, gy, rx, ry);
      const T lx = owx + rx, ly = owy + ry;
      fx = fx + gx;
      fy = fy + gy;
      tau = tau + (lx * gy - ly * gx);
    }
  }
  const T m = bc[o].mass, I = bc[o].inertia;
  T nvx = (b.vx + fx / m * dt) * W.lin_decay;
  T nvy = (b.vy + fy / m * dt) * W.lin_decay;
  const T nom = (b.om + tau / I * dt) * W.ang_decay;
  T nx = b.qx + nvx * dt, ny = b.qy + nvy * dt;
  out.fx = fx;
  out.fy = fy;
  out.tau = tau;
  out.nvx_pre = nvx;
  out.nvy_pre = nvy;
  out.nx_pre = nx;
  out.ny_pre = ny;
  out.clamp_x = out.clamp_y = false;
  if (clamp) {
    const T lox = wmin(W.bx0 + ext, (W.bx0 + W.bx1) * T(0.5));
    const T hix = wmax(W.bx1 - ext, lox);
    const T loy = wmin(W.by0 + ext, (W.by0 + W.by1) * T(0.5));
    const T hiy = wmax(W.by1 - ext, loy);
    const T cx = wclamp(nx, lox, hix), cy = wclamp(ny, loy, hiy);
    if (cx != nx) {
      nvx = T(0);
      out.clamp_x = true;
    }
    if (cy != ny) {
      nvy = T(0);
      out.clamp_y = true;
    }
    nx = cx;
    ny = cy;
  }
  out.next = BodyS<T>{nx, ny, b.th + nom * dt, nvx, nvy, nom};
}

// ------------------------------------------------------------------- adjoint
// VJP of the agent-side force from a CIRCLE obstacle w.r.t. the obstacle's centre and
// velocity (the pair law depends on d = p - c and rv = v - v_obs only).
template <typename T>
__device__ __forceinline__ void circle_obstacle_vjp_pose(T px, T py, T vx, T vy, T ra, T ida,
                                                         const Obs<T>& o, T gx, T gy,
                                                         const WorldC<T>& W, T& gcx, T& gcy,
                                                         T& gvox, T& gvoy) {
  if (bounds_apart(px - o.cx, py - o.cy, ra + W.margin + o.bound)) return;
  T gdx = T(0), gdy = T(0), grx = T(0), gry = T(0);
  pair_force_vjp(px - o.cx, py - o.cy, vx - o.vx, vy - o.vy, ra + o.r + W.margin, ida, gx, gy, W,
                 gdx, gdy, grx, gry);
  gcx -= gdx;
  gcy -= gdy;
  gvox -= grx;
  gvoy -= gry;
}

// Cotangent of a body state.
template <typename T> struct BodyG {
  T qx, qy, th, vx, vy, om;
};

// Chain the cotangent of a circle shape's centre (gcx, gcy) and centre velocity
// (gvx, gvy) through its placement on body state b into gb.
template <typename T>
__device__ __forceinline__ void place_vjp(const BodyS<T>& b, const BodyC<T>& c, T gcx, T gcy, T gvx,
                                          T gvy, BodyG<T>& gb) {
  const T ca = Num<T>::cos_(b.th), sa = Num<T>::sin_(b.th);
  T owx, owy;
  body_offset(ca, sa, c.offx, c.offy, owx, owy);
  // centre = q + ow ; velocity = v + om x ow
  gb.qx += gcx;
  gb.qy += gcy;
  gb.vx += gvx;
  gb.vy += gvy;
  gb.om += -owy * gvx + owx * gvy;
  const T gowx = gcx + b.om * gvy;
  const T gowy = gcy - b.om * gvx;
  // d ow / d th = (-owy, owx)
  gb.th += -owy * gowx + owx * gowy;
}

// Adjoint of body_pass_root for a body of CIRCLE shapes. gnext: cotangent of the new
// body state. Adds: agent cotangents (pos, vel) into gag[a] (x, y, vx, vy), the
// cotangents of other movable shapes' centre/velocity into gshape[o2], and returns the
// cotangent of this body's input state (direct terms; the caller adds the placement
// terms of this body's shapes from gshape).
template <typename T, typename T4>
__device__ __forceinline__ void body_pass_root_vjp(int o, const BodyS<T>& b, const BodyC<T>* bc,
                                                   const Obs<T>* obs, int N, const T4* rec,
                                                   const T* rad, const T* iden, int A,
                                                   const WorldC<T>& W, bool clamp,
                                                   const BodyG<T>& gnext, T4* gag, T4* gshape,
                                                   BodyG<T>& gb) {
  BodyPassOut<T> P;
  body_pass_root(o, b, bc, obs, N, rec, rad, iden, A, W, clamp, P);
  const T dt = W.dt;
  const T m = bc[o].mass, I = bc[o].inertia;
  // position: clamp passes the gradient unless the axis was clamped (then the velocity
  // of that axis is zeroed too)
  T gnvx = P.clamp_x ? T(0) : gnext.vx + gnext.qx * dt;
  T gnvy = P.clamp_y ? T(0) : gnext.vy + gnext.qy * dt;
  gb.qx += P.clamp_x ? T(0) : gnext.qx;
  gb.qy += P.clamp_y ? T(0) : gnext.qy;
  // angle and spin
  gb.th += gnext.th;
  const T gnom = gnext.om + gnext.th * dt;
  gb.om += gnom * W.ang_decay;
  const T gtau = gnom * W.ang_decay / I * dt;
  gb.vx += gnvx * W.lin_decay;
  gb.vy += gnvy * W.lin_decay;
  const T gfx = gnvx * W.lin_decay / m * dt;
  const T gfy = gnvy * W.lin_decay / m * dt;

  const T ca = Num<T>::cos_(b.th), sa = Num<T>::sin_(b.th);
  const T ids = T(1) / (T(1) + W.c * dt / m);
  for (int s = 0; s < N; ++s) {
    if (bc[s].body != o) continue;
    T owx, owy;
    body_offset(ca, sa, bc[s].offx, bc[s].offy, owx, owy);
    Obs<T> sh = obs[s];
    sh.cx = b.qx + owx;
    sh.cy = b.qy + owy;
    sh.ca = ca;
    sh.sa = sa;
    sh.vx = b.vx - b.om * owy;
    sh.vy = b.vy + b.om * owx;
    sh.om = b.om;
    T gcx = T(0), gcy = T(0), gvx = T(0), gvy = T(0), gowx = T(0), gowy = T(0);
    for (int a = 0; a < A; ++a) {
      const T4 q = rec[a];
      if (bounds_apart(q.x - sh.cx, q.y - sh.cy, rad[a] + sh.bound + W.margin)) continue;
      T fx, fy, rx, ry;
      reaction(q.x, q.y, q.z, q.w, rad[a], iden[a], sh, W, fx, fy, rx, ry);  // rx = ry = 0
      // F += f ; tau += ow x f   (lever ow + 0 for a circle)
      const T gx = gfx - owy * gtau, gy = gfy + owx * gtau;
      gowx += fy * gtau;
      gowy += -fx * gtau;
      // f = -pair(p_a - c_s, v_a - v_s)
      T gdx = T(0), gdy = T(0), grx = T(0), gry = T(0);
      pair_force_vjp(q.x - sh.cx, q.y - sh.cy, q.z - sh.vx, q.w - sh.vy, rad[a] + sh.r + W.margin,
                     iden[a], -gx, -gy, W, gdx, gdy, grx, gry);
      T4 ga = gag[a];
      ga.x += gdx;
      ga.y += gdy;
      ga.z += grx;
      ga.w += gry;
      gag[a] = ga;
      gcx -= gdx;
      gcy -= gdy;
      gvx -= grx;
      gvy -= gry;
    }
    for (int o2 = 0; o2 < N; ++o2) {
      if (bc[o2].body == o) continue;
      const Obs<T>& oo = obs[o2];
      if (bounds_apart(oo.cx - sh.cx, oo.cy - sh.cy, sh.bound + oo.bound + W.margin)) continue;
      T fx, fy, rx, ry;
      body_body(sh, oo, ids, W, fx, fy, rx, ry);  // round self: rx = ry = 0
      const T gx = gfx - owy * gtau, gy = gfy + owx * gtau;
      gowx += fy * gtau;
      gowy += -fx * gtau;
      // round self against o2 is the agent-side law with self as the disc
      T gpx = T(0), gpy = T(0), gpvx = T(0), gpvy = T(0);
      obstacle_force_vjp(sh.cx, sh.cy, sh.vx, sh.vy, sh.r, ids, oo, gx, gy, W, gpx, gpy, gpvx,
                         gpvy);
      gcx += gpx;
      gcy += gpy;
      gvx += gpvx;
      gvy += gpvy;
      if (bc[o2].kind == 1 && oo.type == SHAPE_CIRCLE) {
        // other movable circle: its centre/velocity enter as -d and -rv
        T4 gs = gshape[o2];
        T gdx = T(0), gdy = T(0), grx = T(0), gry = T(0);
        pair_force_vjp(sh.cx - oo.cx, sh.cy - oo.cy, sh.vx - oo.vx, sh.vy - oo.vy,
                       sh.r + oo.r + W.margin, ids, gx, gy, W, gdx, gdy, grx, gry);
        gs.x -= gdx;
        gs.y -= gdy;
        gs.z -= grx;
        gs.w -= gry;
        gshape[o2] = gs;
      }
    }
    // shape centre / velocity / offset -> body state
    gb.qx += gcx;
    gb.qy += gcy;
    gb.vx += gvx;
    gb.vy += gvy;
    gb.om += -owy * gvx + owx * gvy;
    gowx += gcx + b.om * gvy;
    gowy += gcy - b.om * gvx;
    gb.th += -owy * gowx + owx * gowy;
  }
}

}  // namespace swarp
