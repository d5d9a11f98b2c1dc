/*
 * CPU restatement (plain C + OpenMP) of swarp's differentiable rollout: forward and
 * hand-written reverse-mode adjoint. TEST INFRASTRUCTURE / CPU BASELINE ONLY: it is the
 * timed CPU baseline of bench.py and a cross-check of the CUDA adjoint in the tests;
 * the product (swarp_b200) never links or calls it.
 *
 * Forward semantics follow the reference (ddebenedittis/swarp) operation by operation,
 * with IEEE division and square root as written there:
 *   clamp_norm            swarp/dynamics/kernels.py:68-71
 *   servo_command         swarp/dynamics/kernels.py:166-190
 *   _step_2d              swarp/dynamics/kernels.py:194-275
 *   disc bounds clamp     swarp/dynamics/kernels.py:395-403
 *   _normal_coeff         swarp/core/collisions.py:87-106
 *   pair_force            swarp/core/collisions.py:109-143
 *   closest_on_segment    swarp/core/collisions.py:156-171
 *   box_force             swarp/core/collisions.py:174-260
 *   shape_bound / bounds_apart  swarp/core/collisions.py:61-84
 *   obstacle / wall forces      swarp/core/collisions.py:690-780
 *   collision_forces_kernel     swarp/core/collisions.py:818-881 (list-order gather)
 *   _brute_force          swarp/core/neighbors.py:76-97
 *   _compute_keys / _query_uniform, static frame
 *                         swarp/core/neighbors.py:182-254, 591-620 (list_order 1: the
 *                         uniform grid's (3 x 3 block cell, index) list order)
 *   substep order         swarp/core/stepper.py:549-648 (neighbors, forces, integrate)
 * The adjoint differentiates these with Warp's branch conventions at kinks (max sends
 * the gradient to the second argument on a tie, clamp passes it on the closed
 * interval, length has zero gradient at the zero vector). Envs run in parallel
 * (OpenMP); within an env the adjoint scatters pair contributions sequentially.
 *
 * Compiled once per precision: REAL=float -> *_f32 symbols, REAL=double -> *_f64.
 */
#include <tgmath.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifndef REAL
#define REAL double
#define SFX(name) name##_f64
#endif
typedef REAL real;

#define EPS2 ((real)1.0e-10)

typedef struct {
  int n_envs, n_agents, act_dim, substeps, horizon;
  double dt;
  int collisions;
  double k, c, margin, max_overlap, neighbor_radius;
  int max_neighbors;
  int bounds_mode; /* 0 none, 1 soft walls, 2 clamp */
  double bounds[4];
  const double* params; /* [A,22] or [E,A,22] */
  long params_env_stride;
  const int* model_tag;
  const int* ctrl_mode;
  int n_obstacles;
  const double *obs_pos, *obs_angle, *obs_vel, *obs_ang_vel, *obs_radius, *obs_half;
  const int* obs_shape;
  int threads;
  /* 0: ascending index (brute force); 1: the radix-sort uniform grid's order with a
     static frame: cells clamp((p - origin) / cell, 0, bins - 1) per axis */
  int list_order, grid_bins;
  double grid_origin[2], grid_cell;
} cpu_world_t;

typedef struct {
  real radius, mass, max_speed, min_speed, max_accel, max_ang_vel, max_ang_accel;
  real l_f, l_r, max_steer, gain_v, gain_w;
  int tag, mode;
} prm_t;

typedef struct { real px, py, th, vx, vy, s, w; } st_t;

typedef struct {
  real dt, k, c, margin, mo;
  real bx0, bx1, by0, by1;
  real R;
  int K, bounds_mode;
  int order, bins; /* list order (cpu_world_t.list_order) and grid cells per axis */
  real ox, oy, cs;
} wc_t;

static inline real wmax(real a, real b) { return a > b ? a : b; }
static inline real wmin(real a, real b) { return a < b ? a : b; }
static inline real wclamp(real x, real lo, real hi) { return wmin(wmax(lo, x), hi); }
static inline int pass(real x, real lo, real hi) { return !(x < lo) && !(x > hi); }

/* ------------------------------------------------------------ contact law */
static inline real ncoef(real ov, real vn, real denom, const wc_t* W) {
  real ovs = ov;
  if (W->mo > 0) ovs = W->mo * tanh(ov / W->mo);
  return wmax((W->k * ovs - W->c * vn) / denom, (real)0);
}
static inline void ncoef_vjp(real ov, real vn, real denom, real g, const wc_t* W, real* gov,
                             real* gvn) {
  real ovs = ov, th = 0;
  if (W->mo > 0) {
    th = tanh(ov / W->mo);
    ovs = W->mo * th;
  }
  real x = (W->k * ovs - W->c * vn) / denom;
  if (x > 0) {
    real gn = g / denom;
    *gvn = -W->c * gn;
    *gov = W->mo > 0 ? W->k * gn * (1 - th * th) : W->k * gn;
  } else {
    *gov = 0;
    *gvn = 0;
  }
}
static inline void pair_f(real dx, real dy, real rvx, real rvy, real md, real denom,
                          const wc_t* W, real* fx, real* fy) {
  real dist = sqrt(wmax(dx * dx + dy * dy, EPS2));
  real ov = md - dist;
  *fx = 0;
  *fy = 0;
  if (ov > 0) {
    real nx = dx / dist, ny = dy / dist;
    real cf = ncoef(ov, rvx * nx + rvy * ny, denom, W);
    *fx = cf * nx;
    *fy = cf * ny;
  }
}
/* adds d(g.f)/dd and d(g.f)/drv */
static inline void pair_vjp(real dx, real dy, real rvx, real rvy, real md, real denom, real gx,
                            real gy, const wc_t* W, real* gdx, real* gdy, real* grx, real* gry) {
  real d2 = dx * dx + dy * dy;
  real dist = sqrt(wmax(d2, EPS2));
  real ov = md - dist;
  if (!(ov > 0)) return;
  real nx = dx / dist, ny = dy / dist;
  real vn = rvx * nx + rvy * ny;
  real cf = ncoef(ov, vn, denom, W);
  real gcf = gx * nx + gy * ny;
  real gnx = cf * gx, gny = cf * gy, gov, gvn;
  ncoef_vjp(ov, vn, denom, gcf, W, &gov, &gvn);
  *grx += gvn * nx;
  *gry += gvn * ny;
  gnx += gvn * rvx;
  gny += gvn * rvy;
  real gdist = -gov - (gnx * nx + gny * ny) / dist;
  real ddx = gnx / dist, ddy = gny / dist;
  if (d2 > EPS2) {
    real gd2 = gdist * 0.5 / dist;
    ddx += 2 * dx * gd2;
    ddy += 2 * dy * gd2;
  }
  *gdx += ddx;
  *gdy += ddy;
}

/* ------------------------------------------------------------ obstacles */
typedef struct { real cx, cy, ang, vx, vy, om, r, hx, hy; int type; } ob_t;

static inline real shape_bound(const ob_t* o) {
  if (o->type == 1) return sqrt(o->hx * o->hx + o->hy * o->hy);
  if (o->type == 2) return o->hx + o->r;
  return o->r;
}
static inline int apart(real dx, real dy, real reach) {
  real lim = reach * (real)1.0001 + (real)1.0e-6;
  return dx * dx + dy * dy > lim * lim;
}

static void box_f(real px, real py, real vx, real vy, const ob_t* o, real reach, real denom,
                  const wc_t* W, real* fx, real* fy, real* gpx, real* gpy, real* gvx, real* gvy,
                  real gx, real gy) {
  /* forward if gpx == NULL, else VJP with cotangent (gx, gy) */
  real ca = cos(o->ang), sa = sin(o->ang);
  real dx = px - o->cx, dy = py - o->cy;
  real lx = ca * dx + sa * dy, ly = -sa * dx + ca * dy;
  real qx = fabs(lx) - o->hx, qy = fabs(ly) - o->hy;
  real cx = wclamp(lx, -o->hx, o->hx), cy = wclamp(ly, -o->hy, o->hy);
  real ox = lx - cx, oy = ly - cy, od2 = ox * ox + oy * oy;
  real s, nlx, nly;
  int ext = od2 > EPS2, ux = qx > qy;
  if (ext) {
    s = sqrt(od2);
    nlx = ox / s;
    nly = oy / s;
  } else if (ux) {
    s = qx;
    nlx = lx >= 0 ? 1 : -1;
    nly = 0;
  } else {
    s = qy;
    nlx = 0;
    nly = ly >= 0 ? 1 : -1;
  }
  real ov = reach - s;
  if (fx) {
    *fx = 0;
    *fy = 0;
  }
  if (!(ov > 0)) return;
  real nx = ca * nlx - sa * nly, ny = sa * nlx + ca * nly;
  real spx = lx - s * nlx, spy = ly - s * nly;
  real rx = ca * spx - sa * spy, ry = sa * spx + ca * spy;
  real vsx = o->vx + (-o->om * ry), vsy = o->vy + o->om * rx;
  real relx = vx - vsx, rely = vy - vsy;
  real vn = relx * nx + rely * ny;
  real cf = ncoef(ov, vn, denom, W);
  if (fx) {
    *fx = cf * nx;
    *fy = cf * ny;
    return;
  }
  real gcf = gx * nx + gy * ny, gnx = cf * gx, gny = cf * gy, gov, gvn;
  ncoef_vjp(ov, vn, denom, gcf, W, &gov, &gvn);
  real grelx = gvn * nx, grely = gvn * ny;
  gnx += gvn * relx;
  gny += gvn * rely;
  *gvx += grelx;
  *gvy += grely;
  real grx = o->om * (-grely), gry = -o->om * (-grelx);
  real gspx = ca * grx + sa * gry, gspy = -sa * grx + ca * gry;
  real glx = gspx, gly = gspy;
  real gs = -(nlx * gspx + nly * gspy) - gov;
  real gnlx = -s * gspx + (ca * gnx + sa * gny);
  real gnly = -s * gspy + (-sa * gnx + ca * gny);
  if (ext) {
    real gox = gnlx / s, goy = gnly / s;
    gs -= (gnlx * nlx + gnly * nly) / s;
    real god2 = gs * 0.5 / s;
    gox += 2 * ox * god2;
    goy += 2 * oy * god2;
    glx += gox - (pass(lx, -o->hx, o->hx) ? gox : 0);
    gly += goy - (pass(ly, -o->hy, o->hy) ? goy : 0);
  } else if (ux) {
    glx += lx < 0 ? -gs : gs;
  } else {
    gly += ly < 0 ? -gs : gs;
  }
  *gpx += ca * glx - sa * gly;
  *gpy += sa * glx + ca * gly;
}

static void obstacle_f(real px, real py, real vx, real vy, real ra, real denom, const ob_t* o,
                       const wc_t* W, real* fx, real* fy) {
  *fx = 0;
  *fy = 0;
  if (apart(px - o->cx, py - o->cy, ra + W->margin + shape_bound(o))) return;
  if (o->type == 1) {
    box_f(px, py, vx, vy, o, ra + W->margin, denom, W, fx, fy, 0, 0, 0, 0, 0, 0);
  } else if (o->type == 2) {
    real ux = cos(o->ang), uy = sin(o->ang);
    real t = wclamp((px - o->cx) * ux + (py - o->cy) * uy, -o->hx, o->hx);
    real qx = o->cx + t * ux, qy = o->cy + t * uy;
    real rx = qx - o->cx, ry = qy - o->cy;
    pair_f(px - qx, py - qy, vx - (o->vx + (-o->om * ry)), vy - (o->vy + o->om * rx),
           ra + o->r + W->margin, denom, W, fx, fy);
  } else {
    pair_f(px - o->cx, py - o->cy, vx - o->vx, vy - o->vy, ra + o->r + W->margin, denom, W, fx,
           fy);
  }
}

static void obstacle_vjp(real px, real py, real vx, real vy, real ra, real denom, const ob_t* o,
                         const wc_t* W, real gx, real gy, real* gpx, real* gpy, real* gvx,
                         real* gvy) {
  if (apart(px - o->cx, py - o->cy, ra + W->margin + shape_bound(o))) return;
  if (o->type == 1) {
    box_f(px, py, vx, vy, o, ra + W->margin, denom, W, 0, 0, gpx, gpy, gvx, gvy, gx, gy);
  } else if (o->type == 2) {
    real ux = cos(o->ang), uy = sin(o->ang);
    real sp = (px - o->cx) * ux + (py - o->cy) * uy;
    real t = wclamp(sp, -o->hx, o->hx);
    real qx = o->cx + t * ux, qy = o->cy + t * uy;
    real rx = qx - o->cx, ry = qy - o->cy;
    real gdx = 0, gdy = 0, grx = 0, gry = 0;
    pair_vjp(px - qx, py - qy, vx - (o->vx + (-o->om * ry)), vy - (o->vy + o->om * rx),
             ra + o->r + W->margin, denom, gx, gy, W, &gdx, &gdy, &grx, &gry);
    *gpx += gdx;
    *gpy += gdy;
    *gvx += grx;
    *gvy += gry;
    real gqx = -gdx + o->om * (-gry), gqy = -gdy - o->om * (-grx);
    real gt = gqx * ux + gqy * uy;
    if (pass(sp, -o->hx, o->hx)) {
      *gpx += gt * ux;
      *gpy += gt * uy;
    }
  } else {
    real gdx = 0, gdy = 0, grx = 0, gry = 0;
    pair_vjp(px - o->cx, py - o->cy, vx - o->vx, vy - o->vy, ra + o->r + W->margin, denom, gx, gy,
             W, &gdx, &gdy, &grx, &gry);
    *gpx += gdx;
    *gpy += gdy;
    *gvx += grx;
    *gvy += gry;
  }
}

/* ------------------------------------------------------------------ walls */
static void wall_f(real px, real py, real vx, real vy, real ra, real denom, const wc_t* W,
                   real* fx, real* fy) {
  real reach = ra + W->margin, pen;
  *fx = 0;
  *fy = 0;
  pen = reach - (px - W->bx0);
  if (pen > 0) *fx += ncoef(pen, vx, denom, W);
  pen = reach - (W->bx1 - px);
  if (pen > 0) *fx += -ncoef(pen, -vx, denom, W);
  pen = reach - (py - W->by0);
  if (pen > 0) *fy += ncoef(pen, vy, denom, W);
  pen = reach - (W->by1 - py);
  if (pen > 0) *fy += -ncoef(pen, -vy, denom, W);
}
static void wall_vjp(real px, real py, real vx, real vy, real ra, real denom, const wc_t* W,
                     real gx, real gy, real* gpx, real* gpy, real* gvx, real* gvy) {
  real reach = ra + W->margin, pen, gov, gvn;
  pen = reach - (px - W->bx0);
  if (pen > 0) {
    ncoef_vjp(pen, vx, denom, gx, W, &gov, &gvn);
    *gpx -= gov;
    *gvx += gvn;
  }
  pen = reach - (W->bx1 - px);
  if (pen > 0) {
    ncoef_vjp(pen, -vx, denom, -gx, W, &gov, &gvn);
    *gpx += gov;
    *gvx -= gvn;
  }
  pen = reach - (py - W->by0);
  if (pen > 0) {
    ncoef_vjp(pen, vy, denom, gy, W, &gov, &gvn);
    *gpy -= gov;
    *gvy += gvn;
  }
  pen = reach - (W->by1 - py);
  if (pen > 0) {
    ncoef_vjp(pen, -vy, denom, -gy, W, &gov, &gvn);
    *gpy += gov;
    *gvy -= gvn;
  }
}

/* -------------------------------------------------------------- integrate */
static inline void cnorm(real x, real y, real L, real* ox, real* oy) {
  real n = sqrt(x * x + y * y);
  real sc = L / wmax(n, L);
  *ox = x * sc;
  *oy = y * sc;
}
static inline void cnorm_vjp(real x, real y, real L, real gx, real gy, real* rx, real* ry) {
  real n = sqrt(x * x + y * y), mx = wmax(n, L), sc = L / mx;
  *rx = gx * sc;
  *ry = gy * sc;
  if (n > L) {
    real gn = -(gx * x + gy * y) * sc / mx;
    *rx += x / n * gn;
    *ry += y / n * gn;
  }
}
static inline void servo(real a0, real a1, real s, real w, const prm_t* P, real dt, real* c0,
                         real* c1) {
  real tv = wclamp(a0, -P->max_speed, P->max_speed) * P->gain_v;
  real tw = wclamp(a1, -P->max_ang_vel, P->max_ang_vel) * P->gain_w;
  real dv = P->max_accel * dt, dw = P->max_ang_accel * dt;
  *c0 = s + wclamp(tv - s, -dv, dv);
  *c1 = w + wclamp(tw - w, -dw, dw);
}

static void integ(const st_t* in, real a0, real a1, real fx, real fy, const prm_t* P,
                  const wc_t* W, st_t* out) {
  real dt = W->dt;
  int mode = P->mode;
  if (mode == 2) {
    servo(a0, a1, in->s, in->w, P, dt, &a0, &a1);
    mode = 0;
  }
  real dvx = fx * (dt / P->mass), dvy = fy * (dt / P->mass);
  if (P->tag == 0) {
    real vx, vy;
    if (mode == 0) {
      cnorm(a0, a1, P->max_speed, &vx, &vy);
    } else {
      real ax, ay;
      cnorm(a0, a1, P->max_accel, &ax, &ay);
      cnorm(in->vx + ax * dt, in->vy + ay * dt, P->max_speed, &vx, &vy);
    }
    vx = vx + dvx;
    vy = vy + dvy;
    out->px = in->px + vx * dt;
    out->py = in->py + vy * dt;
    out->th = in->th;
    out->vx = vx;
    out->vy = vy;
    out->s = sqrt(vx * vx + vy * vy);
    out->w = 0;
  } else if (P->tag == 1) {
    real sn, wn;
    if (mode == 0) {
      sn = wclamp(a0, -P->max_speed, P->max_speed);
      wn = wclamp(a1, -P->max_ang_vel, P->max_ang_vel);
    } else {
      sn = wclamp(in->s + wclamp(a0, -P->max_accel, P->max_accel) * dt, -P->max_speed, P->max_speed);
      wn = wclamp(in->w + wclamp(a1, -P->max_ang_accel, P->max_ang_accel) * dt, -P->max_ang_vel,
                  P->max_ang_vel);
    }
    real vx = sn * cos(in->th) + dvx, vy = sn * sin(in->th) + dvy;
    out->px = in->px + vx * dt;
    out->py = in->py + vy * dt;
    out->th = in->th + wn * dt;
    out->vx = vx;
    out->vy = vy;
    out->s = sn;
    out->w = wn;
  } else {
    real acc = wclamp(a0, -P->max_accel, P->max_accel);
    real delta = wclamp(a1, -P->max_steer, P->max_steer);
    real sn = wclamp(in->s + acc * dt, P->min_speed, P->max_speed);
    real wb = P->l_f + P->l_r;
    real beta = atan(tan(delta) * P->l_r / wb);
    real vx = sn * cos(in->th + beta) + dvx, vy = sn * sin(in->th + beta) + dvy;
    real wn = sn / wb * cos(beta) * tan(delta);
    out->px = in->px + vx * dt;
    out->py = in->py + vy * dt;
    out->th = in->th + wn * dt;
    out->vx = vx;
    out->vy = vy;
    out->s = sn;
    out->w = wn;
  }
  if (W->bounds_mode == 2) {
    out->px = wclamp(out->px, W->bx0 + P->radius, W->bx1 - P->radius);
    out->py = wclamp(out->py, W->by0 + P->radius, W->by1 - P->radius);
  }
}

/* VJP of integ: gin <- direct input gradients, (gfx, gfy) force cotangent, ga += action */
static void integ_vjp(const st_t* in, real a0, real a1, const st_t* out, const st_t* g,
                      const prm_t* P, const wc_t* W, st_t* gin, real* gfx, real* gfy, real* ga0,
                      real* ga1) {
  real dt = W->dt;
  memset(gin, 0, sizeof(*gin));
  real gpx = g->px, gpy = g->py;
  if (W->bounds_mode == 2) {
    if (!pass(in->px + out->vx * dt, W->bx0 + P->radius, W->bx1 - P->radius)) gpx = 0;
    if (!pass(in->py + out->vy * dt, W->by0 + P->radius, W->by1 - P->radius)) gpy = 0;
  }
  int mode = P->mode;
  real c0 = a0, c1 = a1, gc0 = 0, gc1 = 0;
  if (mode == 2) {
    servo(a0, a1, in->s, in->w, P, dt, &c0, &c1);
    mode = 0;
  }
  gin->px = gpx;
  gin->py = gpy;
  real gvx = g->vx + gpx * dt, gvy = g->vy + gpy * dt;
  real k = dt / P->mass;
  if (P->tag == 0) {
    real n = sqrt(out->vx * out->vx + out->vy * out->vy);
    if (n > 0) {
      gvx += out->vx / n * g->s;
      gvy += out->vy / n * g->s;
    }
    gin->th = g->th;
    *gfx = gvx * k;
    *gfy = gvy * k;
    if (mode == 0) {
      cnorm_vjp(c0, c1, P->max_speed, gvx, gvy, &gc0, &gc1);
    } else {
      real ax, ay, gux, guy;
      cnorm(c0, c1, P->max_accel, &ax, &ay);
      cnorm_vjp(in->vx + ax * dt, in->vy + ay * dt, P->max_speed, gvx, gvy, &gux, &guy);
      gin->vx = gux;
      gin->vy = guy;
      cnorm_vjp(c0, c1, P->max_accel, gux * dt, guy * dt, &gc0, &gc1);
    }
  } else if (P->tag == 1) {
    real c = cos(in->th), s = sin(in->th), sn = out->s;
    *gfx = gvx * k;
    *gfy = gvy * k;
    real gsn = g->s + gvx * c + gvy * s;
    gin->th = g->th + sn * (c * gvy - s * gvx);
    real gwn = g->w + g->th * dt;
    if (mode == 0) {
      gc0 = pass(c0, -P->max_speed, P->max_speed) ? gsn : 0;
      gc1 = pass(c1, -P->max_ang_vel, P->max_ang_vel) ? gwn : 0;
    } else {
      real acc = wclamp(c0, -P->max_accel, P->max_accel);
      real alp = wclamp(c1, -P->max_ang_accel, P->max_ang_accel);
      real gus = pass(in->s + acc * dt, -P->max_speed, P->max_speed) ? gsn : 0;
      real guw = pass(in->w + alp * dt, -P->max_ang_vel, P->max_ang_vel) ? gwn : 0;
      gin->s = gus;
      gin->w = guw;
      gc0 = pass(c0, -P->max_accel, P->max_accel) ? gus * dt : 0;
      gc1 = pass(c1, -P->max_ang_accel, P->max_ang_accel) ? guw * dt : 0;
    }
  } else {
    real acc = wclamp(c0, -P->max_accel, P->max_accel);
    real delta = wclamp(c1, -P->max_steer, P->max_steer);
    real us = in->s + acc * dt, sn = out->s, wb = P->l_f + P->l_r;
    real td = tan(delta), z = td * P->l_r / wb, beta = atan(z);
    real ca = cos(in->th + beta), sa = sin(in->th + beta), cb = cos(beta), sb = sin(beta);
    *gfx = gvx * k;
    *gfy = gvy * k;
    real gwn = g->w + g->th * dt;
    real gsn = g->s + gvx * ca + gvy * sa;
    real gang = sn * (ca * gvy - sa * gvx);
    gin->th = g->th + gang;
    real q = sn / wb, sec2 = 1 + td * td;
    gsn += gwn * td * cb / wb;
    real gbeta = gang - gwn * td * q * sb;
    real gdelta = gwn * q * cb * sec2 + gbeta / (1 + z * z) * P->l_r / wb * sec2;
    real gus = pass(us, P->min_speed, P->max_speed) ? gsn : 0;
    gin->s = gus;
    gc0 = pass(c0, -P->max_accel, P->max_accel) ? gus * dt : 0;
    gc1 = pass(c1, -P->max_steer, P->max_steer) ? gdelta : 0;
  }
  if (P->mode == 2) {
    real tv = wclamp(a0, -P->max_speed, P->max_speed) * P->gain_v;
    real tw = wclamp(a1, -P->max_ang_vel, P->max_ang_vel) * P->gain_w;
    real dv = P->max_accel * dt, dw = P->max_ang_accel * dt;
    real gd0 = pass(tv - in->s, -dv, dv) ? gc0 : 0, gd1 = pass(tw - in->w, -dw, dw) ? gc1 : 0;
    gin->s += gc0 - gd0;
    gin->w += gc1 - gd1;
    *ga0 += pass(a0, -P->max_speed, P->max_speed) ? gd0 * P->gain_v : 0;
    *ga1 += pass(a1, -P->max_ang_vel, P->max_ang_vel) ? gd1 * P->gain_w : 0;
  } else {
    *ga0 += gc0;
    *ga1 += gc1;
  }
}

/* ------------------------------------------------------------- one env */
typedef struct {
  int A, K;
  int* list;   /* [A*A] neighbor indices per agent (capped, in list order) */
  int* nlist;  /* [A] */
  int *cell, *cstart, *cfill, *csorted; /* grid order: [A] cells, [bins^2+1] starts,
                                          [bins^2] cursors, [A] agents by cell */
  real *fx, *fy, *gfx, *gfy;
  st_t *sub;   /* [S+1][A] substep states of the current step */
} scratch_t;

static inline int grid_cell(real p, real o, const wc_t* W) {
  int c = (int)((p - o) / W->cs); /* truncation toward zero, as wp.int32() */
  return c < 0 ? 0 : (c > W->bins - 1 ? W->bins - 1 : c);
}

/* The uniform grid's lists: agents bucketed by cell in ascending index (the stable radix
   sort), then per agent the 3 x 3 block, rows dy = -1..1, columns dx = -1..1. */
static void grid_lists(const st_t* x, int A, const wc_t* W, scratch_t* sc) {
  const int B = W->bins, NC = B * B;
  for (int c = 0; c <= NC; ++c) sc->cstart[c] = 0;
  for (int a = 0; a < A; ++a) {
    sc->cell[a] = grid_cell(x[a].py, W->oy, W) * B + grid_cell(x[a].px, W->ox, W);
    ++sc->cstart[sc->cell[a] + 1];
  }
  for (int c = 0; c < NC; ++c) sc->cstart[c + 1] += sc->cstart[c];
  for (int c = 0; c < NC; ++c) sc->cfill[c] = sc->cstart[c];
  for (int a = 0; a < A; ++a) sc->csorted[sc->cfill[sc->cell[a]]++] = a;  /* stable */
  for (int a = 0; a < A; ++a) {
    const int cy = sc->cell[a] / B, cx = sc->cell[a] - cy * B;
    int n = 0;
    for (int dy = -1; dy <= 1; ++dy) {
      const int ny = cy + dy;
      if (ny < 0 || ny >= B) continue;
      for (int dx = -1; dx <= 1; ++dx) {
        const int nx = cx + dx;
        if (nx < 0 || nx >= B) continue;
        const int c = ny * B + nx;
        for (int i = sc->cstart[c]; i < sc->cstart[c + 1]; ++i) {
          const int b = sc->csorted[i];
          if (b == a) continue;
          real ddx = x[b].px - x[a].px, ddy = x[b].py - x[a].py;
          if (sqrt(ddx * ddx + ddy * ddy) <= W->R) {
            if (n < W->K) sc->list[a * A + n] = b;
            ++n;
          }
        }
      }
    }
    sc->nlist[a] = n < W->K ? n : W->K;
  }
}

static void neighbor_lists(const st_t* x, int A, const wc_t* W, scratch_t* sc) {
  if (W->order == 1) {
    grid_lists(x, A, W, sc);
    return;
  }
  for (int a = 0; a < A; ++a) {
    int n = 0;
    for (int b = 0; b < A; ++b) {
      if (b == a) continue;
      real dx = x[b].px - x[a].px, dy = x[b].py - x[a].py;
      if (sqrt(dx * dx + dy * dy) <= W->R) {
        if (n < W->K) sc->list[a * A + n] = b;
        ++n;
      }
    }
    sc->nlist[a] = n < W->K ? n : W->K;
  }
}

static void forces(const st_t* x, const prm_t* P, const ob_t* obs, int N, const wc_t* W,
                   int coll, scratch_t* sc) {
  const int A = sc->A;
  if (coll) neighbor_lists(x, A, W, sc);
  for (int a = 0; a < A; ++a) {
    real denom = 1 + W->c * W->dt / P[a].mass, fx = 0, fy = 0, gx, gy;
    if (coll) {
      for (int i = 0; i < sc->nlist[a]; ++i) {
        int b = sc->list[a * A + i];
        pair_f(x[a].px - x[b].px, x[a].py - x[b].py, x[a].vx - x[b].vx, x[a].vy - x[b].vy,
               P[a].radius + P[b].radius + W->margin, denom, W, &gx, &gy);
        fx += gx;
        fy += gy;
      }
    }
    real sx = 0, sy = 0;
    for (int o = 0; o < N; ++o) {
      obstacle_f(x[a].px, x[a].py, x[a].vx, x[a].vy, P[a].radius, denom, &obs[o], W, &gx, &gy);
      sx += gx;
      sy += gy;
    }
    if (W->bounds_mode == 1) {
      wall_f(x[a].px, x[a].py, x[a].vx, x[a].vy, P[a].radius, denom, W, &gx, &gy);
      sx += gx;
      sy += gy;
    }
    sc->fx[a] = fx + sx;
    sc->fy[a] = fy + sy;
  }
}

/* adjoint of forces(): adds into gin (pos/vel) of every agent given force cotangents */
static void forces_vjp(const st_t* x, const prm_t* P, const ob_t* obs, int N, const wc_t* W,
                       int coll, scratch_t* sc, st_t* gin) {
  const int A = sc->A;
  if (coll) neighbor_lists(x, A, W, sc);
  for (int a = 0; a < A; ++a) {
    real denom = 1 + W->c * W->dt / P[a].mass, gx = sc->gfx[a], gy = sc->gfy[a];
    if (coll) {
      for (int i = 0; i < sc->nlist[a]; ++i) {
        int b = sc->list[a * A + i];
        real gdx = 0, gdy = 0, grx = 0, gry = 0;
        pair_vjp(x[a].px - x[b].px, x[a].py - x[b].py, x[a].vx - x[b].vx, x[a].vy - x[b].vy,
                 P[a].radius + P[b].radius + W->margin, denom, gx, gy, W, &gdx, &gdy, &grx, &gry);
        gin[a].px += gdx;
        gin[a].py += gdy;
        gin[a].vx += grx;
        gin[a].vy += gry;
        gin[b].px -= gdx;
        gin[b].py -= gdy;
        gin[b].vx -= grx;
        gin[b].vy -= gry;
      }
    }
    for (int o = 0; o < N; ++o)
      obstacle_vjp(x[a].px, x[a].py, x[a].vx, x[a].vy, P[a].radius, denom, &obs[o], W, gx, gy,
                   &gin[a].px, &gin[a].py, &gin[a].vx, &gin[a].vy);
    if (W->bounds_mode == 1)
      wall_vjp(x[a].px, x[a].py, x[a].vx, x[a].vy, P[a].radius, denom, W, gx, gy, &gin[a].px,
               &gin[a].py, &gin[a].vx, &gin[a].vy);
  }
}

static inline void load_st(const real* pos, const real* th, const real* vel, const real* s,
                           const real* w, long i, st_t* x) {
  x->px = pos[2 * i];
  x->py = pos[2 * i + 1];
  x->vx = vel[2 * i];
  x->vy = vel[2 * i + 1];
  x->th = th[i];
  x->s = s[i];
  x->w = w[i];
}
static inline void store_st(real* pos, real* th, real* vel, real* s, real* w, long i,
                            const st_t* x) {
  pos[2 * i] = x->px;
  pos[2 * i + 1] = x->py;
  vel[2 * i] = x->vx;
  vel[2 * i + 1] = x->vy;
  th[i] = x->th;
  s[i] = x->s;
  w[i] = x->w;
}

/*
 * Forward rollout of every env, then (if g_act != NULL) the adjoint of
 * L = <gf, final state> over all envs. State arrays: pos/vel [.., 2], scalars [..].
 * traj_* [H, E, A(,2)] receive the state after every step. Returns 0.
 */
int SFX(swarp_cpu_rollout)(const cpu_world_t* w, const real* i_pos, const real* i_th,
                           const real* i_vel, const real* i_s, const real* i_w, const real* act,
                           real* t_pos, real* t_th, real* t_vel, real* t_s, real* t_w,
                           const real* gf_pos, real* g_act, real* gi_pos, real* gi_th,
                           real* gi_vel, real* gi_s, real* gi_w) {
  const int E = w->n_envs, A = w->n_agents, H = w->horizon, S = w->substeps, D = w->act_dim;
  const long EA = (long)E * A;
  wc_t W;
  W.dt = (real)(w->dt / S);
  W.k = (real)w->k;
  W.c = (real)w->c;
  W.margin = (real)w->margin;
  W.mo = (real)w->max_overlap;
  W.bx0 = (real)w->bounds[0];
  W.bx1 = (real)w->bounds[1];
  W.by0 = (real)w->bounds[2];
  W.by1 = (real)w->bounds[3];
  W.R = (real)w->neighbor_radius;
  W.K = w->max_neighbors;
  W.bounds_mode = w->bounds_mode;
  W.order = w->list_order;
  W.bins = w->grid_bins > 0 ? w->grid_bins : 1;
  W.ox = (real)w->grid_origin[0];
  W.oy = (real)w->grid_origin[1];
  W.cs = (real)w->grid_cell;
  if (W.order == 1 && !(W.cs > 0)) return -1;
#ifdef _OPENMP
  if (w->threads > 0) omp_set_num_threads(w->threads);
#pragma omp parallel
#endif
  {
    scratch_t sc;
    sc.A = A;
    sc.K = W.K;
    sc.list = (int*)malloc(sizeof(int) * A * A);
    sc.nlist = (int*)malloc(sizeof(int) * A);
    sc.fx = (real*)malloc(sizeof(real) * A * 4);
    sc.fy = sc.fx + A;
    sc.gfx = sc.fx + 2 * A;
    sc.gfy = sc.fx + 3 * A;
    sc.sub = (st_t*)malloc(sizeof(st_t) * A * (S + 1));
    const int NC = W.order == 1 ? W.bins * W.bins : 0;
    sc.cell = (int*)malloc(sizeof(int) * (2 * A + 2 * NC + 1));
    sc.csorted = sc.cell + A;
    sc.cstart = sc.cell + 2 * A;
    sc.cfill = sc.cstart + NC + 1;
    prm_t* P = (prm_t*)malloc(sizeof(prm_t) * A);
    ob_t* obs = (ob_t*)malloc(sizeof(ob_t) * (w->n_obstacles > 0 ? w->n_obstacles : 1));
    st_t* g = (st_t*)malloc(sizeof(st_t) * A * 2);
    st_t* gin = g + A;
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int e = 0; e < E; ++e) {
      for (int a = 0; a < A; ++a) {
        const double* r = w->params + (long)e * w->params_env_stride + (long)a * 22;
        prm_t* p = &P[a];
        p->radius = (real)r[0];
        p->mass = (real)r[1];
        p->max_speed = (real)r[2];
        p->max_accel = (real)r[3];
        p->max_ang_vel = (real)r[4];
        p->max_ang_accel = (real)r[5];
        p->l_f = (real)r[6];
        p->l_r = (real)r[7];
        p->max_steer = (real)r[8];
        p->min_speed = (real)r[16];
        p->gain_v = (real)r[20];
        p->gain_w = (real)r[21];
        p->tag = w->model_tag[a];
        p->mode = w->ctrl_mode[a];
      }
      for (int o = 0; o < w->n_obstacles; ++o) {
        long eo = (long)e * w->n_obstacles + o;
        ob_t* ob = &obs[o];
        ob->cx = (real)w->obs_pos[2 * eo];
        ob->cy = (real)w->obs_pos[2 * eo + 1];
        ob->ang = (real)w->obs_angle[eo];
        ob->vx = (real)w->obs_vel[2 * eo];
        ob->vy = (real)w->obs_vel[2 * eo + 1];
        ob->om = (real)w->obs_ang_vel[eo];
        ob->r = (real)w->obs_radius[o];
        ob->hx = (real)w->obs_half[2 * o];
        ob->hy = (real)w->obs_half[2 * o + 1];
        ob->type = w->obs_shape[o];
      }
      st_t* x = sc.sub;
      for (int a = 0; a < A; ++a) load_st(i_pos, i_th, i_vel, i_s, i_w, (long)e * A + a, &x[a]);
      /* forward */
      for (int t = 0; t < H; ++t) {
        for (int k = 0; k < S; ++k) {
          forces(x, P, obs, w->n_obstacles, &W, w->collisions, &sc);
          st_t* y = sc.sub + A;
          for (int a = 0; a < A; ++a) {
            const real* ap = act + (((long)t * E + e) * A + a) * D;
            integ(&x[a], ap[0], ap[1], sc.fx[a], sc.fy[a], &P[a], &W, &y[a]);
          }
          memcpy(x, y, sizeof(st_t) * A);
        }
        for (int a = 0; a < A; ++a)
          store_st(t_pos, t_th, t_vel, t_s, t_w, (long)t * EA + (long)e * A + a, &x[a]);
      }
      if (!g_act) continue;
      /* adjoint of <gf_pos, final pos> */
      memset(g, 0, sizeof(st_t) * A);
      for (int a = 0; a < A; ++a) {
        long i = (long)e * A + a;
        g[a].px = gf_pos[2 * i];
        g[a].py = gf_pos[2 * i + 1];
      }
      for (int t = H - 1; t >= 0; --t) {
        /* recompute the substep chain of step t from its checkpointed input */
        st_t* chain = sc.sub; /* [S+1][A] */
        for (int a = 0; a < A; ++a) {
          if (t > 0)
            load_st(t_pos, t_th, t_vel, t_s, t_w, (long)(t - 1) * EA + (long)e * A + a, &chain[a]);
          else
            load_st(i_pos, i_th, i_vel, i_s, i_w, (long)e * A + a, &chain[a]);
        }
        for (int k = 0; k < S; ++k) {
          forces(&chain[k * A], P, obs, w->n_obstacles, &W, w->collisions, &sc);
          for (int a = 0; a < A; ++a) {
            const real* ap = act + (((long)t * E + e) * A + a) * D;
            integ(&chain[k * A + a], ap[0], ap[1], sc.fx[a], sc.fy[a], &P[a], &W,
                  &chain[(k + 1) * A + a]);
          }
        }
        real* ga = g_act + ((long)t * E + e) * A * D;
        for (int j = 0; j < A * D; ++j) ga[j] = 0;
        for (int k = S - 1; k >= 0; --k) {
          for (int a = 0; a < A; ++a) {
            const real* ap = act + (((long)t * E + e) * A + a) * D;
            integ_vjp(&chain[k * A + a], ap[0], ap[1], &chain[(k + 1) * A + a], &g[a], &P[a], &W,
                      &gin[a], &sc.gfx[a], &sc.gfy[a], &ga[a * D], &ga[a * D + 1]);
          }
          forces_vjp(&chain[k * A], P, obs, w->n_obstacles, &W, w->collisions, &sc, gin);
          memcpy(g, gin, sizeof(st_t) * A);
        }
      }
      for (int a = 0; a < A; ++a)
        store_st(gi_pos, gi_th, gi_vel, gi_s, gi_w, (long)e * A + a, &g[a]);
    }
    free(sc.list);
    free(sc.nlist);
    free(sc.fx);
    free(sc.sub);
    free(sc.cell);
    free(P);
    free(obs);
    free(g);
  }
  return 0;
}
