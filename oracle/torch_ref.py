"""CPU restatement of swarp's differentiable step, in torch (float64 by default).

TEST INFRASTRUCTURE ONLY. This module is the parity checker for the CUDA path: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
it. The product (``swarp_b200``) never calls it and has no CPU fallback.

What it restates (reference = ddebenedittis/swarp, paths relative to that project):

* ``swarp/dynamics/kernels.py:68-71``  ``clamp_norm``
* ``swarp/dynamics/kernels.py:166-190`` ``servo_command``
* ``swarp/dynamics/kernels.py:194-275`` ``_step_2d`` (holonomic / diff-drive / bicycle)
* ``swarp/dynamics/kernels.py:395-403`` the disc bounds clamp of ``_integrate_agent``
* ``swarp/core/collisions.py:48``      ``_EPS2``
* ``swarp/core/collisions.py:61-84``   ``shape_bound``, ``bounds_apart``
* ``swarp/core/collisions.py:87-143``  ``_normal_coeff``, ``pair_force``
* ``swarp/core/collisions.py:156-260`` ``closest_on_segment``, ``box_force``
* ``swarp/core/collisions.py:690-815`` obstacle, wall and static forces
* ``swarp/core/collisions.py:818-881`` ``collision_forces_kernel`` (list-order gather)
* ``swarp/core/neighbors.py:76-97``    ``_brute_force`` (ascending index, cap, true count)
* ``swarp/core/neighbors.py:135-254, 388-394, 591-620`` the radix-sort uniform grid that
  ``"auto"`` picks above 512 agents per env (its frame, cells and list order)
* ``swarp/core/bodies.py:79-127,167-255,367-569`` movable compound-body pass
* ``swarp/core/stepper.py:549-648``    substep order: neighbors, forces, bodies, integrate
* ``swarp/dynamics/kernels.py:102-163,349-369,494-508,758-768`` the 6-DOF drone (Euler, RK4)
* ``swarp/core/collisions.py:262-690`` box agents; ``swarp/dynamics/kernels.py:80-99``
  footprint clamp

Gradients come from torch autograd over this restatement. Warp's adjoint conventions
at kinks are reproduced with ``torch.where`` forms: ``max(a, b)`` sends the gradient
to ``b`` on a tie, ``clamp`` passes it to ``x`` on the closed interval (else to the active
bound), ``length`` and
``abs`` follow Warp's ``adj_length`` (zero at the zero vector) and ``adj_abs`` (+1 at
0). Movable bodies are not differentiated by the reference (its body pass is
untaped, ``swarp/core/bodies.py:40-43``); here they are, which makes this module the
gradient oracle for bodies (pinned by finite differences in the tests).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

# Parameter-row columns (same layout as swarp/dynamics/base.py:114-169).
P_RADIUS, P_MASS, P_MAX_SPEED, P_MAX_ACCEL, P_MAX_ANG_VEL, P_MAX_ANG_ACCEL = 0, 1, 2, 3, 4, 5
P_LF, P_LR, P_MAX_STEER, P_MIN_SPEED = 6, 7, 8, 16
P_CMD_GAIN_V, P_CMD_GAIN_W = 20, 21
P_SHAPE, P_HALF_X, P_HALF_Y = 17, 18, 19
P_THRUST_MAX, P_ARM, P_IXX, P_IYY, P_IZZ, P_KAPPA, P_GRAVITY = 9, 10, 11, 12, 13, 14, 15
HOLONOMIC, DIFF_DRIVE, BICYCLE, DRONE = 0, 1, 2, 3
VELOCITY, ACCELERATION, SERVO = 0, 1, 2
CIRCLE, BOX, SEGMENT = 0, 1, 2
EPS2 = 1.0e-10


# --------------------------------------------------------------------------- kinks


def wmax(a, b):
    """Warp ``max``: value max(a, b); gradient to ``a`` iff ``a > b``."""
    return torch.where(a > b, a, b)


def wmin(a, b):
    return torch.where(a < b, a, b)


def wclamp(x, lo, hi):
    """Warp ``clamp``: value ``min(max(lo, x), hi)``; Warp's adjoint routes the gradient to
    ``lo`` where x < lo, to ``hi`` where x > hi and to ``x`` otherwise (the bounds carry a
    gradient only where they depend on the state, e.g. a box's support extents at its
    heading in the footprint clamp). The routing terms are exact zeros in value."""
    x_t = torch.as_tensor(x)
    lo = torch.as_tensor(lo, dtype=x_t.dtype, device=x_t.device)
    hi = torch.as_tensor(hi, dtype=x_t.dtype, device=x_t.device)
    val = torch.minimum(torch.maximum(lo, x_t), hi).detach()
    route = torch.where(x_t < lo, lo - lo.detach(),
                        torch.where(x_t > hi, hi - hi.detach(), x_t - x_t.detach()))
    return val + route


def wabs(x):
    return torch.where(x < 0, -x, x)


def wlength(x, y):
    """Warp ``length``: sqrt(x*x + y*y), zero gradient at the zero vector."""
    d2 = x * x + y * y
    pos = d2 > 0
    return torch.where(pos, torch.sqrt(torch.where(pos, d2, torch.ones_like(d2))), d2 * 0)


def _zeros_like(x):
    return torch.zeros_like(x)


# ----------------------------------------------------------------------- world spec


@dataclass
class RefObstacles:
    """Per-env obstacle state (``[E,N]``) and per-shape constants (``[N]``)."""

    pos: torch.Tensor  # [E,N,2]
    angle: torch.Tensor  # [E,N]
    vel: torch.Tensor  # [E,N,2]
    ang_vel: torch.Tensor  # [E,N]
    radius: torch.Tensor  # [N]
    half: torch.Tensor  # [N,2]
    shape: list  # [N] ints
    kind: list = field(default_factory=list)  # [N] ints (0 immovable, 1 movable)
    mass: torch.Tensor | None = None  # [N]
    inertia: torch.Tensor | None = None  # [N]
    body: list = field(default_factory=list)  # [N] root index per shape
    body_off: torch.Tensor | None = None  # [N,2]
    # body state per root index [E,N,...] (only movable roots are meaningful)
    body_pos: torch.Tensor | None = None
    body_angle: torch.Tensor | None = None
    body_vel: torch.Tensor | None = None
    body_ang_vel: torch.Tensor | None = None

    @property
    def n(self) -> int:
        return self.pos.shape[1]

    def any_movable(self) -> bool:
        return any(int(k) == 1 for k in self.kind)


@dataclass
class RefWorld:
    params: torch.Tensor  # [A,22] or [E,A,22]
    model_tag: list
    ctrl_mode: list
    dt: float
    substeps: int = 1
    collisions: bool = True
    k: float = 100.0
    c: float = 1.0
    margin: float = 0.02
    max_overlap: float = 0.0
    neighbor_radius: float = 0.0
    max_neighbors: int = 32
    bounds: tuple | None = None
    soft_walls: bool = False
    clamp_bounds: bool = False
    lin_damping: float = 10.0
    ang_damping: float = 10.0
    bodies_move: bool = True
    rk4: bool = False  # Integrator.RK4 instead of semi-implicit Euler
    # "brute" (ascending index), "uniform_grid" (the radix-sort grid's order; frame from
    # ``bounds`` when given, else from the batch) or "auto" (the grid above 512 agents)
    neighbor_method: str = "brute"
    uniform_bins: int | None = None

    def col(self, j):
        """Parameter column ``j`` broadcastable to ``[E, A]``."""
        p = self.params
        return p[..., j] if p.dim() == 3 else p[:, j].unsqueeze(0)


# ------------------------------------------------------------------- contact law


def normal_coeff(ov, vn, k, c, denom, max_overlap):
    """``swarp/core/collisions.py:87-106``: implicit damping, clamped repulsive."""
    ovs = max_overlap * torch.tanh(ov / max_overlap) if max_overlap > 0.0 else ov
    x = (k * ovs - c * vn) / denom
    return wmax(x, torch.zeros_like(x))


def pair_force(dx, dy, rvx, rvy, min_dist, k, c, denom, max_overlap):
    """``swarp/core/collisions.py:109-143``: force on self from a disc at -d."""
    d2 = dx * dx + dy * dy
    dist = torch.sqrt(wmax(d2, torch.full_like(d2, EPS2)))
    ov = min_dist - dist
    active = ov > 0
    nx = dx / dist
    ny = dy / dist
    vn = rvx * nx + rvy * ny
    cf = normal_coeff(ov, vn, k, c, denom, max_overlap)
    z = torch.zeros_like(d2)
    return torch.where(active, cf * nx, z), torch.where(active, cf * ny, z)


def closest_on_segment(px, py, cx, cy, angle, half_len):
    """``swarp/core/collisions.py:156-171``."""
    ux, uy = torch.cos(angle), torch.sin(angle)
    t = wclamp((px - cx) * ux + (py - cy) * uy, -half_len, half_len)
    return cx + t * ux, cy + t * uy


def box_force(px, py, vx, vy, cx, cy, angle, hx, hy, reach, k, c, denom, max_overlap, vox, voy, om):
    """``swarp/core/collisions.py:174-260``: oriented-box SDF contact."""
    ca, sa = torch.cos(angle), torch.sin(angle)
    dx, dy = px - cx, py - cy
    lx = ca * dx + sa * dy
    ly = -sa * dx + ca * dy
    qx = wabs(lx) - hx
    qy = wabs(ly) - hy
    clx = wclamp(lx, -hx, hx)
    cly = wclamp(ly, -hy, hy)
    ox, oy = lx - clx, ly - cly
    od2 = ox * ox + oy * oy
    ext = od2 > EPS2
    one = torch.ones_like(od2)
    s_e = torch.sqrt(torch.where(ext, od2, one))
    nlx_e, nly_e = ox / s_e, oy / s_e
    use_x = qx > qy
    sgx = torch.where(lx >= 0, one, -one)
    sgy = torch.where(ly >= 0, one, -one)
    zero = torch.zeros_like(od2)
    s_i = torch.where(use_x, qx, qy)
    nlx_i = torch.where(use_x, sgx, zero)
    nly_i = torch.where(use_x, zero, sgy)
    s = torch.where(ext, s_e, s_i)
    nlx = torch.where(ext, nlx_e, nlx_i)
    nly = torch.where(ext, nly_e, nly_i)
    overlap = reach - s
    active = overlap > 0
    nx = ca * nlx - sa * nly
    ny = sa * nlx + ca * nly
    spx = lx - s * nlx
    spy = ly - s * nly
    rx = ca * spx - sa * spy
    ry = sa * spx + ca * spy
    vsx = vox + (-om * ry)
    vsy = voy + om * rx
    relx, rely = vx - vsx, vy - vsy
    vn = relx * nx + rely * ny
    cf = normal_coeff(overlap, vn, k, c, denom, max_overlap)
    return torch.where(active, cf * nx, zero), torch.where(active, cf * ny, zero)


def shape_bound(st: int, r, hx, hy):
    if st == BOX:
        return torch.sqrt(hx * hx + hy * hy)
    if st == SEGMENT:
        return hx + r
    return r


def bounds_apart(dx, dy, reach):
    lim = reach * 1.0001 + 1.0e-6
    return dx * dx + dy * dy > lim * lim


def obstacle_forces(px, py, vx, vy, ra, obs: RefObstacles, w: RefWorld, denom):
    """``swarp/core/collisions.py:690-742``: sum over obstacles in index order."""
    fx = torch.zeros_like(px)
    fy = torch.zeros_like(py)
    if obs is None:
        return fx, fy
    k, c, margin, mo = w.k, w.c, w.margin, w.max_overlap
    for o in range(obs.n):
        st = int(obs.shape[o])
        cx = obs.pos[:, o, 0].unsqueeze(1)
        cy = obs.pos[:, o, 1].unsqueeze(1)
        ang = obs.angle[:, o].unsqueeze(1)
        r_o = obs.radius[o]
        hx, hy = obs.half[o, 0], obs.half[o, 1]
        apart = bounds_apart(px - cx, py - cy, ra + margin + shape_bound(st, r_o, hx, hy))
        vox = obs.vel[:, o, 0].unsqueeze(1)
        voy = obs.vel[:, o, 1].unsqueeze(1)
        om = obs.ang_vel[:, o].unsqueeze(1)
        if st == BOX:
            gx, gy = box_force(px, py, vx, vy, cx, cy, ang, hx, hy, ra + margin, k, c, denom, mo,
                               vox, voy, om)
        elif st == SEGMENT:
            qx, qy = closest_on_segment(px, py, cx, cy, ang, hx)
            rx, ry = qx - cx, qy - cy
            vsx = vox + (-om * ry)
            vsy = voy + om * rx
            gx, gy = pair_force(px - qx, py - qy, vx - vsx, vy - vsy, ra + r_o + margin, k, c,
                                denom, mo)
        else:
            gx, gy = pair_force(px - cx, py - cy, vx - vox, vy - voy, ra + r_o + margin, k, c,
                                denom, mo)
        z = torch.zeros_like(gx)
        fx = fx + torch.where(apart, z, gx)
        fy = fy + torch.where(apart, z, gy)
    return fx, fy


def wall_forces(px, py, vx, vy, ra, w: RefWorld, denom):
    """``swarp/core/collisions.py:745-780``: four soft walls, static closing velocity."""
    x0, x1, y0, y1 = w.bounds
    k, c, mo = w.k, w.c, w.max_overlap
    reach = ra + w.margin
    fx = torch.zeros_like(px)
    fy = torch.zeros_like(py)
    z = torch.zeros_like(px)
    pen = reach - (px - x0)
    fx = fx + torch.where(pen > 0, normal_coeff(pen, vx, k, c, denom, mo), z)
    pen = reach - (x1 - px)
    fx = fx + torch.where(pen > 0, -normal_coeff(pen, -vx, k, c, denom, mo), z)
    pen = reach - (py - y0)
    fy = fy + torch.where(pen > 0, normal_coeff(pen, vy, k, c, denom, mo), z)
    pen = reach - (y1 - py)
    fy = fy + torch.where(pen > 0, -normal_coeff(pen, -vy, k, c, denom, mo), z)
    return fx, fy


# ------------------------------------------------------------------ box agents


def _point_box(vx, vy, cx, cy, ca, sa, hx, hy):
    """``swarp/core/collisions.py:270-288``: distance and closest point from an exterior
    point to an oriented box (distance floored like pair_force's)."""
    dx, dy = vx - cx, vy - cy
    lx = ca * dx + sa * dy
    ly = -sa * dx + ca * dy
    clx = wclamp(lx, -hx, hx)
    cly = wclamp(ly, -hy, hy)
    ox, oy = lx - clx, ly - cly
    d2 = ox * ox + oy * oy
    dist = torch.sqrt(wmax(d2, torch.full_like(d2, EPS2)))
    return dist, cx + (ca * clx - sa * cly), cy + (sa * clx + ca * cly)


def obb_contact(cax, cay, tha, hax, hay, cbx, cby, thb, hbx, hby, reach):
    """``swarp/core/collisions.py:311-444``: signed distance, unit normal (B to A) and
    contact point of two oriented boxes. SAT over the four face normals first; beyond
    ``reach`` no contact; disjoint within reach: the closest of the eight vertex-versus-
    box distances; overlapping: the least-overlap axis and the middle of the overlap of
    the two projections on its reference face. Branches are selected per element."""
    caA, saA, caB, saB = torch.cos(tha), torch.sin(tha), torch.cos(thb), torch.sin(thb)
    uA0, uA1 = (caA, saA), (-saA, caA)
    uB0, uB1 = (caB, saB), (-saB, caB)
    dot = lambda u, v: u[0] * v[0] + u[1] * v[1]  # noqa: E731
    d = (cax - cbx, cay - cby)
    a00, a01 = wabs(dot(uA0, uB0)), wabs(dot(uA0, uB1))
    a10, a11 = wabs(dot(uA1, uB0)), wabs(dot(uA1, uB1))
    dA0, dA1, dB0, dB1 = dot(d, uA0), dot(d, uA1), dot(d, uB0), dot(d, uB1)
    gaps = [wabs(dA0) - hax - (hbx * a00 + hby * a01), wabs(dA1) - hay - (hbx * a10 + hby * a11),
            wabs(dB0) - hbx - (hax * a00 + hay * a10), wabs(dB1) - hby - (hax * a01 + hay * a11)]
    s = gaps[0]
    axis = torch.zeros_like(s, dtype=torch.int64)
    for i in (1, 2, 3):
        take = gaps[i] > s
        s = torch.where(take, gaps[i], s)
        axis = torch.where(take, torch.full_like(axis, i), axis)
    zero = torch.zeros_like(s)
    # disjoint: vertices of A against B (flip +1), then of B against A (flip -1)
    eA0 = (uA0[0] * hax, uA0[1] * hax)
    eA1 = (uA1[0] * hay, uA1[1] * hay)
    eB0 = (uB0[0] * hbx, uB0[1] * hbx)
    eB1 = (uB1[0] * hby, uB1[1] * hby)
    best = torch.full_like(s, 1.0e30)
    bnx, bny, bxx, bxy = zero, zero, cax, cay
    verts = []
    for sx, sy in ((1, 1), (-1, 1), (-1, -1), (1, -1)):
        verts.append(((cax + sx * eA0[0]) + sy * eA1[0], (cay + sx * eA0[1]) + sy * eA1[1],
                      cbx, cby, caB, saB, hbx, hby, 1.0))
    for sx, sy in ((1, 1), (-1, 1), (-1, -1), (1, -1)):
        verts.append(((cbx + sx * eB0[0]) + sy * eB1[0], (cby + sx * eB0[1]) + sy * eB1[1],
                      cax, cay, caA, saA, hax, hay, -1.0))
    for vx, vy, cx, cy, ca, sa, hx, hy, flip in verts:
        dist, qx, qy = _point_box(vx, vy, cx, cy, ca, sa, hx, hy)
        take = dist < best
        best = torch.where(take, dist, best)
        bnx = torch.where(take, (vx - qx) * (flip / dist), bnx)
        bny = torch.where(take, (vy - qy) * (flip / dist), bny)
        bxx = torch.where(take, (vx + qx) * 0.5, bxx)
        bxy = torch.where(take, (vy + qy) * 0.5, bxy)
    # overlapping: the least-overlap axis, oriented B -> A, and its reference face
    sel = lambda vals: torch.where(axis == 0, vals[0], torch.where(  # noqa: E731
        axis == 1, vals[1], torch.where(axis == 2, vals[2], vals[3])))
    ux = sel([uA0[0], uA1[0], uB0[0], uB1[0]])
    uy = sel([uA0[1], uA1[1], uB0[1], uB1[1]])
    tx = sel([uA1[0], uA0[0], uB1[0], uB0[0]])
    ty = sel([uA1[1], uA0[1], uB1[1], uB0[1]])
    dn = sel([dA0, dA1, dB0, dB1])
    h_n = sel([hax, hay, hbx, hby])
    h_t = sel([hay, hax, hby, hbx])
    r_t = sel([hbx * a10 + hby * a11, hbx * a00 + hby * a01, hax * a01 + hay * a11,
               hax * a00 + hay * a10])
    sgn = torch.where(dn < 0, -torch.ones_like(dn), torch.ones_like(dn))
    onx, ony = ux * sgn, uy * sgn
    b_axis = axis >= 2
    crx, cry = torch.where(b_axis, cbx, cax), torch.where(b_axis, cby, cay)
    cix, ciy = torch.where(b_axis, cax, cbx), torch.where(b_axis, cay, cby)
    xn = torch.where(b_axis, (cbx * onx + cby * ony) + h_n, (cax * onx + cay * ony) - h_n)
    ct_ref = crx * tx + cry * ty
    ct_inc = cix * tx + ciy * ty
    lo = wmax(ct_ref - h_t, ct_inc - r_t)
    hi = wmin(ct_ref + h_t, ct_inc + r_t)
    mid = 0.5 * (lo + hi)
    oxx, oxy = onx * xn + tx * mid, ony * xn + ty * mid
    far = s > reach
    disjoint = (~far) & (s > 0)
    s_out = torch.where(disjoint, best, s)
    nx = torch.where(far, zero, torch.where(disjoint, bnx, onx))
    ny = torch.where(far, zero, torch.where(disjoint, bny, ony))
    px = torch.where(far, cax, torch.where(disjoint, bxx, oxx))
    py = torch.where(far, cay, torch.where(disjoint, bxy, oxy))
    return s_out, nx, ny, px, py


def obb_force(cax, cay, tha, hax, hay, vax, vay, wa, cbx, cby, thb, hbx, hby, vbx, vby, wb, reach,
              k, c, denom, max_overlap):
    """``swarp/core/collisions.py:447-486``: force on box A from box B."""
    fx, fy, _, _ = obb_force_at(cax, cay, tha, hax, hay, vax, vay, wa, cbx, cby, thb, hbx, hby,
                                vbx, vby, wb, reach, k, c, denom, max_overlap)
    return fx, fy


def obb_force_at(cax, cay, tha, hax, hay, vax, vay, wa, cbx, cby, thb, hbx, hby, vbx, vby, wb,
                 reach, k, c, denom, max_overlap):
    """obb_force with the contact point it acts at (``collisions.py:447-486`` returns both)."""
    s, nx, ny, xx, xy = obb_contact(cax, cay, tha, hax, hay, cbx, cby, thb, hbx, hby, reach)
    ov = reach - s
    rax, ray = xx - cax, xy - cay
    rbx, rby = xx - cbx, xy - cby
    rvx = (vax + (-wa * ray)) - (vbx + (-wb * rby))
    rvy = (vay + wa * rax) - (vby + wb * rbx)
    cf = normal_coeff(ov, rvx * nx + rvy * ny, k, c, denom, max_overlap)
    z = torch.zeros_like(s)
    active = ov > 0
    return torch.where(active, cf * nx, z), torch.where(active, cf * ny, z), xx, xy


def agent_pair_force(a_lt_b, box_a, box_b, pax, pay, tha, vax, vay, wa, ra, hax, hay,
                     pbx, pby, thb, vbx, vby, wb, rb, hbx, hby, w: RefWorld, denom):
    """``swarp/core/collisions.py:490-537``: the force on agent a from agent b for any
    shapes: disc-disc pair_force; disc-box box_force (negated on the box); box-box
    obb_force with the lower index as A on both agents, negated on the higher one."""
    k, c, mo, m = w.k, w.c, w.max_overlap, w.margin
    dd = pair_force(pax - pbx, pay - pby, vax - vbx, vay - vby, ra + rb + m, k, c, denom, mo)
    db = box_force(pax, pay, vax, vay, pbx, pby, thb, hbx, hby, ra + m, k, c, denom, mo, vbx, vby, wb)
    bd = box_force(pbx, pby, vbx, vby, pax, pay, tha, hax, hay, rb + m, k, c, denom, mo, vax, vay, wa)
    lo = obb_force(pax, pay, tha, hax, hay, vax, vay, wa, pbx, pby, thb, hbx, hby, vbx, vby, wb, m,
                   k, c, denom, mo)
    hi = obb_force(pbx, pby, thb, hbx, hby, vbx, vby, wb, pax, pay, tha, hax, hay, vax, vay, wa, m,
                   k, c, denom, mo)
    out = []
    for i in range(2):
        bb = torch.where(a_lt_b, lo[i], -hi[i])
        v = torch.where(box_a, torch.where(box_b, bb, -bd[i]), torch.where(box_b, db[i], dd[i]))
        out.append(v)
    return out[0], out[1]


def box_obstacle_forces(px, py, th, vx, vy, om, hax, hay, obs, w: RefWorld, denom):
    """``swarp/core/collisions.py:540-630``: obstacles on a box agent: BOX = obb_force with
    reach = margin; SEGMENT = obb_force against the degenerate box (half_len, 0) with reach
    = radius + margin; CIRCLE = -box_force with the circle centre as the point."""
    fx = torch.zeros_like(px)
    fy = torch.zeros_like(py)
    if obs is None:
        return fx, fy
    k, c, m, mo = w.k, w.c, w.margin, w.max_overlap
    ra = wlength(hax, hay)
    for o in range(obs.n):
        st = int(obs.shape[o])
        cx, cy = obs.pos[:, o, 0].unsqueeze(1), obs.pos[:, o, 1].unsqueeze(1)
        ang = obs.angle[:, o].unsqueeze(1)
        vox, voy = obs.vel[:, o, 0].unsqueeze(1), obs.vel[:, o, 1].unsqueeze(1)
        omo = obs.ang_vel[:, o].unsqueeze(1)
        r_o, hx, hy = obs.radius[o], obs.half[o, 0], obs.half[o, 1]
        apart = bounds_apart(px - cx, py - cy, ra + m + shape_bound(st, r_o, hx, hy))
        if st == BOX:
            gx, gy = obb_force(px, py, th, hax, hay, vx, vy, om, cx, cy, ang, hx + 0 * cx,
                               hy + 0 * cx, vox, voy, omo, m, k, c, denom, mo)
        elif st == SEGMENT:
            gx, gy = obb_force(px, py, th, hax, hay, vx, vy, om, cx, cy, ang, hx + 0 * cx, 0 * cx,
                               vox, voy, omo, r_o + m, k, c, denom, mo)
        else:
            gx, gy = box_force(cx, cy, vox, voy, px, py, th, hax, hay, r_o + m, k, c, denom, mo,
                               vx, vy, om)
            gx, gy = -gx, -gy
        z = torch.zeros_like(gx)
        fx = fx + torch.where(apart, z, gx)
        fy = fy + torch.where(apart, z, gy)
    return fx, fy


def _sgn0(x):
    one = torch.ones_like(x)
    return torch.where(x > 0, one, torch.where(x < 0, -one, torch.zeros_like(x)))


def wall_forces_box(px, py, th, vx, vy, om, hax, hay, w: RefWorld, denom):
    """``swarp/core/collisions.py:646-690``: walls against a box's support extents, damped by
    the velocity of the touching support vertex."""
    x0, x1, y0, y1 = w.bounds
    k, c, m, mo = w.k, w.c, w.margin, w.max_overlap
    ca, sa = torch.cos(th), torch.sin(th)
    ex = hax * wabs(ca) + hay * wabs(sa)
    ey = hax * wabs(sa) + hay * wabs(ca)
    sc, ss = _sgn0(ca), _sgn0(sa)
    rl_y = -sc * hax * sa + ss * hay * ca
    rb_x = -ss * hax * ca + sc * hay * sa
    z = torch.zeros_like(px)
    fx, fy = z, z
    pen = ex + m - (px - x0)
    fx = fx + torch.where(pen > 0, normal_coeff(pen, vx - om * rl_y, k, c, denom, mo), z)
    pen = ex + m - (x1 - px)
    fx = fx + torch.where(pen > 0, -normal_coeff(pen, -(vx + om * rl_y), k, c, denom, mo), z)
    pen = ey + m - (py - y0)
    fy = fy + torch.where(pen > 0, normal_coeff(pen, vy + om * rb_x, k, c, denom, mo), z)
    pen = ey + m - (y1 - py)
    fy = fy + torch.where(pen > 0, -normal_coeff(pen, -(vy - om * rb_x), k, c, denom, mo), z)
    return fx, fy


def clamp_footprint(npx, npy, nth, w: RefWorld, col):
    """``swarp/dynamics/kernels.py:80-99``: keep the footprint inside the bounds (a box by
    its support extents at the new heading, a disc by its radius)."""
    x0, x1, y0, y1 = w.bounds
    r = col(P_RADIUS)
    box = col(P_SHAPE) > 0.5
    ca, sa = wabs(torch.cos(nth)), wabs(torch.sin(nth))
    hx, hy = col(P_HALF_X), col(P_HALF_Y)
    ex = torch.where(box, hx * ca + hy * sa, r)
    ey = torch.where(box, hx * sa + hy * ca, r)
    return wclamp(npx, x0 + ex, x1 - ex), wclamp(npy, y0 + ey, y1 - ey)


# ------------------------------------------------------------------ neighbor lists


@torch.no_grad()
def brute_neighbors(pos, radius: float, max_neighbors: int):
    """``swarp/core/neighbors.py:76-97``: ascending-index within-radius lists.

    Returns ``(in_list [E,A,A] bool, idx [E,A,K] int64 padded with -1, count [E,A],
    true_count [E,A])``. ``in_list[e,a,b]`` is True iff b is among the first
    ``max_neighbors`` agents (by index) within ``radius`` of a.
    """
    E, A, _ = pos.shape
    dxy = pos.unsqueeze(1) - pos.unsqueeze(2)  # [E, a, b, 2] = p_b - p_a
    dist = wlength(dxy[..., 0], dxy[..., 1])
    eye = torch.eye(A, dtype=torch.bool, device=pos.device).unsqueeze(0)
    inr = (dist <= radius) & ~eye
    before = torch.cumsum(inr.to(torch.int64), dim=-1) - inr.to(torch.int64)
    in_list = inr & (before < max_neighbors)
    true_count = inr.sum(-1)
    count = in_list.sum(-1)
    K = max_neighbors
    idx = torch.full((E, A, K), -1, dtype=torch.int64, device=pos.device)
    order = torch.where(in_list, before, torch.full_like(before, K))
    ar = torch.arange(A, device=pos.device).expand(E, A, A)
    sel = order < K
    idx[sel.nonzero(as_tuple=True)[0], sel.nonzero(as_tuple=True)[1], order[sel]] = ar[sel]
    return in_list, idx, count, true_count


def default_uniform_bins(n_agents: int) -> int:
    """``swarp/core/neighbors.py:394``: cells per axis, about sqrt(n_agents), in [4, 128]."""
    return max(4, min(128, int(math.ceil(math.sqrt(n_agents)))))


def auto_neighbor_method(n_agents: int) -> str:
    """``swarp/core/neighbors.py:388-389``: ``"auto"`` picks the uniform grid above 512
    agents per env, brute force otherwise."""
    return "uniform_grid" if n_agents > 512 else "brute"


def uniform_grid_frame(pos, radius: float, bins: int, bounds=None):
    """Grid origin and cell size, in the dtype of ``pos``.

    With a pinned world rectangle (``swarp/core/neighbors.py:591-620``) the origin is its
    lower corner and the cell size ``max(radius, extent / bins)``, both computed in Python
    floats and stored in the position dtype. Without one (``_bounds_reduce`` /
    ``_finalize_grid``, ``neighbors.py:149-178``) they come from the minimum and maximum
    coordinates over the WHOLE batch, all envs together, in the position dtype.
    """
    dt = pos.dtype
    if bounds is not None:
        x_min, x_max, y_min, y_max = bounds
        extent = max(x_max - x_min, y_max - y_min)
        origin = torch.tensor([x_min, y_min], dtype=dt)
        cell = torch.tensor(max(radius, extent / bins), dtype=dt)
        return origin, cell
    lo = pos.reshape(-1, 2).min(0).values
    hi = pos.reshape(-1, 2).max(0).values
    ext = torch.maximum(hi[0] - lo[0], hi[1] - lo[1])
    cell = torch.maximum(torch.tensor(radius, dtype=dt), ext / torch.tensor(bins, dtype=dt))
    return lo.clone(), cell


def uniform_grid_neighbors(pos, radius: float, max_neighbors: int, bins: int | None = None,
                           bounds=None):
    """``swarp/core/neighbors.py:182-254`` (``_compute_keys``, radix sort, ``_build_offsets``,
    ``_query_uniform``): the uniform-grid lists, in the reference's list order.

    Each agent falls in cell ``clamp(int((p - origin) / cell), 0, bins - 1)`` per axis (the
    division in the position dtype, truncation toward zero). A query visits the 3 x 3
    block of cells around its own, rows ``dy = -1, 0, 1`` and in each row ``dx = -1, 0, 1``,
    and each cell's agents in ascending index (the radix sort is stable and its values
    start in index order); it keeps ``b != a`` with ``length(p_b - p_a) <= radius`` and
    lists the first ``max_neighbors`` of them. So the list order is (block cell, index)
    rather than the brute force's index order: both give the same sets when no list
    truncates, different ones when a list truncates.

    Returns ``(in_list [E,A,A] bool, idx [E,A,K] int64 padded with -1, count [E,A],
    true_count [E,A])`` like :func:`brute_neighbors`, ``idx`` in the grid's list order.
    """
    E, A, _ = pos.shape
    bins = bins or default_uniform_bins(A)
    origin, cell = uniform_grid_frame(pos, radius, bins, bounds)
    c = ((pos - origin) / cell).to(torch.int32).clamp(0, bins - 1).to(torch.int64)  # [E,A,2]
    dcx = c[..., 0].unsqueeze(1) - c[..., 0].unsqueeze(2)  # [E, a, b] = cx_b - cx_a
    dcy = c[..., 1].unsqueeze(1) - c[..., 1].unsqueeze(2)
    in_block = (dcx.abs() <= 1) & (dcy.abs() <= 1)
    dxy = pos.unsqueeze(1) - pos.unsqueeze(2)  # p_b - p_a
    dist = wlength(dxy[..., 0], dxy[..., 1])
    eye = torch.eye(A, dtype=torch.bool).unsqueeze(0)
    member = in_block & (dist <= radius) & ~eye
    ar = torch.arange(A).expand(E, A, A)
    key = ((dcy + 1) * 3 + (dcx + 1)) * A + ar  # visit order of the candidates
    key = torch.where(member, key, torch.full_like(key, 9 * A))
    order = torch.argsort(key, dim=-1, stable=True)  # [E, a, rank] -> b
    ranked = torch.gather(member, -1, order)
    true_count = member.sum(-1)
    K = max_neighbors
    count = torch.clamp(true_count, max=K)
    idx = torch.full((E, A, K), -1, dtype=torch.int64)
    take = min(K, A)
    first = order[..., :take]
    idx[..., :take] = torch.where(ranked[..., :take], first, torch.full_like(first, -1))
    in_list = torch.zeros((E, A, A), dtype=torch.bool)
    rank = torch.arange(A).expand(E, A, A)
    listed_rank = ranked & (rank < K)
    in_list.scatter_(-1, order, listed_rank)
    return in_list, idx, count, true_count


def collision_forces(state, w: RefWorld, obs: RefObstacles | None):
    """``swarp/core/collisions.py:818-881``: neighbor gather in list order + static."""
    pos, _, vel, _, _ = state[:5]
    px, py = pos[..., 0], pos[..., 1]
    vx, vy = vel[..., 0], vel[..., 1]
    E, A = px.shape
    ra = w.col(P_RADIUS).expand(E, A)
    denom = 1.0 + w.c * (w.dt / w.substeps) / w.col(P_MASS).expand(E, A)
    fx = torch.zeros_like(px)
    fy = torch.zeros_like(py)
    true_count = torch.zeros(E, A, dtype=torch.int64, device=px.device)
    box = w.col(P_SHAPE).expand(E, A) > 0.5
    any_box = bool(box.any())
    th, om = state[1], state[4]
    hax, hay = w.col(P_HALF_X).expand(E, A), w.col(P_HALF_Y).expand(E, A)
    if w.collisions:
        method = w.neighbor_method
        if method == "auto":
            method = auto_neighbor_method(A)
        if method == "uniform_grid":
            in_list, _, _, true_count = uniform_grid_neighbors(
                pos.detach(), w.neighbor_radius, w.max_neighbors, bins=w.uniform_bins,
                bounds=w.bounds)
        elif method == "brute":
            in_list, _, _, true_count = brute_neighbors(pos.detach(), w.neighbor_radius,
                                                        w.max_neighbors)
        else:
            raise ValueError(f"neighbor_method {method!r} is not restated")
        ar = torch.arange(A, device=px.device).unsqueeze(0)
        for b in range(A):
            sel = in_list[:, :, b]
            if not bool(sel.any()):
                continue
            sl = slice(b, b + 1)
            if any_box:
                gx, gy = agent_pair_force(
                    ar < b, box, box[:, sl], px, py, th, vx, vy, om, ra, hax, hay,
                    px[:, sl], py[:, sl], th[:, sl], vx[:, sl], vy[:, sl], om[:, sl], ra[:, sl],
                    hax[:, sl], hay[:, sl], w, denom)
            else:
                gx, gy = pair_force(
                    px - px[:, sl], py - py[:, sl], vx - vx[:, sl], vy - vy[:, sl],
                    ra + ra[:, sl] + w.margin, w.k, w.c, denom, w.max_overlap,
                )
            z = torch.zeros_like(gx)
            fx = fx + torch.where(sel, gx, z)
            fy = fy + torch.where(sel, gy, z)
    sx, sy = obstacle_forces(px, py, vx, vy, ra, obs, w, denom)
    if w.soft_walls:
        wx, wy = wall_forces(px, py, vx, vy, ra, w, denom)
        sx, sy = sx + wx, sy + wy
    if any_box:  # collisions.py:951-994: box agents take the oriented static forces
        bx_, by_ = box_obstacle_forces(px, py, th, vx, vy, om, hax, hay, obs, w, denom)
        if w.soft_walls:
            wx, wy = wall_forces_box(px, py, th, vx, vy, om, hax, hay, w, denom)
            bx_, by_ = bx_ + wx, by_ + wy
        sx, sy = torch.where(box, bx_, sx), torch.where(box, by_, sy)
    return fx + sx, fy + sy, true_count


# ------------------------------------------------------------------------ dynamics


def clamp_norm(x, y, limit):
    """``swarp/dynamics/kernels.py:68-71``: ``v * (limit / max(|v|, limit))``."""
    n = wlength(x, y)
    s = limit / wmax(n, limit * torch.ones_like(n))
    return x * s, y * s


def integrate(state, act, fx, fy, w: RefWorld):
    """``swarp/dynamics/kernels.py:166-275,395-403`` for one substep, per agent model."""
    pos, th, vel, s, om = state[:5]
    E, A = th.shape
    dt = w.dt / w.substeps
    a0, a1 = act[..., 0], act[..., 1]
    col = lambda j: w.col(j).expand(E, A)  # noqa: E731
    max_speed, min_speed = col(P_MAX_SPEED), col(P_MIN_SPEED)
    max_accel, max_ang_vel, max_ang_acc = col(P_MAX_ACCEL), col(P_MAX_ANG_VEL), col(P_MAX_ANG_ACCEL)
    l_f, l_r, max_steer, mass = col(P_LF), col(P_LR), col(P_MAX_STEER), col(P_MASS)
    px, py = pos[..., 0], pos[..., 1]
    vx, vy = vel[..., 0], vel[..., 1]
    tag = torch.tensor(w.model_tag, device=th.device).unsqueeze(0).expand(E, A)
    mode = torch.tensor(w.ctrl_mode, device=th.device).unsqueeze(0).expand(E, A)

    # SERVO -> the VELOCITY command it amounts to (kernels.py:166-190, 856-871)
    servo = mode == SERVO
    if bool(servo.any()):
        tv = wclamp(a0, -max_speed, max_speed) * col(P_CMD_GAIN_V)
        tw = wclamp(a1, -max_ang_vel, max_ang_vel) * col(P_CMD_GAIN_W)
        dv, dw = max_accel * dt, max_ang_acc * dt
        a0 = torch.where(servo, s + wclamp(tv - s, -dv, dv), a0)
        a1 = torch.where(servo, om + wclamp(tw - om, -dw, dw), a1)
        mode = torch.where(servo, torch.zeros_like(mode), mode)

    k_dt = dt / mass
    dvx, dvy = fx * k_dt, fy * k_dt
    zero = torch.zeros_like(th)

    # holonomic
    cvx, cvy = clamp_norm(a0, a1, max_speed)
    ax_, ay_ = clamp_norm(a0, a1, max_accel)
    ux, uy = clamp_norm(vx + ax_ * dt, vy + ay_ * dt, max_speed)
    hvx = torch.where(mode == VELOCITY, cvx, ux) + dvx
    hvy = torch.where(mode == VELOCITY, cvy, uy) + dvy
    h = (px + hvx * dt, py + hvy * dt, th, hvx, hvy, wlength(hvx, hvy), zero)

    # diff drive
    s_vel = wclamp(a0, -max_speed, max_speed)
    w_vel = wclamp(a1, -max_ang_vel, max_ang_vel)
    s_acc = wclamp(s + wclamp(a0, -max_accel, max_accel) * dt, -max_speed, max_speed)
    w_acc = wclamp(om + wclamp(a1, -max_ang_acc, max_ang_acc) * dt, -max_ang_vel, max_ang_vel)
    s_dd = torch.where(mode == VELOCITY, s_vel, s_acc)
    w_dd = torch.where(mode == VELOCITY, w_vel, w_acc)
    dvtx = s_dd * torch.cos(th) + dvx
    dvty = s_dd * torch.sin(th) + dvy
    d = (px + dvtx * dt, py + dvty * dt, th + w_dd * dt, dvtx, dvty, s_dd, w_dd)

    # kinematic bicycle (Polack et al. 2017, eq. 2)
    acc = wclamp(a0, -max_accel, max_accel)
    delta = wclamp(a1, -max_steer, max_steer)
    s_b = wclamp(s + acc * dt, min_speed, max_speed)
    wb = l_f + l_r
    beta = torch.atan(torch.tan(delta) * l_r / wb)
    bvx = s_b * torch.cos(th + beta) + dvx
    bvy = s_b * torch.sin(th + beta) + dvy
    w_b = s_b / wb * torch.cos(beta) * torch.tan(delta)
    b = (px + bvx * dt, py + bvy * dt, th + w_b * dt, bvx, bvy, s_b, w_b)

    hold = (px, py, th, vx, vy, s, om)
    out = []
    for i in range(7):
        v = torch.where(tag == HOLONOMIC, h[i],
                        torch.where(tag == DIFF_DRIVE, d[i],
                                    torch.where(tag == BICYCLE, b[i], hold[i])))
        out.append(v)
    drone = None
    if len(state) == 9:  # kernels.py:349-369: the 6-DOF branch; 2-D agents pass it through
        a2, a3 = _act_slot(act, 2), _act_slot(act, 3)
        dr = _drone_euler(px, py, vx, vy, dvx, dvy, state[5:], a0, a1, a2, a3, col, dt)
        is_d = tag == DRONE
        for i, j in ((0, 0), (1, 1), (3, 2), (4, 3)):
            out[i] = torch.where(is_d, dr[j], out[i])
        drone = _merge_drone(is_d, dr[4:], state[5:])
    npx, npy, nth, nvx, nvy, ns, nw = out
    if w.clamp_bounds:
        npx, npy = clamp_footprint(npx, npy, nth, w, col)
    res = (torch.stack([npx, npy], -1), nth, torch.stack([nvx, nvy], -1), ns, nw)
    return res if drone is None else res + drone


def _rk4_deriv(px, py, th, vx, vy, s, om, a0, a1, tag, mode, c):
    """``swarp/dynamics/kernels.py:420-518`` (``_deriv``): the continuous-time derivative of
    each 2-D model's independent states; derived quantities have zero rate."""
    zero = torch.zeros_like(th)
    vel_mode = mode == VELOCITY
    hax, hay = clamp_norm(a0, a1, c["max_accel"])
    h = (vx, vy, zero, torch.where(vel_mode, zero, hax), torch.where(vel_mode, zero, hay), zero,
         zero)
    d = (s * torch.cos(th), s * torch.sin(th), om, zero, zero,
         torch.where(vel_mode, zero, wclamp(a0, -c["max_accel"], c["max_accel"])),
         torch.where(vel_mode, zero, wclamp(a1, -c["max_ang_acc"], c["max_ang_acc"])))
    wb = c["l_f"] + c["l_r"]
    delta = wclamp(a1, -c["max_steer"], c["max_steer"])
    beta = torch.atan(torch.tan(delta) * c["l_r"] / wb)
    b = (s * torch.cos(th + beta), s * torch.sin(th + beta),
         s / wb * torch.cos(beta) * torch.tan(delta), zero, zero,
         wclamp(a0, -c["max_accel"], c["max_accel"]), zero)
    return tuple(torch.where(tag == HOLONOMIC, h[i],
                             torch.where(tag == DIFF_DRIVE, d[i],
                                         torch.where(tag == BICYCLE, b[i], zero)))
                 for i in range(7))


def integrate_rk4(state, act, fx, fy, w: RefWorld):
    """``swarp/dynamics/kernels.py:521-793`` (``_integrate_rk4``) for one substep: classic
    RK4 over four derivative evaluations with the actions held; velocity-mode commands set
    the velocity-level state first; limits apply to the combined result; the contact force
    enters as the Euler path's ``F/m dt`` velocity term (and ``F/m dt^2`` in the pose)."""
    pos, th, vel, s, om = state[:5]
    E, A = th.shape
    dt = w.dt / w.substeps
    a0, a1 = act[..., 0], act[..., 1]
    col = lambda j: w.col(j).expand(E, A)  # noqa: E731
    c = {"max_speed": col(P_MAX_SPEED), "min_speed": col(P_MIN_SPEED),
         "max_accel": col(P_MAX_ACCEL), "max_ang_vel": col(P_MAX_ANG_VEL),
         "max_ang_acc": col(P_MAX_ANG_ACCEL), "l_f": col(P_LF), "l_r": col(P_LR),
         "max_steer": col(P_MAX_STEER), "mass": col(P_MASS)}
    tag = torch.tensor(w.model_tag, device=th.device).unsqueeze(0).expand(E, A)
    mode = torch.tensor(w.ctrl_mode, device=th.device).unsqueeze(0).expand(E, A)
    servo = mode == SERVO
    if bool(servo.any()):  # kernels.py:846-861: SERVO becomes its VELOCITY command
        tv = wclamp(a0, -c["max_speed"], c["max_speed"]) * col(P_CMD_GAIN_V)
        tw = wclamp(a1, -c["max_ang_vel"], c["max_ang_vel"]) * col(P_CMD_GAIN_W)
        dv_, dw_ = c["max_accel"] * dt, c["max_ang_acc"] * dt
        a0 = torch.where(servo, s + wclamp(tv - s, -dv_, dv_), a0)
        a1 = torch.where(servo, om + wclamp(tw - om, -dw_, dw_), a1)
        mode = torch.where(servo, torch.zeros_like(mode), mode)
    px, py, vx, vy = pos[..., 0], pos[..., 1], vel[..., 0], vel[..., 1]
    vel_mode = mode == VELOCITY
    cvx, cvy = clamp_norm(a0, a1, c["max_speed"])
    vx = torch.where(vel_mode & (tag == HOLONOMIC), cvx, vx)
    vy = torch.where(vel_mode & (tag == HOLONOMIC), cvy, vy)
    s = torch.where(vel_mode & (tag == DIFF_DRIVE), wclamp(a0, -c["max_speed"], c["max_speed"]), s)
    om = torch.where(vel_mode & (tag == DIFF_DRIVE),
                     wclamp(a1, -c["max_ang_vel"], c["max_ang_vel"]), om)
    x = (px, py, th, vx, vy, s, om)
    dt2, sixth = dt * 0.5, dt / 6.0
    k1 = _rk4_deriv(*x, a0, a1, tag, mode, c)
    k2 = _rk4_deriv(*(xi + ki * dt2 for xi, ki in zip(x, k1)), a0, a1, tag, mode, c)
    k3 = _rk4_deriv(*(xi + ki * dt2 for xi, ki in zip(x, k2)), a0, a1, tag, mode, c)
    k4 = _rk4_deriv(*(xi + ki * dt for xi, ki in zip(x, k3)), a0, a1, tag, mode, c)
    ipx, ipy, ith, ivx, ivy, i_s, iom = (
        xi + (q1 + q2 * 2.0 + q3 * 2.0 + q4) * sixth for xi, q1, q2, q3, q4 in zip(x, k1, k2, k3, k4))
    k_dt = dt / c["mass"]
    dvx, dvy = fx * k_dt, fy * k_dt
    zero = torch.zeros_like(th)
    ppx, ppy = ipx + dvx * dt, ipy + dvy * dt
    hvx, hvy = clamp_norm(ivx, ivy, c["max_speed"])
    hvx, hvy = hvx + dvx, hvy + dvy
    h = (ppx, ppy, th, hvx, hvy, wlength(hvx, hvy), zero)
    ds_ = wclamp(i_s, -c["max_speed"], c["max_speed"])
    dw_ = wclamp(iom, -c["max_ang_vel"], c["max_ang_vel"])
    d = (ppx, ppy, ith, ds_ * torch.cos(ith) + dvx, ds_ * torch.sin(ith) + dvy, ds_, dw_)
    bs = wclamp(i_s, c["min_speed"], c["max_speed"])
    wb = c["l_f"] + c["l_r"]
    delta = wclamp(a1, -c["max_steer"], c["max_steer"])
    beta = torch.atan(torch.tan(delta) * c["l_r"] / wb)
    bw = bs / wb * torch.cos(beta) * torch.tan(delta)
    b = (ppx, ppy, ith, bs * torch.cos(ith + beta) + dvx, bs * torch.sin(ith + beta) + dvy, bs, bw)
    hold = (pos[..., 0], pos[..., 1], th, vel[..., 0], vel[..., 1], state[3], state[4])
    out = [torch.where(tag == HOLONOMIC, h[i], torch.where(tag == DIFF_DRIVE, d[i],
                                                            torch.where(tag == BICYCLE, b[i], hold[i])))
           for i in range(7)]
    drone = None
    if len(state) == 9:  # kernels.py:494-518, 758-768: the drone's RK4 over its 6-DOF state
        a2, a3 = _act_slot(act, 2), _act_slot(act, 3)
        dr = _drone_rk4(pos[..., 0], pos[..., 1], vel[..., 0], vel[..., 1], dvx, dvy, state[5:],
                        a0, a1, a2, a3, col, dt)
        is_d = tag == DRONE
        for i, j in ((0, 0), (1, 1), (3, 2), (4, 3)):
            out[i] = torch.where(is_d, dr[j], out[i])
        drone = _merge_drone(is_d, dr[4:], state[5:])
    npx, npy, nth, nvx, nvy, ns, nw = out
    if w.clamp_bounds:
        npx, npy = clamp_footprint(npx, npy, nth, w, col)
    res = (torch.stack([npx, npy], -1), nth, torch.stack([nvx, nvy], -1), ns, nw)
    return res if drone is None else res + drone


# -------------------------------------------------------------------------- drone


def _act_slot(act, j):
    """``swarp/dynamics/kernels.py:797-810`` (``_load_actions``): slot j, zero past act_dim."""
    return act[..., j] if act.shape[-1] > j else torch.zeros_like(act[..., 0])


def _cross3(ax, ay, az, bx, by, bz):
    return ay * bz - az * by, az * bx - ax * bz, ax * by - ay * bx


def _quat_rotate(qx, qy, qz, qw, vx, vy, vz):
    """``swarp/dynamics/kernels.py:107-114``: v rotated by the unit quaternion (x, y, z, w),
    ``v + w t + u x t`` with ``t = 2 u x v``."""
    cx, cy, cz = _cross3(qx, qy, qz, vx, vy, vz)
    tx, ty, tz = 2.0 * cx, 2.0 * cy, 2.0 * cz
    ux, uy, uz = _cross3(qx, qy, qz, tx, ty, tz)
    return vx + qw * tx + ux, vy + qw * ty + uy, vz + qw * tz + uz


def _quat_deriv(qx, qy, qz, qw, wx, wy, wz):
    """``swarp/dynamics/kernels.py:117-126``: ``0.5 q (x) (w, 0)`` (Hamilton)."""
    return (0.5 * (qw * wx + qy * wz - qz * wy), 0.5 * (qw * wy - qx * wz + qz * wx),
            0.5 * (qw * wz + qx * wy - qy * wx), 0.5 * (-qx * wx - qy * wy - qz * wz))


def _normalize4(q):
    """Warp ``normalize`` of a 4-vector: q / |q| (zero for the zero vector)."""
    n2 = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]
    pos = n2 > 0
    n = torch.where(pos, torch.sqrt(torch.where(pos, n2, torch.ones_like(n2))), torch.ones_like(n2))
    return tuple(torch.where(pos, x / n, torch.zeros_like(x)) for x in q)


def _drone_rates(f0, f1, f2, f3, q, br, col):
    """``swarp/dynamics/kernels.py:130-163``: world acceleration and body angular
    acceleration of a "+" quadrotor (rotors 0/2 on body x, 1/3 on body y)."""
    mass, g = col(P_MASS), col(P_GRAVITY)
    arm, kappa = col(P_ARM), col(P_KAPPA)
    ixx, iyy, izz = col(P_IXX), col(P_IYY), col(P_IZZ)
    thrust = f0 + f1 + f2 + f3
    z0 = torch.zeros_like(thrust)
    fx, fy, fz = _quat_rotate(*q, z0, z0, thrust)
    acc = (fx / mass - 0.0, fy / mass - 0.0, fz / mass - g)
    tx = arm * (f1 - f3)
    ty = arm * (f2 - f0)
    tz = kappa * (f0 - f1 + f2 - f3)
    bx, by, bz = br
    ang = ((tx - (izz - iyy) * by * bz) / ixx, (ty - (ixx - izz) * bz * bx) / iyy,
           (tz - (iyy - ixx) * bx * by) / izz)
    return acc, ang


def _thrusts(a0, a1, a2, a3, col):
    tmax = col(P_THRUST_MAX)
    z = torch.zeros_like(tmax)
    return tuple(wclamp(a, z, tmax) for a in (a0, a1, a2, a3))


def _drone_euler(px, py, vx, vy, dvx, dvy, d, a0, a1, a2, a3, col, dt):
    """``swarp/dynamics/kernels.py:349-369``: semi-implicit Euler of the 6-DOF state (rates
    and velocities first, then attitude with the new rates and positions with the new
    velocities). Returns (px, py, vx, vy, z, vz, attitude, body_rates)."""
    z, vz, att, br = d
    q = tuple(att[..., i] for i in range(4))
    b = tuple(br[..., i] for i in range(3))
    acc, ang = _drone_rates(*_thrusts(a0, a1, a2, a3, col), q, b, col)
    nb = tuple(b[i] + ang[i] * dt for i in range(3))
    nvz = vz + acc[2] * dt
    nvx = vx + acc[0] * dt + dvx
    nvy = vy + acc[1] * dt + dvy
    qd = _quat_deriv(*q, *nb)
    nq = _normalize4(tuple(q[i] + qd[i] * dt for i in range(4)))
    return (px + nvx * dt, py + nvy * dt, nvx, nvy, z + nvz * dt, nvz,
            torch.stack(nq, -1), torch.stack(nb, -1))


def _drone_deriv(vx, vy, vz, q, b, f, col):
    """The drone rows of ``_deriv`` (``swarp/dynamics/kernels.py:494-508``)."""
    acc, ang = _drone_rates(*f, q, b, col)
    return (vx, vy, acc[0], acc[1], vz, acc[2], _quat_deriv(*q, *b), ang)


def _drone_rk4(px, py, vx, vy, dvx, dvy, d, a0, a1, a2, a3, col, dt):
    """``swarp/dynamics/kernels.py:521-793`` for a drone: RK4 over (p, v, z, vz, q, rates)
    with the thrusts held, the contact force as the Euler path's F/m dt velocity term,
    the attitude renormalized after the combine."""
    z, vz, att, br = d
    f = _thrusts(a0, a1, a2, a3, col)
    x = [px, py, vx, vy, z, vz] + [att[..., i] for i in range(4)] + [br[..., i] for i in range(3)]

    def deriv(x):
        k = _drone_deriv(x[2], x[3], x[5], tuple(x[6:10]), tuple(x[10:13]), f, col)
        return [k[0], k[1], k[2], k[3], k[4], k[5], *k[6], *k[7]]

    dt2, sixth = dt * 0.5, dt / 6.0
    k1 = deriv(x)
    k2 = deriv([xi + ki * dt2 for xi, ki in zip(x, k1)])
    k3 = deriv([xi + ki * dt2 for xi, ki in zip(x, k2)])
    k4 = deriv([xi + ki * dt for xi, ki in zip(x, k3)])
    xi = [x0 + (q1 + q2 * 2.0 + q3 * 2.0 + q4) * sixth for x0, q1, q2, q3, q4 in zip(x, k1, k2, k3, k4)]
    nq = _normalize4(tuple(xi[6:10]))
    return (xi[0] + dvx * dt, xi[1] + dvy * dt, xi[2] + dvx, xi[3] + dvy, xi[4], xi[5],
            torch.stack(nq, -1), torch.stack(xi[10:13], -1))


def _merge_drone(is_d, new, old):
    """Drone agents take the new 6-DOF fields, every other agent passes them through."""
    out = []
    for n, o in zip(new, old):
        m = is_d if n.dim() == is_d.dim() else is_d.unsqueeze(-1)
        out.append(torch.where(m, n, o))
    return tuple(out)


# -------------------------------------------------------------------------- bodies


def _reaction(px, py, vx, vy, ra, am, cx, cy, ang, st, r_o, hx, hy, vox, voy, om, w: RefWorld):
    """``swarp/core/bodies.py:79-127``: force on the body from one agent, and its lever."""
    denom = 1.0 + w.c * (w.dt / w.substeps) / am
    k, c, margin, mo = w.k, w.c, w.margin, w.max_overlap
    z = torch.zeros_like(px)
    if st == BOX:
        fx, fy = box_force(px, py, vx, vy, cx, cy, ang, hx, hy, ra + margin, k, c, denom, mo,
                           vox, voy, om)
        rx, ry = px - cx, py - cy
    elif st == SEGMENT:
        qx, qy = closest_on_segment(px, py, cx, cy, ang, hx)
        rrx, rry = qx - cx, qy - cy
        vsx = vox + (-om * rry)
        vsy = voy + om * rrx
        fx, fy = pair_force(px - qx, py - qy, vx - vsx, vy - vsy, ra + r_o + margin, k, c, denom,
                            mo)
        rx, ry = rrx, rry
    else:
        fx, fy = pair_force(px - cx, py - cy, vx - vox, vy - voy, ra + r_o + margin, k, c, denom,
                            mo)
        rx, ry = z, z
    return -fx, -fy, rx, ry


def _reaction_box(px, py, th, vx, vy, wa, hax, hay, am, cx, cy, ang, st, r_o, hx, hy, vox, voy,
                  om, w: RefWorld):
    """``swarp/core/bodies.py:131-166``: force on the body from a box agent, and its lever
    from the shape centre: the negated ``_box_obstacle_force`` (``collisions.py:544-582``)
    and its contact point (a circle shape: its centre)."""
    denom = 1.0 + w.c * (w.dt / w.substeps) / am
    k, c, m, mo = w.k, w.c, w.margin, w.max_overlap
    zc = torch.zeros_like(px)
    if st == BOX:
        fx, fy, xx, xy = obb_force_at(px, py, th, hax, hay, vx, vy, wa, cx, cy, ang, hx + zc,
                                      hy + zc, vox, voy, om, m, k, c, denom, mo)
    elif st == SEGMENT:
        fx, fy, xx, xy = obb_force_at(px, py, th, hax, hay, vx, vy, wa, cx, cy, ang, hx + zc, zc,
                                      vox, voy, om, r_o + m, k, c, denom, mo)
    else:
        gx, gy = box_force(cx, cy, vox, voy, px, py, th, hax, hay, r_o + m, k, c, denom, mo,
                           vx, vy, wa)
        fx, fy, xx, xy = -gx, -gy, cx + zc, cy + zc
    return -fx, -fy, xx - cx, xy - cy


def _closest_in_box(dx, dy, ang, hx, hy):
    ca, sa = torch.cos(ang), torch.sin(ang)
    lx = ca * dx + sa * dy
    ly = -sa * dx + ca * dy
    cx = wclamp(lx, -hx, hx)
    cy = wclamp(ly, -hy, hy)
    return ca * cx - sa * cy, sa * cx + ca * cy


def _body_body(qx, qy, tvx, tvy, th, om_s, st, r_s, hxs, hys,
               q2x, q2y, tv2x, tv2y, th2, om2, st2, r2, hx2, hy2, w: RefWorld, denom):
    """``swarp/core/bodies.py:167-255``: contact on shape ``self`` from another shape."""
    k, c, margin, mo = w.k, w.c, w.margin, w.max_overlap
    z = torch.zeros_like(qx)
    if st == BOX:
        if st2 == BOX:
            return z, z, z, z
        c2x, c2y, v2x, v2y = q2x, q2y, tv2x, tv2y
        if st2 == SEGMENT:
            c2x, c2y = closest_on_segment(qx, qy, q2x, q2y, th2, hx2)
            rrx, rry = c2x - q2x, c2y - q2y
            v2x = tv2x + (-om2 * rry)
            v2y = tv2y + om2 * rrx
        fox, foy = box_force(c2x, c2y, v2x, v2y, qx, qy, th, hxs, hys, r2 + margin, k, c, denom, mo,
                             tvx, tvy, om_s)
        rx, ry = _closest_in_box(c2x - qx, c2y - qy, th, hxs, hys)
        return -fox, -foy, rx, ry
    if st2 == BOX:
        fx, fy = box_force(qx, qy, tvx, tvy, q2x, q2y, th2, hx2, hy2, r_s + margin, k, c, denom, mo,
                           tv2x, tv2y, om2)
        return fx, fy, z, z
    if st2 == SEGMENT:
        cpx, cpy = closest_on_segment(qx, qy, q2x, q2y, th2, hx2)
        rrx, rry = cpx - q2x, cpy - q2y
        vs2x = tv2x + (-om2 * rry)
        vs2y = tv2y + om2 * rrx
        fx, fy = pair_force(qx - cpx, qy - cpy, tvx - vs2x, tvy - vs2y, r_s + r2 + margin, k, c,
                            denom, mo)
        return fx, fy, z, z
    fx, fy = pair_force(qx - q2x, qy - q2y, tvx - tv2x, tvy - tv2y, r_s + r2 + margin, k, c, denom,
                        mo)
    return fx, fy, z, z


def body_pass(state, obs: RefObstacles, w: RefWorld):
    """``swarp/core/bodies.py:367-569``: one substep of every movable body root.

    Every body reads the other shapes' pre-pass poses (the reference kernel reads
    ``obs_pos`` of other bodies while their own threads rewrite it; with one movable
    body, as in every configuration here, the two readings coincide).
    Returns a new :class:`RefObstacles`.
    """
    pos, theta, vel, _, ang_vel = state[:5]
    px, py = pos[..., 0], pos[..., 1]
    vx, vy = vel[..., 0], vel[..., 1]
    E, A = px.shape
    dt = w.dt / w.substeps
    ra_all = w.col(P_RADIUS).expand(E, A)
    am_all = w.col(P_MASS).expand(E, A)
    box_all = (w.col(P_SHAPE) > 0.5).expand(E, A)
    hx_all, hy_all = w.col(P_HALF_X).expand(E, A), w.col(P_HALF_Y).expand(E, A)
    any_box = bool(box_all.any())
    N = obs.n
    new = {
        "pos": [obs.pos[:, s] for s in range(N)],
        "angle": [obs.angle[:, s] for s in range(N)],
        "vel": [obs.vel[:, s] for s in range(N)],
        "ang_vel": [obs.ang_vel[:, s] for s in range(N)],
        "bpos": [obs.body_pos[:, s] for s in range(N)],
        "bang": [obs.body_angle[:, s] for s in range(N)],
        "bvel": [obs.body_vel[:, s] for s in range(N)],
        "bom": [obs.body_ang_vel[:, s] for s in range(N)],
    }
    for o in range(N):
        if int(obs.body[o]) != o or int(obs.kind[o]) != 1:
            continue
        qx, qy = obs.body_pos[:, o, 0], obs.body_pos[:, o, 1]
        tvx, tvy = obs.body_vel[:, o, 0], obs.body_vel[:, o, 1]
        th = obs.body_angle[:, o]
        om = obs.body_ang_vel[:, o]
        ca, sa = torch.cos(th), torch.sin(th)
        fx = torch.zeros_like(qx)
        fy = torch.zeros_like(qx)
        tau = torch.zeros_like(qx)
        denom_self = 1.0 + w.c * dt / obs.mass[o]
        ext = torch.zeros_like(qx)
        for s_ in range(N):
            if int(obs.body[s_]) != o:
                continue
            offx, offy = obs.body_off[s_, 0], obs.body_off[s_, 1]
            owx = ca * offx - sa * offy
            owy = sa * offx + ca * offy
            csx, csy = qx + owx, qy + owy
            vsx, vsy = tvx - om * owy, tvy + om * owx
            st = int(obs.shape[s_])
            r_o = obs.radius[s_]
            hx, hy = obs.half[s_, 0], obs.half[s_, 1]
            ax, ay = wabs(offx), wabs(offy)
            if st == BOX:
                reach = torch.sqrt((ax + hx) * (ax + hx) + (ay + hy) * (ay + hy))
            elif st == SEGMENT:
                reach = torch.sqrt((ax + hx) * (ax + hx) + ay * ay) + r_o
            else:
                reach = torch.sqrt(ax * ax + ay * ay) + r_o
            ext = wmax(ext, reach * torch.ones_like(ext))
            bound = shape_bound(st, r_o, hx, hy)
            for a in range(A):
                pax, pay = px[:, a], py[:, a]
                ra = ra_all[:, a]
                if any_box:  # a box agent's bounding disc: max(radius, half-diagonal)
                    isb = box_all[:, a]
                    hxa, hya = hx_all[:, a], hy_all[:, a]
                    ra = torch.where(isb, wmax(ra, torch.sqrt(hxa * hxa + hya * hya)), ra)
                apart = bounds_apart(pax - csx, pay - csy, ra + bound + w.margin)
                rfx, rfy, rx, ry = _reaction(pax, pay, vx[:, a], vy[:, a], ra_all[:, a],
                                             am_all[:, a], csx, csy, th, st, r_o, hx, hy, vsx,
                                             vsy, om, w)
                if any_box:
                    bfx, bfy, brx, bry = _reaction_box(
                        pax, pay, theta[:, a], vx[:, a], vy[:, a], ang_vel[:, a], hxa, hya,
                        am_all[:, a], csx, csy, th, st, r_o, hx, hy, vsx, vsy, om, w)
                    rfx, rfy = torch.where(isb, bfx, rfx), torch.where(isb, bfy, rfy)
                    rx, ry = torch.where(isb, brx, rx), torch.where(isb, bry, ry)
                lx, ly = owx + rx, owy + ry
                z = torch.zeros_like(fx)
                fx = fx + torch.where(apart, z, rfx)
                fy = fy + torch.where(apart, z, rfy)
                tau = tau + torch.where(apart, z, lx * rfy - ly * rfx)
            for o2 in range(N):
                if int(obs.body[o2]) == o:
                    continue
                st2 = int(obs.shape[o2])
                q2x, q2y = obs.pos[:, o2, 0], obs.pos[:, o2, 1]
                apart = bounds_apart(
                    q2x - csx, q2y - csy,
                    bound + shape_bound(st2, obs.radius[o2], obs.half[o2, 0], obs.half[o2, 1])
                    + w.margin,
                )
                f2x, f2y, r2x, r2y = _body_body(
                    csx, csy, vsx, vsy, th, om, st, r_o, hx, hy,
                    q2x, q2y, obs.vel[:, o2, 0], obs.vel[:, o2, 1], obs.angle[:, o2],
                    obs.ang_vel[:, o2], st2, obs.radius[o2], obs.half[o2, 0], obs.half[o2, 1],
                    w, denom_self,
                )
                lx, ly = owx + r2x, owy + r2y
                z = torch.zeros_like(fx)
                fx = fx + torch.where(apart, z, f2x)
                fy = fy + torch.where(apart, z, f2y)
                tau = tau + torch.where(apart, z, lx * f2y - ly * f2x)
        lin_decay = 1.0 - w.lin_damping * dt
        ang_decay = 1.0 - w.ang_damping * dt
        nvx = (tvx + fx / obs.mass[o] * dt) * lin_decay
        nvy = (tvy + fy / obs.mass[o] * dt) * lin_decay
        nom = (om + tau / obs.inertia[o] * dt) * ang_decay
        nx = qx + nvx * dt
        ny = qy + nvy * dt
        if w.bounds is not None:
            x0, x1, y0, y1 = w.bounds
            lo_x = wmin(x0 + ext, torch.full_like(ext, (x0 + x1) * 0.5))
            hi_x = wmax(x1 - ext, lo_x)
            lo_y = wmin(y0 + ext, torch.full_like(ext, (y0 + y1) * 0.5))
            hi_y = wmax(y1 - ext, lo_y)
            cx_ = wclamp(nx, lo_x, hi_x)
            cy_ = wclamp(ny, lo_y, hi_y)
            nvx = torch.where(cx_ != nx, torch.zeros_like(nvx), nvx)
            nvy = torch.where(cy_ != ny, torch.zeros_like(nvy), nvy)
            nx, ny = cx_, cy_
        nth = th + nom * dt
        new["bvel"][o] = torch.stack([nvx, nvy], -1)
        new["bom"][o] = nom
        new["bpos"][o] = torch.stack([nx, ny], -1)
        new["bang"][o] = nth
        nca, nsa = torch.cos(nth), torch.sin(nth)
        for s_ in range(N):
            if int(obs.body[s_]) != o:
                continue
            offx, offy = obs.body_off[s_, 0], obs.body_off[s_, 1]
            owx = nca * offx - nsa * offy
            owy = nsa * offx + nca * offy
            new["pos"][s_] = torch.stack([nx + owx, ny + owy], -1)
            new["angle"][s_] = nth
            new["vel"][s_] = torch.stack([nvx - nom * owy, nvy + nom * owx], -1)
            new["ang_vel"][s_] = nom
    st = lambda key: torch.stack(new[key], 1)  # noqa: E731
    return RefObstacles(
        pos=st("pos"), angle=st("angle"), vel=st("vel"), ang_vel=st("ang_vel"),
        radius=obs.radius, half=obs.half, shape=obs.shape, kind=obs.kind, mass=obs.mass,
        inertia=obs.inertia, body=obs.body, body_off=obs.body_off,
        body_pos=st("bpos"), body_angle=st("bang"), body_vel=st("bvel"), body_ang_vel=st("bom"),
    )


def seed_bodies(obs: RefObstacles) -> RefObstacles:
    """Body state derived from the root shapes' world poses (``stepper.py`` ``_body_seed``)."""
    root = torch.tensor([int(b) for b in obs.body], device=obs.pos.device)
    r_ang = obs.angle[:, root]
    r_off = obs.body_off[root]
    ca, sa = torch.cos(r_ang), torch.sin(r_ang)
    wx = ca * r_off[:, 0] - sa * r_off[:, 1]
    wy = sa * r_off[:, 0] + ca * r_off[:, 1]
    obs.body_pos = obs.pos[:, root] - torch.stack([wx, wy], -1)
    obs.body_angle = r_ang
    obs.body_vel = obs.vel[:, root]
    obs.body_ang_vel = obs.ang_vel[:, root]
    return obs


# ---------------------------------------------------------------------------- step


def step(state, act, w: RefWorld, obs: RefObstacles | None = None):
    """One env step (all substeps). Returns ``(state, obs, max_true_count)``."""
    tmax = None
    for _ in range(w.substeps):
        fx, fy, tc = collision_forces(state, w, obs)
        tmax = tc if tmax is None else torch.maximum(tmax, tc)
        if obs is not None and w.bodies_move and obs.any_movable():
            obs_next = body_pass(state, obs, w)
        else:
            obs_next = obs
        state = (integrate_rk4 if w.rk4 else integrate)(state, act, fx, fy, w)
        obs = obs_next
    return state, obs, tmax


def rollout(state, actions_seq, w: RefWorld, obs: RefObstacles | None = None):
    """``swarp/interop/autograd.py:341-369`` restated: T steps, returns final + trajectory."""
    traj = []
    body_traj = []
    for t in range(actions_seq.shape[0]):
        state, obs, _ = step(state, actions_seq[t], w, obs)
        traj.append(state)
        body_traj.append(obs)
    return state, traj, body_traj
