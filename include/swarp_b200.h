/*
 * swarp_b200 — C ABI of the B200 (sm_100a) differentiable batched physics step.
 *
 * This is the boundary the Python layer (swarp_b200.interop / swarp_b200.core) calls
 * through ctypes. Every entry point takes plain pointers and sizes, allocates nothing,
 * launches on the caller's CUDA stream, never aborts, and returns SWARP_OK (0) or a
 * negative error code (see swarp_error_string). All device pointers address
 * contiguous row-major arrays in the dtype named by swarp_world_t.dtype.
 *
 * What each entry point replaces in the reference (ddebenedittis/swarp):
 *   swarp_rollout_fwd  -> the forward half of swarp/interop/autograd.py:341-369
 *                         (rollout: T x warp_step, each Stepper.launch_substeps at
 *                         swarp/core/stepper.py:784-1011: neighbor build
 *                         swarp/core/neighbors.py:76-97, collision_forces_kernel
 *                         swarp/core/collisions.py:818-881, obstacle_dynamics_kernel
 *                         swarp/core/bodies.py:367-569, integrate_kernel
 *                         swarp/dynamics/kernels.py:812-971)
 *   swarp_rollout_bwd  -> the backward half: _WarpStepFn.backward
 *                         swarp/interop/autograd.py:277-296 (wp.Tape.backward replay of
 *                         Warp's generated adjoints), T times in reverse
 *   swarp_neighbors    -> NeighborGrid brute build + overflow view
 *                         swarp/core/neighbors.py:76-97, 465-492, 709-714
 */
#ifndef SWARP_B200_H
#define SWARP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SWARP_OK 0
#define SWARP_ERR_INVALID_ARG (-1)   /* null pointer, bad size or inconsistent config */
#define SWARP_ERR_UNSUPPORTED (-2)   /* model / option this build does not run       */
#define SWARP_ERR_TOO_MANY_AGENTS (-3) /* n_agents above SWARP_MAX_AGENTS            */
#define SWARP_ERR_CUDA (-4)          /* a CUDA launch or attribute call failed       */
#define SWARP_ERR_WORKSPACE (-5)     /* workspace pointer null or too small          */
#define SWARP_ERR_SCRATCH_LIMIT (-6) /* swarp_rollout_noalloc: rollout needs more workspace
                                        than SWARP_NOALLOC_SCRATCH_BYTES                 */

/* Agents per env. Envs of up to SWARP_MAX_CTA_AGENTS agents run in one CTA; larger envs
 * run one env per thread-block cluster of up to 8 CTAs (2-D disc fleets: no movable
 * bodies, box agents or drones, which return SWARP_ERR_UNSUPPORTED there). The reference
 * has no per-env agent limit (swarp/core/neighbors.py:135-254 grids any count). */
#define SWARP_MAX_AGENTS 4096
#define SWARP_MAX_CTA_AGENTS 1024
#define SWARP_NUM_PARAMS 22

typedef enum { SWARP_F32 = 0, SWARP_F64 = 1 } swarp_dtype_t;
typedef enum { SWARP_BOUNDS_NONE = 0, SWARP_BOUNDS_SOFT = 1, SWARP_BOUNDS_CLAMP = 2 } swarp_bounds_t;

/* The five live 2-D agent fields, structure of arrays. For a state at one time the
 * shapes are pos/vel [E, A, 2] and theta/speed/ang_vel [E, A]; for a trajectory a
 * leading [T] is added. A NULL field means "absent" where the entry point says so. */
typedef struct {
  void* pos;
  void* theta;
  void* vel;
  void* speed;
  void* ang_vel;
  /* 6-DOF drone fields (swarp/core/state.py WorldState.z/vz/attitude/body_rates); read and
   * written only in worlds with drone agents (fleet_models bit 3), NULL otherwise */
  void* z;          /* [.., E, A]    */
  void* vz;         /* [.., E, A]    */
  void* attitude;   /* [.., E, A, 4] unit quaternion (x, y, z, w), body to world */
  void* body_rates; /* [.., E, A, 3] */
} swarp_state_t;

/* Obstacle set (E envs, N shapes). Poses and motion are per env, extents per shape.
 * Movable compound bodies (kind == 1) are integrated inside the substep loop. */
typedef struct {
  int32_t n_obstacles;   /* N; 0 = no obstacles (all other fields ignored) */
  const void* pos;       /* [E, N, 2] */
  const void* angle;     /* [E, N]    */
  const void* vel;       /* [E, N, 2] */
  const void* ang_vel;   /* [E, N]    */
  const void* radius;    /* [N]       */
  const void* half;      /* [N, 2]    */
  const int32_t* shape;  /* [N] 0 circle, 1 box, 2 segment */
  const int32_t* kind;   /* [N] 0 immovable, 1 movable */
  const void* mass;      /* [N] */
  const void* inertia;   /* [N] */
  const int32_t* body;   /* [N] body root index of each shape */
  const void* body_off;  /* [N, 2] shape placement in its body frame */
  int32_t any_movable;   /* 1 when any kind == 1 (host-known; selects the body pass) */
  int32_t bodies_move;   /* 0 freezes movable bodies (the reference's taped-step rule) */
  int32_t movable_shapes; /* host-known bitmask (1 << shape) over the shapes of movable
                             bodies; the adjoint differentiates circle bodies only */
  int32_t poses_from_bodies; /* 1: moving shapes start at the poses placed from the bodies'
                                initial state (a continuing rollout); 0: at the installed
                                pos/angle/vel/ang_vel (the first substep after an install) */
} swarp_obstacles_t;

/* Movable-body state per shape slot (only body-root slots are meaningful):
 * pos/vel [E, N, 2], angle/ang_vel [E, N]; a trajectory adds a leading [T]. */
typedef struct {
  void* pos;
  void* angle;
  void* vel;
  void* ang_vel;
} swarp_bodies_t;

typedef struct {
  int32_t dtype;          /* swarp_dtype_t */
  int32_t n_envs;         /* E */
  int32_t n_agents;       /* A, 1..SWARP_MAX_AGENTS */
  int32_t act_dim;        /* action slots per agent, >= 2 (slots past 2 are ignored) */
  int32_t substeps;       /* >= 1 */
  double dt;              /* env step; the substep is dt / substeps */
  int32_t collisions;     /* agent-agent contacts on/off */
  double k, c, margin, max_overlap;
  double neighbor_radius; /* R of the within-radius lists */
  int32_t max_neighbors;  /* K, list cap (first K by agent index) */
  int32_t bounds_mode;    /* swarp_bounds_t */
  double bounds[4];       /* x_min, x_max, y_min, y_max */
  double lin_damping, ang_damping; /* movable-body drag */
  const void* params;     /* [A, 22] shared, or [E, A, 22] per env */
  int64_t params_env_stride; /* elements between consecutive envs' rows; 0 = shared */
  const int32_t* model_tag;  /* [A] DynamicsModel (0..2 run here) */
  const int32_t* ctrl_mode;  /* [A] ControlMode */
  int32_t fleet_models;      /* host-known bitmask of the DynamicsModel values in model_tag */
  int32_t fleet_modes;       /* host-known bitmask of the ControlMode values in ctrl_mode */
  swarp_obstacles_t obstacles;
  int32_t integrator;        /* 0 semi-implicit Euler, 1 classic RK4 (dynamics/kernels.py:521-793) */
  int32_t box_agents;        /* host-known: some params row has shape BOX (P_SHAPE = 1); the
                                oriented-box contacts of swarp/core/collisions.py:262-690 */
} swarp_world_t;

/* The fused goal loss L = sum over envs and agents of |pos_T - goal|^2 (pos_T: the
 * positions after the last step). goal [E, A, 2] in the world's dtype, NULL = no loss.
 * swarp_rollout_fwd writes L (one scalar of the world's dtype) to `loss`, reduced in a
 * fixed order from per-CTA partials in the workspace's tail; swarp_rollout_bwd adds
 * loss_grad[0] * dL/dpos_T (loss_grad: one device scalar, dL'/dL of the caller's loss)
 * to the final-position cotangent. This is a fused fast path of the library: the
 * reference's callers form such losses in torch after the rollout. */
typedef struct {
  const void* goal;
  void* loss;             /* swarp_rollout_fwd output */
  const void* loss_grad;  /* swarp_rollout_bwd input  */
} swarp_goal_loss_t;

/* Bytes of device workspace for this world and horizon: the contact checkpoint that
 * swarp_rollout_fwd fills and swarp_rollout_bwd reads, then the adjoint's per-CTA
 * partial sums for adj_actions_sqnorm (0 for an invalid world). */
size_t swarp_rollout_workspace_bytes(const swarp_world_t* w, int32_t horizon);

/* Forward rollout of `horizon` steps from `init`.
 *   actions   [T, E, A, act_dim]
 *   traj      out: the state after every step, [T, E, A(,2)] (all five fields required)
 *   final     out (fields may be NULL): the state after the last step
 *   true_count_max  out [E, A] int32 or NULL: max over all substeps of the uncapped
 *             within-radius neighbor count (overflow <=> > max_neighbors)
 *   bodies_init / bodies_traj: movable-body state at t=0 and after every step
 *             (required only when obstacles.any_movable)
 *   goal_loss: the fused goal loss (goal NULL = none; loss required with a goal)
 *   workspace: device scratch of swarp_rollout_workspace_bytes() bytes, kept for the
 *             matching swarp_rollout_bwd call. */
int swarp_rollout_fwd(const swarp_world_t* w, int32_t horizon, swarp_state_t init,
                      const void* actions, swarp_state_t traj, swarp_state_t final_out,
                      int32_t* true_count_max, swarp_bodies_t bodies_init,
                      swarp_bodies_t bodies_traj, swarp_goal_loss_t goal_loss,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Adjoint of swarp_rollout_fwd (same world, horizon, init, actions, traj, bodies and
 * workspace). Cotangents: adj_traj [T, ...] and adj_final (any field may be NULL =
 * zero), adj_bodies_final (fields may be NULL; body pos/angle/vel/ang_vel after the
 * last step). Outputs: adj_actions [T, E, A, act_dim] and adj_init (all five fields
 * required); adj_actions_sqnorm (NULL = not computed): one scalar of the world's dtype,
 * the sum of squares of adj_actions, reduced in the kernel's epilogue (the per-CTA
 * partials go to the workspace's tail) instead of a second pass over adj_actions.
 * Deterministic: no atomics, fixed summation order. Moving bodies are differentiated
 * when all their shapes are circles (SWARP_ERR_UNSUPPORTED otherwise). The fused norm
 * has no counterpart in the reference (its callers compute it from the gradient).
 * goal_loss: with a goal, loss_grad (required) seeds the goal loss's cotangent. */
int swarp_rollout_bwd(const swarp_world_t* w, int32_t horizon, swarp_state_t init,
                      const void* actions, swarp_state_t traj, swarp_state_t adj_traj,
                      swarp_state_t adj_final, swarp_bodies_t bodies_init,
                      swarp_bodies_t bodies_traj, swarp_bodies_t adj_bodies_final,
                      void* adj_actions, swarp_state_t adj_init, void* adj_actions_sqnorm,
                      swarp_goal_loss_t goal_loss, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Padded within-radius neighbor lists of positions pos [E, A, 2] (brute force, ascending
 * agent index, capped at max_neighbors): idx [E, A, K] int32 (unused slots untouched),
 * count [E, A], true_count [E, A] (uncapped). */
int swarp_neighbors(const swarp_world_t* w, const void* pos, int32_t* idx, int32_t* count,
                    int32_t* true_count, void* stream);

/* Allocation-free BPTT rollout: swarp_rollout_fwd followed by swarp_rollout_bwd in one
 * call, for callers that cannot allocate device memory (a plugin under another
 * runtime's memory manager, such as an XLA/JAX custom call, must not allocate behind
 * that manager's back; a real-time control loop cannot wait on cudaMalloc, which may
 * synchronize the device). This entry point has no counterpart in the reference. The two kernels' shared
 * workspace lives in a static device array of SWARP_NOALLOC_SCRATCH_BYTES that the
 * library owns (one per GPU that loads it, held until the process exits); nothing else
 * is allocated. Arguments mean what they mean for swarp_rollout_fwd / _bwd (final_out,
 * adj_traj, adj_final fields may be NULL); movable bodies are not accepted here.
 * Returns SWARP_ERR_SCRATCH_LIMIT when swarp_rollout_workspace_bytes() exceeds
 * SWARP_NOALLOC_SCRATCH_BYTES. The first call on each device resolves the array's
 * device address (cudaGetSymbolAddress) with that device current: make it before any
 * stream capture. The address is kept for the life of the process: after a
 * cudaDeviceReset of a device, do not call this entry point on that device again. All
 * calls share the array, so calls that overlap on one GPU race on it; serialize them. */
#define SWARP_NOALLOC_SCRATCH_BYTES (16u << 20)
int swarp_rollout_noalloc(const swarp_world_t* w, int32_t horizon, swarp_state_t init,
                          const void* actions, swarp_state_t traj, swarp_state_t final_out,
                          swarp_state_t adj_traj, swarp_state_t adj_final, void* adj_actions,
                          swarp_state_t adj_init, void* stream);

/* Strided asynchronous copy of `rows` rows of `row_bytes` each, between any two of host
 * (pinned) and device memory (cudaMemcpy2DAsync, direction from the pointers), on
 * `stream`. This is host plumbing with no counterpart in the reference: it moves one env
 * slice of a [T, E, ...] array (T rows, one per step) in one call, which the streamed
 * BPTT front end (swarp_b200.interop.streamed) uses to pipeline host inputs and gradients
 * against the kernels env chunk by env chunk. */
int swarp_copy_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch,
                    size_t row_bytes, size_t rows, void* stream);

/* Static description of a return code. */
const char* swarp_error_string(int code);

/* ABI version of this library (bumped on any signature change). */
int32_t swarp_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SWARP_B200_H */
