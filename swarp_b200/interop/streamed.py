"""BPTT steps over a batch that lives in host memory, streamed through the GPU in env chunks.

A BPTT step whose inputs (actions ``[T, E, A, D]``, initial state) start in host memory and
whose result (the action gradient, same shape) must end there moves far more bytes over
the host link than the kernels move in HBM: at 16,000 envs x 16 agents x 64 steps, 136 MB
in and 131 MB out against about 0.4 ms of kernel time. Done one after the other, the two
copies and the kernels add up. :class:`StreamedRollout` splits the envs into chunks
(environments are independent, so a chunk's results equal the whole batch's for its envs,
bit for bit) and runs three streams: host-to-device copies of chunk i+1, the captured BPTT
step (:class:`~swarp_b200.interop.graphs.GraphedRollout`) of chunk i, and device-to-host
copies of chunk i-1's gradient and loss. The host link carries both directions at once,
so a step costs about the larger of the two copies rather than their sum plus the
kernels. Consecutive calls overlap as well (the next step's input copies run beside this
step's last output copies), so few large chunks keep both directions busy; every copy has
a fixed cost, so more chunks cost more (measured at 16,000 envs: 2 chunks 3.3 ms per step,
4 chunks 3.4 ms, 8 chunks 3.9-4.5 ms). Each chunk's slice of a ``[T, E, ...]`` host array is one strided copy
(``swarp_copy_rows``, a ``cudaMemcpy2DAsync``).

The reference has no counterpart: its ``rollout`` takes device tensors
(``swarp/interop/autograd.py:341-369``). Host tensors must be pinned for the copies to be
asynchronous.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch

from swarp_b200 import _lib
from swarp_b200.core.stepper import Stepper
from swarp_b200.interop.autograd import FusedGoalLoss, TorchState, Trajectory
from swarp_b200.interop.graphs import GraphedRollout


def _chunks(n_envs: int, want: int) -> int:
    """The largest chunk count <= want that divides n_envs (equal chunks share graphs)."""
    for c in range(max(1, min(want, n_envs)), 0, -1):
        if n_envs % c == 0:
            return c
    return 1


class StreamedRollout:
    """``loss_fn(final, trajectory, *aux) -> scalar`` and its gradient w.r.t. the actions,
    for a batch held in pinned host memory, pipelined over env chunks.

    ``aux_like`` are example tensors ``[E, ...]`` of the extra per-env inputs ``loss_fn``
    reads (goals, weights); they are chunked along the env axis like the state
    (``loss_fn="goal"``: the fused goal loss, ``aux_like[0]`` the goals). Calling the
    object with host tensors enqueues one BPTT step of the whole batch and returns at once:
    the gradient lands in ``grad_out`` (host, ``[T, E, A, D]``) and the per-chunk losses in
    ``loss_out`` (host, ``[chunks]``, float64) when :meth:`synchronize` returns. Consecutive
    calls overlap (the next step's input copies start while this step's last chunks run).
    """

    def __init__(self, stepper: Stepper, n_envs: int, horizon: int, act_dim: int,
                 loss_fn: Callable[..., torch.Tensor], aux_like: Sequence[torch.Tensor] = (),
                 *, chunks: int = 2, slots: int = 3) -> None:
        if stepper.any_movable or stepper.has_drones:
            raise NotImplementedError("StreamedRollout captures 2-D fleets without movable "
                                      "bodies (as GraphedRollout)")
        dev = stepper.device
        self.stepper = stepper
        self.E, self.H, self.D, self.A = n_envs, horizon, act_dim, stepper.n_agents
        self.n_chunks = _chunks(n_envs, chunks)
        self.Ec = n_envs // self.n_chunks
        self.lib = _lib.load()
        opts = {"device": dev, "dtype": stepper.dtype}
        Ec, A = self.Ec, self.A
        # Per-env world data (obstacle poses, per-env parameters): every chunk has its own
        # stepper over its envs' slice, and so its own captured step (one slot per chunk).
        # Otherwise the chunks share `slots` captured steps round-robin.
        self.per_chunk = stepper.n_obstacles > 0 or stepper.params_per_env is not None
        n_slots = self.n_chunks if self.per_chunk else max(2, slots)
        self.slots = []
        for i in range(n_slots):
            st_i = stepper.env_slice(i * Ec, (i + 1) * Ec) if self.per_chunk else stepper
            aux = tuple(torch.zeros((Ec, *t.shape[1:]), device=dev, dtype=t.dtype)
                        for t in aux_like)
            st = TorchState(torch.zeros(Ec, A, 2, **opts), torch.zeros(Ec, A, **opts),
                            torch.zeros(Ec, A, 2, **opts), torch.zeros(Ec, A, **opts),
                            torch.zeros(Ec, A, **opts))
            acts = torch.zeros(horizon, Ec, A, act_dim, **opts)

            if loss_fn == "goal":  # the fused goal loss on the first auxiliary input
                fn = FusedGoalLoss(aux[0])
            else:
                def fn(final, traj: Trajectory, _aux=aux):
                    return loss_fn(final, traj, *_aux)

            g = GraphedRollout(st_i, st, acts, fn, grad_norm=False)
            loss64 = torch.zeros(1, device=dev, dtype=torch.float64)
            self.slots.append({"graph": g, "aux": aux, "loss64": loss64,
                               "ev_in": torch.cuda.Event(), "ev_done": torch.cuda.Event(),
                               "ev_out": torch.cuda.Event(), "used": False})
        self.s_in = torch.cuda.Stream(device=dev)
        self.s_run = torch.cuda.Stream(device=dev)
        self.s_out = torch.cuda.Stream(device=dev)
        self.done = torch.cuda.Event()
        self._next = 0

    def _copy(self, dst: torch.Tensor, dst_pitch: int, src: torch.Tensor, src_pitch: int,
              row_bytes: int, rows: int, src_off: int, dst_off: int, stream) -> None:
        rc = self.lib.swarp_copy_rows(dst.data_ptr() + dst_off, dst_pitch, src.data_ptr() + src_off,
                                      src_pitch, row_bytes, rows, stream.cuda_stream)
        _lib.check(rc, "swarp_copy_rows")

    def _env_slab(self, dst: torch.Tensor, src: torch.Tensor, e0: int, stream) -> None:
        """dst [Ec, ...] <- src[e0:e0+Ec] (host [E, ...], contiguous)."""
        per_env = src[0].numel() * src.element_size()
        n = per_env * self.Ec
        self._copy(dst, n, src, n, n, 1, e0 * per_env, 0, stream)

    def __call__(self, state: TorchState, actions: torch.Tensor, aux: Sequence[torch.Tensor],
                 grad_out: torch.Tensor, loss_out: torch.Tensor) -> None:
        """Enqueue one BPTT step of the whole batch (see the class docstring)."""
        H, E, A, D, Ec = self.H, self.E, self.A, self.D, self.Ec
        if tuple(actions.shape) != (H, E, A, D) or tuple(grad_out.shape) != (H, E, A, D):
            raise ValueError(f"actions and grad_out must be [{H}, {E}, {A}, {D}]")
        if loss_out.numel() < self.n_chunks or loss_out.dtype != torch.float64:
            raise ValueError(f"loss_out must hold {self.n_chunks} float64 values")
        for t in (actions, grad_out, loss_out, *tuple(state)[:5], *aux):
            if t is not None and not t.is_contiguous():
                raise ValueError("host tensors must be contiguous")
        esz = actions.element_size()
        row_full, row_chunk = E * A * D * esz, Ec * A * D * esz
        for c in range(self.n_chunks):
            s = self.slots[c if self.per_chunk else self._next % len(self.slots)]
            self._next += 1
            g: GraphedRollout = s["graph"]
            e0 = c * Ec
            # inputs: wait until the graph last run on this slot has read them
            if s["used"]:
                self.s_in.wait_event(s["ev_done"])
            self._copy(g.actions, row_chunk, actions, row_full, row_chunk, H, e0 * A * D * esz, 0,
                       self.s_in)
            for dst, src in zip(g.state[:5], tuple(state)[:5], strict=True):
                if src is not None:
                    self._env_slab(dst, src, e0, self.s_in)
            for dst, src in zip(s["aux"], aux, strict=True):
                self._env_slab(dst, src, e0, self.s_in)
            s["ev_in"].record(self.s_in)
            # the step: after its inputs, and after the last read of its outputs
            self.s_run.wait_event(s["ev_in"])
            if s["used"]:
                self.s_run.wait_event(s["ev_out"])
            with torch.cuda.stream(self.s_run):
                g.graph.replay()
                s["loss64"].copy_(g.loss.reshape(1))
            s["ev_done"].record(self.s_run)
            # outputs
            self.s_out.wait_event(s["ev_done"])
            self._copy(grad_out, row_full, g.grad_actions, row_chunk, row_chunk, H, 0,
                       e0 * A * D * esz, self.s_out)
            self._copy(loss_out, 8, s["loss64"], 8, 8, 1, 0, c * 8, self.s_out)
            s["ev_out"].record(self.s_out)
            s["used"] = True
        self.done.record(self.s_out)

    def begin(self) -> None:
        """Order the following calls after the work already on the current stream."""
        cur = torch.cuda.current_stream(self.stepper.device)
        for st in (self.s_in, self.s_run, self.s_out):
            st.wait_stream(cur)

    def end(self) -> None:
        """Order the current stream's next work after every call enqueued so far."""
        torch.cuda.current_stream(self.stepper.device).wait_event(self.done)

    def synchronize(self) -> None:
        """Wait until every enqueued step's gradient and losses are in host memory."""
        self.done.synchronize()

    def release(self) -> None:
        for s in self.slots:
            s["graph"].release()
        self.slots = []
