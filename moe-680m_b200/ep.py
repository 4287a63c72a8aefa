"""Expert-parallel prefill over torch.distributed: the exchange around the library's kernels.

Rank r of N holds routed experts [r*E/N, (r+1)*E/N) plus replicas of the router and of the
shared expert, and its own M_r tokens.  One layer forward (the exchange steps of the
expert-parallel layout; the single-device reference, src/inference.rs:663-766, has no
counterpart):

  1. route the local tokens (f32 router, softmax, top-k: every rank routes with the full router);
  2. dispatch: for each destination rank d, a block of ``capacity`` rows holding, in token
     order, the tokens with at least one expert on d (every token in the rank's own block, which
     also carries the shared expert), each with its routing record reduced to d's experts;
  3. all-to-all of the blocks (f32 rows, exact, and records): fixed equal splits, so no counts
     are exchanged and nothing waits on the host;
  4. the rank's experts on the N*capacity rows it received (padding rows have empty records and
     cost nothing) -> one partial row per received row, sum of w_j E_j(x), unscaled;
  5. all-to-all of the partial rows back to their owners (same layout);
  6. out = resid + scale * (sum of the returned partials in rank order).

This module runs the exchange with the caller's own process group, for callers that already
have one; the library runs the same steps by itself in ``moe_forward_ep`` (its own NCCL group,
or stores and loads over NVLink peer memory).  The per-rank compute goes through an ``ops``
object: ``LibraryEpOps`` (the CUDA library, tensors aliasing the context's arena); a test
stand-in with the same methods drives the same exchange on CPU ranks over gloo.  With no host
synchronisation inside, a step of LibraryEpOps can be captured in a CUDA graph together with
the NCCL collectives.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import host


@dataclass
class EpShape:
    hidden: int
    n_experts: int
    top_k: int
    n_ranks: int
    capacity: int  # rows per destination block >= the largest per-rank token count

    @property
    def rows(self) -> int:  # rows of the send (and of the receive) buffer
        return self.capacity * self.n_ranks


def exchange_forward(ops, group, m: int, scale: float):
    """Runs steps 1-6 for the m local tokens held by ``ops`` (see the module docstring).

    ``ops`` provides route(m), dispatch(m), send() / recv() -> (x rows, record rows) tensors of
    ``rows`` rows, experts(), y_recv() / y_back() -> partial-row tensors, and combine(m, scale).
    An ops object with a ``stream`` (a torch CUDA stream) runs the step on it, ordered after the
    caller's current stream and before the caller's later work."""
    s = getattr(ops, "stream", None)
    if s is None:
        return _exchange(ops, group, m, scale)
    caller = torch.cuda.current_stream(s.device)
    s.wait_stream(caller)
    with torch.cuda.stream(s):
        _exchange(ops, group, m, scale)
    caller.wait_stream(s)


def _exchange(ops, group, m, scale):
    ops.route(m)
    ops.dispatch(m)
    sx, srec = ops.send()
    rx, rrec = ops.recv()
    dist.all_to_all_single(rx, sx, group=group)
    dist.all_to_all_single(rrec, srec, group=group)
    ops.experts()
    dist.all_to_all_single(ops.y_back(), ops.y_recv(), group=group)
    ops.combine(m, scale)


class LibraryEpOps:
    """Per-rank compute of the exchange through libmoe_b200, on buffers in the context's arena.

    The arena is a torch uint8 tensor (``arena``) wrapped by ``ctx`` (moe_ctx_create_external),
    so the collectives run directly on arena memory.  Library kernels and NCCL collectives are
    ordered on one stream: torch's current stream at construction, or a new stream when that is
    the legacy default stream (the library treats a NULL stream as its own private stream)."""

    def __init__(self, ctx: host.Context, arena: torch.Tensor, layer_id: int, shape: EpShape, rank: int,
                 x_off: int, resid_off: int, out_off: int):
        self.ctx, self.arena, self.layer, self.sh, self.rank = ctx, arena, layer_id, shape, rank
        self.device = arena.device
        self.x_off, self.resid_off, self.out_off = x_off, resid_off, out_off
        H, k = shape.hidden, shape.top_k
        rec = (k + 1) * 8
        self.topk = ctx.alloc(shape.capacity * rec)
        self.plan = ctx.alloc(int(host.lib().moe_ep_plan_bytes(shape.capacity, shape.n_ranks)))
        self.send_x = ctx.alloc(shape.rows * H * 4)
        self.send_rec = ctx.alloc(shape.rows * rec)
        self.recv_x = ctx.alloc(shape.rows * H * 4)
        self.recv_rec = ctx.alloc(shape.rows * rec)
        self.yr_off = ctx.alloc(shape.rows * H * 4)
        self.yb_off = ctx.alloc(shape.rows * H * 4)
        ctx.reserve(layer_id, shape.rows)
        ctx.sync()  # work issued so far on the context's previous stream
        cur = torch.cuda.current_stream(self.device)
        self.stream = cur if cur.cuda_stream else torch.cuda.Stream(self.device)
        ctx.set_stream(self.stream.cuda_stream)

    def _view(self, off: int, width: int, dtype) -> torch.Tensor:
        n = self.sh.rows
        esz = torch.empty((), dtype=dtype).element_size()
        return self.arena[off: off + n * width * esz].view(dtype).view(n, width)

    def route(self, m):
        if m:
            self.ctx.route(self.layer, self.x_off, m, self.topk)

    def dispatch(self, m):
        sh = self.sh
        self.ctx.ep_dispatch(sh.n_experts, sh.top_k, sh.n_ranks, self.rank, sh.capacity, self.topk,
                             self.x_off, m, sh.hidden, self.plan, self.send_x, self.send_rec)

    def send(self):
        return (self._view(self.send_x, self.sh.hidden, torch.float32),
                self._view(self.send_rec, 2 * (self.sh.top_k + 1), torch.int32))

    def recv(self):
        return (self._view(self.recv_x, self.sh.hidden, torch.float32),
                self._view(self.recv_rec, 2 * (self.sh.top_k + 1), torch.int32))

    def y_recv(self):
        return self._view(self.yr_off, self.sh.hidden, torch.float32)

    def y_back(self):
        return self._view(self.yb_off, self.sh.hidden, torch.float32)

    def experts(self):
        self.ctx.forward_topk(self.layer, self.recv_x, 0, self.yr_off, self.sh.rows, self.recv_rec,
                              host.MOE_FT_UNSCALED)

    def combine(self, m, scale):
        self.ctx.ep_combine(self.sh.n_ranks, self.sh.capacity, self.sh.hidden, m, self.plan, self.yb_off,
                            self.resid_off, self.out_off, scale)


class CapturedExchange:
    """One layer step of ``exchange_forward`` captured in a CUDA graph (library kernels and
    NCCL collectives), replayed with ``replay()``: no per-step host work beyond one launch.
    The captured step reads its tokens at ``ops.x_off`` and writes ``ops.out_off``; callers
    copy new tokens there between replays.  Run one eager step first (the library caches its
    tensor maps and workspace on first use; nothing may allocate during capture)."""

    def __init__(self, ops: LibraryEpOps, group, m: int, scale: float):
        self.ops = ops
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(ops.device)
        with torch.cuda.graph(self.graph, stream=ops.stream):
            _exchange(ops, group, m, scale)
        torch.cuda.synchronize(ops.device)

    def replay(self):
        caller = torch.cuda.current_stream(self.ops.device)
        self.ops.stream.wait_stream(caller)
        with torch.cuda.stream(self.ops.stream):
            self.graph.replay()
        caller.wait_stream(self.ops.stream)
