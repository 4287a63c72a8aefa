"""Expert-parallel prefill over torch.distributed: the exchange around the library's kernels.

Rank d of N holds routed experts [d*E/N, (d+1)*E/N) plus a replica of the router and of the
shared expert, and its own M_d tokens.  One layer forward (the exchange steps of the
expert-parallel layout; the single-device reference, src/inference.rs:663-766, has no
counterpart):

  1. route the local tokens (f32 router, softmax, top-k: every rank routes with the full router);
  2. dispatch plan: one (token, destination rank) pair per rank a token visits, rank-major,
     token order inside a rank; per-destination pair counts;
  3. all-to-all of the counts, then of the pair rows (f32, exact) and of their routing records
     (only the destination's experts kept);
  4. the rank's experts on the rows it received -> one partial row per received pair
     (sum of w_j E_j(x) over its experts, unscaled);
  5. all-to-all of the partial rows back to their owners (same splits, reversed);
  6. the shared expert on the local tokens, then out = resid + scale * (sum of the returned
     partials in rank order + gate * S(x)).

The per-rank compute goes through an ``ops`` object: ``LibraryEpOps`` (the CUDA library,
tensors aliasing the context's arena) is the product; a test stand-in with the same methods can
drive the same exchange on CPU ranks over gloo.
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
    max_tokens: int  # per rank
    has_shared: bool = True

    @property
    def max_pairs(self) -> int:  # rows one rank can send
        return self.max_tokens * min(self.top_k, self.n_ranks)

    @property
    def max_recv(self) -> int:  # rows one rank can receive
        return self.max_tokens * self.n_ranks


def exchange_forward(ops, group, m: int, scale: float):
    """Runs steps 1-6 for the m local tokens held by ``ops`` (see the module docstring).

    ``ops`` provides: route(m), dispatch(m) -> send counts, recv_views(n_rows) -> (x, rec)
    tensors to receive into, send_views(n_rows) -> (x, rec) tensors to send, experts(n_rows),
    y_recv_view(n_rows), y_back_view(n_rows), shared(m), combine(m, scale) and ``device``."""
    n = dist.get_world_size(group)
    ops.route(m)
    send_counts = ops.dispatch(m)
    sc = torch.tensor(send_counts, dtype=torch.int64, device=ops.device)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    recv_counts = [int(v) for v in rc.tolist()]
    n_send, n_recv = sum(send_counts), sum(recv_counts)
    sx, srec = ops.send_views(n_send)
    rx, rrec = ops.recv_views(n_recv)
    dist.all_to_all_single(rx, sx, recv_counts, send_counts, group=group)
    dist.all_to_all_single(rrec, srec, recv_counts, send_counts, group=group)
    ops.experts(n_recv)
    dist.all_to_all_single(ops.y_back_view(n_send), ops.y_recv_view(n_recv), send_counts,
                           recv_counts, group=group)
    ops.shared(m)
    ops.combine(m, scale)
    assert len(send_counts) == n
    return send_counts, recv_counts


class LibraryEpOps:
    """Per-rank compute of the exchange through libmoe_b200, on buffers in the context's arena.

    The arena is a torch uint8 tensor (``arena``) wrapped by ``ctx`` (moe_ctx_create_external),
    so the collectives run directly on arena memory; the context's stream is set to torch's
    current stream, so library kernels and NCCL collectives are ordered on one stream."""

    def __init__(self, ctx: host.Context, arena: torch.Tensor, layer_id: int, shape: EpShape,
                 x_off: int, resid_off: int, out_off: int):
        self.ctx, self.arena, self.layer, self.sh = ctx, arena, layer_id, shape
        self.device = arena.device
        self.x_off, self.resid_off, self.out_off = x_off, resid_off, out_off
        H, k = shape.hidden, shape.top_k
        rec = (k + 1) * 8
        self.topk = ctx.alloc(shape.max_tokens * rec)
        self.plan = ctx.alloc(int(host.lib().moe_ep_plan_bytes(shape.max_tokens, shape.n_ranks)))
        self.send_x = ctx.alloc(shape.max_pairs * H * 4)
        self.send_rec = ctx.alloc(shape.max_pairs * rec)
        self.recv_x = ctx.alloc(shape.max_recv * H * 4)
        self.recv_rec = ctx.alloc(shape.max_recv * rec)
        self.y_recv = ctx.alloc(shape.max_recv * H * 4)
        self.y_back = ctx.alloc(shape.max_pairs * H * 4)
        self.shared_y = ctx.alloc(shape.max_tokens * H * 4)
        ctx.reserve(layer_id, shape.max_recv)
        ctx.sync()  # work issued so far on the context's previous stream
        ctx.set_stream(torch.cuda.current_stream(self.device).cuda_stream)

    def _rows(self, off: int, n: int, width: int, dtype) -> torch.Tensor:
        esz = torch.empty((), dtype=dtype).element_size()
        return self.arena[off: off + max(n, 1) * width * esz].view(dtype).view(max(n, 1), width)[:n]

    def route(self, m):
        self.ctx.route(self.layer, self.x_off, m, self.topk)

    def dispatch(self, m):
        sh = self.sh
        return self.ctx.ep_dispatch(sh.n_experts, sh.top_k, sh.n_ranks, self.topk, self.x_off, m,
                                    sh.hidden, self.plan, self.send_x, self.send_rec)

    def send_views(self, n):
        k1 = 2 * (self.sh.top_k + 1)
        return (self._rows(self.send_x, n, self.sh.hidden, torch.float32),
                self._rows(self.send_rec, n, k1, torch.int32))

    def recv_views(self, n):
        k1 = 2 * (self.sh.top_k + 1)
        return (self._rows(self.recv_x, n, self.sh.hidden, torch.float32),
                self._rows(self.recv_rec, n, k1, torch.int32))

    def y_recv_view(self, n):
        return self._rows(self.y_recv, n, self.sh.hidden, torch.float32)

    def y_back_view(self, n):
        return self._rows(self.y_back, n, self.sh.hidden, torch.float32)

    def experts(self, n):
        if n:
            self.ctx.forward_topk(self.layer, self.recv_x, 0, self.y_recv, n, self.recv_rec,
                                  host.MOE_FT_NO_SHARED | host.MOE_FT_UNSCALED)

    def shared(self, m):
        if self.sh.has_shared:
            self.ctx.forward_topk(self.layer, self.x_off, 0, self.shared_y, m, self.topk,
                                  host.MOE_FT_SHARED_ONLY | host.MOE_FT_UNSCALED)

    def combine(self, m, scale):
        self.ctx.ep_combine(self.sh.n_ranks, self.sh.hidden, m, self.plan, self.y_back,
                            self.shared_y if self.sh.has_shared else 0, self.resid_off, self.out_off,
                            scale)
