"""Expert-parallel exchange (moe-680m_b200/ep.py ``exchange_forward``) on CPU ranks over gloo.

The exchange logic (count all-to-all, rank-major dispatch, partial rows returned in send
order, ordered combine) is the product code; the per-rank compute is a stand-in built on the
oracle, so these tests need no GPU.  World sizes 2 and 4, uneven token counts per rank
(including a rank with no tokens); the result must equal the single-process oracle layer.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import conftest  # noqa: F401  (registers the package for spawned ranks too)
import moe_oracle as orc
from moe680m_b200 import ep, synth

SEED = 4242
SH = synth.LayerShapes(hidden=256, inter=256, n_experts=8, top_k=3, shared_inter=256)
NO_EXPERT = 0xFFFFFFFF


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Model:
    def __init__(self):
        self.wr, self.g, self.bias = synth.float_tensors(SEED, 0, SH, 1.1)
        self.cache = {}

    def expert(self, e):
        if e not in self.cache:
            w1, w3, w2 = synth.expert_weights(SEED, 0, e, SH)
            self.cache[e] = (orc.dequant_matrix(w1, SH.inter, SH.hidden),
                             orc.dequant_matrix(w3, SH.inter, SH.hidden),
                             orc.dequant_matrix(w2, SH.hidden, SH.inter))
        return self.cache[e]


class OracleEpOps:
    """Stand-in per-rank compute with LibraryEpOps' interface (f64 oracle, CPU tensors)."""

    def __init__(self, model, shape: ep.EpShape, rank: int, x: np.ndarray, resid: np.ndarray):
        self.m_, self.sh, self.rank = model, shape, rank
        self.device = torch.device("cpu")
        self.x, self.resid = x, resid
        H, k1 = shape.hidden, 2 * (shape.top_k + 1)
        self.send_x = torch.zeros(shape.max_pairs, H)
        self.send_rec = torch.zeros(shape.max_pairs, k1, dtype=torch.int32)
        self.recv_x = torch.zeros(shape.max_recv, H)
        self.recv_rec = torch.zeros(shape.max_recv, k1, dtype=torch.int32)
        self.y_recv = torch.zeros(shape.max_recv, H)
        self.y_back = torch.zeros(shape.max_pairs, H)

    def route(self, m):
        _, _, ids, w = orc.route(self.x[:m], self.m_.wr, self.m_.bias, self.sh.top_k)
        gate = 1.0 / (1.0 + np.exp(-(self.x[:m].astype(np.float64) @ self.m_.g.astype(np.float64))))
        rec = np.zeros((m, self.sh.top_k + 1, 2), np.uint32)
        rec[:, 0, 0] = self.sh.n_experts
        rec[:, 0, 1] = gate.astype(np.float32).view(np.uint32)
        rec[:, 1:, 0] = ids
        rec[:, 1:, 1] = w.view(np.uint32)
        self.rec, self.gate = rec, gate

    def dispatch(self, m):
        n, epr = self.sh.n_ranks, self.sh.n_experts // self.sh.n_ranks
        self.pairs = [[t for t in range(m) if any(self.rec[t, 1:, 0] // epr == d)] for d in range(n)]
        p = 0
        for d in range(n):
            for t in self.pairs[d]:
                r = self.rec[t].copy()
                keep = r[1:, 0] // epr == d
                r[1:, 0] = np.where(keep, r[1:, 0], NO_EXPERT)
                self.send_x[p] = torch.from_numpy(self.x[t])
                self.send_rec[p] = torch.from_numpy(r.reshape(-1).view(np.int32))
                p += 1
        return [len(v) for v in self.pairs]

    def send_views(self, n):
        return self.send_x[:n], self.send_rec[:n]

    def recv_views(self, n):
        return self.recv_x[:n], self.recv_rec[:n]

    def y_recv_view(self, n):
        return self.y_recv[:n]

    def y_back_view(self, n):
        return self.y_back[:n]

    def experts(self, n):
        xr = self.recv_x[:n].numpy().astype(np.float64)
        rec = self.recv_rec[:n].numpy().view(np.uint32).reshape(n, self.sh.top_k + 1, 2)
        y = np.zeros((n, self.sh.hidden))
        for i in range(n):
            for s in range(1, self.sh.top_k + 1):
                e = int(rec[i, s, 0])
                if e == NO_EXPERT:
                    continue
                assert e // (self.sh.n_experts // self.sh.n_ranks) == self.rank, "foreign expert"
                w = float(rec[i, s, 1:2].view(np.float32)[0])
                y[i] += w * orc.expert_ffn(xr[i:i + 1], *self.m_.expert(e))[0]
        self.y_recv[:n] = torch.from_numpy(y)

    def shared(self, m):
        self.shared_y = self.gate[:, None] * orc.expert_ffn(self.x[:m].astype(np.float64),
                                                           *self.m_.expert(self.sh.n_experts))

    def combine(self, m, scale):
        acc = self.shared_y.copy()
        p = 0
        back = self.y_back.numpy()
        for d in range(self.sh.n_ranks):
            for t in self.pairs[d]:
                acc[t] += back[p]
                p += 1
        self.out = self.resid[:m].astype(np.float64) + scale * acc


def _rank_tokens(world, counts):
    x_all = synth.tokens(SEED, 0, sum(counts), SH.hidden)
    starts = np.cumsum([0] + counts)
    return x_all, [x_all[starts[r]:starts[r + 1]] for r in range(world)]


def _worker(rank, world, port, counts, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _Model()
        _, parts = _rank_tokens(world, counts)
        x = parts[rank]
        m = x.shape[0]
        shape = ep.EpShape(SH.hidden, SH.n_experts, SH.top_k, world, max(max(counts), 1))
        ops = OracleEpOps(model, shape, rank, x, x)
        sent, recv = ep.exchange_forward(ops, None, m, 0.5)
        q.put((rank, ops.out if m else np.zeros((0, SH.hidden)), sent, recv))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,counts", [(2, [7, 5]), (4, [6, 0, 9, 3])])
def test_exchange_matches_single_process(world, counts):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, counts, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out, sent, recv = q.get(timeout=120)
            res[r] = (out, sent, recv)
    finally:
        for p in procs:
            if p.is_alive() and len(res) < world:
                p.kill()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # counts are consistent: what r sent to d is what d received from r
    for r in range(world):
        for d in range(world):
            assert res[r][1][d] == res[d][2][r]
    model = _Model()
    x_all, _ = _rank_tokens(world, counts)
    ref = orc.moe_forward(x_all, x_all, model.wr, model.bias, model.g, 0.5, model.expert,
                          SH.n_experts, SH.top_k)["out"]
    got = np.concatenate([res[r][0] for r in range(world)])
    assert got.shape == ref.shape
    # partial rows travel as f32: agreement to f32 rounding of the partial sums
    assert orc.rel_l2(got, ref) < 1e-6
