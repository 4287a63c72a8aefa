"""Expert-parallel exchange (moe-680m_b200/ep.py ``exchange_forward``) on CPU ranks over gloo.

The exchange logic (fixed-capacity rank blocks, all-to-all of rows and records, partial rows
returned in send layout, ordered combine) is the product code; the per-rank compute is a stand-in built on the
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
        self.x, self.resid = x, resid
        H, k1, n = shape.hidden, 2 * (shape.top_k + 1), shape.rows
        self.send_x, self.recv_x = torch.zeros(n, H), torch.zeros(n, H)
        self.send_rec = torch.full((n, k1), -1, dtype=torch.int32)
        self.recv_rec = torch.zeros(n, k1, dtype=torch.int32)
        self.yr, self.yb = torch.zeros(n, H), torch.zeros(n, H)

    def route(self, m):
        _, _, ids, w = orc.route(self.x[:m], self.m_.wr, self.m_.bias, self.sh.top_k)
        gate = 1.0 / (1.0 + np.exp(-(self.x[:m].astype(np.float64) @ self.m_.g.astype(np.float64))))
        rec = np.zeros((m, self.sh.top_k + 1, 2), np.uint32)
        rec[:, 0, 0] = self.sh.n_experts
        rec[:, 0, 1] = gate.astype(np.float32).view(np.uint32)
        rec[:, 1:, 0] = ids
        rec[:, 1:, 1] = w.view(np.uint32)
        self.rec = rec

    def dispatch(self, m):
        n, epr, cap = self.sh.n_ranks, self.sh.n_experts // self.sh.n_ranks, self.sh.capacity
        self.pairs = [[t for t in range(m) if d == self.rank or any(self.rec[t, 1:, 0] // epr == d)]
                      for d in range(n)]
        self.send_rec.fill_(-1)
        for d in range(n):
            for i, t in enumerate(self.pairs[d]):
                r = self.rec[t].copy()
                r[1:, 0] = np.where(r[1:, 0] // epr == d, r[1:, 0], NO_EXPERT)
                if d != self.rank:
                    r[0, 0] = NO_EXPERT
                self.send_x[d * cap + i] = torch.from_numpy(self.x[t])
                self.send_rec[d * cap + i] = torch.from_numpy(r.reshape(-1).view(np.int32))

    def send(self):
        return self.send_x, self.send_rec

    def recv(self):
        return self.recv_x, self.recv_rec

    def y_recv(self):
        return self.yr

    def y_back(self):
        return self.yb

    def experts(self):
        n, k = self.sh.rows, self.sh.top_k
        xr = self.recv_x.numpy().astype(np.float64)
        rec = self.recv_rec.numpy().view(np.uint32).reshape(n, k + 1, 2)
        y = np.zeros((n, self.sh.hidden))
        for i in range(n):
            for s in range(k + 1):
                e = int(rec[i, s, 0])
                if e == NO_EXPERT:
                    continue
                if s > 0:
                    assert e // (self.sh.n_experts // self.sh.n_ranks) == self.rank, "foreign expert"
                w = float(rec[i, s, 1:2].view(np.float32)[0])
                y[i] += w * orc.expert_ffn(xr[i:i + 1], *self.m_.expert(e))[0]
        self.yr[:] = torch.from_numpy(y)

    def combine(self, m, scale):
        acc = np.zeros((m, self.sh.hidden))
        back = self.yb.numpy()
        for d in range(self.sh.n_ranks):
            for i, t in enumerate(self.pairs[d]):
                acc[t] += back[d * self.sh.capacity + i]
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
        ep.exchange_forward(ops, None, m, 0.5)
        q.put((rank, ops.out if m else np.zeros((0, SH.hidden))))
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
            r, out = q.get(timeout=120)
            res[r] = out
    finally:
        for p in procs:
            if p.is_alive() and len(res) < world:
                p.kill()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    model = _Model()
    x_all, _ = _rank_tokens(world, counts)
    ref = orc.moe_forward(x_all, x_all, model.wr, model.bias, model.g, 0.5, model.expert,
                          SH.n_experts, SH.top_k)["out"]
    got = np.concatenate([res[r] for r in range(world)])
    assert got.shape == ref.shape
    # partial rows travel as f32: agreement to f32 rounding of the partial sums
    assert orc.rel_l2(got, ref) < 1e-6


def test_bench_ep_exchange_bytes():
    """The NVLink byte count the bench's expert-parallel roofline uses, on a hand-checked case:
    2 ranks, 4 experts each, 2 tokens per rank, top-2."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parent.parent / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    routed = np.array([[0, 1],    # rank 0 token: own experts only
                       [2, 5],    # rank 0 token: visits rank 1
                       [6, 7],    # rank 1 token: own experts only
                       [0, 4]])   # rank 1 token: visits rank 0
    b = bench.ep_exchange_bytes(routed, world=2, m=2, epr=4, hidden=8, k=2)
    row_in, row_back = 8 * 4 + 3 * 8, 8 * 4
    assert b.tolist() == [[row_in + row_back, row_in + row_back], [row_in + row_back, row_in + row_back]]
    routed[3] = [6, 7]  # now only rank 0 sends
    b = bench.ep_exchange_bytes(routed, world=2, m=2, epr=4, hidden=8, k=2)
    assert b.tolist() == [[row_in, row_back], [row_back, row_in]]
