"""GPU tests of the expert-parallel building blocks (all through the C ABI) and of the
expert-parallel layer over NCCL.

* moe_forward_topk: flags 0 equals moe_forward bit for bit on the same routing; the partial
  (routed only, unscaled) plus the shared-only part, scaled, plus the residual equals it to f32
  rounding; empty routed entries (MOE_NO_EXPERT) are skipped (checked against the oracle).
* moe_ep_dispatch: the rank blocks (rows, reduced records, empty padding) equal a NumPy
  restatement exactly.
* one-rank expert-parallel layer (an NCCL group of 1): equals moe_forward to f32 rounding and
  the f64 oracle to the layer tolerance.
* two ranks on two GPUs (skipped with fewer GPUs): each rank's output equals the single-GPU
  layer on the same tokens to f32 rounding.
"""
import os
import socket

import numpy as np
import pytest
import torch

import coracle
import conftest  # noqa: F401  (registers the package for spawned ranks too)
import moe_oracle as O
from moe680m_b200 import ep, host, synth

pytestmark = pytest.mark.gpu

FULL = synth.LayerShapes(2048, 512, 256, 8, 512)
SEED = 777


@pytest.fixture(scope="module")
def full():
    ctx = host.Context(0, 2 << 30)
    _, _, ids = host.build_synthetic_model(ctx, SEED, 1, FULL, 1.1)
    yield ctx, ids[0]
    ctx.close()


def _route(ctx, lid, x):
    m = x.shape[0]
    xo = ctx.put(x)
    topk = ctx.alloc(m * 9 * 8)
    ctx.route(lid, xo, m, topk)
    return xo, topk


@pytest.mark.parametrize("m", [37, 300])
def test_forward_topk_matches_forward(full, m):
    ctx, lid = full
    x = synth.tokens(SEED, m, m, FULL.hidden)
    xo, topk = _route(ctx, lid, x)
    ref_o, a_o, p_o, s_o = (ctx.alloc(x.nbytes) for _ in range(4))
    ctx.forward(lid, xo, xo, ref_o, m)
    ctx.forward_topk(lid, xo, xo, a_o, m, topk, 0)
    ctx.forward_topk(lid, xo, 0, p_o, m, topk, host.MOE_FT_NO_SHARED | host.MOE_FT_UNSCALED)
    ctx.forward_topk(lid, xo, 0, s_o, m, topk, host.MOE_FT_SHARED_ONLY | host.MOE_FT_UNSCALED)
    ctx.sync()
    ref = ctx.download(ref_o, (m, FULL.hidden))
    assert np.array_equal(ctx.download(a_o, (m, FULL.hidden)).view(np.uint32), ref.view(np.uint32))
    parts = ctx.download(p_o, (m, FULL.hidden)).astype(np.float64) + ctx.download(s_o, (m, FULL.hidden))
    assert O.rel_l2(x.astype(np.float64) + parts, ref) < 1e-6


def test_forward_topk_empty_slots(full):
    ctx, lid = full
    m = 50
    x = synth.tokens(SEED, 5, m, FULL.hidden)
    xo, topk = _route(ctx, lid, x)
    rec = ctx.download(topk, (m, 9, 2), np.uint32)
    rng = np.random.default_rng(1)
    drop = rng.random((m, 8)) < 0.5
    rec[:, 1:, 0] = np.where(drop, host.MOE_NO_EXPERT, rec[:, 1:, 0])
    ctx.upload(topk, rec)
    out = ctx.alloc(x.nbytes)
    ctx.forward_topk(lid, xo, 0, out, m, topk, host.MOE_FT_NO_SHARED)
    ctx.sync()
    got = ctx.download(out, (m, FULL.hidden))
    hl = coracle.synthetic_layer(SEED, 0, FULL, 1.1)
    ref = np.zeros((m, FULL.hidden))
    x64 = x.astype(np.float64)
    for t in range(m):
        for s in range(8):
            e = int(rec[t, 1 + s, 0])
            if e == host.MOE_NO_EXPERT:
                continue
            w = float(rec[t, 1 + s, 1:2].view(np.float32)[0])
            ws = [O.dequant_matrix(raw, r, c) for raw, r, c in
                  zip(hl.experts[e], (512, 512, 2048), (2048, 2048, 512))]
            ref[t] += w * O.expert_ffn(x64[t:t + 1], *ws)[0]
    assert O.rel_l2(got, ref) <= 1e-3


@pytest.mark.parametrize("n_ranks,my_rank", [(1, 0), (2, 1), (4, 2), (8, 7)])
def test_ep_dispatch_exact(full, n_ranks, my_rank):
    ctx, lid = full
    m, H, k, E = 300, FULL.hidden, 8, 256
    cap = 320
    x = synth.tokens(SEED, 9, m, H)
    xo, topk = _route(ctx, lid, x)
    rec = ctx.download(topk, (m, k + 1, 2), np.uint32)
    plan = ctx.alloc(int(host.lib().moe_ep_plan_bytes(m, n_ranks)))
    rows = n_ranks * cap
    sx, sr = ctx.alloc(rows * H * 4), ctx.alloc(rows * (k + 1) * 8)
    ctx.ep_dispatch(E, k, n_ranks, my_rank, cap, topk, xo, m, H, plan, sx, sr)
    ctx.sync()
    got_x = ctx.download(sx, (rows, H))
    got_r = ctx.download(sr, (rows, k + 1, 2), np.uint32)
    epr = E // n_ranks
    for d in range(n_ranks):
        toks = [t for t in range(m) if d == my_rank or np.any(rec[t, 1:, 0] // epr == d)]
        for i, t in enumerate(toks):
            assert np.array_equal(got_x[d * cap + i], x[t])
            r = rec[t].copy()
            r[1:, 0] = np.where(r[1:, 0] // epr == d, r[1:, 0], host.MOE_NO_EXPERT)
            if d != my_rank:
                r[0, 0] = host.MOE_NO_EXPERT
            assert np.array_equal(got_r[d * cap + i], r)
        assert (got_r[d * cap + len(toks):(d + 1) * cap, :, 0] == host.MOE_NO_EXPERT).all()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_rank_forward(rank, world, tokens_per_rank, seed):
    """Builds this rank's expert subset and runs one expert-parallel forward of its tokens."""
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    E, H = FULL.n_experts, FULL.hidden
    epr = E // world
    m_max = max(tokens_per_rank)
    arena_bytes = 1 << 30
    arena = torch.empty(arena_bytes, dtype=torch.uint8, device=dev)
    ctx = host.Context(rank, arena_bytes, external_ptr=arena.data_ptr())
    _, _, ids = host.build_synthetic_model(ctx, seed, 1, FULL, 1.1, experts=range(rank * epr, (rank + 1) * epr))
    m = tokens_per_rank[rank]
    x_all = synth.tokens(seed, 1, sum(tokens_per_rank), H)
    start = sum(tokens_per_rank[:rank])
    x = x_all[start:start + m]
    xo = ctx.put(x if m else np.zeros((1, H), np.float32))
    out = ctx.alloc(max(m, 1) * H * 4)
    ops = ep.LibraryEpOps(ctx, arena, ids[0], ep.EpShape(H, E, FULL.top_k, world, m_max), rank, xo, xo, out)
    for _ in range(2):  # a second step checks that reused buffers hold nothing stale
        ep.exchange_forward(ops, None, m, 1.0)
    torch.cuda.synchronize(dev)
    ctx.sync()
    got = ctx.download(out, (m, H)) if m else np.zeros((0, H), np.float32)
    ctx.close()
    del arena
    dist.barrier()
    return x, got


def _ep_worker(rank, world, port, tokens_per_rank, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        x, got = _ep_rank_forward(rank, world, tokens_per_rank, SEED)
        q.put((rank, x, got))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _run_ranks(world, tokens_per_rank):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, tokens_per_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, x, got = q.get(timeout=300)
            assert x is not None, f"rank {r}: {got}"
            res[r] = (x, got)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


def _single_gpu_reference(x):
    ctx = host.Context(0, 2 << 30)
    try:
        _, _, ids = host.build_synthetic_model(ctx, SEED, 1, FULL, 1.1)
        xo = ctx.put(x)
        out = ctx.alloc(x.nbytes)
        ctx.forward(ids[0], xo, xo, out, x.shape[0])
        ctx.sync()
        return ctx.download(out, x.shape)
    finally:
        ctx.close()


def test_ep_one_rank_matches_forward():
    res = _run_ranks(1, [260])
    x, got = res[0]
    ref = _single_gpu_reference(x)
    assert O.rel_l2(got, ref) < 1e-6
    hl = coracle.synthetic_layer(SEED, 0, FULL, 1.1)
    oref = coracle.moe_forward(hl, x, x)["out64"]
    assert O.rel_l2(got, oref) <= 1e-3


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_ranks_match_single_gpu():
    res = _run_ranks(2, [300, 212])
    x = np.concatenate([res[0][0], res[1][0]])
    got = np.concatenate([res[0][1], res[1][1]])
    ref = _single_gpu_reference(x)
    assert O.rel_l2(got, ref) < 1e-6


# ---- the C-level expert-parallel layer (moe_ep_init / moe_forward_ep, NCCL inside the library) --

@pytest.mark.parametrize("transport", [host.MOE_EP_TRANSPORT_PEER, host.MOE_EP_TRANSPORT_NCCL])
def test_c_abi_ep_one_rank(full, transport):
    ctx, lid = full
    ctx.ep_set_transport(transport)
    ctx.ep_init(host.Context.ep_unique_id(), 1, 0)
    m = 260
    x = synth.tokens(SEED, 5, m, FULL.hidden)
    xo = ctx.put(x)
    ref_o, ep_o = ctx.alloc(x.nbytes), ctx.alloc(x.nbytes)
    ctx.forward(lid, xo, xo, ref_o, m)
    for cap in (m, 300, 300):  # a larger capacity regrows the exchange buffers; then a reuse
        ctx.forward_ep(lid, xo, xo, ep_o, m, cap)
        ctx.sync()
        got = ctx.download(ep_o, (m, FULL.hidden))
        assert O.rel_l2(got, ctx.download(ref_o, (m, FULL.hidden))) < 1e-6
    assert ctx.ep_transport() == transport
    ctx.forward_ep(lid, xo, xo, ep_o, 0, 8)  # a rank without tokens still takes part
    ctx.sync()
    with pytest.raises(host.MoeError):
        ctx.forward_ep(lid, xo, xo, ep_o, m, m - 1)  # capacity below the local tokens


def _c_ep_worker(rank, world, uid, tokens_per_rank, transport, q):
    try:
        E, H = FULL.n_experts, FULL.hidden
        epr = E // world
        ctx = host.Context(rank, 1 << 30)
        _, _, ids = host.build_synthetic_model(ctx, SEED, 1, FULL, 1.1, experts=range(rank * epr, (rank + 1) * epr))
        ctx.ep_set_transport(transport)
        ctx.ep_init(uid, world, rank)
        m = tokens_per_rank[rank]
        x_all = synth.tokens(SEED, 1, sum(tokens_per_rank), H)
        start = sum(tokens_per_rank[:rank])
        x = x_all[start:start + m]
        xo = ctx.put(x if m else np.zeros((1, H), np.float32))
        out = ctx.alloc(max(m, 1) * H * 4)
        for _ in range(3):  # later steps reuse the exchange buffers and step flags
            ctx.forward_ep(ids[0], xo, xo, out, m, max(tokens_per_rank))
        ctx.sync()
        got = ctx.download(out, (m, H)) if m else np.zeros((0, H), np.float32)
        used = ctx.ep_transport()
        ctx.close()
        q.put((rank, x, (got, used)))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("transport,tpr", [(host.MOE_EP_TRANSPORT_PEER, [300, 212]),
                                           (host.MOE_EP_TRANSPORT_PEER, [0, 97]),
                                           (host.MOE_EP_TRANSPORT_NCCL, [300, 212])])
def test_c_abi_ep_two_ranks_match_single_gpu(transport, tpr):
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    world = 2
    uid = host.Context.ep_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_c_ep_worker, args=(r, world, uid, tpr, transport, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, x, got = q.get(timeout=300)
            assert x is not None, f"rank {r}: {got}"
            res[r] = (x, got)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[0][1][1] == transport and res[1][1][1] == transport
    x = np.concatenate([res[0][0], res[1][0]])
    got = np.concatenate([res[0][1][0], res[1][1][0]])
    assert O.rel_l2(got, _single_gpu_reference(x)) < 1e-6


def _c_ep_mismatch_worker(rank, world, uid, caps, q):
    try:
        E, H = FULL.n_experts, FULL.hidden
        epr = E // world
        ctx = host.Context(rank, 1 << 30)
        _, _, ids = host.build_synthetic_model(ctx, SEED, 1, FULL, 1.1, experts=range(rank * epr, (rank + 1) * epr))
        ctx.ep_init(uid, world, rank)
        xo = ctx.put(synth.tokens(SEED, 9, 8, H))
        out = ctx.alloc(8 * H * 4)
        try:
            ctx.forward_ep(ids[0], xo, xo, out, 8, caps[rank])
            q.put((rank, "no error"))
        except host.MoeError as e:
            q.put((rank, str(e)))
        ctx.close()
    except Exception as e:  # reported to the parent
        q.put((rank, "worker failed: " + repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_c_abi_ep_two_ranks_reject_different_capacities():
    """Ranks that pass different capacities get an error on every rank, before any exchange."""
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    uid = host.Context.ep_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_c_ep_mismatch_worker, args=(r, 2, uid, [64, 96], q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, msg = q.get(timeout=300)
            res[r] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all("disagree" in m for m in res.values()), res


def test_c_abi_ep_abort_one_rank(full):
    """moe_ep_abort ends the group: later moe_forward_ep calls fail; a new moe_ep_init recovers."""
    ctx, lid = full
    ctx.ep_init(host.Context.ep_unique_id(), 1, 0)
    m = 64
    x = synth.tokens(SEED, 6, m, FULL.hidden)
    xo = ctx.put(x)
    ref_o, ep_o = ctx.alloc(x.nbytes), ctx.alloc(x.nbytes)
    ctx.forward(lid, xo, xo, ref_o, m)
    ctx.forward_ep(lid, xo, xo, ep_o, m, m)
    ctx.sync()
    ctx.ep_abort()
    ctx.ep_abort()  # idempotent
    with pytest.raises(host.MoeError):
        ctx.forward_ep(lid, xo, xo, ep_o, m, m)
    ctx.ep_init(host.Context.ep_unique_id(), 1, 0)
    ctx.forward_ep(lid, xo, xo, ep_o, m, m)
    ctx.sync()
    assert O.rel_l2(ctx.download(ep_o, (m, FULL.hidden)), ctx.download(ref_o, (m, FULL.hidden))) < 1e-6


def _c_ep_bad_rank_worker(rank, world, uid, m, cap, q):
    try:
        E, H = FULL.n_experts, FULL.hidden
        epr = E // world
        ctx = host.Context(rank, 1 << 30)
        _, _, ids = host.build_synthetic_model(ctx, SEED, 1, FULL, 1.1, experts=range(rank * epr, (rank + 1) * epr))
        ctx.ep_init(uid, world, rank)
        x = synth.tokens(SEED, 11 + rank, m, H)
        xo = ctx.put(x)
        out = ctx.alloc(m * H * 4)
        try:
            # rank 1 passes more tokens than the capacity: it must fail without stalling rank 0
            ctx.forward_ep(ids[0], xo, xo, out, m if rank == 0 else cap + 5, cap)
            ctx.sync()
            q.put((rank, x, ctx.download(out, (m, H))))
        except host.MoeError as e:
            q.put((rank, None, str(e)))
        ctx.close()
    except Exception as e:  # reported to the parent
        q.put((rank, None, "worker failed: " + repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_c_abi_ep_bad_rank_does_not_stall_the_group():
    """A rank with invalid token arguments reports its error; the other rank's step completes
    with results equal to the single-GPU layer (the bad rank served its experts)."""
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    uid = host.Context.ep_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_c_ep_bad_rank_worker, args=(r, 2, uid, 96, 128, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, x, got = q.get(timeout=300)
            res[r] = (x, got)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[1][0] is None and "capacity" in res[1][1], res[1]
    x0, got0 = res[0]
    assert x0 is not None, got0
    assert O.rel_l2(got0, _single_gpu_reference(x0)) < 1e-6
