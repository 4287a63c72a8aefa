"""GPU parity tests: every call goes through the C ABI (libmoe_b200.so via ctypes) and is
checked against the CPU oracle (oracle/) on the same seeded inputs.

Tolerances (the contract's): top-k expert ids exact (ties to the lower index) except tokens whose
k-th/(k+1)-th logits are within 1e-5 (reported, expected none); decoded weights bit-exact; layer
outputs relative L2 <= 1e-3 and max|d| / max|ref| <= 2e-3 against the f64 oracle.
"""
import numpy as np
import pytest

import coracle
import moe_oracle as O
from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
MAX_REL = 2e-3
FULL = synth.LayerShapes(2048, 512, 256, 8, 512)


@pytest.fixture(scope="module")
def ctx():
    c = host.Context(0, 3 << 30)
    yield c
    c.close()


_models = {}


def model(ctx, seed, shapes, zipf=None, flags=host.MOE_F_SHARED | host.MOE_F_SHARED_GATE, scale=1.0):
    key = (seed, shapes.hidden, shapes.inter, shapes.n_experts, shapes.top_k, zipf, flags, scale)
    if key not in _models:
        _, lw, ids = host.build_synthetic_model(ctx, seed, 1, shapes, zipf, flags, scale)
        hl = coracle.synthetic_layer(seed, 0, shapes, zipf, bool(flags & host.MOE_F_SHARED),
                                     bool(flags & host.MOE_F_SHARED_GATE), scale)
        _models[key] = (ids[0], hl)
    return _models[key]


def run_forward(ctx, lid, x, resid=None, routed=None):
    m, H = x.shape
    xo = ctx.put(x)
    ro = ctx.put(resid) if resid is not None else 0
    oo = ctx.alloc(x.nbytes)
    if routed is None:
        ctx.forward(lid, xo, ro, oo, m)
    else:
        ctx.forward_routed(lid, xo, ro, oo, m, *routed)
    ctx.sync()
    return ctx.download(oo, (m, H)), xo


def check_close(got, ref, what=""):
    rl2 = O.rel_l2(got, ref)
    mr = O.max_rel(got, ref)
    assert np.isfinite(got).all(), what
    assert rl2 <= REL_L2 and mr <= MAX_REL, f"{what}: rel_l2={rl2:.3e} max_rel={mr:.3e}"
    return rl2, mr


def test_synth_device_matches_host(ctx):
    key = synth.tensor_key(99, 1, 2, synth.W3)
    n = 5000
    off = ctx.alloc(n * 136)
    ctx.synth_iq4xs(off, key, 17, n)
    got = ctx.download(off, (n, 136), np.uint8)
    assert np.array_equal(got, synth.iq4xs_blocks(key, 17, n))


def test_dequant_bit_exact(ctx):
    n = 1 << 18
    src = ctx.alloc(n * 136)
    ctx.synth_iq4xs(src, synth.tensor_key(3, 0, 0, synth.W1), 0, n)
    dst = ctx.alloc(n * 1024)
    ctx.dequant(src, n, dst)
    got = ctx.download(dst, (n, 256))
    ref = coracle.dequant(coracle.synth_iq4xs(synth.tensor_key(3, 0, 0, synth.W1), 0, n))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_golden(ctx):
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / "iq4xs_decode.npz")
    blocks = np.ascontiguousarray(z["blocks"])
    n = blocks.shape[0]
    src = ctx.alloc(n * 136)
    ctx.upload(src, blocks)
    dst = ctx.alloc(n * 1024)
    ctx.dequant(src, n, dst)
    got = ctx.download(dst, (n, 256))
    assert np.array_equal(got.view(np.uint32), z["expected"].view(np.uint32))


@pytest.mark.parametrize("name", ["a", "b", "compat"])
def test_forward_golden_small(ctx, name):
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / f"moe_small_{name}.npz")
    H, I, E, k, M = (int(z[n]) for n in ("H", "I", "E", "k", "M"))
    zipf = None if np.isnan(z["zipf"]) else float(z["zipf"])
    flags = host.MOE_F_SHARED | (host.MOE_F_SHARED_GATE if bool(z["gate"]) else 0)
    lid, _ = model(ctx, int(z["seed"]), synth.LayerShapes(H, I, E, k, I), zipf, flags, float(z["scale"]))
    out, xo = run_forward(ctx, lid, z["x"], z["resid"])
    check_close(out, z["out"], name)
    routed, w, g = ctx.do_route(lid, xo, M, k)
    assert np.array_equal(routed.astype(np.int32), z["ids"])
    assert np.allclose(w, z["w"], rtol=1e-5, atol=1e-7)


def near_ties(hl, x, k):
    lg = x.astype(np.float64) @ hl.router_w.astype(np.float64).T
    if hl.bias is not None:
        lg += hl.bias
    return set(O.near_tie_tokens(lg, k).tolist())


@pytest.mark.parametrize("m,zipf", [(1, None), (2, None), (3, None), (7, None), (64, None),
                                    (512, 1.1)])
def test_forward_full_shapes(ctx, m, zipf):
    lid, hl = model(ctx, 1234, FULL, zipf)
    x = synth.tokens(1234, 7 + m, m, FULL.hidden)
    resid = synth.tokens(1234, 8 + m, m, FULL.hidden)
    out, xo = run_forward(ctx, lid, x, resid)
    ref = coracle.moe_forward(hl, x, resid, acc64=True)
    routed, w, g = ctx.do_route(lid, xo, m, FULL.top_k)
    ties = near_ties(hl, x, FULL.top_k)
    ok = np.array([t not in ties for t in range(m)])
    assert np.array_equal(routed.astype(np.int32)[ok], ref["ids"][ok])
    # softmax weights from f32-accurate logits (f32 CUDA-core or 3xTF32 tensor-core router)
    assert np.allclose(w[ok], ref["w"][ok], rtol=2e-5, atol=1e-9)
    assert np.allclose(g, ref["gate"], rtol=1e-5)
    if ok.all():
        check_close(out, ref["out64"], f"M={m}")
    else:
        check_close(out[ok], ref["out64"][ok], f"M={m} (near ties {sorted(ties)})")


def test_exact_ties_pick_lower_index(ctx):
    sh = synth.LayerShapes(256, 256, 16, 4, 256)
    lid, hl = model(ctx, 77, sh)
    # overwrite router rows 3, 9 and 12 with row 3 -> bit-identical logits on the device
    wr = hl.router_w.copy()
    wr[9] = wr[3]
    wr[12] = wr[3]
    lw_off = ctx.put(wr)
    spec = host.LayerSpec(256, 256, 16, 4, 0, 1.0, lw_off)
    e_off = [ctx.alloc(synth.matrix_bytes(256, 256)) for _ in range(3)]
    lid2 = ctx.layer_create(spec, [e_off[0]] * 16, [e_off[1]] * 16, [e_off[2]] * 16)
    x = synth.tokens(77, 0, 32, 256) + 40.0 * wr[3] / np.linalg.norm(wr[3])
    xo = ctx.put(x.astype(np.float32))
    routed, w, _ = ctx.do_route(lid2, xo, 32, 4)
    assert (routed[:, :3] == np.array([3, 9, 12])).all()
    assert (w[:, 0] == w[:, 1]).all() and (w[:, 1] == w[:, 2]).all()


@pytest.mark.parametrize("m", [700, 1024, 1500, 3000])  # one-launch path (<= 1024 tokens), three-launch path
def test_bucket_matches_oracle(ctx, m):
    lid, hl = model(ctx, 1234, FULL, 1.1)
    x = synth.tokens(1234, 99, m, FULL.hidden)
    xo = ctx.put(x)
    k, E = FULL.top_k, FULL.n_experts
    topk = ctx.alloc(m * (k + 1) * 8)
    ctx.route(lid, xo, m, topk)
    S = m * (k + 1)
    r_off, t_off, w_off, p_off = (ctx.alloc((E + 2) * 4), ctx.alloc(S * 4), ctx.alloc(S * 4),
                                  ctx.alloc(S * 4))
    ctx.bucket(E, k, True, topk, m, r_off, t_off, w_off, p_off)
    ctx.sync()
    rec = ctx.download(topk, (m, k + 1, 2), np.uint32)
    ids = rec[:, 1:, 0].astype(np.int32)
    w = rec[:, 1:, 1].copy().view(np.float32)
    g = rec[:, 0, 1].copy().view(np.float32)
    assert (rec[:, 0, 0] == E).all()
    ranges, tok, sw, pos = coracle.bucket(ids, w, g, E, True)
    assert np.array_equal(ctx.download(r_off, (E + 2,), np.int32), ranges)
    assert np.array_equal(ctx.download(t_off, (S,), np.int32), tok)
    assert np.array_equal(ctx.download(w_off, (S,), np.float32), sw)
    assert np.array_equal(ctx.download(p_off, (m, k + 1), np.int32), pos)


def test_deterministic_reruns(ctx):
    lid, _ = model(ctx, 1234, FULL, 1.1)
    x = synth.tokens(5, 5, 300, FULL.hidden)
    a, _ = run_forward(ctx, lid, x, x)
    b, _ = run_forward(ctx, lid, x, x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_forward_routed_reference_compat(ctx):
    """The reference's own combine semantics: shared weight 1.0, global scale 1/9."""
    flags = host.MOE_F_SHARED
    lid, hl = model(ctx, 4321, FULL, None, flags, 1.0 / 9.0)
    m = 5
    x = synth.tokens(4321, 0, m, FULL.hidden)
    ref = coracle.moe_forward(hl, x, x, acc64=True)
    out, _ = run_forward(ctx, lid, x, x, routed=(ref["ids"].astype(np.uint16), ref["w"], None))
    check_close(out, ref["out64"], "compat")


def test_engine_mirror(ctx):
    lid, hl = model(ctx, 1234, FULL, None)
    eng = host.MoeEngine(ctx, [lid], FULL, max_tokens=4)
    x = synth.tokens(1, 2, 3, FULL.hidden)
    ctx.upload(eng.hi(True), x)
    routing = eng.do_route(0, 3, ping=True)
    eng.record_and_submit_moe(0, routing, 3, ping=True)
    out = ctx.download(eng.ho(True), (3, FULL.hidden))
    ref = coracle.moe_forward(hl, x, x, acc64=True)
    assert all((r.routed == ref["ids"][t]).all() for t, r in enumerate(routing))
    check_close(out, ref["out64"], "engine")


def test_rms_norm(ctx):
    x = synth.tokens(3, 3, 9, 2048) * 3.0
    xo = ctx.put(x)
    yo = ctx.alloc(x.nbytes)
    ctx.rms_norm(xo, yo, 9, 2048, 1e-6)
    y = ctx.download(yo, x.shape)
    assert np.allclose(y, O.rms_norm(x), rtol=1e-5, atol=1e-6)


def test_invalid_arguments(ctx):
    lid, _ = model(ctx, 1234, FULL, None)
    with pytest.raises(host.MoeError):
        ctx.forward(lid, 0, 0, 256, 1)          # offset 0 = missing tensor
    with pytest.raises(host.MoeError):
        ctx.forward(lid, 256, 0, ctx.arena_bytes - 16, 4)  # outside the arena
    with pytest.raises(host.MoeError):
        ctx.forward(99, 256, 0, 512, 1)         # unknown layer
    with pytest.raises(host.MoeError):
        ctx.forward_routed(lid, 256, 0, 8448, 1, np.array([[300] * 8], np.uint16),
                           np.ones((1, 8), np.float32))   # expert id out of range
    spec = host.LayerSpec(2048, 768, 256, 8, 0, 1.0, 256)
    with pytest.raises(host.MoeError):
        ctx.layer_create(spec, [256] * 256, [256] * 256, [256] * 256)  # unsupported inter


def test_graph_replay_new_pointers(ctx):
    """Repeated forwards of one (layer, M) replay one captured CUDA graph; each call's own
    input/residual/output buffers must be used."""
    lid, hl = model(ctx, 1234, FULL, None)
    m = 24
    xs = [synth.tokens(77, i, m, FULL.hidden) for i in range(3)]
    outs = [run_forward(ctx, lid, x, x)[0] for x in xs]
    for x, out in zip(xs, outs):
        ref = coracle.moe_forward(hl, x, x, acc64=True)
        check_close(out, ref["out64"], "graph replay")


@pytest.mark.parametrize("name", ["a", "b", "compat"])
def test_decode_single_token_small(ctx, name):
    """M = 1 runs the fused single-launch decode kernel; small shapes, with and without gate."""
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / f"moe_small_{name}.npz")
    H, I, E, k = (int(z[n]) for n in ("H", "I", "E", "k"))
    zipf = None if np.isnan(z["zipf"]) else float(z["zipf"])
    gate = bool(z["gate"])
    flags = host.MOE_F_SHARED | (host.MOE_F_SHARED_GATE if gate else 0)
    sh = synth.LayerShapes(H, I, E, k, I)
    lid, hl = model(ctx, int(z["seed"]), sh, zipf, flags, float(z["scale"]))
    for t in range(2):  # two calls in a row exercise the self-resetting grid synchronisation
        x = np.ascontiguousarray(z["x"][t:t + 1])
        out, _ = run_forward(ctx, lid, x, x)
        ref = coracle.moe_forward(hl, x, x, acc64=True)
        check_close(out, ref["out64"], f"decode {name} t={t}")


def test_dequant_ref36_bit_exact(ctx):
    """The reference's own 36-byte block decode (shaders/common.glsl:59-86) on the device,
    bit-exact against the oracle restatement, over random blocks including subnormal, inf and
    NaN scales."""
    rng = np.random.default_rng(36)
    n = 50000
    blk = rng.integers(0, 256, size=(n, 36), dtype=np.uint8)
    special = np.array([0x0001, 0x8001, 0x7C00, 0xFC00, 0x7E00, 0x0400, 0x3C00], np.uint16)
    blk[:len(special), 0:2] = special.view(np.uint8).reshape(-1, 2)
    src = ctx.put(blk)
    dst = ctx.alloc(n * 128)
    ctx.dequant_ref36(src, n, dst)
    ctx.sync()
    got = ctx.download(dst, (n, 32))
    ref = O.dequant_ref36(blk)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)  # NaN payloads are not compared
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


@pytest.mark.parametrize("m", [1, 17])
def test_forward_norm_matches_oracle(ctx, m):
    """out = x + MoE(RMSNorm(x)) (one step of the config-2 layer stack): the fused decode kernel
    for one token, RMSNorm + layer otherwise; against the f64 oracle and against the separate
    moe_rms_norm + moe_forward calls."""
    lid, hl = model(ctx, 21, FULL)
    x = synth.tokens(21, 50 + m, m, FULL.hidden) * 3.0
    xo = ctx.put(x)
    out = ctx.alloc(x.nbytes)
    ctx.forward_norm(lid, xo, out, m, 1e-6)
    xn = ctx.alloc(x.nbytes)
    out2 = ctx.alloc(x.nbytes)
    ctx.rms_norm(xo, xn, m, FULL.hidden, 1e-6)
    ctx.forward(lid, xn, xo, out2, m)
    ctx.sync()
    got = ctx.download(out, x.shape)
    sep = ctx.download(out2, x.shape)
    xn_ref = O.rms_norm(x, 1e-6)
    ref = coracle.moe_forward(hl, xn_ref.astype(np.float32), x)["out64"]
    check_close(got, ref, f"forward_norm m={m}")
    assert O.rel_l2(got, sep) < 1e-5


def test_layer_set_next_keeps_results(ctx):
    """Prefetching the next layer's fixed weights into L2 changes no result bit."""
    lid, _ = model(ctx, 21, FULL)
    x = synth.tokens(21, 77, 1, FULL.hidden)
    xo = ctx.put(x)
    o1, o2 = ctx.alloc(x.nbytes), ctx.alloc(x.nbytes)
    ctx.forward_norm(lid, xo, o1, 1)
    ctx.layer_set_next(lid, lid)
    ctx.forward_norm(lid, xo, o2, 1)
    ctx.layer_set_next(lid, -1)
    ctx.sync()
    assert np.array_equal(ctx.download(o1, x.shape).view(np.uint32), ctx.download(o2, x.shape).view(np.uint32))
