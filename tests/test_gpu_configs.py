"""GPU parity at the benchmark's own configurations (3 and 4), through the C
ABI against the CPU oracle:

* config 3: one layer over 8192 tokens, uniform router logits and the Zipf(1.1) skew -- sampled
  output rows against the f64 oracle, top-k ids exact on those rows (except near ties);
* config 2: the 40-layer stack x <- x + MoE(RMSNorm(x)), 2 token steps of 40 layers each: every
  layer's output against the oracle applied to the GPU's own input of that layer (so a near tie
  in one layer cannot hide or fake an error in the next), and the stack's final state against the
  free-running oracle chain;
* config 4: the CUDA-core GEMV expert path forced at M=64 against the oracle.

Tolerances: relative L2 <= 1e-3 and max|d| / max|ref| <= 2e-3 per layer output (the contract's);
the 40-layer chain's final state within relative L2 1e-2 of the free-running oracle chain when
both chains route every layer alike (a routing flip is allowed only at a near tie).
"""
import numpy as np
import pytest

import coracle
import moe_oracle as O
from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
MAX_REL = 2e-3
STACK_REL_L2 = 1e-2  # final state of the 40-layer chain against the free-running oracle chain
FULL = synth.LayerShapes(2048, 512, 256, 8, 512)


def check_close(got, ref, what):
    rl2, mr = O.rel_l2(got, ref), O.max_rel(got, ref)
    assert np.isfinite(got).all(), what
    assert rl2 <= REL_L2 and mr <= MAX_REL, f"{what}: rel_l2={rl2:.3e} max_rel={mr:.3e}"


def sparse_host_layer(seed, layer, sh, zipf, needed):
    """Host copy of a seeded layer holding only the experts in `needed` (+ the shared expert);
    the others point at the shared expert's bytes and must not be routed to."""
    wr, g, bias = synth.float_tensors(seed, layer, sh, zipf)
    nb13, nb2 = sh.w13_bytes // 136, sh.w2_bytes // 136

    def exp(e):
        return (coracle.synth_iq4xs(synth.tensor_key(seed, layer, e, synth.W1), 0, nb13),
                coracle.synth_iq4xs(synth.tensor_key(seed, layer, e, synth.W3), 0, nb13),
                coracle.synth_iq4xs(synth.tensor_key(seed, layer, e, synth.W2), 0, nb2))
    shared = exp(sh.n_experts)
    experts = [exp(e) if e in needed else shared for e in range(sh.n_experts)]
    return coracle.HostLayer(sh.hidden, sh.inter, sh.n_experts, sh.top_k, wr, bias, g, experts, shared, 1.0, True)


def near_ties(hl, x, k):
    lg = x.astype(np.float64) @ hl.router_w.astype(np.float64).T
    if hl.bias is not None:
        lg += hl.bias
    return set(O.near_tie_tokens(lg, k).tolist())


@pytest.mark.parametrize("zipf", [None, 1.1], ids=["uniform", "zipf1.1"])
def test_config3_8192_tokens(zipf):
    m, seed = 8192, 303
    ctx = host.Context(0, 2 << 30)
    try:
        _, _, ids = host.build_synthetic_model(ctx, seed, 1, FULL, zipf)
        lid = ids[0]
        x = synth.tokens(seed, 1, m, FULL.hidden)
        xo = ctx.put(x)
        oo = ctx.alloc(x.nbytes)
        ctx.forward(lid, xo, xo, oo, m)
        ctx.sync()
        out = ctx.download(oo, x.shape)
        routed, _, _ = ctx.do_route(lid, xo, m, FULL.top_k)
        assert np.isfinite(out).all()
        rows = np.sort(np.random.default_rng(3).choice(m, 192, replace=False))
        rows = np.unique(np.concatenate([rows, [0, m - 1]]))
        hl = coracle.synthetic_layer(seed, 0, FULL, zipf)
        xr = np.ascontiguousarray(x[rows])
        ref = coracle.moe_forward(hl, xr, xr, acc64=True)
        check_close(out[rows], ref["out64"], f"config3 {zipf}")
        ties = near_ties(hl, xr, FULL.top_k)
        bad = [i for i in range(len(rows)) if i not in ties and
               not np.array_equal(routed[rows[i]].astype(np.int32), ref["ids"][i])]
        assert not bad, bad[:5]
        # bucket occupancy is what the grouped kernels see: every routed expert appears
        assert len(np.unique(routed)) > (200 if zipf is None else 60)
    finally:
        ctx.close()


def test_config2_layer_stack_two_steps():
    n_layers, steps, seed, eps = 40, 2, 404, 1e-6
    sh = FULL
    ctx = host.Context(0, n_layers * sh.expert_bytes * (sh.n_experts + 1) + (1 << 30))
    try:
        _, _, ids = host.build_synthetic_model(ctx, seed, n_layers, sh, None)
        a, b = ctx.alloc(sh.hidden * 4), ctx.alloc(sh.hidden * 4)
        finals = []
        for t in range(steps):
            x0 = synth.tokens(seed, 100 + t, 1, sh.hidden)
            ctx.upload(a, x0)
            xs = [x0]
            for li, lid in enumerate(ids):
                src, dst = (a, b) if li % 2 == 0 else (b, a)
                ctx.forward_norm(lid, src, dst, 1, eps)
                ctx.sync()
                xs.append(ctx.download(dst, (1, sh.hidden)))
            free = x0.astype(np.float32)
            flip = None  # first layer whose routing differs between the two chains
            for li in range(n_layers):
                xin = xs[li]
                xn = O.rms_norm(xin, eps).astype(np.float32)
                hl_full_router = synth.float_tensors(seed, li, sh, None)
                lg = xn.astype(np.float64) @ hl_full_router[0].astype(np.float64).T
                top = set(np.argsort(-lg[0])[:sh.top_k + 4].tolist())
                # teacher forcing: the oracle layer on the GPU's own layer input
                fn = O.rms_norm(free, eps).astype(np.float32)
                lgf = fn.astype(np.float64) @ hl_full_router[0].astype(np.float64).T
                top |= set(np.argsort(-lgf[0])[:sh.top_k + 4].tolist())
                hl = sparse_host_layer(seed, li, sh, None, top)
                ref = coracle.moe_forward(hl, xn, xin, acc64=True)
                check_close(xs[li + 1], ref["out64"], f"step {t} layer {li}")
                fr = coracle.moe_forward(hl, fn, free, acc64=True)
                if flip is None and set(fr["ids"][0].tolist()) != set(ref["ids"][0].tolist()):
                    flip = li
                    # the chains' inputs differ by rounding only, so a routing difference must
                    # come from a near tie between the k-th and (k+1)-th logits
                    srt = np.sort(lgf[0])[::-1]
                    assert srt[sh.top_k - 1] - srt[sh.top_k] < 1e-3 * max(abs(srt[0]), 1.0), (t, li)
                free = fr["out64"].astype(np.float32)
            finals.append(xs[-1])
            # without a routing flip, the free-running oracle chain ends where the stack does: 40
            # residual layers compound the per-layer differences, so the bound is looser than one
            # layer's (after a flip the chains follow different experts and are not compared)
            if flip is None:
                assert O.rel_l2(xs[-1], free) <= STACK_REL_L2, (t, O.rel_l2(xs[-1], free))
        assert not np.array_equal(finals[0], finals[1])
    finally:
        ctx.close()


def test_config4_gemv_path_m64():
    m, seed = 64, 505
    ctx = host.Context(0, 1 << 30)
    try:
        _, _, ids = host.build_synthetic_model(ctx, seed, 1, FULL, None)
        lid = ids[0]
        x = synth.tokens(seed, 2, m, FULL.hidden)
        xo = ctx.put(x)
        outs = {}
        for path in (host.PATH_GEMV, host.PATH_TC_TMEM_A):
            ctx.set_path(path)
            oo = ctx.alloc(x.nbytes)
            ctx.forward(lid, xo, xo, oo, m)
            ctx.sync()
            outs[path] = ctx.download(oo, x.shape)
        ctx.set_path(host.PATH_AUTO)
        hl = coracle.synthetic_layer(seed, 0, FULL, None)
        ref = coracle.moe_forward(hl, x, x, acc64=True)["out64"]
        check_close(outs[host.PATH_GEMV], ref, "gemv m=64")
        check_close(outs[host.PATH_TC_TMEM_A], ref, "tcgen05 m=64")
    finally:
        ctx.close()
