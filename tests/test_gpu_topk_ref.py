"""GPU routing against the literal restatement of the reference's top-k shader
(oracle/router_topk_ref.py, shaders/router_topk.comp:36-93), on logits chosen exactly: the
router weight is zero and the router bias carries the logits, so every token of a layer has the
same, exactly known logits.  Checked: the routed ids (ties to the lower expert index, later equal
probabilities never displacing earlier ones, routed expert 0 next to the shared expert) through
the batch router (moe_do_route at M = 16) and the CUDA-core router (M = 1); the probabilities
within 2e-6 relative; and the single-token fused layer (moe_forward, M = 1) against
moe_forward_routed given the restatement's routing."""
import numpy as np
import pytest

import moe_oracle as O
import router_topk_ref as R
from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu
FULL = synth.LayerShapes(2048, 512, 256, 8, 512)


def cases():
    rng = np.random.default_rng(9)
    tie = np.full(256, -5.0, np.float32)
    tie[[200, 17, 3, 99]] = 2.0
    tie[[250, 251]] = 1.5
    tie[[10, 11, 12]] = 1.0
    zero = np.zeros(256, np.float32)
    zero[0] = 3.0
    flat = np.zeros(256, np.float32)  # every probability equal: experts 0..7
    return {"ties": tie, "expert0": zero, "flat": flat,
            "random": (rng.normal(0, 2, 256)).astype(np.float32)}


@pytest.fixture(scope="module")
def env():
    ctx = host.Context(0, 1 << 30)
    _, lw, ids = host.build_synthetic_model(ctx, 11, 1, FULL, None)
    yield ctx, lw
    ctx.close()


@pytest.mark.parametrize("name", list(cases()))
def test_routing_matches_shader_restatement(env, name):
    ctx, lw = env
    lg = cases()[name]
    E, H = FULL.n_experts, FULL.hidden
    spec = host.LayerSpec(H, FULL.inter, E, FULL.top_k, host.MOE_F_SHARED | host.MOE_F_SHARED_GATE, 1.0,
                          ctx.put(np.zeros((E, H), np.float32)), ctx.put(lg), lw.shared_gate[0],
                          lw.shared_w1[0], lw.shared_w3[0], lw.shared_w2[0])
    w1, w3, w2 = lw.expert_tables(0)
    lid = ctx.layer_create(spec, w1, w3, w2)
    ref = R.route_token(lg)
    ref_ids = np.array([e for e, _ in ref[1:]], np.int32)
    ref_w = np.array([v for _, v in ref[1:]], np.float32)
    for m in (1, 16):
        x = synth.tokens(11, m, m, H)
        xo = ctx.put(x)
        routed, w, _ = ctx.do_route(lid, xo, m, FULL.top_k)
        assert (routed.astype(np.int32) == ref_ids[None]).all(), (name, m, routed[0], ref_ids)
        assert np.allclose(w, ref_w[None], rtol=2e-6, atol=0), (name, m)
    # the fused single-token layer routes the same way: equal to the layer run with the
    # restatement's routing given explicitly
    x = synth.tokens(12, 0, 1, H)
    xo = ctx.put(x)
    o1, o2 = ctx.alloc(x.nbytes), ctx.alloc(x.nbytes)
    ctx.forward(lid, xo, xo, o1, 1)
    _, _, g = ctx.do_route(lid, xo, 1, FULL.top_k)
    ctx.forward_routed(lid, xo, xo, o2, 1, ref_ids[None].astype(np.uint16), ref_w[None], g)
    ctx.sync()
    a, b = ctx.download(o1, x.shape), ctx.download(o2, x.shape)
    assert O.rel_l2(a, b) <= 1e-3 and O.max_rel(a, b) <= 2e-3, name
