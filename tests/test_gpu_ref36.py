"""GPU layer forward on the reference's own weight format (MOE_F_REF36): 36-byte blocks of 32
weights (shaders/common.glsl:59-86), each matrix stored [in][out] with weight (k, n) at flat
index k*out + n (shaders/w1_w3_fused_m1.comp:46-47, w2_scatter_m1.comp:41), with the reference's
weighting (combine scale 1/9, shared expert weight 1).  Checked against the f64 oracle built on
moe_oracle.dequant_ref36 (itself bit-exact with the shaders' decode, tests/test_gpu_parity.py)
within the contract's tolerances."""
import numpy as np
import pytest

import moe_oracle as O
from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu


def ref36_matrix(rng, k_in, n_out):
    """Random reference-format matrix [k_in][n_out]: random codes, f16 scales in +-[0.002, 0.01]."""
    nb = k_in * n_out // 32
    b = rng.integers(0, 256, size=(nb, 36), dtype=np.uint8)
    d = (rng.uniform(0.002, 0.01, size=(nb, 2)) * rng.choice([-1.0, 1.0], size=(nb, 2))).astype(np.float16)
    b[:, 0:4] = d.view(np.uint8).reshape(nb, 4)
    return b


@pytest.mark.parametrize("H,I,E,k,ms", [(512, 512, 16, 4, (1, 3, 8, 17)), (2048, 512, 32, 8, (1, 5, 40))])
def test_ref36_layer_matches_oracle(H, I, E, k, ms):
    rng = np.random.default_rng(H + E)
    ctx = host.Context(0, 1 << 30)
    try:
        mats = {}
        offs = {}
        for e in range(E + 1):  # index E: the shared expert
            m1, m3, m2 = ref36_matrix(rng, H, I), ref36_matrix(rng, H, I), ref36_matrix(rng, I, H)
            mats[e] = (O.dequant_ref36(m1).reshape(H, I).T, O.dequant_ref36(m3).reshape(H, I).T,
                       O.dequant_ref36(m2).reshape(I, H).T)
            offs[e] = (ctx.put(m1), ctx.put(m3), ctx.put(m2))
        wr = rng.normal(0, 0.02, size=(E, H)).astype(np.float32)
        spec = host.LayerSpec(H, I, E, k, host.MOE_F_SHARED | host.MOE_F_REF36, 1.0 / 9.0, ctx.put(wr), 0, 0,
                              *offs[E])
        lid = ctx.layer_create(spec, [offs[e][0] for e in range(E)], [offs[e][1] for e in range(E)],
                               [offs[e][2] for e in range(E)])
        for m in ms:
            x = rng.normal(0, 1, size=(m, H)).astype(np.float32)
            resid = rng.normal(0, 1, size=(m, H)).astype(np.float32)
            xo, ro, oo = ctx.put(x), ctx.put(resid), ctx.alloc(x.nbytes)
            for _ in range(2):  # a second call reuses the scratch and the captured graph
                ctx.forward(lid, xo, ro, oo, m)
            ctx.sync()
            got = ctx.download(oo, x.shape)
            ref = O.moe_forward(x, resid, wr, None, None, 1.0 / 9.0, lambda e: mats[e], E, k, True)
            rl2, mr = O.rel_l2(got, ref["out"]), O.max_rel(got, ref["out"])
            assert rl2 <= 1e-3 and mr <= 2e-3, (m, rl2, mr)
            routed, _, _ = ctx.do_route(lid, xo, m, k)
            assert np.array_equal(routed.astype(np.int32), ref["ids"]), m
    finally:
        ctx.close()


def test_ref36_rejects_tensor_core_path():
    ctx = host.Context(0, 1 << 28)
    try:
        rng = np.random.default_rng(1)
        H, I, E, k = 512, 512, 4, 2
        o = [ctx.put(ref36_matrix(rng, H, I)) for _ in range(2)] + [ctx.put(ref36_matrix(rng, I, H))]
        spec = host.LayerSpec(H, I, E, k, host.MOE_F_REF36, 1.0, ctx.put(np.zeros((E, H), np.float32)))
        lid = ctx.layer_create(spec, [o[0]] * E, [o[1]] * E, [o[2]] * E)
        ctx.set_path(host.PATH_TC_TMEM_A)
        x = ctx.put(np.ones((16, H), np.float32))
        with pytest.raises(host.MoeError):
            ctx.forward(lid, x, x, ctx.alloc(16 * H * 4), 16)
    finally:
        ctx.close()
