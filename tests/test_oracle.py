"""CPU tests of the oracle itself (no GPU): pinned IQ4_XS decode, generator twins, routing /
bucketing / layer restatements (NumPy vs C) and the golden fixtures."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

import coracle
import moe_oracle as O
from moe680m_b200 import synth

GOLD = Path(__file__).resolve().parent / "golden"


def test_decode_matches_gguf_golden():
    z = np.load(GOLD / "iq4xs_decode.npz")
    blocks, expected = z["blocks"], z["expected"]
    got_np = O.dequant_iq4xs(blocks)
    got_c = coracle.dequant(blocks)
    assert np.array_equal(got_np.view(np.uint32), expected.view(np.uint32))
    assert np.array_equal(got_c.view(np.uint32), expected.view(np.uint32))


def test_decode_kat_values():
    # d = 1, sub-block ib has scale ls = ib (first KAT block), nibble j -> kv[j]
    z = np.load(GOLD / "iq4xs_decode.npz")
    b = z["blocks"][0]
    v = O.dequant_iq4xs(b[None])[0]
    for ib in range(8):
        for j in range(16):
            assert v[32 * ib + j] == (ib - 32) * int(O.KVALUES_IQ4NL[j])
            assert v[32 * ib + 16 + j] == (ib - 32) * int(O.KVALUES_IQ4NL[(j + ib) % 16])


def test_decode_covers_every_scale_and_code():
    z = np.load(GOLD / "iq4xs_decode.npz")
    kat = z["blocks"][:8]
    seen = set()
    for b in kat:
        sh = int(b[2]) | int(b[3]) << 8
        for ib in range(8):
            seen.add(((b[4 + ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4))
    assert seen == set(range(64))


def test_generator_numpy_c_twins():
    key = synth.tensor_key(5, 3, 17, synth.W2)
    a = synth.iq4xs_blocks(key, 100, 300)
    b = coracle.synth_iq4xs(key, 100, 300)
    assert np.array_equal(a, b)
    d = a[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert d.min() >= 0.005 - 1e-5 and d.max() <= 0.02 + 1e-5


def test_generator_distribution():
    raw = synth.iq4xs_blocks(synth.tensor_key(1, 0, 0, synth.W1), 0, 4000)
    sl = raw[:, 4:8]
    sh = raw[:, 2:4].copy().view(np.uint16).astype(np.uint32)
    ls = np.concatenate([((sl[:, i // 2] >> (4 * (i % 2))) & 0xF) | (((sh[:, 0] >> (2 * i)) & 3) << 4)
                         for i in range(8)])
    hist = np.bincount(ls, minlength=64)
    assert hist.min() > 0.8 * hist.mean()
    codes = np.concatenate([raw[:, 8:] & 0xF, raw[:, 8:] >> 4]).reshape(-1)
    ch = np.bincount(codes, minlength=16)
    assert ch.min() > 0.95 * ch.mean()


def test_topk_ties_lower_index():
    p = np.array([[0.1, 0.3, 0.3, 0.2, 0.3, 0.1]], np.float32)
    ids, w = O.topk_desc(p, 3)
    assert ids.tolist() == [[1, 2, 4]]
    # C oracle: duplicated router rows give equal logits -> lower index first
    H, E = 256, 8
    rng = np.random.default_rng(0)
    wr = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    wr[5] = wr[2]
    wr[7] = wr[2]
    x = rng.normal(0, 1, (16, H)).astype(np.float32)
    x[:, :] += 10 * wr[2] / np.linalg.norm(wr[2])  # make expert 2/5/7 the top three
    zero = np.zeros((256, 136), np.uint8)
    layer = coracle.HostLayer(H, 256, E, 3, wr, None, None, [(zero, zero, zero)] * E)
    ids, w, g, lg = coracle.route(layer, x)
    assert (ids == np.array([2, 5, 7])).all()


def _check_fixture(name):
    z = np.load(GOLD / f"moe_small_{name}.npz")
    H, I, E, k, M = (int(z[n]) for n in ("H", "I", "E", "k", "M"))
    seed = int(z["seed"])
    zipf = None if np.isnan(z["zipf"]) else float(z["zipf"])
    sh = synth.LayerShapes(H, I, E, k, I)
    exps = [synth.expert_weights(seed, 0, e, sh) for e in range(E + 1)]
    h = hashlib.sha256()
    for t in exps:
        for m in t:
            h.update(np.ascontiguousarray(m).tobytes())
    assert h.hexdigest() == str(z["weights_sha256"])
    wr, g, bias = synth.float_tensors(seed, 0, sh, zipf)
    assert np.array_equal(wr, z["wr"]) and np.array_equal(g, z["g"])
    gate = bool(z["gate"])
    dec = [tuple(O.dequant_matrix(m, *shape) for m, shape in zip(t, [(I, H), (I, H), (H, I)]))
           for t in exps]
    r = O.moe_forward(z["x"], z["resid"], wr, bias, g if gate else None, float(z["scale"]),
                      lambda e: dec[e], E, k)
    assert np.array_equal(r["ids"], z["ids"])
    assert O.rel_l2(r["out"], z["out"]) < 1e-12
    # C oracle restatement agrees with the NumPy one
    hl = coracle.HostLayer(H, I, E, k, wr, bias, g if gate else None, exps[:E], exps[E],
                           float(z["scale"]), gate)
    c = coracle.moe_forward(hl, z["x"], z["resid"], acc64=True)
    assert np.array_equal(c["ids"], z["ids"])
    assert O.rel_l2(c["out64"], z["out"]) < 1e-6  # C keeps the shared gate in f32
    c32 = coracle.moe_forward(hl, z["x"], z["resid"], acc64=False)
    assert O.rel_l2(c32["out64"], z["out"]) < 1e-4


@pytest.mark.parametrize("name", ["a", "b", "compat"])
def test_golden_moe_small(name):
    _check_fixture(name)


def test_bucket_numpy_vs_c():
    rng = np.random.default_rng(3)
    M, E, k = 300, 32, 4
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(M)]).astype(np.int32)
    w = rng.random((M, k)).astype(np.float32)
    g = rng.random(M).astype(np.float32)
    st, sw, ranges, pos = O.build_expert_batches(ids, w, E, True, g)
    r2, t2, w2, p2 = coracle.bucket(ids, w, g, E, True)
    assert np.array_equal(ranges, r2) and np.array_equal(st, t2)
    assert np.array_equal(sw, w2) and np.array_equal(pos, p2)
    # stable: tokens ascending in every bucket
    for e in range(E + 1):
        seg = st[ranges[e]:ranges[e + 1]]
        assert (np.diff(seg) > 0).all()
    # empty buckets allowed
    ids2 = np.tile(np.arange(k, dtype=np.int32), (5, 1))
    r3, t3, _, _ = coracle.bucket(ids2, np.ones((5, k), np.float32), None, E, False)
    assert r3[k] == r3[E + 1] == 5 * k


def test_ref36_decode_known_answers():
    """The reference's 36-byte block: hand-built known answers (scales 1.0 / -0.5, a subnormal
    scale flushed to zero, codes 0, 8, 31 through the fifth-bit byte)."""
    blk = np.zeros((2, 36), np.uint8)
    blk[0, 0:2] = np.array([1.0], np.float16).view(np.uint8)
    blk[0, 2:4] = np.array([-0.5], np.float16).view(np.uint8)
    blk[0, 4] = 0x80          # weight 0: low nibble 0; weight 1: high nibble 8
    blk[0, 4 + 8] = 0x0F      # weight 16: low nibble 15
    blk[0, 20 + 2] = 0x01     # weight 16: fifth bit -> q = 31
    blk[1, 0:2] = np.array([1], np.uint16).view(np.uint8)  # subnormal f16: flushed
    blk[1, 4] = 0x33
    w = O.dequant_ref36(blk)
    assert w[0, 0] == -8.0 and w[0, 1] == 0.0 and w[0, 16] == (31 - 8) * -0.5
    assert w[0, 2] == -8.0 and w[0, 17] == 4.0    # q = 0 under both scales
    assert np.all(w[1, :16] == 0.0)


def test_argmax_first_follows_the_reference():
    """src/util.rs:66-76: strict '>' from -inf, so ties keep the first index, NaN and -inf never
    win, and no value above -inf gives index 0."""
    assert O.argmax_first([1.0, 3.0, 3.0, 2.0]) == 1
    assert O.argmax_first([np.nan, 0.5, np.nan, 0.7]) == 3
    assert O.argmax_first([-np.inf, -np.inf]) == 0
    assert O.argmax_first([np.nan, np.nan]) == 0
    assert O.argmax_first([-0.0, 0.0]) == 0
    assert O.argmax_first([-5.0, -np.inf, -1.0]) == 2


def test_vocab_logits_is_the_dequantised_product():
    raw = synth.iq4xs_matrix(synth.tensor_key(1, 90, 0, 0), 37, 512)
    x = np.random.default_rng(0).standard_normal((3, 512)).astype(np.float32)
    w = O.dequant_matrix(raw, 37, 512)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.array_equal(O.vocab_logits(x, raw, 37, 512), ref)
