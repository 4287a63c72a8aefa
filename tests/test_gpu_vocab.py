"""Vocabulary projection (moe_vocab_logits: the LM head of src/inference.rs:319-330 and its greedy
argmax, src/util.rs:66-76) through the C ABI against the f64 oracle.

Tolerances: logits relative L2 <= 1e-4 and max|d| / max|ref| <= 1e-3 against the f64 oracle
(activations are rounded to 16-bit fixed point, relative step 2^-15 of the row maximum); the
argmax id is exact against the reference's argmax over the returned logits, and its oracle logit
lies within 1e-3 * max|logit| of the oracle's maximum."""
import numpy as np
import pytest

import moe_oracle as O
from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-4
MAX_REL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = host.Context(0, 1 << 30)
    yield c
    c.close()


def head(seed, vocab, hidden):
    return synth.iq4xs_matrix(synth.tensor_key(seed, 90, 0, 0), vocab, hidden)


def run(ctx, raw, vocab, hidden, x, logits=True, ids=True):
    m = x.shape[0]
    wo = ctx.put(raw)
    xo = ctx.put(np.ascontiguousarray(x, np.float32))
    lo = ctx.alloc(m * vocab * 4) if logits else 0
    io = ctx.alloc(256) if ids else 0
    ctx.vocab_logits(wo, vocab, hidden, xo, m, lo, io)
    ctx.sync()
    lg = ctx.download(lo, (m, vocab)) if logits else None
    ii = ctx.download(io, (m,), np.uint32) if ids else None
    return lg, ii


def check(lg, ids, ref):
    assert np.isfinite(lg).all()
    rl2, mr = O.rel_l2(lg, ref), O.max_rel(lg, ref)
    assert rl2 <= REL_L2 and mr <= MAX_REL, f"rel_l2={rl2:.3e} max_rel={mr:.3e}"
    for t in range(lg.shape[0]):
        assert int(ids[t]) == O.argmax_first(lg[t])
        assert ref[t, ids[t]] >= ref[t].max() - 1e-3 * np.abs(ref[t]).max()


@pytest.mark.parametrize("vocab,hidden,m", [(1000, 2048, 1), (999, 2048, 2), (4099, 2048, 3),
                                            (1500, 1024, 1), (1501, 1024, 2), (2053, 1024, 8),
                                            (16, 512, 2), (777, 4096, 5), (300, 4096, 1), (1, 2048, 1)])
def test_logits_and_argmax(ctx, vocab, hidden, m):
    raw = head(7, vocab, hidden)
    x = synth.tokens(7, vocab % 97, m, hidden)
    lg, ids = run(ctx, raw, vocab, hidden, x)
    check(lg, ids, O.vocab_logits(x, raw, vocab, hidden))


def test_argmax_only_and_relaunch(ctx):
    vocab, hidden = 3001, 2048
    raw = head(8, vocab, hidden)
    x = synth.tokens(8, 1, 4, hidden)
    lg, ids = run(ctx, raw, vocab, hidden, x)
    for _ in range(3):  # keys and ticket are reset by each launch's last CTA
        _, ids2 = run(ctx, raw, vocab, hidden, x, logits=False)
        assert np.array_equal(ids, ids2)
    x2 = synth.tokens(8, 2, 4, hidden)
    lg2, ids3 = run(ctx, raw, vocab, hidden, x2)
    assert [O.argmax_first(r) for r in lg2] == ids3.tolist()


def test_ties_take_the_lowest_index(ctx):
    vocab, hidden = 700, 2048
    raw = head(9, vocab, hidden).reshape(vocab, -1).copy()
    x = synth.tokens(9, 0, 2, hidden)
    lg, _ = run(ctx, raw.reshape(-1), vocab, hidden, x)
    best = int(np.argmax(lg[0]))
    for dup in (5, 333, 699):  # exact copies of the winning row tie exactly
        raw[dup] = raw[best]
    lg, ids = run(ctx, raw.reshape(-1), vocab, hidden, x)
    assert int(ids[0]) == min(5, best)
    assert int(ids[0]) == O.argmax_first(lg[0])
    same = np.repeat(raw[:1], vocab, axis=0)  # every row equal: index 0
    _, ids = run(ctx, same.reshape(-1), vocab, hidden, x)
    assert ids.tolist() == [0, 0]


def test_nonfinite_row(ctx):
    vocab, hidden = 500, 1024
    raw = head(10, vocab, hidden)
    x = synth.tokens(10, 0, 3, hidden)
    x[1, 17] = np.nan
    x[2, 3] = np.inf
    lg, ids = run(ctx, raw, vocab, hidden, x)
    assert np.isnan(lg[1]).all() and np.isnan(lg[2]).all()
    assert ids[1] == 0 and ids[2] == 0
    ref = O.vocab_logits(x[:1], raw, vocab, hidden)
    check(lg[:1], ids[:1], ref)


def test_zero_activations(ctx):
    vocab, hidden = 300, 512
    raw = head(11, vocab, hidden)
    lg, ids = run(ctx, raw, vocab, hidden, np.zeros((1, hidden), np.float32))
    assert not lg.any() and ids[0] == 0


def test_rejects_unsupported(ctx):
    raw = head(12, 64, 512)
    wo = ctx.put(raw)
    xo = ctx.put(np.zeros((9, 512), np.float32))
    lo = ctx.alloc(9 * 64 * 4)
    for args in ((64, 512, xo, 9, lo, 0), (64, 256, xo, 1, lo, 0), (64, 768, xo, 1, lo, 0),
                 (64, 512, xo, 1, 0, 0)):
        with pytest.raises(host.MoeError):
            ctx.vocab_logits(wo, *args)
    with pytest.raises(host.MoeError):  # weight range past the arena
        ctx.vocab_logits(wo, 1 << 26, 512, xo, 1, lo, 0)


def test_full_vocab_sampled_rows(ctx):
    """The 248,320 x 2048 head (generated on the device); 4096 sampled rows against the oracle,
    the argmax against the reference's argmax over all returned logits."""
    vocab, hidden, m = 248320, 2048, 2
    key = synth.tensor_key(13, 91, 0, 0)
    bpr = hidden // 256
    wo = ctx.alloc(vocab * bpr * 136)
    ctx.synth_iq4xs(wo, key, 0, vocab * bpr)
    x = synth.tokens(13, 0, m, hidden)
    xo = ctx.put(x)
    lo = ctx.alloc(m * vocab * 4)
    io = ctx.alloc(256)
    ctx.vocab_logits(wo, vocab, hidden, xo, m, lo, io)
    ctx.sync()
    lg = ctx.download(lo, (m, vocab))
    ids = ctx.download(io, (m,), np.uint32)
    rows = np.random.default_rng(13).choice(vocab, 4096, replace=False)
    rows[:2] = [0, vocab - 1]
    raw = np.concatenate([synth.iq4xs_blocks(key, int(r) * bpr, bpr).reshape(-1) for r in rows])
    ref = O.vocab_logits(x, raw, len(rows), hidden)
    assert O.rel_l2(lg[:, rows], ref) <= REL_L2 and O.max_rel(lg[:, rows], ref) <= MAX_REL
    for t in range(m):
        assert int(ids[t]) == O.argmax_first(lg[t])


def test_silu_mul(ctx):
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(5000) * 4).astype(np.float32)
    u = rng.standard_normal(5000).astype(np.float32)
    go, uo, yo = ctx.put(g), ctx.put(u), ctx.alloc(g.nbytes)
    ctx.silu_mul(go, uo, yo, g.size)
    ctx.silu_mul(go, 0, go, g.size)  # in place, no up operand
    ctx.sync()
    ref = O.silu(g.astype(np.float64))
    assert O.max_rel(ctx.download(yo, g.shape), ref * u) <= 1e-6
    assert O.max_rel(ctx.download(go, g.shape), ref) <= 1e-6


def test_mtp_head_chain(ctx):
    """MTP head (src/inference.rs:335-360): z = W1 . h (V = H), a = silu(z), draft = argmax(W2 . a)."""
    hidden, vocab = 2048, 5003
    w1 = synth.iq4xs_matrix(synth.tensor_key(14, 92, 0, 0), hidden, hidden)
    w2 = synth.iq4xs_matrix(synth.tensor_key(14, 93, 0, 0), vocab, hidden)
    x = synth.tokens(14, 0, 1, hidden)
    w1o, w2o, xo = ctx.put(w1), ctx.put(w2), ctx.put(x)
    zo, lo, io = ctx.alloc(hidden * 4), ctx.alloc(vocab * 4), ctx.alloc(256)
    ctx.vocab_logits(w1o, hidden, hidden, xo, 1, zo, 0)
    ctx.silu_mul(zo, 0, zo, hidden)
    ctx.vocab_logits(w2o, vocab, hidden, zo, 1, lo, io)
    ctx.sync()
    a = O.silu(O.vocab_logits(x, w1, hidden, hidden))
    ref = O.vocab_logits(a, w2, vocab, hidden)
    check(ctx.download(lo, (1, vocab)), ctx.download(io, (1,), np.uint32), ref)
