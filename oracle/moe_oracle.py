"""CPU oracle for the MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this module, and only as the checker.  The product path (the CUDA library behind
``include/moe_b200.h``) never calls it.

This is a NumPy restatement of moe-680m's MoE layer (reference paths relative to the
moe-680m source tree), with the contract's semantics where the reference has known defects:

* IQ4_XS decode: GGUF type 23 (136-byte block, f16 d, 6-bit sub-block scales, 4-bit codes
  into kvalues_iq4nl).  The reference's own decoder (shaders/common.glsl:59-86) decodes a
  private 36-byte block instead; this oracle follows the GGUF definition, pinned against the
  ``gguf`` 0.19.0 package's ``IQ4_XS.dequantize_blocks`` by tests/golden fixtures.
* Router: logits = x . Wr^T (+ bias) (shaders/router.comp:21-60, f32 weight instead of the
  reference's quantised ffn_gate); softmax with max subtraction, exp, sum, divide
  (shaders/router_topk.comp:36-60, src/router.rs:23-35); top-8 by probability, descending,
  ties to the lower expert index (strict '>' insertion, shaders/router_topk.comp:67-85);
  weights are the probabilities, not renormalised.
* Bucketing: count per expert, exclusive prefix sum, stable fill in token order
  (src/router.rs:55-97).  The shared expert gets its own bucket (index E) rather than
  sharing bucket ``shared_id = 0`` with routed expert 0 (src/router.rs:66,93).
* Experts: g = W1 x, u = W3 x (shaders/w1_w3_fused.comp:40-59); h = silu(g) * u with
  silu(v) = v / (1 + e^-v) (shaders/common.glsl:106-108, shaders/w2_scatter.comp:31-41);
  y = W2 h (shaders/w2.comp:28-49).  Every expert reads the unmodified token rows (the
  reference gathers nothing in prefill and accumulates in place, src/inference.rs:709-748).
* Combine: out = resid + scale * (sum_k p_k y_k + gate * y_shared), gate = sigmoid(g . x) or 1
  (shaders/moe_combine.comp:32-45 without its division by the expert count;
  shaders/w2_scatter.comp:67-86 for the weighted scatter-add).
"""
from __future__ import annotations

import numpy as np

KVALUES_IQ4NL = np.array([-127, -104, -83, -65, -49, -35, -22, -10,
                          1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int8)
QK_K = 256
BLOCK_BYTES = 136


def dequant_iq4xs(blocks: np.ndarray) -> np.ndarray:
    """Decode IQ4_XS blocks [n x 136] uint8 -> f32 [n x 256] (exact in f32).

    Block: f16 d @0, u16 scales_h @2, u8 scales_l[4] @4, u8 qs[128] @8.  Sub-block ib (32
    weights) has ls = (scales_l[ib/2] >> 4*(ib%2) & 0xF) | ((scales_h >> 2*ib & 3) << 4);
    weight 32*ib + j (j < 16) is the low nibble of qs[16*ib + j], weight 32*ib + 16 + j its high
    nibble; value = d * (ls - 32) * kvalues_iq4nl[nibble]."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, BLOCK_BYTES)
    n = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(n, 1)
    sh = b[:, 2:4].copy().view(np.uint16).astype(np.uint32).reshape(n, 1)
    sl = b[:, 4:8].astype(np.uint32)
    ib = np.arange(8)
    ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4)
    dl = d * (ls.astype(np.float32) - np.float32(32.0))                # [n, 8] exact
    qs = b[:, 8:].reshape(n, 8, 16)
    codes = np.concatenate([qs & 0xF, qs >> 4], axis=2)                  # [n, 8, 32]
    kv = KVALUES_IQ4NL[codes].astype(np.float32)
    return (dl[:, :, None] * kv).reshape(n, QK_K).astype(np.float32)


def ref36_f16_to_f32(bits: np.ndarray) -> np.ndarray:
    """The reference shaders' f16 -> f32 conversion (shaders/common.glsl:20-36): subnormals
    flush to signed zero, exponent 31 maps to 255 (inf / NaN), otherwise exponent + 112."""
    b = bits.astype(np.uint32)
    s = (b & 0x8000) << 16
    e = (b & 0x7C00) >> 10
    m = b & 0x03FF
    e32 = np.where(e == 31, 255, e + 112)
    out = np.where(e == 0, s, s | (e32 << 23) | (m << 13)).astype(np.uint32)
    return out.view(np.float32)


def dequant_ref36(blocks: np.ndarray) -> np.ndarray:
    """The reference's own 36-byte block (shaders/common.glsl:66-86) -> f32 [n x 32]: d0 @0
    (weights 0-15), d2 @2 (16-31), low nibble of weight p in byte 4 + p/2 (even p: low half),
    fifth bit in byte 20 + p/8 bit p%8; w = (q - 8) * d in f32."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 36)
    n = b.shape[0]
    d0 = ref36_f16_to_f32(b[:, 0].astype(np.uint32) | (b[:, 1].astype(np.uint32) << 8))
    d2 = ref36_f16_to_f32(b[:, 2].astype(np.uint32) | (b[:, 3].astype(np.uint32) << 8))
    p = np.arange(32)
    q = (b[:, 4 + (p >> 1)] >> ((p & 1) * 4)) & 0xF
    q = q.astype(np.uint32) | (((b[:, 20 + (p >> 3)] >> (p & 7)) & 1).astype(np.uint32) << 4)
    d = np.where(p[None, :] < 16, d0[:, None], d2[:, None]).astype(np.float32)
    return ((q.astype(np.float32) - np.float32(8.0)) * d).astype(np.float32)


def dequant_matrix(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return dequant_iq4xs(raw.reshape(-1, BLOCK_BYTES)).reshape(rows, cols)


def router_logits(x: np.ndarray, wr: np.ndarray, bias: np.ndarray | None) -> np.ndarray:
    """f32 logits [M x E]: f64 dot products rounded once to f32 (+ f32 bias)."""
    lg = (x.astype(np.float64) @ wr.astype(np.float64).T).astype(np.float32)
    if bias is not None:
        lg = (lg + bias.astype(np.float32)).astype(np.float32)
    return lg


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    lg = logits.astype(np.float32)
    mx = lg.max(axis=1, keepdims=True)
    e = np.exp(lg - mx).astype(np.float32)
    s = e.sum(axis=1, keepdims=True, dtype=np.float32)
    return (e / s).astype(np.float32)


def topk_desc(p: np.ndarray, k: int):
    """Top-k by value, descending, ties to the lower index -> (ids int32 [M,k], w f32 [M,k])."""
    order = np.argsort(-p, axis=1, kind="stable")[:, :k]
    return order.astype(np.int32), np.take_along_axis(p, order, axis=1).astype(np.float32)


def route(x, wr, bias, k=8):
    lg = router_logits(x, wr, bias)
    p = softmax_f32(lg)
    ids, w = topk_desc(p, k)
    return lg, p, ids, w


def near_tie_tokens(logits_f64: np.ndarray, k: int, rel: float = 1e-5) -> np.ndarray:
    """Tokens whose k-th and (k+1)-th largest logits are within ``rel`` (relative to the
    logit spread): their top-k set is not well defined under f32 reordering."""
    s = np.sort(logits_f64, axis=1)[:, ::-1]
    gap = s[:, k - 1] - s[:, k]
    scale = np.maximum(np.abs(s[:, 0]), 1.0)
    return np.nonzero(gap < rel * scale)[0]


def build_expert_batches(ids: np.ndarray, w: np.ndarray, n_experts: int, has_shared: bool = True,
                         shared_w: np.ndarray | None = None):
    """Bucket (token, slot) pairs by expert (src/router.rs:55-97).

    Returns (sorted_tokens int32[S], sorted_weights f32[S], ranges int32[E+2], pos int32[M, k+1]):
    bucket e in [ranges[e], ranges[e+1]); bucket E is the shared expert (all tokens, weight =
    shared gate, 1.0 if none); tokens ascending inside each bucket; pos[t, s] is the sorted
    position of token t's slot s (slot k = shared)."""
    m, k = ids.shape
    nb = n_experts + 1
    counts = np.bincount(ids.reshape(-1), minlength=nb).astype(np.int64)
    if has_shared:
        counts[n_experts] += m
    ranges = np.zeros(nb + 1, dtype=np.int64)
    ranges[1:] = np.cumsum(counts)
    total = int(ranges[-1])
    st = np.zeros(total, np.int32)
    sw = np.zeros(total, np.float32)
    pos = np.full((m, k + 1), -1, np.int32)
    cur = ranges[:-1].copy()
    for t in range(m):
        for s in range(k):
            e = int(ids[t, s])
            p = cur[e]
            cur[e] += 1
            st[p] = t
            sw[p] = w[t, s]
            pos[t, s] = p
        if has_shared:
            p = cur[n_experts]
            cur[n_experts] += 1
            st[p] = t
            sw[p] = 1.0 if shared_w is None else shared_w[t]
            pos[t, k] = p
    return st, sw, ranges.astype(np.int32), pos


def silu(v):
    with np.errstate(over="ignore"):
        return v / (1.0 + np.exp(-v))


def expert_ffn(xrows64: np.ndarray, w1: np.ndarray, w3: np.ndarray, w2: np.ndarray) -> np.ndarray:
    """SwiGLU expert in f64 on decoded weights: y = W2 (silu(W1 x) * W3 x)."""
    g = xrows64 @ w1.astype(np.float64).T
    u = xrows64 @ w3.astype(np.float64).T
    h = silu(g) * u
    return h @ w2.astype(np.float64).T


def moe_forward(x, resid, wr, bias, gate_w, scale, get_expert, n_experts, k=8, has_shared=True,
                route_result=None):
    """Full MoE layer in f64 accumulation.  ``get_expert(e)`` returns decoded f32 (W1, W3, W2)
    for routed expert e or the shared expert (e == n_experts).

    Returns dict(out f64 [M,H], ids, w, logits, gate)."""
    m = x.shape[0]
    if route_result is None:
        lg, _, ids, w = route(x, wr, bias, k)
    else:
        lg, ids, w = route_result
    x64 = x.astype(np.float64)
    if gate_w is not None:
        gate = 1.0 / (1.0 + np.exp(-(x64 @ gate_w.astype(np.float64))))
    else:
        gate = np.ones(m)
    acc = np.zeros((m, x.shape[1]), np.float64)
    for e in np.unique(ids):
        tok, slot = np.nonzero(ids == e)
        w1, w3, w2 = get_expert(int(e))
        y = expert_ffn(x64[tok], w1, w3, w2)
        acc[tok] += w[tok, slot].astype(np.float64)[:, None] * y
    if has_shared:
        w1, w3, w2 = get_expert(n_experts)
        acc += gate[:, None] * expert_ffn(x64, w1, w3, w2)
    out = resid.astype(np.float64) + scale * acc
    return dict(out=out, ids=ids, w=w, logits=lg, gate=gate)


def rms_norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Per-token RMSNorm without gamma (shaders/rms_norm.comp:36-58)."""
    x64 = x.astype(np.float64)
    return x64 / np.sqrt((x64 * x64).mean(axis=1, keepdims=True) + eps)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def max_rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


def vocab_logits(x: np.ndarray, w_raw: np.ndarray, vocab: int, hidden: int) -> np.ndarray:
    """LM-head projection, f64: logits[m][n] = sum_h x[m][h] * W[n][h] with W an IQ4_XS matrix of
    ``vocab`` rows in GGUF row layout.  The reference computes the same product on
    shaders/attn_output.comp with M = 1, N = vocab, K = hidden (src/inference.rs:319-330), from
    its own weight layout and f16 activations."""
    w = dequant_matrix(np.asarray(w_raw, np.uint8), vocab, hidden).astype(np.float64)
    return np.asarray(x, np.float64) @ w.T


def argmax_first(v) -> int:
    """Greedy sampling's argmax (src/util.rs:66-76): the first index whose value is strictly
    greater than every earlier one, starting from -inf, so NaN and -inf never win and an input
    with no value above -inf gives 0."""
    best_i, best_v = 0, -np.inf
    for i, x in enumerate(np.asarray(v, np.float32).tolist()):
        if x > best_v:
            best_i, best_v = i, x
    return best_i
