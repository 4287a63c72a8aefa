"""Seeded synthetic MoE-layer inputs (the benchmark configurations' shapes and distributions).

Integer data (IQ4_XS weight bytes) comes from a counter-based generator, splitmix64
(Steele, Lea & Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014),
evaluated on (tensor key, word index).  The same generator is implemented in the CUDA
library (``moe_synth_iq4xs``) so multi-GB weight sets can be produced directly in HBM
while the CPU oracle regenerates exactly the same bytes for the experts it needs.

Floating-point tensors (router weight, shared-expert gate, tokens, Zipf bias) are small and
come from NumPy's PCG64 ``default_rng`` seeded from the same seed, generated on the host.

Distributions:
  * IQ4_XS block (GGUF type 23, 136 bytes / 256 weights): f16 ``d`` ~ U(0.005, 0.02);
    the 6-bit sub-block scales and the 4-bit codes are uniform (every other byte of the
    block is a uniform random byte, which makes every packed field uniform).
  * router weight f32 [E x H] ~ N(0, 0.02^2); shared gate g f32 [H] ~ N(0, 0.02^2);
  * tokens x f32 [M x H] ~ N(0, 1);
  * Zipf skew: bias_e = -s * ln(rank_e), rank a seeded permutation of 1..E, s = 1.1.
"""
from __future__ import annotations

import numpy as np

QK_K = 256
IQ4XS_BLOCK_BYTES = 136
MASK64 = (1 << 64) - 1

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

# matrix ids inside an expert
W1, W3, W2 = 1, 3, 2


def splitmix64_np(z: np.ndarray) -> np.ndarray:
    """Vectorised splitmix64 finaliser on uint64 (wrapping arithmetic)."""
    with np.errstate(over="ignore"):
        z = (z + _GOLDEN).astype(np.uint64)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def splitmix64_int(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def tensor_key(seed: int, layer: int, expert: int, matrix: int) -> int:
    """64-bit key of one weight matrix; ``expert == n_experts`` denotes the shared expert."""
    k = splitmix64_int(seed & MASK64)
    k = splitmix64_int(k ^ ((layer & 0xFFFF) << 32 | (expert & 0xFFFF) << 8 | (matrix & 0xFF)))
    return k


def iq4xs_blocks(key: int, block_start: int, n_blocks: int) -> np.ndarray:
    """Bytes of ``n_blocks`` IQ4_XS blocks [n_blocks x 136] uint8, blocks numbered from
    ``block_start`` inside the tensor with ``key``.  Each block is 17 uint64 words
    w_i = splitmix64(key + 17*block + i), little-endian; bytes 0..1 (f16 d) are then
    replaced by d = f16(0.005 + 0.015 * u), u = (w_0 >> 40) * 2^-24 in f32 arithmetic."""
    idx = (np.arange(n_blocks, dtype=np.uint64)[:, None] + np.uint64(block_start)) * np.uint64(17) \
        + np.arange(17, dtype=np.uint64)[None, :]
    with np.errstate(over="ignore"):
        words = splitmix64_np(idx + np.uint64(key))
    raw = words.view(np.uint8).reshape(n_blocks, IQ4XS_BLOCK_BYTES).copy()
    u = (words[:, 0] >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
    v = np.float32(0.005) + np.float32(0.015) * u          # two separately rounded f32 ops
    d = v.astype(np.float32).astype(np.float16)
    raw[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    return raw


def matrix_bytes(rows: int, cols: int) -> int:
    assert cols % QK_K == 0
    return rows * (cols // QK_K) * IQ4XS_BLOCK_BYTES


def iq4xs_matrix(key: int, rows: int, cols: int) -> np.ndarray:
    """One IQ4_XS matrix [rows x cols] as raw bytes [rows x cols/256 x 136]."""
    nb = rows * (cols // QK_K)
    return iq4xs_blocks(key, 0, nb).reshape(rows, cols // QK_K, IQ4XS_BLOCK_BYTES)


class LayerShapes:
    def __init__(self, hidden=2048, inter=512, n_experts=256, top_k=8, shared_inter=512):
        self.hidden, self.inter, self.n_experts, self.top_k = hidden, inter, n_experts, top_k
        self.shared_inter = shared_inter
        assert shared_inter == inter, "shared expert uses the routed expert shapes"

    @property
    def w13_bytes(self):
        return matrix_bytes(self.inter, self.hidden)

    @property
    def w2_bytes(self):
        return matrix_bytes(self.hidden, self.inter)

    @property
    def expert_bytes(self):
        return 2 * self.w13_bytes + self.w2_bytes


def float_tensors(seed: int, layer: int, sh: LayerShapes, zipf_s: float | None = None):
    """Router weight [E x H], shared gate [H] and optional Zipf bias [E] of one layer."""
    rng = np.random.default_rng([seed, layer, 0x5EED])
    wr = rng.normal(0.0, 0.02, size=(sh.n_experts, sh.hidden)).astype(np.float32)
    g = rng.normal(0.0, 0.02, size=(sh.hidden,)).astype(np.float32)
    bias = None
    if zipf_s is not None:
        rank = rng.permutation(sh.n_experts) + 1
        bias = (-zipf_s * np.log(rank.astype(np.float64))).astype(np.float32)
    return wr, g, bias


def tokens(seed: int, step: int, m: int, hidden: int) -> np.ndarray:
    rng = np.random.default_rng([seed, step, 0x70C])
    return rng.normal(0.0, 1.0, size=(m, hidden)).astype(np.float32)


def expert_weights(seed: int, layer: int, expert: int, sh: LayerShapes):
    """(W1, W3, W2) raw IQ4_XS bytes for one expert (expert == n_experts: shared)."""
    w1 = iq4xs_matrix(tensor_key(seed, layer, expert, W1), sh.inter, sh.hidden)
    w3 = iq4xs_matrix(tensor_key(seed, layer, expert, W3), sh.inter, sh.hidden)
    w2 = iq4xs_matrix(tensor_key(seed, layer, expert, W2), sh.hidden, sh.inter)
    return w1, w3, w2
