"""A second, literal restatement of the reference's routing step -- TEST INFRASTRUCTURE ONLY.

Independent of moe_oracle.py's vectorised top-k: this follows shaders/router_topk.comp line by
line for one token (pure Python loops over f32 NumPy scalars; small cases only):

* router_topk.comp:36-44: max by a tree reduction over 256 lanes (s = 128, 64, ..., 1,
  v[i] = max(v[i], v[i + s]));
* :47-49: e_i = exp(logit_i - max) (f32);
* :52-58: sum by the same tree reduction with +=, in f32;
* :61: prob_i = e_i / sum if sum > 0 else 0;
* :67-85: thread 0's insertion of the 256 probabilities into 8 slots initialised to (0, -1.0):
  a probability enters slot k at the first k with p > vals[k] (strict), shifting the lower
  slots down -- so equal probabilities keep index order (the lower expert index first) and a
  later equal probability never displaces an earlier one;
* :88-93: entry 0 = {id 0, weight 1.0} (the shared expert), entries 1..8 the routed slots.

The library's record differs in one documented way: its entry 0 carries the shared expert's own
id E (and its gate), because the reference's id 0 collides with routed expert 0 in bucketing
(src/router.rs:69-72, :88-93).  `to_library_record` states that mapping.
"""
from __future__ import annotations

import numpy as np


def _tree(v: list, op) -> np.float32:
    v = list(v)
    s = len(v) // 2
    while s > 0:
        for i in range(s):
            v[i] = op(v[i], v[i + s])
        s //= 2
    return v[0]


def route_token(logits) -> list:
    """Nine (id, weight) entries for one token's 256 f32 logits (router_topk.comp:28-93)."""
    lg = [np.float32(v) for v in logits]
    assert len(lg) == 256
    mx = _tree(lg, lambda a, b: max(a, b))
    e = [np.float32(np.exp(np.float32(v - mx))) for v in lg]
    ssum = _tree(e, lambda a, b: np.float32(a + b))
    prob = [np.float32(v / ssum) if ssum > 0 else np.float32(0.0) for v in e]
    ids = [0] * 9
    vals = [np.float32(1.0)] + [np.float32(-1.0)] * 8
    for j in range(256):
        p = prob[j]
        for k in range(1, 9):
            if p > vals[k]:
                for s in range(8, k, -1):
                    ids[s] = ids[s - 1]
                    vals[s] = vals[s - 1]
                ids[k] = j
                vals[k] = p
                break
    return list(zip(ids, vals))


def to_library_record(entries, n_experts: int, gate: float = 1.0) -> list:
    """The reference's 9 entries in the library's record convention: entry 0 -> (E, gate)."""
    return [(n_experts, np.float32(gate))] + list(entries[1:])
