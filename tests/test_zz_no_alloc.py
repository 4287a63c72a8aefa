"""GPU test of moe_bucket_static, the allocation-free bucketing entry point.

It exists for callers that cannot allocate device memory (an engine that sized its arena up
front, or code where cudaMalloc is not allowed): instead of a context workspace grown with
cudaMalloc it uses a fixed static device array.  Its results must equal moe_bucket's exactly
(bucketing is integer work), on two calls in a row, since calls share and reuse that array.
This file is collected last so that a run stopping at the first failure has run all the others.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu


def test_bucket_static_matches_bucket():
    sh = synth.LayerShapes(2048, 512, 256, 8, 512)
    ctx = host.Context(0, 1 << 30)
    try:
        _, _, ids = host.build_synthetic_model(ctx, 31337, 1, sh, 1.1)
        lid, k, E = ids[0], sh.top_k, sh.n_experts
        L = host.lib()
        for call, m in enumerate((700, 333)):
            x = synth.tokens(31337, call, m, sh.hidden)
            xo = ctx.put(x)
            topk = ctx.alloc(m * (k + 1) * 8)
            ctx.route(lid, xo, m, topk)
            S = m * (k + 1)
            ref = [ctx.alloc((E + 2) * 4), ctx.alloc(S * 4), ctx.alloc(S * 4), ctx.alloc(S * 4)]
            got = [ctx.alloc((E + 2) * 4), ctx.alloc(S * 4), ctx.alloc(S * 4), ctx.alloc(S * 4)]
            ctx.bucket(E, k, True, topk, m, *ref)
            ctx.sync()
            rc = L.moe_bucket_static(E, k, 1, C.c_void_p(ctx.ptr(topk)), m,
                                     *[C.c_void_p(ctx.ptr(o)) for o in got], None)
            assert rc == 0
            torch.cuda.synchronize()  # the call above ran on the legacy default stream
            for (ro, go), (n, dt) in zip(zip(ref, got), [((E + 2,), np.int32), ((S,), np.int32),
                                                           ((S,), np.float32), ((S,), np.int32)]):
                a = ctx.download(ro, n, dt)
                b = ctx.download(go, n, dt)
                assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"call {call}"
        # sizes beyond the fixed scratch are refused, not overrun
        assert L.moe_bucket_static(E, k, 1, C.c_void_p(ctx.ptr(topk)), 9000,
                                   *[C.c_void_p(ctx.ptr(o)) for o in got], None) == -4
    finally:
        ctx.close()
