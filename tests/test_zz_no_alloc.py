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
        # an out-of-range routed id is dropped (slot_pos -1), the rest bucketed as usual
        m = 3
        rec = np.zeros((m, k + 1, 2), np.uint32)
        rec[:, 0, 0] = E
        rec[:, 0, 1] = np.float32(1.0).view(np.uint32)
        rec[:, 1:, 0] = np.arange(k)[None, :]
        rec[:, 1:, 1] = np.float32(0.125).view(np.uint32)
        rec[1, 3, 0] = E + 7  # bad id in token 1, slot 2
        ro = ctx.put(rec)
        S = m * (k + 1)
        outs = [ctx.alloc((E + 2) * 4), ctx.alloc(S * 4), ctx.alloc(S * 4), ctx.alloc(S * 4)]
        assert L.moe_bucket_static(E, k, 1, C.c_void_p(ctx.ptr(ro)), m,
                                   *[C.c_void_p(ctx.ptr(o)) for o in outs], None) == 0
        torch.cuda.synchronize()
        ranges = ctx.download(outs[0], (E + 2,), np.int32)
        sp = ctx.download(outs[3], (m, k + 1), np.int32)
        assert sp[1, 2] == -1 and (np.delete(sp.ravel(), 1 * (k + 1) + 2) >= 0).all()
        assert ranges[E + 1] == S - 1 and ranges[3] - ranges[2] == 2  # expert 2 lost token 1
        # sizes beyond the fixed scratch are refused, not overrun
        assert L.moe_bucket_static(E, k, 1, C.c_void_p(ctx.ptr(topk)), 9000,
                                   *[C.c_void_p(ctx.ptr(o)) for o in got], None) == -4
    finally:
        ctx.close()
