"""moe_forward_host (asynchronous forward from and to host memory, double-buffered staging)
against moe_forward on arena buffers: the same bits, over several calls in a row issued before
one sync (so the staging slots are reused while earlier calls are still in flight), for the
tensor-core batch path and the single-token decode path, with and without the residual."""
import numpy as np
import pytest

from moe680m_b200 import host, synth

pytestmark = pytest.mark.gpu

SH = synth.LayerShapes(2048, 512, 256, 8, 512)


@pytest.mark.parametrize("m", [1, 512])
def test_forward_host_matches_forward(m):
    ctx = host.Context(0, 2 << 30)
    try:
        _, _, ids = host.build_synthetic_model(ctx, 83, 2, SH, None)
        xs = [np.ascontiguousarray(synth.tokens(83, 10 + i, m, SH.hidden)) for i in range(5)]
        ref = []
        for i, x in enumerate(xs):
            xo = ctx.put(x)
            oo = ctx.alloc(x.nbytes)
            ctx.forward(ids[i % 2], xo, xo if i % 3 else 0, oo, m)
            ctx.sync()
            ref.append(ctx.download(oo, x.shape))
        outs = [np.full_like(x, np.nan) for x in xs]
        for i, x in enumerate(xs):
            ctx.forward_host(ids[i % 2], x.ctypes.data, outs[i].ctypes.data, m, add_residual=bool(i % 3))
        ctx.sync()
        for i in range(len(xs)):
            assert np.isfinite(outs[i]).all(), i
            assert np.array_equal(outs[i], ref[i]), (i, float(np.abs(outs[i] - ref[i]).max()))
    finally:
        ctx.close()
