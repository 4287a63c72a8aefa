"""The concurrent shared-expert pass of large tensor-core batches (the shared expert on a second
stream, its rows added by the combine after the routed slots) against the single pass
(MOE_B200_SHARED_SPLIT=0): the same bits, for the plain forward and its captured graph, with
and without the shared gate, and with the layer scale."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys, numpy as np
sys.path.insert(0, {root!r} + "/tests")
import conftest
conftest.load_pkg()
from moe680m_b200 import host, synth
sh = synth.LayerShapes(2048, 512, 256, 8, 512)
ctx = host.Context(0, 2 << 30)
outs = []
for flags, scale in ((host.MOE_F_SHARED | host.MOE_F_SHARED_GATE, 1.0), (host.MOE_F_SHARED, 0.75)):
    _, _, ids = host.build_synthetic_model(ctx, 71, 1, sh, None, flags, scale)
    for m in (64, 700):
        x = synth.tokens(71, m, m, sh.hidden)
        xo = ctx.put(x)
        oo = ctx.alloc(x.nbytes)
        for rep in range(3):  # the first call runs eagerly, later ones replay the graph
            ctx.forward(ids[0], xo, xo, oo, m)
            ctx.sync()
            outs.append(ctx.download(oo, x.shape))
ctx.close()
np.save({out!r}, np.concatenate([o.ravel() for o in outs]))
"""


def run(tmp_path, split):
    out = str(tmp_path / f"out{split}.npy")
    env = dict(os.environ, MOE_B200_SHARED_SPLIT=str(split))
    subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT, out=out)], env=env, check=True, timeout=600)
    return np.load(out)


def test_shared_split_bit_identical(tmp_path):
    a, b = run(tmp_path, 1), run(tmp_path, 0)
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)
