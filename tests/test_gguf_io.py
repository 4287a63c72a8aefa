"""GGUF reader (moe-680m_b200/gguf_io.py) against files written by the independent ``gguf``
0.19.0 package: metadata, tensor index, byte ranges and shapes must agree with its own reader;
corrupt files are rejected.  The GPU test loads the MoE tensors of such a file into a context
and checks the layer against the f64 oracle on the same weights."""
import numpy as np
import pytest

import moe_oracle as O
from moe680m_b200 import gguf_io, host, synth

gguf = pytest.importorskip("gguf")

SEED = 99
SH = synth.LayerShapes(hidden=512, inter=512, n_experts=8, top_k=2, shared_inter=512)
ARCH = "qwen3moe"


def _weights(layer):
    E = SH.n_experts
    ex = [synth.expert_weights(SEED, layer, e, SH) for e in range(E + 1)]  # E = shared
    wr, g, _ = synth.float_tensors(SEED, layer, SH)
    return wr, g, ex


def write_model(path, n_layers=2, router_dtype="f32"):
    w = gguf.GGUFWriter(str(path), arch=ARCH)
    w.add_block_count(n_layers)
    w.add_uint32(f"{ARCH}.expert_count", SH.n_experts)
    w.add_uint32(f"{ARCH}.expert_used_count", SH.top_k)
    w.add_uint32(f"{ARCH}.embedding_length", SH.hidden)
    w.add_string("general.note", "synthetic MoE layers for reader tests")
    w.add_array("general.tags", [1, 2, 3])
    IQ = gguf.GGMLQuantizationType.IQ4_XS
    for l in range(n_layers):
        wr, g, ex = _weights(l)
        if router_dtype == "f16":
            w.add_tensor(f"blk.{l}.ffn_gate_inp.weight", wr.astype(np.float16))
        else:
            w.add_tensor(f"blk.{l}.ffn_gate_inp.weight", wr)
        for key, m in (("ffn_gate_exps", 0), ("ffn_up_exps", 1), ("ffn_down_exps", 2)):
            stacked = np.stack([ex[e][m] for e in range(SH.n_experts)])  # [E][rows][blocks][136]
            E_, rows, nb, _ = stacked.shape
            w.add_tensor(f"blk.{l}.{key}.weight", stacked.reshape(E_, rows, nb * 136), raw_dtype=IQ)
        for key, m in (("ffn_gate_shexp", 0), ("ffn_up_shexp", 1), ("ffn_down_shexp", 2)):
            a = ex[SH.n_experts][m]
            w.add_tensor(f"blk.{l}.{key}.weight", a.reshape(a.shape[0], -1), raw_dtype=IQ)
        w.add_tensor(f"blk.{l}.ffn_gate_inp_shexp.weight", g)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("gguf") / "moe.gguf"
    write_model(p)
    return p


def test_reader_matches_gguf_package(model_file):
    mine = gguf_io.read_gguf(model_file)
    ref = gguf.GGUFReader(str(model_file))
    assert mine.metadata["general.architecture"] == ARCH
    assert mine.arch_int("expert_count") == SH.n_experts
    assert mine.metadata["general.tags"] == [1, 2, 3]
    assert set(mine.tensors) == {t.name for t in ref.tensors}
    for t in ref.tensors:
        m = mine.tensors[t.name]
        assert m.ggml_type == int(t.tensor_type)
        assert m.file_offset == int(t.data_offset)
        assert m.nbytes == int(t.n_bytes)
        assert list(m.dims) == [int(d) for d in t.shape]
        assert np.array_equal(np.asarray(mine.array(t.name)), np.asarray(t.data).reshape(-1).view(np.uint8))


def test_iq4xs_is_type_23_with_136_byte_blocks(model_file):
    g = gguf_io.read_gguf(model_file)
    t = g.tensors["blk.0.ffn_gate_exps.weight"]
    assert t.ggml_type == 23
    assert t.shape == (SH.n_experts, SH.inter, SH.hidden)
    assert t.nbytes == SH.n_experts * SH.inter * SH.hidden // 256 * 136


def test_rejects_corrupt_files(tmp_path, model_file):
    data = model_file.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + data[4:])
    with pytest.raises(gguf_io.GgufError):
        gguf_io.read_gguf(bad)
    bad.write_bytes(data[: len(data) // 2])
    with pytest.raises(gguf_io.GgufError):
        gguf_io.read_gguf(bad)


@pytest.mark.gpu
@pytest.mark.parametrize("router_dtype", ["f32", "f16"])
def test_load_and_forward_matches_oracle(tmp_path, router_dtype):
    p = tmp_path / "moe.gguf"
    write_model(p, n_layers=2, router_dtype=router_dtype)
    g = gguf_io.read_gguf(p)
    ctx = host.Context(0, 256 << 20)
    try:
        reg, ids = gguf_io.load_moe_layers(ctx, g)
        assert len(ids) == 2 and reg.lookup("blk.1.ffn_down_exps.weight") > 0
        m = 40
        x = synth.tokens(SEED, 3, m, SH.hidden)
        xo = ctx.put(x)
        oo = ctx.alloc(x.nbytes)
        ctx.forward(ids[1], xo, xo, oo, m)
        ctx.sync()
        got = ctx.download(oo, x.shape)
        wr, gw, ex = _weights(1)
        if router_dtype == "f16":
            wr = wr.astype(np.float16).astype(np.float32)
        dec = {e: (O.dequant_matrix(ex[e][0], SH.inter, SH.hidden), O.dequant_matrix(ex[e][1], SH.inter, SH.hidden),
                   O.dequant_matrix(ex[e][2], SH.hidden, SH.inter)) for e in range(SH.n_experts + 1)}
        ref = O.moe_forward(x, x, wr, None, gw, 1.0, lambda e: dec[e], SH.n_experts, SH.top_k)["out"]
        assert O.rel_l2(got, ref) <= 1e-3 and O.max_rel(got, ref) <= 2e-3
    finally:
        ctx.close()


class _ArenaStandIn:
    """Host-memory stand-in for host.Context with the three calls load_moe_layers makes (put,
    layer_create) so the tensor-name mapping is checked without a GPU."""

    def __init__(self):
        self.mem = bytearray(256)
        self.layers = []

    def put(self, arr):
        off = (len(self.mem) + 255) // 256 * 256
        data = np.ascontiguousarray(arr).view(np.uint8).reshape(-1).tobytes()
        self.mem.extend(b"\0" * (off - len(self.mem)))
        self.mem.extend(data)
        return off

    def alloc(self, nbytes):
        return self.put(np.zeros(nbytes, np.uint8))

    def dequant(self, src, n_blocks, dst):  # moe_dequant_iq4xs, here by the oracle
        raw = np.frombuffer(bytes(self.mem[src:src + n_blocks * 136]), np.uint8).reshape(n_blocks, 136)
        f = O.dequant_iq4xs(raw).astype(np.float32).tobytes()
        self.mem[dst:dst + len(f)] = f

    def layer_create(self, spec, w1, w3, w2):
        self.layers.append((spec, list(w1), list(w3), list(w2)))
        return len(self.layers) - 1


@pytest.mark.parametrize("router_dtype", ["f32", "f16"])
def test_load_maps_tensor_names_without_gpu(model_file, tmp_path, router_dtype):
    """Every expert's W1/W3/W2 offset points at its own slice of the stacked tensor, the shared
    expert and gate are wired with their flags, the router lands as f32."""
    p = model_file
    if router_dtype == "f16":
        p = tmp_path / "f16.gguf"
        write_model(p, router_dtype="f16")
    g = gguf_io.read_gguf(p)
    arena = _ArenaStandIn()
    reg, ids = gguf_io.load_moe_layers(arena, g, scale=0.5)
    assert ids == [0, 1]
    E, H, I = SH.n_experts, SH.hidden, SH.inter
    b13, b2 = I * (H // 256) * 136, H * (I // 256) * 136
    for l, (spec, w1, w3, w2) in enumerate(arena.layers):
        assert (spec.hidden, spec.inter, spec.n_experts, spec.top_k) == (H, I, E, SH.top_k)
        assert spec.flags == host.MOE_F_SHARED | host.MOE_F_SHARED_GATE and spec.scale == 0.5
        wr, gate, ex = _weights(l)
        if router_dtype == "f16":
            wr = wr.astype(np.float16).astype(np.float32)
        got_wr = np.frombuffer(bytes(arena.mem[spec.router_w:spec.router_w + wr.nbytes]), np.float32)
        assert np.array_equal(got_wr, wr.reshape(-1))
        assert reg.lookup(f"blk.{l}.ffn_gate_inp.weight") == spec.router_w
        for e in range(E):
            for offs, m, nb in ((w1, 0, b13), (w3, 1, b13), (w2, 2, b2)):
                assert bytes(arena.mem[offs[e]:offs[e] + nb]) == ex[e][m].tobytes()
        for off, m, nb in ((spec.shared_w1, 0, b13), (spec.shared_w3, 1, b13), (spec.shared_w2, 2, b2)):
            assert bytes(arena.mem[off:off + nb]) == ex[E][m].tobytes()
        got_g = np.frombuffer(bytes(arena.mem[spec.shared_gate:spec.shared_gate + gate.nbytes]), np.float32)
        assert np.array_equal(got_g, gate.reshape(-1))


def test_load_rejects_missing_expert_tensor(tmp_path):
    p = tmp_path / "bad.gguf"
    w = gguf.GGUFWriter(str(p), arch=ARCH)
    w.add_block_count(1)
    w.add_uint32(f"{ARCH}.expert_count", SH.n_experts)
    w.add_uint32(f"{ARCH}.expert_used_count", SH.top_k)
    wr, _, _ = _weights(0)
    w.add_tensor("blk.0.ffn_gate_inp.weight", wr)
    w.add_tensor("blk.0.ffn_gate_exps.weight", np.zeros((SH.n_experts, SH.inter, SH.hidden), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(gguf_io.GgufError):
        gguf_io.load_moe_layers(_ArenaStandIn(), gguf_io.read_gguf(p))


def write_reference_named(path, router="f32"):
    """One block under the reference registry's names (src/memory.rs:147-175): ffn_gate router,
    experts.E.w1/w3/w2 per expert, shared_expert.w1/w3/w2, and the llama.* expert keys the
    reference reads whatever the architecture."""
    w = gguf.GGUFWriter(str(path), arch="qwen35moe")
    w.add_uint32("llama.expert_count", SH.n_experts)
    w.add_uint32("llama.expert_used_count", SH.top_k)
    wr, _, ex = _weights(0)
    IQ = gguf.GGMLQuantizationType.IQ4_XS
    if router == "iq4":
        raw = synth.iq4xs_matrix(synth.tensor_key(SEED, 50, 0, 0), SH.n_experts, SH.hidden)
        w.add_tensor("blk.0.ffn_gate.weight", raw.reshape(SH.n_experts, -1), raw_dtype=IQ)
    else:
        w.add_tensor("blk.0.ffn_gate.weight", wr)
    for e in range(SH.n_experts + 1):
        pre = f"blk.0.experts.{e}." if e < SH.n_experts else "blk.0.shared_expert."
        for m, name in ((0, "w1"), (1, "w3"), (2, "w2")):
            a = ex[e][m]
            w.add_tensor(pre + name + ".weight", a.reshape(a.shape[0], -1), raw_dtype=IQ)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.mark.parametrize("router", ["f32", "iq4"])
def test_load_reference_registry_names(tmp_path, router):
    p = tmp_path / "ref.gguf"
    write_reference_named(p, router)
    g = gguf_io.read_gguf(p)
    arena = _ArenaStandIn()
    reg, ids = gguf_io.load_moe_layers(arena, g, scale=1.0 / 9.0)
    assert ids == [0]
    spec, w1, w3, w2 = arena.layers[0]
    E, H, I = SH.n_experts, SH.hidden, SH.inter
    assert (spec.hidden, spec.inter, spec.n_experts, spec.top_k) == (H, I, E, SH.top_k)
    assert spec.flags == host.MOE_F_SHARED and spec.shared_gate == 0  # reference: no shared gate
    assert abs(spec.scale - 1.0 / 9.0) < 1e-7
    wr, _, ex = _weights(0)
    if router == "iq4":
        raw = synth.iq4xs_matrix(synth.tensor_key(SEED, 50, 0, 0), E, H)
        wr = O.dequant_matrix(raw, E, H).astype(np.float32)
    got = np.frombuffer(bytes(arena.mem[spec.router_w:spec.router_w + wr.nbytes]), np.float32)
    assert np.array_equal(got, wr.reshape(-1))
    b13, b2 = I * (H // 256) * 136, H * (I // 256) * 136
    for e in range(E):
        for offs, m, nb in ((w1, 0, b13), (w3, 1, b13), (w2, 2, b2)):
            assert bytes(arena.mem[offs[e]:offs[e] + nb]) == ex[e][m].tobytes()
            assert reg.lookup(f"blk.0.experts.{e}.{('w1', 'w3', 'w2')[m]}.weight") == offs[e]
    for off, m, nb in ((spec.shared_w1, 0, b13), (spec.shared_w3, 1, b13), (spec.shared_w2, 2, b2)):
        assert bytes(arena.mem[off:off + nb]) == ex[E][m].tobytes()
