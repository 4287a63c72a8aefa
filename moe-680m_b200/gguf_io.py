"""GGUF reader for the MoE layers of a model file, and loading them into a library context.

The reference's parser (src/gguf.rs) reads the header, metadata and tensor index of a GGUF file;
it maps IQ4_XS to type 30 with 32-weight / 36-byte blocks (src/gguf.rs:27,55,67), ignores
``general.alignment`` and reads the expert counts under the ``llama.`` prefix whatever the
architecture.  This reader follows the GGUF format itself (versions 2 and 3): IQ4_XS is type 23
with 256-weight / 136-byte blocks, the tensor data section starts at the next multiple of
``general.alignment`` (32 when absent), and hyper-parameters are read under
``<general.architecture>.``.

``load_moe_layers`` maps MoE tensors onto the library's layer description (the registry shape of
src/memory.rs:120-290), under the reference registry's own names (``blk.L.ffn_gate``,
``blk.L.experts.E.w1/w3/w2``, ``blk.L.shared_expert.w1/w3/w2``) or the Qwen-MoE names of
llama.cpp files:

  blk.L.ffn_gate_inp.weight        router [E][H]           (F32; F16 / BF16 converted to f32)
  blk.L.ffn_gate_exps.weight       W1 of all experts [E][I][H]   IQ4_XS, stacked
  blk.L.ffn_up_exps.weight         W3 [E][I][H]                  IQ4_XS
  blk.L.ffn_down_exps.weight       W2 [E][H][I]                  IQ4_XS
  blk.L.ffn_gate_shexp / ffn_up_shexp / ffn_down_shexp .weight   shared expert, IQ4_XS
  blk.L.ffn_gate_inp_shexp.weight  shared-expert gate g [H]      (optional)

The stacked expert tensors are uploaded once; expert e's matrices are slices at
e * (rows x row bytes), so no per-expert copy is made.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import host

GGUF_MAGIC = b"GGUF"

# GGML tensor types this reader sizes: type -> (weights per block, bytes per block)
GGML_BLOCK = {
    0: (1, 4),       # F32
    1: (1, 2),       # F16
    8: (32, 34),     # Q8_0
    23: (256, 136),  # IQ4_XS
    30: (1, 2),      # BF16
}
GGML_NAMES = {0: "F32", 1: "F16", 8: "Q8_0", 23: "IQ4_XS", 30: "BF16"}

# metadata value types
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


class GgufError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    dims: tuple          # GGUF order: dims[0] is the contiguous (innermost) dimension
    ggml_type: int
    offset: int          # relative to the tensor data section
    nbytes: int
    file_offset: int = 0  # absolute

    @property
    def shape(self) -> tuple:  # row-major (outermost first)
        return tuple(reversed(self.dims))


@dataclass
class GgufFile:
    path: Path
    version: int
    metadata: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    alignment: int = 32
    data_offset: int = 0

    def array(self, name: str) -> np.ndarray:
        """The tensor's bytes (read-only memory map of the file)."""
        t = self.tensors[name]
        return np.memmap(self.path, dtype=np.uint8, mode="r", offset=t.file_offset, shape=(t.nbytes,))

    def arch_int(self, key: str, default=None):
        arch = self.metadata.get("general.architecture", "")
        v = self.metadata.get(f"{arch}.{key}", default)
        return int(v) if v is not None else None


def _tensor_bytes(dims, ggml_type: int, name: str) -> int:
    if ggml_type not in GGML_BLOCK:
        raise GgufError(f"{name}: unsupported GGML type {ggml_type}")
    bw, bb = GGML_BLOCK[ggml_type]
    n = 1
    for d in dims:
        n *= int(d)
    if int(dims[0]) % bw:
        raise GgufError(f"{name}: innermost dimension {dims[0]} not a multiple of the block size {bw}")
    return n // bw * bb


def read_gguf(path) -> GgufFile:
    """Parse the header, metadata and tensor index of a GGUF v2/v3 file."""
    path = Path(path)
    with open(path, "rb") as f:
        buf = f.read()
    pos = 0

    def take(fmt):
        nonlocal pos
        size = struct.calcsize(fmt)
        if pos + size > len(buf):
            raise GgufError("truncated file")
        v = struct.unpack_from(fmt, buf, pos)
        pos += size
        return v[0] if len(v) == 1 else v

    def string():
        nonlocal pos
        n = take("<Q")
        if pos + n > len(buf):
            raise GgufError("truncated string")
        s = buf[pos:pos + n].decode("utf-8", errors="replace")
        pos += n
        return s

    def value(t):
        if t in _SCALARS:
            return take(_SCALARS[t])
        if t == _STRING:
            return string()
        if t == _ARRAY:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        raise GgufError(f"unknown metadata type {t}")

    if buf[:4] != GGUF_MAGIC:
        raise GgufError("not a GGUF file (bad magic)")
    pos = 4
    version = take("<I")
    if version not in (2, 3):
        raise GgufError(f"unsupported GGUF version {version}")
    n_tensors, n_kv = take("<Q"), take("<Q")
    g = GgufFile(path, version)
    for _ in range(n_kv):
        key = string()
        g.metadata[key] = value(take("<I"))
    infos = []
    for _ in range(n_tensors):
        name = string()
        nd = take("<I")
        dims = tuple(take("<Q") for _ in range(nd))
        ty = take("<I")
        off = take("<Q")
        infos.append(TensorInfo(name, dims, ty, off, _tensor_bytes(dims, ty, name)))
    g.alignment = int(g.metadata.get("general.alignment", 32))
    g.data_offset = (pos + g.alignment - 1) // g.alignment * g.alignment
    for t in infos:
        t.file_offset = g.data_offset + t.offset
        if t.file_offset + t.nbytes > len(buf):
            raise GgufError(f"{t.name}: data outside the file")
        g.tensors[t.name] = t
    return g


def _router_f32(g: GgufFile, t: TensorInfo) -> np.ndarray:
    raw = np.asarray(g.array(t.name))
    if t.ggml_type == 0:
        return raw.view(np.float32).reshape(t.shape)
    if t.ggml_type == 1:
        return raw.view(np.float16).astype(np.float32).reshape(t.shape)
    if t.ggml_type == 30:  # bf16: the upper half of an f32
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(t.shape)
    raise GgufError(f"{t.name}: router type {GGML_NAMES.get(t.ggml_type, t.ggml_type)} not supported")


def _moe_blocks(g: GgufFile) -> list:
    """Blocks with MoE experts under either naming: llama.cpp's stacked ``ffn_*_exps`` tensors or
    the reference registry's per-expert ``experts.E.w1`` tensors (src/memory.rs:159-175)."""
    out = set()
    for n in g.tensors:
        parts = n.split(".")
        if len(parts) > 2 and parts[0] == "blk" and (n.endswith("ffn_gate_exps.weight") or
                                                    n.endswith(".experts.0.w1.weight")):
            out.add(int(parts[1]))
    return sorted(out)


def load_moe_layers(ctx: host.Context, g: GgufFile, layers=None, scale: float = 1.0):
    """Upload the MoE tensors of ``layers`` (default: every block with experts) into the
    context's arena and create one library layer each.  Returns (TensorRegistry, [layer ids]).

    Two tensor namings are read:
      * llama.cpp (Qwen-MoE): ``blk.L.ffn_gate_inp`` router, stacked ``ffn_{gate,up,down}_exps``,
        ``ffn_{gate,up,down}_shexp`` shared expert, optional ``ffn_gate_inp_shexp`` gate;
      * the reference's registry (src/memory.rs:147-175, :236-262): ``blk.L.ffn_gate`` router,
        ``blk.L.experts.E.w1/w3/w2`` per expert, ``blk.L.shared_expert.w1/w3/w2``, no shared
        gate (the reference weights routed experts p/9 and the shared expert 1/9: pass
        ``scale=1/9``).
    The router may be F32, F16, BF16 (converted on the host) or IQ4_XS (decoded to f32 on the
    device with moe_dequant_iq4xs)."""
    reg = host.TensorRegistry()
    layers = _moe_blocks(g) if layers is None else list(layers)
    k = g.arch_int("expert_used_count")
    if k is None and "llama.expert_used_count" in g.metadata:  # the key the reference reads
        k = int(g.metadata["llama.expert_used_count"])
    if k is None:
        raise GgufError("expert_used_count missing from the metadata")
    ids = []

    def put(name, arr=None):
        t = g.tensors.get(name)
        if t is None:
            return 0, None
        data = np.ascontiguousarray(arr if arr is not None else g.array(name))
        off = ctx.put(data)
        reg.add(name, off, data.nbytes, t.ggml_type if arr is None else host.GGML_F32)
        return off, t

    def iq4(name, shape=None):
        off, t = put(name)
        if t is None or t.ggml_type != 23:
            raise GgufError(f"{name} missing or not IQ4_XS")
        if shape is not None and tuple(t.shape) != tuple(shape):
            raise GgufError(f"{name} has shape {t.shape}, expected {tuple(shape)}")
        return off, t

    def router(name):
        t = g.tensors.get(name)
        if t is None:
            raise GgufError(f"{name} missing")
        if t.ggml_type == 23:  # IQ4_XS router: decoded on the device into an f32 [E][H] tensor
            src, _ = put(name)
            E_, H_ = t.shape
            dst = ctx.alloc(E_ * H_ * 4)
            ctx.dequant(src, E_ * H_ // 256, dst)
            reg.add(name + ".f32", dst, E_ * H_ * 4, host.GGML_F32)
            return dst, t
        return put(name, _router_f32(g, t))[0], t

    for l in layers:
        p = f"blk.{l}."
        stacked = p + "ffn_gate_exps.weight" in g.tensors
        if not stacked and p + "experts.0.w1.weight" not in g.tensors:
            raise GgufError(f"{p}: no expert tensors (ffn_gate_exps or experts.0.w1)")
        router_off, rt = router(p + ("ffn_gate_inp.weight" if stacked else "ffn_gate.weight"))
        E, H = rt.shape
        flags = 0
        sh = [0, 0, 0]
        gate_off = 0
        if stacked:
            offs, shapes = {}, {}
            for key in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"):
                off, t = iq4(p + key + ".weight")
                if t.shape[0] != E:
                    raise GgufError(f"{p}{key}.weight has {t.shape[0]} experts, router {E}")
                offs[key], shapes[key] = off, t.shape
            I = shapes["ffn_gate_exps"][1]
            if shapes["ffn_gate_exps"][2] != H or shapes["ffn_down_exps"][1:] != (H, I):
                raise GgufError(f"{p}: expert shapes {shapes} do not match hidden {H}")
            b13 = I * (H // 256) * 136
            b2 = H * (I // 256) * 136
            w1 = [offs["ffn_gate_exps"] + e * b13 for e in range(E)]
            w3 = [offs["ffn_up_exps"] + e * b13 for e in range(E)]
            w2 = [offs["ffn_down_exps"] + e * b2 for e in range(E)]
            shared = ("ffn_gate_shexp", "ffn_up_shexp", "ffn_down_shexp")
        else:
            t1 = g.tensors.get(p + "experts.0.w1.weight")
            I = t1.shape[0]
            w1, w3, w2 = [], [], []
            for e in range(E):
                w1.append(iq4(f"{p}experts.{e}.w1.weight", (I, H))[0])
                w3.append(iq4(f"{p}experts.{e}.w3.weight", (I, H))[0])
                w2.append(iq4(f"{p}experts.{e}.w2.weight", (H, I))[0])
            shared = ("shared_expert.w1", "shared_expert.w3", "shared_expert.w2")
        if p + shared[0] + ".weight" in g.tensors:
            for i, key in enumerate(shared):
                sh[i] = iq4(p + key + ".weight", (H, I) if i == 2 else (I, H))[0]
            flags |= host.MOE_F_SHARED
        gt = g.tensors.get(p + "ffn_gate_inp_shexp.weight")
        if gt is not None and flags & host.MOE_F_SHARED:
            gate_off, _ = put(p + "ffn_gate_inp_shexp.weight", _router_f32(g, gt).reshape(-1))
            flags |= host.MOE_F_SHARED_GATE
        spec = host.LayerSpec(H, I, E, k, flags, scale, router_off, 0, gate_off, sh[0], sh[1], sh[2])
        ids.append(ctx.layer_create(spec, w1, w3, w2))
    return reg, ids
