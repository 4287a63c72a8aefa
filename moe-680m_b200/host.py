"""ctypes binding of libmoe_b200.so and the host-side mirror of the reference MoE engine.

Reference (moe-680m tree): src/inference.rs (InferenceEngine::do_route :622,
record_and_submit_moe :663), src/memory.rs (ArenaLayout, TensorRegistry, LayerWeights),
src/router.rs (RoutingOutput).  Error behaviour follows the reference's ``Result<_, String>``:
every failing call raises ``MoeError`` carrying the library's message.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import synth

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libmoe_b200.so"

MOE_OK = 0
MOE_F_SHARED = 1
MOE_F_SHARED_GATE = 2
MOE_F_EXPERT_SUBSET = 4
MOE_F_REF36 = 8
MOE_NO_EXPERT = 0xFFFFFFFF
MOE_FT_NO_SHARED, MOE_FT_SHARED_ONLY, MOE_FT_UNSCALED = 1, 2, 4
MOE_EP_TRANSPORT_NCCL, MOE_EP_TRANSPORT_PEER = 0, 1

# Every symbol include/moe_b200.h declares.
EXPORTS = (
    "moe_abi_version", "moe_ctx_create", "moe_ctx_create_external", "moe_ctx_destroy",
    "moe_arena_upload", "moe_arena_download", "moe_arena_ptr", "moe_set_stream", "moe_sync",
    "moe_last_error", "moe_layer_create", "moe_reserve", "moe_route", "moe_do_route",
    "moe_bucket", "moe_forward", "moe_forward_host", "moe_forward_routed", "moe_rms_norm", "moe_dequant_iq4xs",
    "moe_synth_iq4xs", "moe_profile", "moe_profile_read", "moe_launch_count", "moe_set_path",
    "moe_bucket_static", "moe_forward_topk", "moe_ep_plan_bytes", "moe_ep_dispatch",
    "moe_ep_combine", "moe_dequant_ref36", "moe_forward_norm", "moe_vocab_logits",
    "moe_ep_unique_id", "moe_ep_init", "moe_forward_ep", "moe_ep_set_transport", "moe_ep_transport", "moe_silu_mul",
    "moe_layer_set_next", "moe_ep_abort",
)

PATH_AUTO, PATH_GEMV, PATH_TC_SMEM_A, PATH_TC_TMEM_A = 0, 1, 2, 3


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class LibraryMissing(RuntimeError):
    pass


class StageStatC(C.Structure):
    _fields_ = [("name", C.c_char * 24), ("calls", C.c_uint32), ("total_ms", C.c_float)]


class LayerSpecC(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("inter", C.c_uint32), ("n_experts", C.c_uint32),
        ("top_k", C.c_uint32), ("flags", C.c_uint32), ("scale", C.c_float),
        ("router_w", C.c_uint64), ("router_bias", C.c_uint64), ("shared_gate", C.c_uint64),
        ("shared_w1", C.c_uint64), ("shared_w3", C.c_uint64), ("shared_w2", C.c_uint64),
    ]


_lib = None


def lib():
    """Load the CUDA library (raises LibraryMissing when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("MOE_B200_LIB", LIB_PATH))
    if not path.exists():
        raise LibraryMissing(f"{path} not built: run python moe-680m_b200/build.py "
                             "(there is no CPU fallback)")
    L = C.CDLL(str(path))
    u32, u64, i32, vp, f32 = C.c_uint32, C.c_uint64, C.c_int, C.c_void_p, C.c_float
    P = C.POINTER
    sig = {
        "moe_abi_version": (i32, []),
        "moe_ctx_create": (i32, [i32, u64, P(vp)]),
        "moe_ctx_create_external": (i32, [i32, vp, u64, P(vp)]),
        "moe_ctx_destroy": (None, [vp]),
        "moe_arena_upload": (i32, [vp, u64, vp, u64]),
        "moe_arena_download": (i32, [vp, u64, vp, u64]),
        "moe_arena_ptr": (i32, [vp, u64, P(vp)]),
        "moe_set_stream": (i32, [vp, vp]),
        "moe_sync": (i32, [vp]),
        "moe_last_error": (i32, [vp, C.c_char_p, C.c_size_t]),
        "moe_layer_create": (i32, [vp, P(LayerSpecC), P(u64), P(u64), P(u64), P(u32)]),
        "moe_reserve": (i32, [vp, u32, u32]),
        "moe_route": (i32, [vp, u32, u64, u32, u64]),
        "moe_do_route": (i32, [vp, u32, u64, u32, P(C.c_uint16), P(f32), P(f32)]),
        "moe_bucket": (i32, [vp, u32, u32, i32, u64, u32, u64, u64, u64, u64]),
        "moe_forward": (i32, [vp, u32, u64, u64, u64, u32]),
        "moe_forward_host": (i32, [vp, u32, vp, vp, u32, C.c_int]),
        "moe_forward_routed": (i32, [vp, u32, u64, u64, u64, u32, P(C.c_uint16), P(f32), P(f32)]),
        "moe_rms_norm": (i32, [vp, u64, u64, u32, u32, f32]),
        "moe_dequant_iq4xs": (i32, [vp, u64, u64, u64]),
        "moe_dequant_ref36": (i32, [vp, u64, u64, u64]),
        "moe_vocab_logits": (i32, [vp, u64, u32, u32, u64, u32, u64, u64]),
        "moe_ep_unique_id": (i32, [vp, C.c_size_t]),
        "moe_ep_init": (i32, [vp, vp, u32, u32]),
        "moe_forward_ep": (i32, [vp, u32, u64, u64, u64, u32, u32]),
        "moe_ep_set_transport": (i32, [vp, i32]),
        "moe_ep_abort": (i32, [vp]),
        "moe_silu_mul": (i32, [vp, u64, u64, u64, u64]),
        "moe_ep_transport": (i32, [vp, P(i32)]),
        "moe_forward_norm": (i32, [vp, u32, u64, u64, u32, f32]),
        "moe_layer_set_next": (i32, [vp, u32, i32]),
        "moe_synth_iq4xs": (i32, [vp, u64, u64, u64, u64]),
        "moe_profile": (i32, [vp, i32]),
        "moe_profile_read": (i32, [vp, P(StageStatC), i32, P(i32)]),
        "moe_launch_count": (i32, [vp, P(u64)]),
        "moe_set_path": (i32, [vp, i32]),
        "moe_bucket_static": (i32, [u32, u32, i32, vp, u32, vp, vp, vp, vp, vp]),
        "moe_forward_topk": (i32, [vp, u32, u64, u64, u64, u32, u64, u32]),
        "moe_ep_plan_bytes": (u64, [u32, u32]),
        "moe_ep_dispatch": (i32, [vp, u32, u32, u32, u32, u32, u64, u64, u32, u32, u64, u64, u64]),
        "moe_ep_combine": (i32, [vp, u32, u32, u32, u32, u64, u64, u64, u64, f32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _err(ctx_handle) -> str:
    buf = C.create_string_buffer(1024)
    lib().moe_last_error(ctx_handle, buf, 1024)
    return buf.value.decode(errors="replace")


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


class Context:
    """One device arena (owned, or wrapping caller memory) and the library context over it."""

    ALIGN = 256

    def __init__(self, device: int = 0, arena_bytes: int = 1 << 30, external_ptr: int | None = None):
        L = lib()
        h = C.c_void_p()
        if external_ptr is None:
            rc = L.moe_ctx_create(device, arena_bytes, C.byref(h))
        else:
            rc = L.moe_ctx_create_external(device, C.c_void_p(external_ptr), arena_bytes, C.byref(h))
        if rc != MOE_OK:
            raise MoeError(rc, _err(None))
        self.h = h
        self.device = device
        self.arena_bytes = arena_bytes
        self._next = self.ALIGN  # offset 0 is the "missing" sentinel (src/memory.rs:33)

    # -- lifetime -----------------------------------------------------------------------------
    def close(self):
        if self.h:
            lib().moe_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != MOE_OK:
            raise MoeError(rc, _err(self.h))

    # -- arena --------------------------------------------------------------------------------
    def alloc(self, nbytes: int, align: int = ALIGN) -> int:
        """Bump-allocate an arena region (ArenaLayout::compute analogue)."""
        off = (self._next + align - 1) // align * align
        if off + nbytes > self.arena_bytes:
            raise MoeError(-3, f"arena exhausted: need {off + nbytes} of {self.arena_bytes} bytes")
        self._next = off + nbytes
        return off

    @property
    def used(self) -> int:
        return self._next

    def upload(self, off: int, arr: np.ndarray):
        a = np.ascontiguousarray(arr)
        self._check(lib().moe_arena_upload(self.h, off, a.ctypes.data_as(C.c_void_p), a.nbytes))

    def upload_ptr(self, off: int, host_ptr: int, nbytes: int):
        self._check(lib().moe_arena_upload(self.h, off, C.c_void_p(host_ptr), nbytes))

    def download(self, off: int, shape, dtype=np.float32) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        self._check(lib().moe_arena_download(self.h, off, out.ctypes.data_as(C.c_void_p), out.nbytes))
        return out

    def download_ptr(self, off: int, host_ptr: int, nbytes: int):
        self._check(lib().moe_arena_download(self.h, off, C.c_void_p(host_ptr), nbytes))

    def put(self, arr: np.ndarray, align: int = ALIGN) -> int:
        a = np.ascontiguousarray(arr)
        off = self.alloc(a.nbytes, align)
        self.upload(off, a)
        return off

    def ptr(self, off: int) -> int:
        p = C.c_void_p()
        self._check(lib().moe_arena_ptr(self.h, off, C.byref(p)))
        return p.value

    def set_stream(self, stream_handle: int | None):
        self._check(lib().moe_set_stream(self.h, C.c_void_p(stream_handle or 0)))

    def sync(self):
        self._check(lib().moe_sync(self.h))

    # -- layers -------------------------------------------------------------------------------
    def layer_create(self, spec: "LayerSpec", w1, w3, w2) -> int:
        c = spec.to_c()
        a1 = np.ascontiguousarray(w1, dtype=np.uint64)
        a3 = np.ascontiguousarray(w3, dtype=np.uint64)
        a2 = np.ascontiguousarray(w2, dtype=np.uint64)
        lid = C.c_uint32()
        self._check(lib().moe_layer_create(self.h, C.byref(c), _ptr(a1, C.c_uint64),
                                           _ptr(a3, C.c_uint64), _ptr(a2, C.c_uint64), C.byref(lid)))
        return lid.value

    def layer_set_next(self, layer: int, next_layer: int):
        self._check(lib().moe_layer_set_next(self.h, layer, next_layer))

    def reserve(self, layer: int, max_tokens: int):
        self._check(lib().moe_reserve(self.h, layer, max_tokens))

    # -- the path -----------------------------------------------------------------------------
    def route(self, layer: int, x_off: int, m: int, topk_off: int):
        self._check(lib().moe_route(self.h, layer, x_off, m, topk_off))

    def do_route(self, layer: int, x_off: int, m: int, k: int):
        routed = np.zeros((m, k), np.uint16)
        w = np.zeros((m, k), np.float32)
        g = np.zeros(m, np.float32)
        self._check(lib().moe_do_route(self.h, layer, x_off, m, _ptr(routed, C.c_uint16),
                                       _ptr(w, C.c_float), _ptr(g, C.c_float)))
        return routed, w, g

    def bucket(self, n_experts, top_k, has_shared, topk_off, m, ranges_off, tokens_off,
               weights_off, slot_pos_off):
        self._check(lib().moe_bucket(self.h, n_experts, top_k, int(has_shared), topk_off, m,
                                     ranges_off, tokens_off, weights_off, slot_pos_off))

    def forward(self, layer: int, x_off: int, resid_off: int, out_off: int, m: int):
        self._check(lib().moe_forward(self.h, layer, x_off, resid_off, out_off, m))

    def forward_host(self, layer: int, x_host_ptr: int, out_host_ptr: int, m: int, add_residual: bool = True):
        """Asynchronous forward from / to host memory (pointers to f32 [m][H]); results are in
        out_host after sync()."""
        self._check(lib().moe_forward_host(self.h, layer, C.c_void_p(x_host_ptr), C.c_void_p(out_host_ptr), m,
                                           int(add_residual)))

    def forward_norm(self, layer: int, x_off: int, out_off: int, m: int, eps: float = 1e-6):
        """out = x + MoE(RMSNorm(x)) (one step of the layer stack)."""
        self._check(lib().moe_forward_norm(self.h, layer, x_off, out_off, m, eps))

    def forward_routed(self, layer, x_off, resid_off, out_off, m, routed, weights, gate=None):
        r = np.ascontiguousarray(routed, np.uint16)
        w = np.ascontiguousarray(weights, np.float32)
        gp = None
        if gate is not None:
            g = np.ascontiguousarray(gate, np.float32)
            gp = _ptr(g, C.c_float)
        self._check(lib().moe_forward_routed(self.h, layer, x_off, resid_off, out_off, m,
                                             _ptr(r, C.c_uint16), _ptr(w, C.c_float), gp))

    def forward_topk(self, layer, x_off, resid_off, out_off, m, topk_off, flags=0):
        self._check(lib().moe_forward_topk(self.h, layer, x_off, resid_off, out_off, m, topk_off, flags))

    def ep_dispatch(self, n_experts, top_k, n_ranks, my_rank, capacity, topk_off, x_off, m, hidden,
                    plan_off, send_x_off, send_topk_off):
        self._check(lib().moe_ep_dispatch(self.h, n_experts, top_k, n_ranks, my_rank, capacity, topk_off,
                                          x_off, m, hidden, plan_off, send_x_off, send_topk_off))

    def ep_combine(self, n_ranks, capacity, hidden, m, plan_off, y_back_off, resid_off, out_off, scale):
        self._check(lib().moe_ep_combine(self.h, n_ranks, capacity, hidden, m, plan_off, y_back_off,
                                         resid_off, out_off, scale))

    def rms_norm(self, x_off, y_off, m, hidden, eps=1e-6):
        self._check(lib().moe_rms_norm(self.h, x_off, y_off, m, hidden, eps))

    def dequant(self, src_off, n_blocks, dst_off):
        self._check(lib().moe_dequant_iq4xs(self.h, src_off, n_blocks, dst_off))

    def dequant_ref36(self, src_off, n_blocks, dst_off):
        self._check(lib().moe_dequant_ref36(self.h, src_off, n_blocks, dst_off))

    def vocab_logits(self, w_off, vocab, hidden, x_off, m, logits_off=0, ids_off=0):
        """LM-head projection (moe_vocab_logits): f32 logits [m][vocab] and/or argmax ids [m]."""
        self._check(lib().moe_vocab_logits(self.h, w_off, vocab, hidden, x_off, m, logits_off, ids_off))

    # -- expert parallelism over NCCL (C level) --------------------------------------------------
    @staticmethod
    def ep_unique_id() -> bytes:
        """A new NCCL unique id (128 bytes) for moe_ep_init; made by rank 0, shared out of band."""
        buf = C.create_string_buffer(128)
        rc = lib().moe_ep_unique_id(buf, 128)
        if rc != 0:
            raise MoeError(rc, _err(None))
        return buf.raw

    def ep_init(self, unique_id: bytes, n_ranks: int, rank: int):
        buf = C.create_string_buffer(bytes(unique_id), 128)
        self._check(lib().moe_ep_init(self.h, buf, n_ranks, rank))

    def ep_set_transport(self, transport: int):
        self._check(lib().moe_ep_set_transport(self.h, transport))

    def ep_transport(self) -> int:
        v = C.c_int(0)
        self._check(lib().moe_ep_transport(self.h, C.byref(v)))
        return v.value

    def ep_abort(self):
        """Abort the group's communicator (a watchdog's call when a peer rank is lost)."""
        self._check(lib().moe_ep_abort(self.h))

    def forward_ep(self, layer_id, x_off, resid_off, out_off, m, capacity):
        self._check(lib().moe_forward_ep(self.h, layer_id, x_off, resid_off, out_off, m, capacity))

    def silu_mul(self, g_off, u_off, y_off, n):
        """y = silu(g) * u (u_off 0: y = silu(g)), n f32 values."""
        self._check(lib().moe_silu_mul(self.h, g_off, u_off, y_off, n))

    def synth_iq4xs(self, dst_off, key, block_start, n_blocks):
        self._check(lib().moe_synth_iq4xs(self.h, dst_off, key, block_start, n_blocks))

    # -- tracing ------------------------------------------------------------------------------
    def profile(self, enable: bool):
        self._check(lib().moe_profile(self.h, int(enable)))

    def profile_read(self) -> dict:
        """{stage name: (calls, total device ms)} since the last moe_profile call."""
        arr = (StageStatC * 32)()
        n = C.c_int()
        self._check(lib().moe_profile_read(self.h, arr, 32, C.byref(n)))
        return {arr[i].name.decode(): (arr[i].calls, arr[i].total_ms) for i in range(min(n.value, 32))}

    def set_path(self, path: int):
        self._check(lib().moe_set_path(self.h, path))

    def launch_count(self) -> int:
        n = C.c_uint64()
        self._check(lib().moe_launch_count(self.h, C.byref(n)))
        return n.value


@dataclass
class LayerSpec:
    hidden: int = 2048
    inter: int = 512
    n_experts: int = 256
    top_k: int = 8
    flags: int = MOE_F_SHARED | MOE_F_SHARED_GATE
    scale: float = 1.0
    router_w: int = 0
    router_bias: int = 0
    shared_gate: int = 0
    shared_w1: int = 0
    shared_w3: int = 0
    shared_w2: int = 0

    def to_c(self) -> LayerSpecC:
        return LayerSpecC(self.hidden, self.inter, self.n_experts, self.top_k, self.flags,
                          self.scale, self.router_w, self.router_bias, self.shared_gate,
                          self.shared_w1, self.shared_w3, self.shared_w2)


@dataclass
class RoutingOutput:
    """src/router.rs:4-8: top-k expert ids and softmax weights of one token."""
    routed: np.ndarray
    weights: np.ndarray
    shared_id: int
    shared_weight: float = 1.0


@dataclass
class TensorRegistry:
    """Name -> arena offset (src/memory.rs:101-198); a missing name looks up as 0."""
    entries: dict = field(default_factory=dict)

    def add(self, name: str, off: int, size: int, ggml_type: int):
        self.entries[name] = (off, size, ggml_type)

    def lookup(self, name: str) -> int:
        e = self.entries.get(name)
        return e[0] if e else 0


GGML_F32 = 0
GGML_IQ4_XS = 23


@dataclass
class LayerWeights:
    """Per-layer offsets resolved from the registry (src/memory.rs:201-290); expert_w* are
    flat [layer * E + e] tables."""
    n_layers: int
    n_experts: int
    ffn_gate: list
    shared_w1: list
    shared_w2: list
    shared_w3: list
    shared_gate: list
    router_bias: list
    expert_w1: list
    expert_w2: list
    expert_w3: list

    @classmethod
    def from_registry(cls, reg: TensorRegistry, n_layers: int, n_experts: int) -> "LayerWeights":
        lk = reg.lookup
        f = lambda pat: [lk(pat.format(l)) for l in range(n_layers)]  # noqa: E731
        ew = lambda w: [lk(f"blk.{l}.experts.{e}.{w}.weight")  # noqa: E731
                        for l in range(n_layers) for e in range(n_experts)]
        return cls(n_layers, n_experts, f("blk.{}.ffn_gate.weight"),
                   f("blk.{}.shared_expert.w1.weight"), f("blk.{}.shared_expert.w2.weight"),
                   f("blk.{}.shared_expert.w3.weight"), f("blk.{}.shared_expert.gate.weight"),
                   f("blk.{}.ffn_gate.bias"), ew("w1"), ew("w2"), ew("w3"))

    def expert_tables(self, layer: int):
        s = slice(layer * self.n_experts, (layer + 1) * self.n_experts)
        return self.expert_w1[s], self.expert_w3[s], self.expert_w2[s]


def build_synthetic_model(ctx: Context, seed: int, n_layers: int = 1,
                          shapes: synth.LayerShapes | None = None, zipf_s: float | None = None,
                          flags: int = MOE_F_SHARED | MOE_F_SHARED_GATE, scale: float = 1.0,
                          experts: range | None = None):
    """Place a seeded synthetic model in the arena (weights generated on the device), register
    every tensor by its GGUF-style name and create one library layer per model layer.

    ``experts``: the routed experts this context holds (an expert-parallel rank); the others
    get no weights and the layers are created with MOE_F_EXPERT_SUBSET.

    Returns (registry, LayerWeights, [layer ids])."""
    sh = shapes or synth.LayerShapes()
    reg = TensorRegistry()
    E, H, I = sh.n_experts, sh.hidden, sh.inter
    b13, b2 = sh.w13_bytes, sh.w2_bytes

    def synth_matrix(name, layer, expert, mat, rows, cols):
        nbytes = synth.matrix_bytes(rows, cols)
        off = ctx.alloc(nbytes)
        key = synth.tensor_key(seed, layer, expert, mat)
        ctx.synth_iq4xs(off, key, 0, nbytes // synth.IQ4XS_BLOCK_BYTES)
        reg.add(name, off, nbytes, GGML_IQ4_XS)

    for l in range(n_layers):
        wr, g, bias = synth.float_tensors(seed, l, sh, zipf_s)
        reg.add(f"blk.{l}.ffn_gate.weight", ctx.put(wr), wr.nbytes, GGML_F32)
        if flags & MOE_F_SHARED_GATE:
            reg.add(f"blk.{l}.shared_expert.gate.weight", ctx.put(g), g.nbytes, GGML_F32)
        if bias is not None:
            reg.add(f"blk.{l}.ffn_gate.bias", ctx.put(bias), bias.nbytes, GGML_F32)
        if flags & MOE_F_SHARED:
            synth_matrix(f"blk.{l}.shared_expert.w1.weight", l, E, synth.W1, I, H)
            synth_matrix(f"blk.{l}.shared_expert.w3.weight", l, E, synth.W3, I, H)
            synth_matrix(f"blk.{l}.shared_expert.w2.weight", l, E, synth.W2, H, I)
        for e in (range(E) if experts is None else experts):
            synth_matrix(f"blk.{l}.experts.{e}.w1.weight", l, e, synth.W1, I, H)
            synth_matrix(f"blk.{l}.experts.{e}.w3.weight", l, e, synth.W3, I, H)
            synth_matrix(f"blk.{l}.experts.{e}.w2.weight", l, e, synth.W2, H, I)
    lw = LayerWeights.from_registry(reg, n_layers, E)
    if experts is not None:
        flags |= MOE_F_EXPERT_SUBSET
    ids = []
    for l in range(n_layers):
        spec = LayerSpec(H, I, E, sh.top_k, flags, scale, lw.ffn_gate[l], lw.router_bias[l],
                         lw.shared_gate[l], lw.shared_w1[l], lw.shared_w3[l], lw.shared_w2[l])
        w1, w3, w2 = lw.expert_tables(l)
        ids.append(ctx.layer_create(spec, w1, w3, w2))
    return reg, lw, ids


class MoeEngine:
    """The MoE half of InferenceEngine (src/inference.rs:60-766) over the library.

    Holds hidden ping/pong buffers in the arena like ArenaLayout (hidden_ping/hidden_pong) and
    exposes the reference's two calls: ``do_route`` and ``record_and_submit_moe``."""

    def __init__(self, ctx: Context, layer_ids, shapes: synth.LayerShapes, max_tokens: int):
        self.ctx, self.layers, self.sh = ctx, list(layer_ids), shapes
        nbytes = max_tokens * shapes.hidden * 4
        self.hidden_ping = ctx.alloc(nbytes)
        self.hidden_pong = ctx.alloc(nbytes)
        self.max_tokens = max_tokens
        for lid in self.layers:
            ctx.reserve(lid, max_tokens)

    def hi(self, ping: bool) -> int:
        return self.hidden_ping if ping else self.hidden_pong

    def ho(self, ping: bool) -> int:
        return self.hidden_pong if ping else self.hidden_ping

    def do_route(self, layer: int, m: int, ping: bool = True):
        """Router + softmax + top-k on the device, RoutingOutput rows back on the host."""
        routed, w, g = self.ctx.do_route(self.layers[layer], self.hi(ping), m, self.sh.top_k)
        return [RoutingOutput(routed[t].copy(), w[t].copy(), self.sh.n_experts, float(g[t]))
                for t in range(m)]

    def record_and_submit_moe(self, layer: int, routing, m: int, ping: bool):
        """Experts + combine for the routed tokens in hi(ping); result in ho(ping) with the
        residual hi(ping) added; waits for completion (the reference's fence wait)."""
        if len(routing) != m:
            raise MoeError(-1, f"routing has {len(routing)} rows for {m} tokens")
        routed = np.stack([r.routed for r in routing]).astype(np.uint16)
        w = np.stack([r.weights for r in routing]).astype(np.float32)
        g = np.array([r.shared_weight for r in routing], np.float32)
        hi, ho = self.hi(ping), self.ho(ping)
        self.ctx.forward_routed(self.layers[layer], hi, hi, ho, m, routed, w, g)
        self.ctx.sync()
