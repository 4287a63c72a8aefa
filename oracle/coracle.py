"""ctypes front-end of the C oracle (oracle/moe_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may use this
module, as the checker or as the timed CPU restatement of the reference's MoE layer.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libmoe_oracle.so"
_lib = None


def build(force: bool = False) -> Path:
    src = HERE / "moe_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "-B" if force else "libmoe_oracle.so"], check=True,
                       capture_output=True)
    return LIB


class OracleLayerC(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32), ("inter", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32),
        ("has_shared", C.c_int32), ("has_gate", C.c_int32), ("scale", C.c_float),
        ("router_w", C.c_void_p), ("router_bias", C.c_void_p), ("gate_w", C.c_void_p),
        ("w1", C.c_void_p), ("w3", C.c_void_p), ("w2", C.c_void_p),
    ]


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        vp, i32, i64, u64 = C.c_void_p, C.c_int, C.c_int64, C.c_uint64
        L.oracle_dequant_iq4xs.argtypes = [vp, i64, vp]
        L.oracle_synth_iq4xs.argtypes = [vp, u64, u64, u64]
        L.oracle_route.argtypes = [C.POINTER(OracleLayerC), vp, i32, i32, vp, vp, vp, vp]
        L.oracle_bucket.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp, vp, vp, vp]
        L.oracle_moe_forward.argtypes = [C.POINTER(OracleLayerC), vp, vp, i32, i32, i32, vp, vp,
                                         vp, vp, vp]
        L.oracle_moe_forward.restype = i32
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def synth_iq4xs(key: int, block_start: int, n_blocks: int) -> np.ndarray:
    out = np.empty((n_blocks, 136), np.uint8)
    lib().oracle_synth_iq4xs(_p(out), key, block_start, n_blocks)
    return out


def dequant(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 136)
    out = np.empty((b.shape[0], 256), np.float32)
    lib().oracle_dequant_iq4xs(_p(b), b.shape[0], _p(out))
    return out


class HostLayer:
    """One MoE layer's tensors in host memory, laid out for the C oracle."""

    def __init__(self, hidden, inter, n_experts, top_k, router_w, bias, gate_w, experts,
                 shared=None, scale=1.0, has_gate=True):
        self.hidden, self.inter, self.n_experts, self.top_k = hidden, inter, n_experts, top_k
        self.router_w = np.ascontiguousarray(router_w, np.float32)
        self.bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.gate_w = None if gate_w is None else np.ascontiguousarray(gate_w, np.float32)
        self.experts = list(experts) + ([shared] if shared is not None else [experts[0]])
        self.has_shared = shared is not None
        self.has_gate = bool(has_gate and gate_w is not None and self.has_shared)
        self.scale = scale
        self._keep = [np.ascontiguousarray(m, np.uint8) for tr in self.experts for m in tr]
        n = len(self.experts)
        self.t1 = (C.c_void_p * n)(*[self._keep[3 * i + 0].ctypes.data for i in range(n)])
        self.t3 = (C.c_void_p * n)(*[self._keep[3 * i + 1].ctypes.data for i in range(n)])
        self.t2 = (C.c_void_p * n)(*[self._keep[3 * i + 2].ctypes.data for i in range(n)])

    def c(self) -> OracleLayerC:
        return OracleLayerC(self.hidden, self.inter, self.n_experts, self.top_k,
                            int(self.has_shared), int(self.has_gate), self.scale,
                            _p(self.router_w), _p(self.bias), _p(self.gate_w),
                            C.cast(self.t1, C.c_void_p), C.cast(self.t3, C.c_void_p),
                            C.cast(self.t2, C.c_void_p))


def route(layer: HostLayer, x: np.ndarray, acc64: bool = True):
    m = x.shape[0]
    x = np.ascontiguousarray(x, np.float32)
    ids = np.empty((m, layer.top_k), np.int32)
    w = np.empty((m, layer.top_k), np.float32)
    g = np.empty(m, np.float32)
    lg = np.empty((m, layer.n_experts), np.float32)
    c = layer.c()
    lib().oracle_route(C.byref(c), _p(x), m, int(acc64), _p(ids), _p(w), _p(g), _p(lg))
    return ids, w, g, lg


def bucket(ids, w, gate, n_experts, has_shared=True):
    m, k = ids.shape
    ns = k + (1 if has_shared else 0)
    S = m * ns
    ranges = np.empty(n_experts + 2, np.int32)
    tok = np.empty(S, np.int32)
    sw = np.empty(S, np.float32)
    pos = np.empty((m, ns), np.int32)
    ids = np.ascontiguousarray(ids, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    gate = None if gate is None else np.ascontiguousarray(gate, np.float32)
    lib().oracle_bucket(_p(ids), _p(w), _p(gate), m, n_experts, k, int(has_shared), _p(ranges),
                        _p(tok), _p(sw), _p(pos))
    return ranges, tok, sw, pos


def moe_forward(layer: HostLayer, x: np.ndarray, resid: np.ndarray | None, acc64: bool = True,
                nthreads: int = 0):
    m = x.shape[0]
    x = np.ascontiguousarray(x, np.float32)
    r = None if resid is None else np.ascontiguousarray(resid, np.float32)
    out = np.empty((m, layer.hidden), np.float32)
    out64 = np.empty((m, layer.hidden), np.float64)
    ids = np.empty((m, layer.top_k), np.int32)
    w = np.empty((m, layer.top_k), np.float32)
    g = np.empty(m, np.float32)
    c = layer.c()
    rc = lib().oracle_moe_forward(C.byref(c), _p(x), _p(r), m, int(acc64), nthreads, _p(out),
                                  _p(out64), _p(ids), _p(w), _p(g))
    if rc != 0:
        raise MemoryError("oracle_moe_forward failed")
    return dict(out=out, out64=out64, ids=ids, w=w, gate=g)


def synthetic_layer(seed: int, layer: int, shapes, zipf_s=None, has_shared=True, has_gate=True,
                    scale=1.0) -> HostLayer:
    """Host copy of the same seeded layer the device generator builds (moe-680m_b200/synth.py)."""
    import importlib.util
    import sys
    pkg = HERE.parent / "moe-680m_b200"
    if "moe680m_b200" not in sys.modules:
        spec = importlib.util.spec_from_file_location("moe680m_b200", pkg / "__init__.py",
                                                      submodule_search_locations=[str(pkg)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["moe680m_b200"] = mod
        spec.loader.exec_module(mod)
    from moe680m_b200 import synth
    sh = shapes
    wr, g, bias = synth.float_tensors(seed, layer, sh, zipf_s)
    nb13 = sh.w13_bytes // 136
    nb2 = sh.w2_bytes // 136

    def exp(e):
        return (synth_iq4xs(synth.tensor_key(seed, layer, e, synth.W1), 0, nb13),
                synth_iq4xs(synth.tensor_key(seed, layer, e, synth.W3), 0, nb13),
                synth_iq4xs(synth.tensor_key(seed, layer, e, synth.W2), 0, nb2))

    experts = [exp(e) for e in range(sh.n_experts)]
    shared = exp(sh.n_experts) if has_shared else None
    return HostLayer(sh.hidden, sh.inter, sh.n_experts, sh.top_k, wr, bias,
                     g if has_gate else None, experts, shared, scale, has_gate)
