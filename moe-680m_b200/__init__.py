"""moe-680m B200 MoE-layer path: Python host mirror of the reference's MoE engine interface.

The compute lives in the CUDA library ``lib/libmoe_b200.so`` (C ABI in include/moe_b200.h).
This package binds it with ctypes and mirrors, for Python callers and tests, the pieces of the
reference host that sit on the path (reference paths relative to the moe-680m tree):

* ``ArenaLayout``-style offsets: every tensor is a byte offset into one device arena, offset 0
  meaning "missing" (src/memory.rs:10-99);
* ``TensorRegistry`` / ``LayerWeights`` name -> offset tables (src/memory.rs:101-290);
* ``RoutingOutput`` (src/router.rs:4-8) and the engine methods ``do_route`` and
  ``record_and_submit_moe`` (src/inference.rs:622-766), in ``MoeEngine``.

There is no CPU fallback: if the library is missing, importing succeeds but every call raises.
"""
from .host import (  # noqa: F401
    MoeError, LibraryMissing, Context, LayerSpec, RoutingOutput, TensorRegistry, LayerWeights,
    MoeEngine, lib, MOE_F_SHARED, MOE_F_SHARED_GATE, build_synthetic_model,
)
