"""CPU tests of the C-ABI boundary: the built library loads, exports every function the header
declares, and fails loudly (status + message, no crash) when no GPU is present; host-side
mirror logic (registry, LayerWeights) without a device."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from moe680m_b200 import host

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "moe_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert header_functions() == sorted(host.EXPORTS)


def test_library_exports_every_symbol():
    lib = C.CDLL(str(host.LIB_PATH))
    for name in header_functions():
        assert hasattr(lib, name), name
    assert host.lib().moe_abi_version() == 1


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_no_gpu_fails_loudly():
    with pytest.raises(host.MoeError) as ei:
        host.Context(0, 1 << 20)
    assert "device" in str(ei.value).lower() or "cuda" in str(ei.value).lower()


def test_null_context_calls_return_status():
    L = host.lib()
    assert L.moe_sync(None) == -1
    assert L.moe_forward(None, 0, 0, 0, 0, 1) == -1
    buf = C.create_string_buffer(64)
    assert L.moe_last_error(None, buf, 64) == 0


def test_layer_spec_layout():
    # the C struct: 5 x u32 + f32, then 6 x u64
    assert C.sizeof(host.LayerSpecC) == 24 + 6 * 8
    assert host.LayerSpecC.router_w.offset == 24


def test_registry_and_layer_weights():
    reg = host.TensorRegistry()
    off = 256
    for l in range(2):
        reg.add(f"blk.{l}.ffn_gate.weight", off, 16, host.GGML_F32); off += 256
        for e in range(4):
            for w in ("w1", "w2", "w3"):
                reg.add(f"blk.{l}.experts.{e}.{w}.weight", off, 16, host.GGML_IQ4_XS); off += 256
    lw = host.LayerWeights.from_registry(reg, 2, 4)
    assert lw.ffn_gate[1] == reg.lookup("blk.1.ffn_gate.weight")
    assert lw.shared_w1 == [0, 0]  # missing tensors resolve to the 0 sentinel
    w1, w3, w2 = lw.expert_tables(1)
    assert w1[2] == reg.lookup("blk.1.experts.2.w1.weight")
    assert len(w3) == 4 and len(w2) == 4


def test_ep_unique_id_without_gpu():
    """moe_ep_unique_id loads NCCL at run time and needs no device; a short buffer is rejected."""
    try:
        a = host.Context.ep_unique_id()
    except host.MoeError as e:
        pytest.skip(f"NCCL not loadable here: {e}")
    assert len(a) == 128 and a != host.Context.ep_unique_id()
    import ctypes
    assert host.lib().moe_ep_unique_id(ctypes.create_string_buffer(64), 64) == -1  # MOE_E_INVALID
