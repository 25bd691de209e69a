"""CPU-side checks of the C-ABI boundary (no kernel launches): the library
loads, exports every entry point include/pulsar_moe.h declares, keeps the
reference's struct layouts, and rejects invalid arguments with 0 before
touching the device (cu:25-29 / klib:212-218 convention)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pulsar_moe.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(?:int|size_t|uint32_t|uint64_t)\s+(pulsar_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    import pulsar_b200
    pulsar_b200.build()
    return pulsar_b200.lib()


def test_exports_every_declared_symbol(L):
    names = declared()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(ROOT, "pulsar_b200", "libpulsar_moe.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (pulsar_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert hasattr(L, n)


def test_struct_layouts(L):
    from pulsar_b200 import ExpertPtrs, LayerDesc
    assert ctypes.sizeof(ExpertPtrs) == 48  # cu:2555-2563
    src = '#include "pulsar_moe.h"\n#include <stdio.h>\n#include <stddef.h>\nint main(){printf("%zu %zu %zu",' \
          'sizeof(pulsar_moe_layer_desc), offsetof(pulsar_moe_layer_desc, shared_gate), sizeof(pulsar_expert_ptrs));}'
    exe = os.path.join("/tmp", "pm_layout_probe")
    subprocess.run(["gcc", "-x", "c", "-", "-I", os.path.dirname(HEADER), "-o", exe], input=src, text=True,
                   check=True)
    size, off, ep = map(int, subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split())
    assert size == ctypes.sizeof(LayerDesc) and off == LayerDesc.shared_gate.offset and ep == 48


def test_invalid_arguments_return_zero(L):
    # each call fails argument validation before any CUDA call
    assert L.pulsar_moe_pair_swiglu(None, None, None, None, 2048, 512, 8, 0, 1152, 2, 0) == 0
    assert L.pulsar_moe_down(1, 1, 1, 512, 2048, 8, 1, 288, 5) == 0          # unsupported quant code (Q3_K)
    assert L.pulsar_moe_down(1, 1, 1, 500, 2048, 8, 1, 288, 2) == 0          # Q4_K needs whole super-blocks
    assert L.pulsar_moe_pair_swiglu(1, 1, 1, 1, 2048, 512, 8, 1, 100, 2, 0) == 0  # row_bytes too small
    assert L.pulsar_router_select(1, 1, 1, 1, 64, 65, 1.0, 1, 0, 0) == 0     # k > n_expert
    assert L.pulsar_router_select(1, 1, 1, 1, 64, 8, 1.0, 1, 1, 2) == 0      # n_shexp outside mode 2
    assert L.pulsar_quantize_q8_K(1, 1, 0, 1) == 0
    assert L.pulsar_moe_slot_sum(1, 1, 0, 8, 1) == 0
    assert L.pulsar_moe_pair_swiglu_grouped(1, 1, 1, 1, 1, 1, 2048, 512, 17, 4, 1152, 2, 0) == 0  # k > 16
    assert L.pulsar_quantize_rows(1, 1, None, 2, 4, 300, None) == 0          # Q4_K row not 256-multiple


def test_layer_descriptor_validation(L):
    from pulsar_b200 import LayerDesc
    d = LayerDesc()
    assert L.pulsar_moe_layer_workspace(ctypes.byref(d), 8) == 0
    d.n_embd, d.n_ff, d.n_expert, d.n_used, d.quant = 2048, 512, 256, 8, 2
    d.row_bytes_gu, d.row_bytes_down = 1152, 288
    d.gate = d.up = d.down = d.router_w = 1
    ws = L.pulsar_moe_layer_workspace(ctypes.byref(d), 8)
    assert ws > 8 * 9 * 512 * 4
    d.n_used = 300
    assert L.pulsar_moe_layer_workspace(ctypes.byref(d), 8) == 0
    d.n_used = 8
    d.router_mode = 2  # the sink mode is not a layer mode
    assert L.pulsar_moe_layer(ctypes.byref(d), 1, 1, None, 1, 1, 1 << 30, None) == 0


def test_row_bytes_match_block_layouts(L):
    # gguf/src/lib.rs:145-170 block sizes
    from pulsar_b200 import row_bytes
    assert row_bytes(2, 2048) == 8 * 144 and row_bytes(0, 4096) == 16 * 84
    assert row_bytes(1, 7168) == 28 * 66 and row_bytes(12, 2880) == 90 * 17 and row_bytes(10, 7168) == 224 * 34


def test_workspace_tensor_core_images(L):
    """Calls of >= 192 tokens carry the tensor-core operand images: the
    expanded weights of the experts that can reach 192 tokens (fp16 hi + lo,
    4 B per weight of gate, up) and the token images; the weight-image region
    is bounded (more experts run in waves)."""
    from pulsar_b200 import LayerDesc
    d = LayerDesc()  # C3 shapes: H 2880, F 2880, 32 MXFP4 experts, top-4
    d.n_embd, d.n_ff, d.n_expert, d.n_used, d.quant, d.router_mode = 2880, 2880, 32, 4, 12, 1
    d.row_bytes_gu = d.row_bytes_down = 90 * 17
    d.gate = d.up = d.down = d.router_w = 1
    below, at = L.pulsar_moe_layer_workspace(ctypes.byref(d), 191), L.pulsar_moe_layer_workspace(ctypes.byref(d), 192)
    per_expert = 2 * 23 * 45 * 2 * 16384  # gate + up, 23 row blocks x 45 K chunks, hi + lo images
    assert at - below >= 4 * per_expert   # 192 x 4 / 192 = 4 experts can reach the threshold
    assert L.pulsar_moe_layer_workspace(ctypes.byref(d), 2048) >= 32 * per_expert
    e = LayerDesc()  # C5 shapes: 256 IQ2_XXS experts of H 7168, F 2048: 30 GB if every expert were expanded at once
    e.n_embd, e.n_ff, e.n_expert, e.n_used, e.quant, e.router_mode = 7168, 2048, 256, 8, 1, 0
    e.row_bytes_gu, e.row_bytes_down = 28 * 66, 8 * 66
    e.gate = e.up = e.down = e.router_w = 1
    assert L.pulsar_moe_layer_workspace(ctypes.byref(e), 4096) < (10 << 30)
