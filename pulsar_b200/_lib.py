"""ctypes binding of libpulsar_moe.so, mirroring the reference's FFI crate.

crates/kernels/src/lib.rs binds the CUDA library from Rust: ExpertPtrs
(:21-48), the QUANT_* codes (:55-73), the extern block (:78-200) and the
`check(ret)` convention (:212-218, 1 = ok, 0 = error).  This module is the
same boundary for Python callers and the tests: every wrapper takes torch
CUDA tensors (plumbing only), passes raw device pointers to the C ABI and
raises KernelError when a call returns 0.  There is no CPU fallback: if
the shared library is missing, import fails loudly.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpulsar_moe.so")
_LIB = None

QUANT_Q2_K = 0
QUANT_IQ2_XXS = 1
QUANT_Q4_K = 2
QUANT_Q8_0 = 10
QUANT_MXFP4 = 12
QUANTS = {"Q2_K": QUANT_Q2_K, "IQ2_XXS": QUANT_IQ2_XXS, "Q4_K": QUANT_Q4_K, "Q8_0": QUANT_Q8_0,
          "MXFP4": QUANT_MXFP4}
Q8K_BLOCK_BYTES = 292
LAYER_NO_I8 = 1     # path_flags: routed Q2_K experts off the integer tensor cores
LAYER_FORCE_I8 = 2  # path_flags: routed Q2_K experts on the integer tensor cores below the default threshold


class KernelError(RuntimeError):
    """A pulsar_* call returned 0 (invalid arguments or a launch error)."""


class ExpertPtrs(ctypes.Structure):
    """pulsar_expert_ptrs / ExpertPtrs: 48 bytes, NULL = not routed."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("gate", "up", "down", "gate_b", "up_b", "down_b")]


class LayerDesc(ctypes.Structure):
    """pulsar_moe_layer_desc (include/pulsar_moe.h)."""
    _fields_ = [
        ("n_embd", ctypes.c_uint32), ("n_ff", ctypes.c_uint32), ("n_expert", ctypes.c_uint32),
        ("n_used", ctypes.c_uint32), ("quant", ctypes.c_uint32), ("act_op", ctypes.c_uint32),
        ("router_mode", ctypes.c_uint32), ("n_group", ctypes.c_uint32), ("topk_group", ctypes.c_uint32),
        ("weight_scale", ctypes.c_float),
        ("row_bytes_gu", ctypes.c_uint64), ("row_bytes_down", ctypes.c_uint64),
        ("expert_stride_gu", ctypes.c_uint64), ("expert_stride_down", ctypes.c_uint64),
        ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
        ("gate_b", ctypes.c_void_p), ("up_b", ctypes.c_void_p), ("down_b", ctypes.c_void_p),
        ("router_w", ctypes.c_void_p), ("router_logit_b", ctypes.c_void_p), ("router_select_b", ctypes.c_void_p),
        ("n_shared", ctypes.c_uint32), ("shared_quant", ctypes.c_uint32), ("shared_n_ff", ctypes.c_uint32),
        ("expert_lo", ctypes.c_uint32), ("expert_hi", ctypes.c_uint32),
        ("shared_row_bytes_gu", ctypes.c_uint64), ("shared_row_bytes_down", ctypes.c_uint64),
        ("shared_gate", ctypes.c_void_p), ("shared_up", ctypes.c_void_p), ("shared_down", ctypes.c_void_p),
        ("wait_cycles", ctypes.c_uint64), ("shared_gate_w", ctypes.c_void_p), ("path_flags", ctypes.c_uint32),
        ("gate_tiles", ctypes.c_void_p), ("up_tiles", ctypes.c_void_p), ("down_tiles", ctypes.c_void_p),
    ]


class WsView(ctypes.Structure):
    _fields_ = [("logits", ctypes.c_void_p), ("selected", ctypes.c_void_p), ("weights", ctypes.c_void_p),
                ("xq", ctypes.c_void_p), ("mid", ctypes.c_void_p),
                ("err", ctypes.c_void_p), ("n_items", ctypes.c_void_p), ("item_expert", ctypes.c_void_p),
                ("item_start", ctypes.c_void_p), ("pairs", ctypes.c_void_p), ("work_item", ctypes.c_void_p),
                ("work_t0", ctypes.c_void_p), ("partial", ctypes.c_void_p), ("tc_tile", ctypes.c_void_p),
                ("n_slot", ctypes.c_uint32), ("f_max", ctypes.c_uint32),
                ("tc_img", ctypes.c_void_p), ("tc_lo", ctypes.c_void_p), ("tc_slot_bytes", ctypes.c_uint64),
                ("tc_slots", ctypes.c_uint32), ("max_tc", ctypes.c_uint32)]


# (name, argtypes) of every C entry point, in header order
_P, _U32, _U64, _F = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float
_SIGS = {
    "pulsar_router_select": [_P, _P, _P, _P, _U32, _U32, _F, _U32, _U32, _U32],
    "pulsar_quantize_q8_K": [_P, _P, _U32, _U32],
    "pulsar_moe_pair_swiglu": [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _U64, _U32, _U32],
    "pulsar_moe_down": [_P, _P, _P, _U32, _U32, _U32, _U32, _U64, _U32],
    "pulsar_moe_pair_swiglu_grouped": [_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U64, _U32, _U32],
    "pulsar_moe_down_grouped": [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U64, _U32],
    "pulsar_moe_slot_sum": [_P, _P, _U32, _U32, _U32],
    "pulsar_moe_down_bias": [_P, _P, _P, _U32, _U32, _U32],
    "pulsar_add_bias_rows": [_P, _P, _U32, _U32],
    "pulsar_matmul_f32": [_P, _P, _P, _U32, _U32, _U32],
    "pulsar_swiglu": [_P, _P, _P, _U32, _F, _F, _U32],
    "pulsar_add": [_P, _P, _P, _U32],
    "pulsar_rms_norm": [_P, _P, _P, _U32, _U32, _F],
    "pulsar_rms_norm_stream": [_P, _P, _P, _U32, _U32, _F, _P],
    "pulsar_router_logits_select": [_P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _F, _U32, _U32, _U32, _U32, _P],
    "pulsar_moe_layer": [ctypes.POINTER(LayerDesc), _P, _P, _P, _U32, _P, ctypes.c_size_t, _P],
    "pulsar_moe_layer_profiled": [ctypes.POINTER(LayerDesc), _P, _P, _P, _U32, _P, ctypes.c_size_t, _P,
                                  ctypes.POINTER(ctypes.c_void_p)],
    "pulsar_moe_layer_ws_view": [ctypes.POINTER(LayerDesc), _U32, _P, ctypes.POINTER(WsView)],
    "pulsar_quantize_rows": [_P, _P, _P, _U32, _U64, _U32, _P],
    "pulsar_repack_q2k_tiles": [_P, _P, _U32, _U32, _U32, _U64, _U64, _P],
}


def build(force: bool = False) -> str:
    """Compile the CUDA library for sm_100a in-tree (nvcc; no GPU needed)."""
    csrc = os.path.join(_HERE, "csrc")
    if force:
        subprocess.run(["make", "-s", "-C", csrc, "clean"], check=True)
    subprocess.run(["make", "-s", "-j8", "-C", csrc], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run pulsar_b200.build() (nvcc, sm_100a) first; "
                              "there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        L.pulsar_moe_layer_workspace.argtypes = [ctypes.POINTER(LayerDesc), _U32]
        L.pulsar_moe_layer_workspace.restype = ctypes.c_size_t
        L.pulsar_moe_layer_ep_workspace.argtypes = [ctypes.POINTER(LayerDesc), _U32, _U32]
        L.pulsar_moe_layer_ep_workspace.restype = ctypes.c_size_t
        L.pulsar_moe_layer_ep.argtypes = [ctypes.POINTER(LayerDesc), _P, _U32, _U32, _P, _P, _P, _U32, _P,
                                          ctypes.c_size_t, _P]
        L.pulsar_moe_layer_ep.restype = ctypes.c_int
        L.pulsar_ep_unique_id.argtypes = [_P]
        L.pulsar_ep_comm_init.argtypes = [ctypes.POINTER(ctypes.c_void_p), _P, _U32, _U32]
        L.pulsar_ep_comm_destroy.argtypes = [_P]
        L.pulsar_row_bytes.argtypes = [_U32, _U32]
        L.pulsar_row_bytes.restype = _U64
        L.pulsar_b200_abi_error.argtypes = []
        L.pulsar_b200_abi_error.restype = _U32
        _LIB = L
    return _LIB


def check(ret: int, op: str) -> None:
    if ret == 0:
        raise KernelError(op)


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None passes through as NULL)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    assert t.is_cuda and t.is_contiguous(), "device tensors must be contiguous CUDA tensors"
    return t.data_ptr()


def row_bytes(quant: int, n: int) -> int:
    return int(lib().pulsar_row_bytes(quant, n))


def abi_error() -> int:
    return int(lib().pulsar_b200_abi_error())
