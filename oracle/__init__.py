"""ctypes binding of the CPU parity oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
the CPU-baseline leg of bench.py.  The product (pulsar_b200) never imports
this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

Q2_K, IQ2_XXS, Q4_K, Q8_0, MXFP4 = 0, 1, 2, 10, 12
Q8K_BYTES = 292


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        P, S, U32, U64, F = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float
        L.orc_quantize_rows.argtypes = [ctypes.c_int, P, S, S, P, P]
        L.orc_row_bytes.argtypes = [ctypes.c_int, U64]
        L.orc_row_bytes.restype = U64
        L.orc_dequant_row.argtypes = [ctypes.c_int, P, S, P]
        L.orc_quantize_q8k_rows.argtypes = [P, S, S, P]
        L.orc_vec_dot.argtypes = [ctypes.c_int, P, P, S]
        L.orc_vec_dot.restype = F
        L.orc_glu.argtypes = [F, F, U32]
        L.orc_glu.restype = F
        L.orc_router_logits.argtypes = [P, P, P, P, U32, U32, U32]
        L.orc_router_select.argtypes = [P, P, P, P, U32, U32, F, U32, U32, U32, U32, U32]
        L.orc_moe_ffn.argtypes = [P, P, P, P, P, U32, U32, U32, U32,
                                  U32, U32, U64, U64, U32, U32, U64, U64, U32, ctypes.c_int]
        L.orc_expf.argtypes = [F]
        L.orc_expf.restype = F
        L.orc_sigmoid.argtypes = [F]
        L.orc_sigmoid.restype = F
        L.orc_iq2xxs_grid.argtypes = [ctypes.c_int]
        L.orc_iq2xxs_grid.restype = U64
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def row_bytes(quant: int, n: int) -> int:
    return int(lib().orc_row_bytes(quant, n))


def quantize(quant: int, x: np.ndarray, qw: np.ndarray | None = None) -> np.ndarray:
    """rows x n f32 -> rows x row_bytes u8 (the crates/quant encoders)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    rows, n = x.shape
    rb = row_bytes(quant, n)
    out = np.zeros((rows, rb), np.uint8)
    q = None if qw is None else np.ascontiguousarray(qw, dtype=np.float32)
    ok = lib().orc_quantize_rows(quant, _p(x), rows, n, None if q is None else _p(q), _p(out))
    assert ok
    return out


def dequant(quant: int, row: np.ndarray, n: int) -> np.ndarray:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    out = np.zeros(n, np.float32)
    assert lib().orc_dequant_row(quant, _p(row), n, _p(out))
    return out


def quantize_q8k(x: np.ndarray) -> np.ndarray:
    """rows x n f32 -> rows x nblk x 292 bytes (q8_K, tail zero-padded)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    rows, n = x.shape
    nb = (n + 255) // 256
    out = np.zeros((rows, nb * Q8K_BYTES), np.uint8)
    lib().orc_quantize_q8k_rows(_p(x), n, rows, _p(out))
    return out


def q8k_fields(blocks: np.ndarray):
    """(d [nb], qs [nb,256] int8, bsums [nb,16] int16) of a q8_K byte array."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, Q8K_BYTES)
    d = b[:, 0:4].copy().view(np.float32).reshape(-1)
    qs = b[:, 4:260].copy().view(np.int8)
    bs = b[:, 260:292].copy().view(np.int16)
    return d, qs, bs


def vec_dot(quant: int, row: np.ndarray, xq: np.ndarray, n: int) -> float:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    return float(lib().orc_vec_dot(quant, _p(row), _p(xq), n))


def router_logits(w: np.ndarray, x: np.ndarray, logit_bias: np.ndarray | None = None) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    E, H = w.shape
    T = x.shape[0]
    out = np.zeros((T, E), np.float32)
    lb = None if logit_bias is None else np.ascontiguousarray(logit_bias, np.float32)
    lib().orc_router_logits(_p(out), _p(w), _p(x), None if lb is None else _p(lb), E, H, T)
    return out


def router_select(logits, bias, k, scale, mode, n_shexp=0, n_group=0, topk_group=0):
    logits = np.ascontiguousarray(logits, np.float32)
    T = logits.shape[0]
    E = logits.shape[1] - (n_shexp if mode == 2 else 0)
    n_slot = k + (n_shexp if mode == 2 else 0)
    sel = np.zeros((T, n_slot), np.int32)
    w = np.zeros((T, n_slot), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ok = lib().orc_router_select(_p(sel), _p(w), _p(logits), None if b is None else _p(b),
                                 E, k, scale, T, mode, n_shexp, n_group, topk_group)
    assert ok
    return sel, w


class ExpertPtrs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("gate", "up", "down", "gate_b", "up_b", "down_b")]


def moe_ffn(x, slots, w, H, n_routed, routed, shared=None, act_op=0, n_threads=0, return_mid=False):
    """Expert FFN of the CPU lane.

    x      [T][H] f32
    slots  list (len T) of lists (len n_slot) of dicts with numpy arrays
           'gate','up','down' (u8 rows, or None) and optional 'gate_b','up_b','down_b'
    w      [T][n_slot] f32 slot weights
    routed (F, quant, rb_gu, rb_down); shared likewise (or None)
    """
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    T = x.shape[0]
    n_slot = w.shape[1]
    arr = (ExpertPtrs * (T * n_slot))()
    keep = []
    for t in range(T):
        for s in range(n_slot):
            d = slots[t][s]
            e = arr[t * n_slot + s]
            for name in ("gate", "up", "down", "gate_b", "up_b", "down_b"):
                a = d.get(name) if d else None
                if a is not None:
                    a = np.ascontiguousarray(a)
                    keep.append(a)
                    setattr(e, name, a.ctypes.data)
    sh = shared or (0, 0, 0, 0)
    Fmax = max(routed[0], sh[0] if n_routed < n_slot else 0)
    out = np.zeros((T, H), np.float32)
    mid = np.zeros((T, n_slot, Fmax), np.float32) if return_mid else None
    ok = lib().orc_moe_ffn(_p(out), None if mid is None else _p(mid), ctypes.cast(arr, ctypes.c_void_p),
                           _p(w), _p(x), H, T, n_slot, n_routed,
                           routed[0], routed[1], routed[2], routed[3], sh[0], sh[1], sh[2], sh[3],
                           act_op, n_threads)
    assert ok
    return (out, mid) if return_mid else out
