"""Tensor-level wrappers of the kernel entry points.

Names and argument order follow the reference's safe wrappers in
crates/kernels/src/lib.rs:1322-1450 (router_select, quantize_q8_k,
moe_pair_swiglu, moe_down, the grouped variants, moe_slot_sum,
moe_down_bias).  Each takes preallocated torch CUDA tensors as the
caller-owned device buffers and raises KernelError on a 0 return.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import ExpertPtrs, KernelError, Q8K_BLOCK_BYTES, check, lib, ptr

__all__ = [
    "q8k_bytes", "expert_ptrs_tensor", "router_select", "quantize_q8_k", "moe_pair_swiglu", "moe_down",
    "moe_pair_swiglu_grouped", "moe_down_grouped", "moe_slot_sum", "moe_down_bias", "add_bias_rows",
    "matmul_f32", "swiglu", "add", "rms_norm", "router_logits_select", "quantize_rows", "KernelError",
]


def q8k_bytes(dim: int, rows: int) -> int:
    return ((dim + 255) // 256) * Q8K_BLOCK_BYTES * rows


def expert_ptrs_tensor(records, device) -> torch.Tensor:
    """Pack a list of dicts/ExpertPtrs (gate, up, down, *_b as ints or tensors)
    into a device array of 48-byte records."""
    arr = (ExpertPtrs * len(records))()
    for i, r in enumerate(records):
        if r is None:
            continue
        for name in ("gate", "up", "down", "gate_b", "up_b", "down_b"):
            v = r.get(name) if isinstance(r, dict) else getattr(r, name)
            if v is not None:
                setattr(arr[i], name, v if isinstance(v, int) else v.data_ptr())
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return host.to(device)


def router_select(selected, weights, logits, bias, n_expert, k_used, weight_scale, n_tok, softmax_mode, n_shexp=0):
    check(lib().pulsar_router_select(ptr(selected), ptr(weights), ptr(logits), ptr(bias), n_expert, k_used,
                                     weight_scale, n_tok, softmax_mode, n_shexp), "router_select")


def quantize_q8_k(out, x, in_dim, n_rows):
    check(lib().pulsar_quantize_q8_K(ptr(out), ptr(x), in_dim, n_rows), "quantize_q8_K")


def moe_pair_swiglu(mid, ptrs, weights, xq, in_dim, mid_dim, n_used, n_tok, row_bytes, quant, act_op):
    check(lib().pulsar_moe_pair_swiglu(ptr(mid), ptr(ptrs), ptr(weights), ptr(xq), in_dim, mid_dim, n_used, n_tok,
                                       row_bytes, quant, act_op), "moe_pair_swiglu")


def moe_down(out, ptrs, midq, mid_dim, out_dim, n_used, n_tok, row_bytes, quant):
    check(lib().pulsar_moe_down(ptr(out), ptr(ptrs), ptr(midq), mid_dim, out_dim, n_used, n_tok, row_bytes, quant),
          "moe_down")


def moe_pair_swiglu_grouped(mid, gptrs, starts, pairs, weights, xq, in_dim, mid_dim, n_used, n_group, row_bytes,
                            quant, act_op):
    check(lib().pulsar_moe_pair_swiglu_grouped(ptr(mid), ptr(gptrs), ptr(starts), ptr(pairs), ptr(weights), ptr(xq),
                                               in_dim, mid_dim, n_used, n_group, row_bytes, quant, act_op),
          "moe_pair_swiglu_grouped")


def moe_down_grouped(partial, gptrs, starts, pairs, midq, mid_dim, out_dim, n_used, n_group, row_bytes, quant):
    check(lib().pulsar_moe_down_grouped(ptr(partial), ptr(gptrs), ptr(starts), ptr(pairs), ptr(midq), mid_dim,
                                        out_dim, n_used, n_group, row_bytes, quant), "moe_down_grouped")


def moe_slot_sum(out, partial, out_dim, n_used, n_tok):
    check(lib().pulsar_moe_slot_sum(ptr(out), ptr(partial), out_dim, n_used, n_tok), "moe_slot_sum")


def moe_down_bias(out, ptrs, weights, out_dim, n_used, n_tok):
    check(lib().pulsar_moe_down_bias(ptr(out), ptr(ptrs), ptr(weights), out_dim, n_used, n_tok), "moe_down_bias")


def add_bias_rows(x, bias, dim, rows):
    check(lib().pulsar_add_bias_rows(ptr(x), ptr(bias), dim, rows), "add_bias_rows")


def matmul_f32(out, w, x, in_dim, out_dim, n_tok):
    check(lib().pulsar_matmul_f32(ptr(out), ptr(w), ptr(x), in_dim, out_dim, n_tok), "matmul_f32")


def swiglu(out, gate, up, n, clamp=0.0, weight=1.0, act_op=0):
    check(lib().pulsar_swiglu(ptr(out), ptr(gate), ptr(up), n, clamp, weight, act_op), "swiglu")


def add(out, a, b, n):
    check(lib().pulsar_add(ptr(out), ptr(a), ptr(b), n), "add")


def rms_norm(out, x, w=None, eps=1e-6, stream=None):
    rows, n = x.shape
    s = torch.cuda.current_stream() if stream is None else stream
    check(lib().pulsar_rms_norm_stream(ptr(out), ptr(x), ptr(w), n, rows, eps, s.cuda_stream), "rms_norm")


def router_logits_select(selected, weights, logits, x, w, logit_bias, select_bias, in_dim, n_expert, k_used,
                         weight_scale, n_tok, mode, n_group=0, topk_group=0, stream=None):
    check(lib().pulsar_router_logits_select(ptr(selected), ptr(weights), ptr(logits), ptr(x), ptr(w),
                                            ptr(logit_bias), ptr(select_bias), in_dim, n_expert, k_used,
                                            weight_scale, n_tok, mode, n_group, topk_group,
                                            None if stream is None else stream.cuda_stream),
          "router_logits_select")


def quantize_rows(out, x, quant, qw=None, stream=None):
    """GPU block encoder: x f32 [rows][n] -> out u8 [rows][row_bytes]."""
    rows, n = x.shape
    s = torch.cuda.current_stream() if stream is None else stream
    check(lib().pulsar_quantize_rows(ptr(out), ptr(x), ptr(qw), quant, rows, n, s.cuda_stream), "quantize_rows")
