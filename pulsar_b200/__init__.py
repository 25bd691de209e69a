"""pulsar_b200: pulsar's routed-expert MoE FFN path, rebuilt for B200 (sm_100a).

The product is libpulsar_moe.so (pulsar_b200/csrc, C ABI in
include/pulsar_moe.h); this package is its host-side mirror of the
reference's FFI crate (crates/kernels/src/lib.rs) plus the layer builder.
"""
from ._lib import (LIB_PATH, QUANT_IQ2_XXS, QUANT_MXFP4, QUANT_Q2_K, QUANT_Q4_K, QUANT_Q8_0, QUANTS, ExpertPtrs,
                   KernelError, LayerDesc, abi_error, build, lib, row_bytes)
from .layer import LayerSpec, MoeLayer, make_layer, seeded_hidden

__all__ = ["LIB_PATH", "QUANT_IQ2_XXS", "QUANT_MXFP4", "QUANT_Q2_K", "QUANT_Q4_K", "QUANT_Q8_0", "QUANTS",
           "ExpertPtrs", "KernelError", "LayerDesc", "abi_error", "build", "lib", "row_bytes", "LayerSpec",
           "MoeLayer", "make_layer", "seeded_hidden"]
