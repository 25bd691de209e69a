/* moe_layer_mxfp4.cu - the fused layer's expert passes (stream-K dp4a and
 * tensor-core tiles) for routed experts in MXFP4, with each shared-expert
 * format; see pm_layer.cuh. */
#include "pm_layer.cuh"

PM_LAYER_FOR_QR(pm_layer_mxfp4, PM_QUANT_MXFP4)
