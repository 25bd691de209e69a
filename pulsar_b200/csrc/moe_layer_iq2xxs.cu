/* moe_layer_iq2xxs.cu - the fused layer's expert passes (stream-K dp4a and
 * tensor-core tiles) for routed experts in IQ2_XXS, with each shared-expert
 * format; see pm_layer.cuh. */
#include "pm_layer.cuh"

PM_LAYER_FOR_QR(pm_layer_iq2xxs, PM_QUANT_IQ2_XXS)
