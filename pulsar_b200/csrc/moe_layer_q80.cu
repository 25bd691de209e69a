/* moe_layer_q80.cu - the fused layer's expert passes (stream-K dp4a and
 * tensor-core tiles) for routed experts in Q8_0, with each shared-expert
 * format; see pm_layer.cuh. */
#include "pm_layer.cuh"

PM_LAYER_FOR_QR(pm_layer_q80, PM_QUANT_Q8_0)
