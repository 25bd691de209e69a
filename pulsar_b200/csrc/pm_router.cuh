/* pm_router.cuh - warp-level top-k selection and route weights shared by
 * the standalone router and the fused layer.  Semantics of
 * crates/kernels/cuda/pulsar_kernels.cu:939-1050 (router_select_kernel),
 * plus group-limited pre-selection; every float operation is an explicit
 * IEEE op so the CPU restatement reproduces the bits. */
#pragma once
#include "pm_device.cuh"

/* ----------------------------------------------------------- select */

__device__ __forceinline__ bool pm_better(float av, uint32_t ai, float bv, uint32_t bi) {
    return av > bv || (av == bv && ai < bi);
}

/* warp argmax over score[lo, hi) with the lower index winning ties */
__device__ __forceinline__ void pm_warp_argmax(const float *score, uint32_t lo, uint32_t hi, uint32_t skip,
                                               float &bv, uint32_t &bi) {
    const uint32_t lane = threadIdx.x & 31u;
    bv = -INFINITY;
    bi = UINT32_MAX;
    for (uint32_t e = lo + lane; e < hi; e += 32u) {
        if (e == skip) continue;
        if (pm_better(score[e], e, bv, bi)) {
            bv = score[e];
            bi = e;
        }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, m);
        if (pm_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
}

/* one warp per token; scores and probabilities staged in shared memory
 * (2 x n_expert floats per warp).  Semantics of cu:939-1050 plus the
 * group-limited pre-selection (n_group > 1). */
__device__ __forceinline__ void pm_select_token(int32_t *selected, float *weights, const float *logits,
                                                const float *bias, uint32_t n_expert, uint32_t k_used,
                                                float weight_scale, uint32_t token, uint32_t mode, uint32_t n_shexp,
                                                uint32_t n_group, uint32_t topk_group, float *score, float *prob,
                                                uint32_t out_stride = 0) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t sink = mode == 2u ? n_shexp : 0u;
    const uint32_t n_logit = n_expert + sink, n_slot = k_used + sink;
    const uint32_t stride = out_stride ? out_stride : n_slot; /* row stride of selected / weights */
    const float *lg = logits + (uint64_t)token * n_logit;
    int32_t *sel = selected + (uint64_t)token * stride;
    float *w = weights + (uint64_t)token * stride;
    for (uint32_t e = lane; e < n_expert; e += 32u) {
        const float raw = lg[e];
        const float p = mode == 1u ? raw : pm_sigmoid(raw);
        prob[e] = mode == 2u ? raw : p;
        score[e] = __fadd_rn(p, bias ? bias[e] : 0.0f);
    }
    __syncwarp();
    if (n_group > 1u && topk_group < n_group) {
        const uint32_t gs = n_expert / n_group;
        /* group scores: sum of the two best scores of each group */
        float gsc = -INFINITY; /* lane g holds group g's score (n_group <= 32) */
        for (uint32_t g = 0; g < n_group; g++) {
            float b1, b2;
            uint32_t i1, i2;
            pm_warp_argmax(score, g * gs, (g + 1) * gs, UINT32_MAX, b1, i1);
            pm_warp_argmax(score, g * gs, (g + 1) * gs, i1, b2, i2);
            if (lane == g) gsc = __fadd_rn(b1, b2);
        }
        uint32_t keep = 0;
        for (uint32_t r = 0; r < topk_group; r++) {
            float bv = lane < n_group && !((keep >> lane) & 1u) ? gsc : -INFINITY;
            uint32_t bi = lane < n_group && !((keep >> lane) & 1u) ? lane : UINT32_MAX;
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, m);
                if (pm_better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            keep |= 1u << bi;
        }
        for (uint32_t e = lane; e < n_expert; e += 32u)
            if (!((keep >> (e / gs)) & 1u)) score[e] = -INFINITY;
        __syncwarp();
    }
    float sum = 0.0f;
    for (uint32_t k = 0; k < k_used; k++) {
        float bv;
        uint32_t bi;
        pm_warp_argmax(score, 0, n_expert, UINT32_MAX, bv, bi);
        /* only NaN scores are left: the slot stays unrouted (-1, weight 0) */
        const float bp = bi < n_expert ? prob[bi] : 0.0f;
        __syncwarp();
        if (lane == 0) {
            sel[k] = bi < n_expert ? (int32_t)bi : -1;
            w[k] = bp;
            if (bi < n_expert) score[bi] = -INFINITY;
        }
        sum = __fadd_rn(sum, bp);
        __syncwarp();
    }
    if (lane == 0) {
        if (mode == 2u) {
            for (uint32_t s = 0; s < sink; s++) {
                sel[k_used + s] = (int32_t)(n_expert + s);
                w[k_used + s] = lg[n_expert + s];
            }
            float m = -INFINITY;
            for (uint32_t k = 0; k < n_slot; k++) {
                const float xv = w[k];
                w[k] = xv < 0.0f ? xv - log1pf(pm_expf(xv)) : -log1pf(pm_expf(-xv));
                m = fmaxf(m, w[k]);
            }
            float es = 0.0f;
            for (uint32_t k = 0; k < n_slot; k++) {
                w[k] = pm_expf(__fsub_rn(w[k], m));
                es = __fadd_rn(es, w[k]);
            }
            for (uint32_t k = 0; k < n_slot; k++) w[k] = __fmul_rn(__fdiv_rn(w[k], es), weight_scale);
        } else if (mode == 1u) {
            float m = -INFINITY;
            for (uint32_t k = 0; k < k_used; k++) m = fmaxf(m, w[k]);
            float es = 0.0f;
            for (uint32_t k = 0; k < k_used; k++) {
                w[k] = pm_expf(__fsub_rn(w[k], m));
                es = __fadd_rn(es, w[k]);
            }
            for (uint32_t k = 0; k < k_used; k++) w[k] = __fmul_rn(__fdiv_rn(w[k], es), weight_scale);
        } else {
            sum = fmaxf(sum, 6.103515625e-5f);
            for (uint32_t k = 0; k < k_used; k++) w[k] = __fmul_rn(__fdiv_rn(w[k], sum), weight_scale);
        }
    }
}

