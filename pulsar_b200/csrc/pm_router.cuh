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


/* compare-exchange by (score desc, index asc) */
__device__ __forceinline__ void pm_cx(float &as, uint32_t &ai, float &bs, uint32_t &bi) {
    if (pm_better(bs, bi, as, ai)) {
        const float ts = as;
        const uint32_t ti = ai;
        as = bs, ai = bi;
        bs = ts, bi = ti;
    }
}

/* 8 pairs into descending order (Batcher odd-even merge sort, 19 exchanges) */
__device__ __forceinline__ void pm_sort8(float *s, uint32_t *i) {
#define PM_CX(a, b) pm_cx(s[a], i[a], s[b], i[b])
    PM_CX(0, 1); PM_CX(2, 3); PM_CX(4, 5); PM_CX(6, 7);
    PM_CX(0, 2); PM_CX(1, 3); PM_CX(4, 6); PM_CX(5, 7);
    PM_CX(1, 2); PM_CX(5, 6);
    PM_CX(0, 4); PM_CX(1, 5); PM_CX(2, 6); PM_CX(3, 7);
    PM_CX(2, 4); PM_CX(3, 5);
    PM_CX(1, 2); PM_CX(3, 4); PM_CX(5, 6);
#undef PM_CX
}

/* a (sorted desc) := the 8 best of a and b (both sorted desc), sorted desc:
 * a[i] vs b[7 - i] keeps the top 8 as a bitonic sequence, then a bitonic
 * merge of 8 */
__device__ __forceinline__ void pm_merge8(float *as, uint32_t *ai, const float *bs, const uint32_t *bi) {
#pragma unroll
    for (int k = 0; k < 8; k++)
        if (pm_better(bs[7 - k], bi[7 - k], as[k], ai[k])) as[k] = bs[7 - k], ai[k] = bi[7 - k];
#define PM_CX(a, b) pm_cx(as[a], ai[a], as[b], ai[b])
    PM_CX(0, 4); PM_CX(1, 5); PM_CX(2, 6); PM_CX(3, 7);
    PM_CX(0, 2); PM_CX(1, 3); PM_CX(4, 6); PM_CX(5, 7);
    PM_CX(0, 1); PM_CX(2, 3); PM_CX(4, 5); PM_CX(6, 7);
#undef PM_CX
}

/* Fast path of pm_select_token for the fused layer: modes 0 and 1, no group
 * limit, n_expert <= 256, k_used <= 32.  Same operations and tie rule as
 * pm_select_token (and the CPU restatement), so the same bits:
 *   - the lane's logits and biases are read with independent loads, the
 *     sigmoid loop stages scores / probabilities in shared memory and each
 *     lane then holds its 8 experts e = lane + 32 i in registers;
 *   - each round is one warp argmax over the lanes' local bests (ties -> lower
 *     index); only the winning lane marks its expert taken (-inf) and rescans
 *     its 8 registers;
 *   - the weight sums keep the sequential slot order; the divisions run on
 *     lanes 0..k-1 in parallel, and lane s writes slot s. */
__device__ __forceinline__ void pm_select_fast(int32_t *selected, float *weights, const float *logits,
                                               const float *bias, uint32_t n_expert, uint32_t k_used,
                                               float weight_scale, uint32_t token, uint32_t mode, float *score,
                                               float *prob, uint32_t out_stride) {
    const uint32_t lane = threadIdx.x & 31u;
    const float *lg = logits + (uint64_t)token * n_expert;
    float raw[8], bv8[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t e = lane + 32u * (uint32_t)i;
        raw[i] = e < n_expert ? __ldcg(lg + e) : 0.0f;
        bv8[i] = bias && e < n_expert ? __ldg(bias + e) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        score[lane + 32 * i] = raw[i];
        prob[lane + 32 * i] = bv8[i];
    }
    __syncwarp();
    for (uint32_t e = lane; e < 32u * 8u; e += 32u) { /* compact loop: sigmoid, score */
        const float r = score[e];
        const float p = mode == 1u ? r : pm_sigmoid(r);
        score[e] = __fadd_rn(p, prob[e]);
        prob[e] = p;
    }
    __syncwarp();
    float sc[8], pr[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t e = lane + 32u * (uint32_t)i;
        sc[i] = score[e];
        pr[i] = prob[e];
    }
    /* top-k by a warp merge when k <= 8 and at least k scores are finite (then the
     * rounds below would pick exactly the k best by (score desc, index asc), in that
     * order); otherwise the rounds, which also cover picks among -inf scores */
    if (k_used <= 8u) {
        float ks[8];
        uint32_t ki[8];
        uint32_t nfin = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t e = lane + 32u * (uint32_t)i;
            const bool ok = e < n_expert && sc[i] > -INFINITY; /* false for NaN */
            ks[i] = ok ? sc[i] : -INFINITY;
            ki[i] = ok ? e : UINT32_MAX;
            nfin += ok ? 1u : 0u;
        }
        for (int o = 16; o > 0; o >>= 1) nfin += __shfl_xor_sync(0xffffffffu, nfin, o);
        if (nfin >= k_used) {
            pm_sort8(ks, ki);
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) {
                float os[8];
                uint32_t oi[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    os[i] = __shfl_xor_sync(0xffffffffu, ks[i], m);
                    oi[i] = __shfl_xor_sync(0xffffffffu, ki[i], m);
                }
                pm_merge8(ks, ki, os, oi);
            }
            /* every lane holds the 8 best in pick order; lane s takes slot s */
            uint32_t e_s = UINT32_MAX;
#pragma unroll
            for (int i = 0; i < 8; i++)
                if ((uint32_t)i == lane) e_s = ki[i];
            float sum = 0.0f, bp_s = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if ((uint32_t)i >= k_used) break;
                const float bp = prob[ki[i]];
                if ((uint32_t)i == lane) bp_s = bp;
                sum = __fadd_rn(sum, bp);
            }
            float w;
            if (mode == 1u) {
                float m = lane < k_used ? bp_s : -INFINITY;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float ex = lane < k_used ? pm_expf(__fsub_rn(bp_s, m)) : 0.0f;
                float es = 0.0f;
                for (uint32_t s2 = 0; s2 < k_used; s2++) es = __fadd_rn(es, __shfl_sync(0xffffffffu, ex, s2));
                w = __fmul_rn(__fdiv_rn(ex, es), weight_scale);
            } else {
                w = __fmul_rn(__fdiv_rn(bp_s, fmaxf(sum, 6.103515625e-5f)), weight_scale);
            }
            if (lane < k_used) {
                selected[(uint64_t)token * out_stride + lane] = (int32_t)e_s;
                weights[(uint64_t)token * out_stride + lane] = w;
            }
            return;
        }
    }
    auto local_best = [&](float &bv, uint32_t &bi) {
        bv = -INFINITY;
        bi = UINT32_MAX;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t e = lane + 32u * (uint32_t)i;
            if (e < n_expert && pm_better(sc[i], e, bv, bi)) {
                bv = sc[i];
                bi = e;
            }
        }
    };
    float lbv;
    uint32_t lbi;
    local_best(lbv, lbi);
    float sum = 0.0f, myw = 0.0f;
    int32_t mysel = -1;
    for (uint32_t r = 0; r < k_used; r++) {
        float bv = lbv;
        uint32_t bi = lbi;
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, m);
            if (pm_better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        const bool hit = bi < n_expert;
        const bool owner = hit && (bi & 31u) == lane;
        float mine = 0.0f;
        if (owner) {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if ((uint32_t)i == (bi >> 5)) {
                    mine = pr[i];
                    sc[i] = -INFINITY;
                }
            local_best(lbv, lbi);
        }
        /* only NaN scores left: the slot stays unrouted (-1, weight 0) */
        const float bp = hit ? __shfl_sync(0xffffffffu, mine, bi & 31u) : 0.0f;
        if (lane == r) {
            mysel = hit ? (int32_t)bi : -1;
            myw = bp;
        }
        sum = __fadd_rn(sum, bp);
    }
    float w = myw;
    if (mode == 1u) {
        float m = lane < k_used ? myw : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float ex = lane < k_used ? pm_expf(__fsub_rn(myw, m)) : 0.0f;
        float es = 0.0f;
        for (uint32_t s = 0; s < k_used; s++) es = __fadd_rn(es, __shfl_sync(0xffffffffu, ex, s));
        w = __fmul_rn(__fdiv_rn(ex, es), weight_scale);
    } else {
        w = __fmul_rn(__fdiv_rn(myw, fmaxf(sum, 6.103515625e-5f)), weight_scale);
    }
    if (lane < k_used) {
        selected[(uint64_t)token * out_stride + lane] = mysel;
        weights[(uint64_t)token * out_stride + lane] = w;
    }
}
