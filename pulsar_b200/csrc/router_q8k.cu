/* router_q8k.cu - q8_K activation quantizer and the router (logits, top-k
 * selection, route weights) on sm_100a.
 *
 * Both are bit-exact with the CPU restatement of the reference:
 *  - q8_K follows the CPU lane's quantize_row_q8_k
 *    (crates/quant/src/cpu_dot.rs:26-50: d = amax/127, q = round half away
 *    from zero of x*127/amax, clamp +-127), not the reference GPU
 *    quantizer (cu:1498, signed-max iscale with rint), because the CPU
 *    lane's bytes are the parity target.  Layout: the reference's
 *    292-byte block_q8_K (cu:1492), tail elements beyond in_dim zero.
 *  - logits are an f32 fused-multiply-add dot in a fixed order (32 lane
 *    partials over i = 128 j + 4 lane + c, then an xor butterfly);
 *    selection scores use pm_expf, so top-k indices and route weights
 *    reproduce exactly on the host.
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "pm_host.h"
#include "pm_device.cuh"

/* ------------------------------------------------------------- q8_K */

/* one warp per 256-value block */
__global__ void pm_q8k_kernel(pm_block_q8K *out, const float *x, uint32_t in_dim, uint32_t n_rows) {
    const uint32_t nb = (in_dim + 255u) / 256u;
    const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= (uint64_t)nb * n_rows) return;
    const uint64_t row = gw / nb;
    const uint32_t b = (uint32_t)(gw % nb);
    const uint32_t bn = in_dim - b * 256u < 256u ? in_dim - b * 256u : 256u;
    pm_q8k_warp(x + row * in_dim + (uint64_t)b * 256u, bn, out + gw);
}

int pm_launch_q8k(void *out, const float *x, uint32_t in_dim, uint32_t n_rows, cudaStream_t st) {
    const uint64_t warps = (uint64_t)((in_dim + 255u) / 256u) * n_rows;
    const uint32_t blocks = (uint32_t)((warps * 32 + 255) / 256);
    pm_q8k_kernel<<<blocks, 256, 0, st>>>((pm_block_q8K *)out, x, in_dim, n_rows);
    return pm_ok(cudaGetLastError(), "q8_K quantize launch");
}

/* cu:1552 pulsar_quantize_q8_K */
extern "C" int pulsar_quantize_q8_K(void *out_dev, const void *x_dev, uint32_t in_dim, uint32_t n_rows) {
    if (!out_dev || !x_dev || in_dim == 0 || n_rows == 0) return 0;
    return pm_launch_q8k(out_dev, (const float *)x_dev, in_dim, n_rows, cudaStreamPerThread);
}

/* ----------------------------------------------------------- logits */

/* warp per (expert, token group of 4): f32 fma partials in the fixed
 * order, then the xor butterfly.  W rows may be any length; the float4
 * path needs in_dim % 4 == 0 (16-byte aligned rows). */
#define PM_RT_TOK 4
__global__ void __launch_bounds__(128) pm_router_logits_kernel(float *logits, const float *__restrict__ w,
                                                               const float *__restrict__ x,
                                                               const float *__restrict__ lbias, uint32_t n_expert,
                                                               uint32_t in_dim, uint32_t n_tok) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint32_t t0 = blockIdx.y * PM_RT_TOK;
    if (e >= n_expert) return;
    const uint32_t nt = n_tok - t0 < PM_RT_TOK ? n_tok - t0 : PM_RT_TOK;
    const float *wr = w + (uint64_t)e * in_dim;
    float p[PM_RT_TOK];
#pragma unroll
    for (int t = 0; t < PM_RT_TOK; t++) p[t] = 0.0f;
    const uint32_t nj = (in_dim + 127u) / 128u;
    if ((in_dim & 127u) == 0) {
        /* whole 128-wide chunks: four chunks of W and x in flight per step */
        uint32_t j = 0;
        for (; j + 4 <= nj; j += 4) {
            float4 wv[4], xv[4][PM_RT_TOK];
#pragma unroll
            for (int q = 0; q < 4; q++) wv[q] = __ldg((const float4 *)(wr + 128u * (j + q) + 4u * lane));
#pragma unroll
            for (int t = 0; t < PM_RT_TOK; t++)
#pragma unroll
                for (int q = 0; q < 4; q++)
                    xv[q][t] = (uint32_t)t < nt ? __ldg((const float4 *)(x + (uint64_t)(t0 + t) * in_dim +
                                                                          128u * (j + q) + 4u * lane))
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
                for (int t = 0; t < PM_RT_TOK; t++) {
                    p[t] = fmaf(wv[q].x, xv[q][t].x, p[t]);
                    p[t] = fmaf(wv[q].y, xv[q][t].y, p[t]);
                    p[t] = fmaf(wv[q].z, xv[q][t].z, p[t]);
                    p[t] = fmaf(wv[q].w, xv[q][t].w, p[t]);
                }
        }
        for (; j < nj; j++) {
            const float4 wv = __ldg((const float4 *)(wr + 128u * j + 4u * lane));
#pragma unroll
            for (int t = 0; t < PM_RT_TOK; t++) {
                if ((uint32_t)t >= nt) break;
                const float4 xv = __ldg((const float4 *)(x + (uint64_t)(t0 + t) * in_dim + 128u * j + 4u * lane));
                p[t] = fmaf(wv.x, xv.x, p[t]);
                p[t] = fmaf(wv.y, xv.y, p[t]);
                p[t] = fmaf(wv.z, xv.z, p[t]);
                p[t] = fmaf(wv.w, xv.w, p[t]);
            }
        }
    } else {
        for (uint32_t j = 0; j < nj; j++) {
            const uint32_t i0 = 128u * j + 4u * lane;
#pragma unroll
            for (int t = 0; t < PM_RT_TOK; t++) {
                if ((uint32_t)t >= nt) break;
                const float *xr = x + (uint64_t)(t0 + t) * in_dim;
#pragma unroll
                for (int c = 0; c < 4; c++)
                    if (i0 + c < in_dim) p[t] = fmaf(wr[i0 + c], xr[i0 + c], p[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < PM_RT_TOK; t++) {
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) p[t] = p[t] + __shfl_xor_sync(0xffffffffu, p[t], m);
    }
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < PM_RT_TOK; t++) {
            if ((uint32_t)t >= nt) break;
            float l = p[t];
            if (lbias) l = __fadd_rn(l, lbias[e]);
            logits[(uint64_t)(t0 + t) * n_expert + e] = l;
        }
    }
}

/* Token-tiled variant (in_dim % 128 == 0): a CTA stages TPB tokens' rows
 * of x in shared memory once, and its 8
 * warps each take one expert, so x is read from L2 and converted once
 * per 8 experts instead of once per expert.  Every (expert, token) dot
 * keeps the fixed order above (lane partials over i = 128 j + 4 lane + c,
 * j and c ascending, xor butterfly), so the bits equal the per-warp
 * kernel's.  With xq set, the CTAs of expert column 0 also write the
 * tile's q8_K rows (CPU-lane quantizer, pm_q8k_warp). */
/* EPW experts per warp: 1 for small batches (more CTAs), 4 for larger ones
 * (each x value read from shared memory serves 4 experts); G 128-wide W
 * chunks per expert are in flight per warp */
template <int TPB, int EPW>
__global__ void __launch_bounds__(256) pm_router_tile_kernel(float *logits, const float *__restrict__ w,
                                                             const float *__restrict__ x,
                                                             const float *__restrict__ lbias, uint32_t n_expert,
                                                             uint32_t in_dim, uint32_t n_tok, pm_block_q8K *xq,
                                                             uint32_t *ctl) {
    constexpr int G = EPW == 1 ? 8 : 2;
    extern __shared__ float4 xs[]; /* [TPB][32 nj]: rows padded with zeros to whole 128-wide chunks */
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t t0 = blockIdx.y * TPB;
    const uint32_t nt = n_tok - t0 < (uint32_t)TPB ? n_tok - t0 : (uint32_t)TPB;
    const uint32_t e0 = (blockIdx.x * (blockDim.x >> 5) + warp) * EPW;
    const uint32_t nj = (in_dim + 127u) / 128u;
    const bool tail = 128u * (nj - 1u) + 4u * lane < in_dim; /* this lane's float4 of the last chunk is real */
    const float *wr[EPW];
#pragma unroll
    for (int ee = 0; ee < EPW; ee++) wr[ee] = w + (uint64_t)(e0 + ee < n_expert ? e0 + ee : 0u) * in_dim;
    /* the first group of W chunks is in flight while x is staged */
    float4 wv[G][EPW];
#pragma unroll
    for (int q = 0; q < G; q++)
#pragma unroll
        for (int ee = 0; ee < EPW; ee++)
            wv[q][ee] = (uint32_t)q < nj && ((uint32_t)q + 1u < nj || tail)
                            ? __ldg((const float4 *)(wr[ee] + 128u * q + 4u * lane))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    /* the first kernel of a layer call clears the call's control words */
    if (ctl && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x < 2) ctl[threadIdx.x] = 0u;
    const uint32_t h4 = 32u * nj, r4 = in_dim / 4u;
    for (uint32_t i = threadIdx.x; i < nt * h4; i += blockDim.x)
        xs[i] = i % h4 < r4 ? __ldg((const float4 *)(x + (uint64_t)(t0 + i / h4) * in_dim) + i % h4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    if (xq && blockIdx.x == 0) {
        const uint32_t nb = (in_dim + 255u) / 256u;
        for (uint32_t job = warp; job < nt * nb; job += blockDim.x >> 5) {
            const uint32_t t = job / nb, b = job % nb;
            const uint32_t bn = in_dim - b * 256u < 256u ? in_dim - b * 256u : 256u;
            const float *src = x + (uint64_t)(t0 + t) * in_dim + b * 256u;
            pm_q8k_warp(src, bn, xq + (uint64_t)(t0 + t) * nb + b);
        }
    }
    __syncthreads();
    if (e0 >= n_expert) return;
    float p[EPW][TPB];
#pragma unroll
    for (int ee = 0; ee < EPW; ee++)
#pragma unroll
        for (int t = 0; t < TPB; t++) p[ee][t] = 0.0f; /* rows t >= nt hold stale data and are never written */
    for (uint32_t g = 0; g < nj; g += G) {
        float4 nx[G][EPW]; /* the next group, loaded while this one is used */
#pragma unroll
        for (int q = 0; q < G; q++) {
            const uint32_t jn = g + G + q;
#pragma unroll
            for (int ee = 0; ee < EPW; ee++)
                nx[q][ee] = jn < nj && (jn + 1u < nj || tail)
                                ? __ldg((const float4 *)(wr[ee] + 128u * jn + 4u * lane))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < G; q++) {
            const uint32_t j = g + q;
            if (j < nj && (j + 1u < nj || tail)) { /* indices past in_dim are skipped, as in the sequential order */
#pragma unroll
                for (int t = 0; t < TPB; t++) {
                    const float4 a = xs[t * h4 + 32u * j + lane];
#pragma unroll
                    for (int ee = 0; ee < EPW; ee++) {
                        p[ee][t] = fmaf(wv[q][ee].x, a.x, p[ee][t]);
                        p[ee][t] = fmaf(wv[q][ee].y, a.y, p[ee][t]);
                        p[ee][t] = fmaf(wv[q][ee].z, a.z, p[ee][t]);
                        p[ee][t] = fmaf(wv[q][ee].w, a.w, p[ee][t]);
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < G; q++)
#pragma unroll
            for (int ee = 0; ee < EPW; ee++) wv[q][ee] = nx[q][ee];
    }
#pragma unroll
    for (int ee = 0; ee < EPW; ee++)
#pragma unroll
        for (int t = 0; t < TPB; t++) {
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) p[ee][t] = p[ee][t] + __shfl_xor_sync(0xffffffffu, p[ee][t], m);
        }
    if (lane == 0) {
#pragma unroll
        for (int ee = 0; ee < EPW; ee++) {
            const uint32_t e = e0 + ee;
            if (e >= n_expert) break;
#pragma unroll
            for (int t = 0; t < TPB; t++) {
                if ((uint32_t)t >= nt) break;
                float l = p[ee][t];
                if (lbias) l = __fadd_rn(l, lbias[e]);
                logits[(uint64_t)(t0 + t) * n_expert + e] = l;
            }
        }
    }
}

template <int TPB, int EPW>
static int pm_launch_router_tile(float *logits, const float *w, const float *x, const float *lbias, uint32_t n_expert,
                                 uint32_t in_dim, uint32_t n_tok, pm_block_q8K *xq, uint32_t *ctl, cudaStream_t st) {
    static uint64_t done = 0;
    const uint32_t smem = TPB * ((in_dim + 127u) / 128u) * 512u;
    if (!pm_smem_attr(pm_router_tile_kernel<TPB, EPW>, smem, &done)) return 0;
    dim3 grid((n_expert + 8u * EPW - 1u) / (8u * EPW), (n_tok + TPB - 1) / TPB);
    pm_router_tile_kernel<TPB, EPW><<<grid, 256, smem, st>>>(logits, w, x, lbias, n_expert, in_dim, n_tok, xq, ctl);
    return pm_ok(cudaGetLastError(), "router logits launch");
}

/* logits (and, with xq, the q8_K rows of x) on stream st */
int pm_launch_router_logits_q8(float *logits, const float *w, const float *x, const float *lbias, uint32_t n_expert,
                               uint32_t in_dim, uint32_t n_tok, void *xq, uint32_t *ctl, cudaStream_t st) {
    if (in_dim % 4u == 0 && in_dim <= 25600u) {
        /* tokens per tile: no more than the batch, x tile (rows padded to 128) within 200 KB */
        const uint32_t row = ((in_dim + 127u) / 128u) * 512u;
        uint32_t tpb = n_tok >= 4 ? 4u : (n_tok >= 2 ? 2u : 1u);
        while (tpb > 1 && tpb * row > 200u * 1024u) tpb >>= 1;
        pm_block_q8K *q = (pm_block_q8K *)xq;
        if (tpb == 4 && n_tok >= 16) /* enough token tiles: 4 experts per warp */
            return pm_launch_router_tile<4, 4>(logits, w, x, lbias, n_expert, in_dim, n_tok, q, ctl, st);
        switch (tpb) {
        case 4: return pm_launch_router_tile<4, 1>(logits, w, x, lbias, n_expert, in_dim, n_tok, q, ctl, st);
        case 2: return pm_launch_router_tile<2, 1>(logits, w, x, lbias, n_expert, in_dim, n_tok, q, ctl, st);
        default: return pm_launch_router_tile<1, 1>(logits, w, x, lbias, n_expert, in_dim, n_tok, q, ctl, st);
        }
    }
    if (ctl && !pm_ok(cudaMemsetAsync(ctl, 0, 8, st), "layer control words")) return 0;
    dim3 grid((n_expert + 3u) / 4u, (n_tok + PM_RT_TOK - 1) / PM_RT_TOK);
    pm_router_logits_kernel<<<grid, 128, 0, st>>>(logits, w, x, lbias, n_expert, in_dim, n_tok);
    if (!pm_ok(cudaGetLastError(), "router logits launch")) return 0;
    return xq ? pm_launch_q8k(xq, x, in_dim, n_tok, st) : 1;
}

int pm_launch_router_logits(float *logits, const float *w, const float *x, const float *lbias, uint32_t n_expert,
                            uint32_t in_dim, uint32_t n_tok, cudaStream_t st) {
    return pm_launch_router_logits_q8(logits, w, x, lbias, n_expert, in_dim, n_tok, nullptr, nullptr, st);
}

/* cu:6526 pulsar_matmul_f32: out[t][r] = W[r] . x[t], here in the fixed
 * f32 order above (deterministic) */
extern "C" int pulsar_matmul_f32(void *out_dev, const void *w_dev, const void *x_dev, uint32_t in_dim,
                                 uint32_t out_dim, uint32_t n_tok) {
    if (!out_dev || !w_dev || !x_dev || in_dim == 0 || out_dim == 0 || n_tok == 0) return 0;
    return pm_launch_router_logits((float *)out_dev, (const float *)w_dev, (const float *)x_dev, nullptr, out_dim,
                                   in_dim, n_tok, cudaStreamPerThread);
}

#include "pm_router.cuh"

/* one warp per token; scores and probabilities staged in shared memory
 * (4 warps x 2 x n_expert floats) */
__global__ void pm_router_select_kernel(int32_t *selected, float *weights, const float *logits, const float *bias,
                                        uint32_t n_expert, uint32_t k_used, float weight_scale, uint32_t n_tok,
                                        uint32_t mode, uint32_t n_shexp, uint32_t n_group, uint32_t topk_group) {
    extern __shared__ float rs[];
    const uint32_t wid = threadIdx.x >> 5;
    const uint32_t token = blockIdx.x * (blockDim.x >> 5) + wid;
    if (token >= n_tok) return;
    float *score = rs + (size_t)wid * 2 * n_expert;
    pm_select_token(selected, weights, logits, bias, n_expert, k_used, weight_scale, token, mode, n_shexp, n_group,
                    topk_group, score, score + n_expert);
}

int pm_router_args_ok(uint32_t n_expert, uint32_t k_used, uint32_t n_tok, uint32_t mode, uint32_t n_shexp,
                      uint32_t n_group, uint32_t topk_group) {
    if (n_expert == 0 || k_used == 0 || k_used > n_expert || n_tok == 0 || mode > 2u) return 0;
    if (mode != 2u && n_shexp != 0) return 0;
    if (n_expert + (mode == 2u ? n_shexp : 0u) > 4096u) return 0;
    if (n_group > 1u) {
        if (n_group > 32u || n_expert % n_group || topk_group == 0 || topk_group > n_group || mode == 2u) return 0;
        if (n_expert / n_group < 2u) return 0;
        if ((uint64_t)(n_expert / n_group) * topk_group < k_used) return 0;
    }
    return 1;
}

int pm_launch_router_select(int32_t *sel, float *w, const float *logits, const float *bias, uint32_t n_expert,
                            uint32_t k_used, float scale, uint32_t n_tok, uint32_t mode, uint32_t n_shexp,
                            uint32_t n_group, uint32_t topk_group, cudaStream_t st) {
    const uint32_t smem = 4u * 2u * n_expert * 4u;
    static uint64_t done = 0;
    if (!pm_smem_attr(pm_router_select_kernel, smem, &done)) return 0;
    pm_router_select_kernel<<<(n_tok + 3u) / 4u, 128, smem, st>>>(sel, w, logits, bias, n_expert, k_used, scale,
                                                                  n_tok, mode, n_shexp, n_group, topk_group);
    return pm_ok(cudaGetLastError(), "router select launch");
}

/* cu:1052 pulsar_router_select (modes 0/1/2; n_expert up to 4096) */
extern "C" int pulsar_router_select(void *selected_dev, void *weights_dev, const void *logits_dev,
                                    const void *bias_dev, uint32_t n_expert, uint32_t k_used, float weight_scale,
                                    uint32_t n_tok, uint32_t softmax_mode, uint32_t n_shexp) {
    if (!selected_dev || !weights_dev || !logits_dev ||
        !pm_router_args_ok(n_expert, k_used, n_tok, softmax_mode, n_shexp, 0, 0))
        return 0;
    return pm_launch_router_select((int32_t *)selected_dev, (float *)weights_dev, (const float *)logits_dev,
                                   (const float *)bias_dev, n_expert, k_used, weight_scale, n_tok, softmax_mode,
                                   n_shexp, 0, 0, cudaStreamPerThread);
}

/* New entry point: logits + optional logit bias + group-limited top-k in
 * one call (router GEMV fused with selection).  No reference counterpart
 * as one call; equals pulsar_matmul_f32 + pulsar_add_bias_rows +
 * pulsar_router_select when n_group <= 1. */
extern "C" int pulsar_router_logits_select(void *selected_dev, void *weights_dev, void *logits_dev,
                                           const void *x_dev, const void *w_dev, const void *logit_bias_dev,
                                           const void *select_bias_dev, uint32_t in_dim, uint32_t n_expert,
                                           uint32_t k_used, float weight_scale, uint32_t n_tok, uint32_t mode,
                                           uint32_t n_group, uint32_t topk_group, void *stream) {
    if (!selected_dev || !weights_dev || !logits_dev || !x_dev || !w_dev || in_dim == 0 || mode == 2u ||
        !pm_router_args_ok(n_expert, k_used, n_tok, mode, 0, n_group, topk_group))
        return 0;
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    return pm_launch_router_logits((float *)logits_dev, (const float *)w_dev, (const float *)x_dev,
                                   (const float *)logit_bias_dev, n_expert, in_dim, n_tok, st) &&
           pm_launch_router_select((int32_t *)selected_dev, (float *)weights_dev, (const float *)logits_dev,
                                   (const float *)select_bias_dev, n_expert, k_used, weight_scale, n_tok, mode, 0,
                                   n_group, topk_group, st);
}
