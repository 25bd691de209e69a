/* pm_gemv.cuh - expert-major decode GEMV engine (token-tile register
 * blocking), used by the fused layer.
 *
 * One CTA owns (expert work item, tile of R weight rows) of NMAT matrices
 * that share geometry (gate + up, or down).  The rows stream through an
 * S-stage shared-memory ring with 1-D TMA bulk copies (pm_stream.cuh
 * primitives).  The item's tokens are processed in tiles of TT: each
 * tile's q8_K activations are staged in shared memory once, split into two
 * 16-byte planes per 32-value unit so a warp's vector loads are
 * conflict-free.  Every 32-value weight unit is decoded ONCE into eight
 * int8x4 words plus a float scale pair, then dotted (dp4a) against all TT
 * tokens held in registers - the unpack cost is amortised over the tile.
 * Units of a row are spread over LPR lanes (32, or 16/8 for short rows so
 * no lane idles), partial sums reduce with shuffles, and the epilogue gets
 * one value per (row, token, matrix).
 *
 * Per-unit contribution (format math of cu:1582-2190 / cpu_dot.rs, with the
 * 16-value Q2_K scales folded into the int8 weights, q*sc <= 45):
 *   yd * (A * sumi - B * (ma * bsum_lo + mb * bsum_hi))
 */
#pragma once
#include "pm_stream.cuh"

struct pm_wunit {
    int32_t w[8];
    float A, B;
    int32_t ma, mb;
};

template <int Q>
__device__ __forceinline__ void pm_decode(const uint8_t *row, uint32_t u, const uint64_t *grid, pm_wunit &o) {
    const uint32_t sb = u >> 3, s = u & 7u;
    if constexpr (Q == PM_QUANT_Q4_K) {
        const uint8_t *b = row + sb * PM_Q4_K_BYTES;
        const uint4 hdr = *(const uint4 *)b;
        int scv, mnv;
        pm_k4_scale_min((int)s, b + 4, &scv, &mnv);
        const uint4 *qp = (const uint4 *)(b + 16 + 32 * (s >> 1));
        const uint4 q0 = qp[0], q1 = qp[1];
        const uint32_t raw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const int sh = (s & 1) * 4;
#pragma unroll
        for (int i = 0; i < 8; i++) o.w[i] = (int32_t)((raw[i] >> sh) & 0x0f0f0f0fu);
        o.A = pm_h2f(hdr.x & 0xffffu) * (float)scv;
        o.B = pm_h2f(hdr.x >> 16);
        o.ma = o.mb = mnv;
    } else if constexpr (Q == PM_QUANT_Q2_K) {
        const uint8_t *b = row + sb * PM_Q2_K_BYTES;
        const uint32_t *q = (const uint32_t *)(b + 16 + 32 * (s >> 2));
        const int sh = 2 * (s & 3);
        const uint32_t scw = *(const uint16_t *)(b + 2 * s);
        const uint32_t sc0 = scw & 15u, sc1 = (scw >> 8) & 15u;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t v = (q[i] >> sh) & 0x03030303u; /* 0..3 per byte */
            o.w[i] = (int32_t)(v * (i < 4 ? sc0 : sc1));   /* <= 45 per byte, no carry */
        }
        const uint32_t dd = *(const uint32_t *)(b + 80);
        o.A = pm_h2f(dd & 0xffffu);
        o.B = pm_h2f(dd >> 16);
        o.ma = (int32_t)((scw >> 4) & 15u);
        o.mb = (int32_t)(scw >> 12);
    } else if constexpr (Q == PM_QUANT_IQ2_XXS) {
        const uint16_t *h = (const uint16_t *)(row + sb * PM_IQ2_XXS_BYTES);
        const uint32_t aux0 = (uint32_t)h[1 + 4 * s] | ((uint32_t)h[2 + 4 * s] << 16);
        const uint32_t aux1 = (uint32_t)h[3 + 4 * s] | ((uint32_t)h[4 + 4 * s] << 16);
#pragma unroll
        for (int k = 0; k < 4; k++)
            pm_iq2_signed(grid[(aux0 >> (8 * k)) & 0xffu], pm_ksigns_dev((aux1 >> (7 * k)) & 127u), o.w[2 * k],
                          o.w[2 * k + 1]);
        o.A = 0.125f * pm_h2f(h[0]) * (float)(2u * (aux1 >> 28) + 1u);
        o.B = 0.0f;
        o.ma = o.mb = 0;
    } else if constexpr (Q == PM_QUANT_MXFP4) {
        const uint8_t *b = row + u * PM_MXFP4_BLOCK;
        uint32_t q[4];
        pm_lds_words<4>(b + 1, q);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            o.w[i] = pm_e2m1x4(q[i] & 0x0f0f0f0fu);
            o.w[4 + i] = pm_e2m1x4((q[i] >> 4) & 0x0f0f0f0fu);
        }
        o.A = pm_mxfp4_scale_half(b[0]);
        o.B = 0.0f;
        o.ma = o.mb = 0;
    } else if constexpr (Q == PM_QUANT_Q8_0) {
        const uint8_t *b = row + u * PM_Q8_0_BLOCK;
        uint32_t q[8];
        pm_lds_words<8>(b + 2, q);
#pragma unroll
        for (int i = 0; i < 8; i++) o.w[i] = (int32_t)q[i];
        o.A = pm_h2f(*(const uint16_t *)b);
        o.B = 0.0f;
        o.ma = o.mb = 0;
    }
}

/* staged activations of one token tile in shared memory:
 *   lo/hi planes: [TT][n_units] x 16 bytes; bs: [TT][n_units] (int16 pair); d: [TT][nblk] */
struct pm_acts {
    uint4 *lo, *hi;
    float *d;
    int32_t *bs;
    uint32_t n_units, nblk;
};

__host__ __device__ __forceinline__ uint32_t pm_acts_bytes(uint32_t TT, uint32_t n_units) {
    const uint32_t nblk = (n_units + 7) / 8;
    return TT * (n_units * 36u + nblk * 4u) + 64u;
}

__device__ __forceinline__ pm_acts pm_acts_carve(uint8_t *p, uint32_t TT, uint32_t n_units) {
    pm_acts a;
    a.n_units = n_units;
    a.nblk = (n_units + 7) / 8;
    a.lo = (uint4 *)p;
    a.hi = a.lo + TT * n_units;
    a.bs = (int32_t *)(a.hi + TT * n_units);
    a.d = (float *)(a.bs + TT * n_units);
    return a;
}

/* copy nt tokens' q8_K rows (292-byte blocks) into the planes; all threads */
__device__ __forceinline__ void pm_acts_stage(const pm_acts &a, uint32_t nt, const pm_block_q8K *const *rows) {
    const uint32_t words = a.n_units * 8u; /* int32 words of qs per token */
    for (uint32_t i = threadIdx.x; i < nt * words; i += blockDim.x) {
        const uint32_t ti = i / words, wdx = i % words;
        const uint32_t u = wdx >> 3, k = wdx & 7u;
        const int32_t v = __ldcg((const int32_t *)((const uint8_t *)(rows[ti] + (u >> 3)) + 4 + 32 * (u & 7u)) + k);
        int32_t *dst = (int32_t *)(k < 4 ? a.lo + ti * a.n_units + u : a.hi + ti * a.n_units + u);
        dst[k & 3u] = v;
    }
    for (uint32_t i = threadIdx.x; i < nt * a.n_units; i += blockDim.x) {
        const uint32_t ti = i / a.n_units, u = i % a.n_units;
        const pm_block_q8K *blk = rows[ti] + (u >> 3);
        a.bs[ti * a.n_units + u] = __ldcg((const int32_t *)((const uint8_t *)blk + 260 + 4 * (u & 7u)));
        if ((u & 7u) == 0) a.d[ti * a.nblk + (u >> 3)] = __ldcg(&blk->d);
    }
}

/* Segment interface for pm_gemv_tile:
 *   const uint8_t* base(m)                 first row of the CTA's tile in matrix m
 *   uint32_t ntok()                         tokens of the item
 *   const pm_block_q8K* tok(ti)             q8_K row of token ti
 *   void epi(row, ti, const float* v)       one lane per (row, token) */
template <int Q, int NMAT, int TT, class Seg>
__device__ bool pm_gemv_tile(Seg &seg, const pm_ring &ring, uint8_t *act_smem, const pm_block_q8K **tokrows,
                             uint32_t nrows, uint32_t rc, uint64_t rb, uint32_t n_units, uint32_t lpr,
                             const uint64_t *grid, uint32_t *err) {
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t n = seg.ntok();
    const uint32_t cps = (nrows + rc - 1) / rc;
    const pm_acts acts = pm_acts_carve(act_smem, TT, n_units);
    const uint32_t rows_per_warp = 32u / lpr;
    const uint32_t sub = lane / lpr, sl = lane % lpr; /* row slot in the warp, lane in the row */
    uint32_t issued = 0; /* chunks issued across token tiles (ring position) */
    for (uint32_t t0 = 0; t0 < n; t0 += TT) {
        const uint32_t nt = n - t0 < TT ? n - t0 : TT;
        if (tid < nt) tokrows[tid] = seg.tok(t0 + tid);
        __syncthreads();
        pm_acts_stage(acts, nt, tokrows);
        const uint32_t base_c = issued;
        if (tid == 0) {
            const uint32_t pro = cps < ring.S - 1 ? cps : ring.S - 1;
            for (uint32_t c = 0; c < pro; c++) {
                const uint8_t *src[NMAT];
                const uint32_t r0 = c * rc, rows = nrows - r0 < rc ? nrows - r0 : rc;
#pragma unroll
                for (int m = 0; m < NMAT; m++) src[m] = seg.base(m) + (size_t)r0 * rb;
                pm_issue_chunk<NMAT>(ring, base_c + c, src, rows * (uint32_t)rb);
            }
        }
        __syncthreads();
        for (uint32_t c = 0; c < cps; c++) {
            const uint32_t gc = base_c + c;
            if (tid == 0 && c + ring.S - 1 < cps) {
                const uint8_t *src[NMAT];
                const uint32_t cc = c + ring.S - 1;
                const uint32_t r0 = cc * rc, rows = nrows - r0 < rc ? nrows - r0 : rc;
#pragma unroll
                for (int m = 0; m < NMAT; m++) src[m] = seg.base(m) + (size_t)r0 * rb;
                pm_issue_chunk<NMAT>(ring, base_c + cc, src, rows * (uint32_t)rb);
            }
            const bool ok = pm_mbar_wait(ring.full + (gc % ring.S), (gc / ring.S) & 1u, err);
            if (__syncthreads_or(!ok)) {
                if (tid == 0) {
                    const uint32_t last = c + ring.S - 1 < cps ? c + ring.S - 1 : cps - 1;
                    for (uint32_t d = c; d <= last; d++)
                        pm_mbar_wait(ring.full + ((base_c + d) % ring.S), ((base_c + d) / ring.S) & 1u, nullptr);
                }
                __syncthreads();
                return false;
            }
            const uint32_t r0 = c * rc, rows = nrows - r0 < rc ? nrows - r0 : rc;
            const uint8_t *rowp[NMAT];
            {
                const uint8_t *src[NMAT];
#pragma unroll
                for (int m = 0; m < NMAT; m++) src[m] = seg.base(m) + (size_t)r0 * rb;
#pragma unroll
                for (int m = 0; m < NMAT; m++) rowp[m] = pm_chunk_ptr<NMAT>(ring, gc, src, rows * (uint32_t)rb, m);
            }
            for (uint32_t jb = warp * rows_per_warp; jb < rows; jb += PM_WARPS * rows_per_warp) {
                const uint32_t j = jb + sub;
                const bool rv = j < rows;
                float acc[NMAT][TT];
#pragma unroll
                for (int m = 0; m < NMAT; m++)
#pragma unroll
                    for (int t = 0; t < TT; t++) acc[m][t] = 0.0f;
                if (rv) {
                    for (uint32_t u = sl; u < n_units; u += lpr) {
#pragma unroll
                        for (int m = 0; m < NMAT; m++) {
                            pm_wunit wu;
                            pm_decode<Q>(rowp[m] + (size_t)j * rb, u, grid, wu);
#pragma unroll
                            for (int t = 0; t < TT; t++) {
                                if (t < (int)nt) {
                                    const uint4 lo = acts.lo[t * n_units + u], hi = acts.hi[t * n_units + u];
                                    int s = __dp4a(wu.w[0], (int)lo.x, 0);
                                    s = __dp4a(wu.w[1], (int)lo.y, s);
                                    s = __dp4a(wu.w[2], (int)lo.z, s);
                                    s = __dp4a(wu.w[3], (int)lo.w, s);
                                    s = __dp4a(wu.w[4], (int)hi.x, s);
                                    s = __dp4a(wu.w[5], (int)hi.y, s);
                                    s = __dp4a(wu.w[6], (int)hi.z, s);
                                    s = __dp4a(wu.w[7], (int)hi.w, s);
                                    const float yd = acts.d[t * acts.nblk + (u >> 3)];
                                    float cv = wu.A * (float)s;
                                    if (Q == PM_QUANT_Q4_K || Q == PM_QUANT_Q2_K) {
                                        const int32_t bp = acts.bs[t * n_units + u];
                                        const int32_t msum = wu.ma * (int32_t)(int16_t)(bp & 0xffff) +
                                                             wu.mb * (int32_t)(int16_t)((uint32_t)bp >> 16);
                                        cv -= wu.B * (float)msum;
                                    }
                                    acc[m][t] += yd * cv;
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < NMAT; m++)
#pragma unroll
                    for (int t = 0; t < TT; t++) {
                        if (t < (int)nt) {
                            float v = acc[m][t];
                            for (uint32_t o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                            acc[m][t] = v;
                        }
                    }
                if (rv) {
                    /* lane sl of the row writes token sl (spreads the epilogue) */
                    for (uint32_t t = sl; t < nt; t += lpr) {
                        float v[NMAT];
#pragma unroll
                        for (int m = 0; m < NMAT; m++) {
                            float pick = 0.0f;
#pragma unroll
                            for (int q = 0; q < TT; q++)
                                if (q == (int)t) pick = acc[m][q];
                            v[m] = pick;
                        }
                        seg.epi(r0 + j, t0 + t, v);
                    }
                }
            }
            __syncthreads();
        }
        issued += cps;
    }
    return true;
}
