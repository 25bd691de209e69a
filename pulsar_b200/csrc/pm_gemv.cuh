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

/* shared-memory layout of one engine pass (computed on the host) */
struct pm_pass {
    uint32_t S;        /* ring stages per warp */
    uint32_t rw;       /* rows per stage */
    uint32_t stage;    /* bytes per stage */
    uint32_t lpr;      /* lanes per row (one lane per pair of units) */
    uint32_t off_bar;  /* PM_WARPS * S mbarriers */
    uint32_t off_acts; /* token-tile planes */
    uint32_t off_tok;  /* TT token-row pointers */
    uint32_t off_ring; /* PM_WARPS rings of S stages */
    uint32_t smem;     /* total dynamic shared memory */
};

/* copy one stage (rows of NMAT matrices) with 1-D bulk copies: each piece
 * is rounded out to 16-byte boundaries, so the staged byte at global
 * address g sits at dst + off(m) + (g & 15); returns expected bytes */
template <int NMAT>
__device__ __forceinline__ void pm_issue_stage(uint8_t *dst, uint64_t *bar, const uint8_t *const *src,
                                               uint32_t bytes) {
    uint32_t total = 0, len[NMAT];
    const uint8_t *lo[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        const uintptr_t s0 = (uintptr_t)src[m];
        lo[m] = (const uint8_t *)(s0 & ~(uintptr_t)15);
        len[m] = (uint32_t)(((s0 + bytes + 15u) & ~(uintptr_t)15) - (s0 & ~(uintptr_t)15));
        total += len[m];
    }
    pm_mbar_expect_tx(bar, total);
    uint32_t off = 0;
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        pm_bulk_g2s(dst + off, lo[m], len[m], bar);
        off += len[m] + 16u;
    }
}

template <int NMAT>
__device__ __forceinline__ const uint8_t *pm_stage_ptr(const uint8_t *dst, const uint8_t *const *src, uint32_t bytes,
                                                      int m) {
    uint32_t off = 0;
#pragma unroll
    for (int i = 0; i < NMAT; i++) {
        if (i == m) break;
        const uintptr_t s0 = (uintptr_t)src[i];
        off += (uint32_t)(((s0 + bytes + 15u) & ~(uintptr_t)15) - (s0 & ~(uintptr_t)15)) + 16u;
    }
    return dst + off + ((uintptr_t)src[m] & 15u);
}

/* quantize nt f32 rows of `n` values to q8_K (CPU-lane math, as
 * pm_q8k_warp) straight into the planes: one warp per (token, 256-block);
 * a lane holds 8 consecutive values = a quarter of one 32-value unit */
__device__ __forceinline__ void pm_acts_stage_f32(const pm_acts &a, uint32_t nt, const float *const *rows,
                                                  uint32_t n) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (uint32_t job = warp; job < nt * a.nblk; job += nw) {
        const uint32_t ti = job / a.nblk, b = job % a.nblk;
        const float *src = rows[ti] + (size_t)b * 256u;
        const uint32_t valid = n - b * 256u < 256u ? n - b * 256u : 256u;
        float v[8], amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t e = lane * 8u + (uint32_t)i;
            v[i] = e < valid ? __ldcg(src + e) : 0.0f;
            amax = fmaxf(amax, fabsf(v[i]));
        }
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        uint32_t qv[8];
        int s = 0;
        const float inv = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float r = amax == 0.0f ? 0.0f : roundf(__fmul_rn(v[i], inv));
            r = fminf(fmaxf(r, -127.0f), 127.0f);
            const int qi = (int)r;
            s += qi;
            qv[i] = (uint32_t)(uint8_t)(int8_t)qi;
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);    /* 16-value group sum (lane pair) */
        const int s_hi = __shfl_down_sync(0xffffffffu, s, 2); /* the unit's second group */
        const uint32_t u = b * 8u + (lane >> 2);
        if (u < a.n_units) {
            const uint32_t q = lane & 3u; /* quarter of the unit */
            uint32_t *dst = (uint32_t *)(q < 2 ? a.lo + ti * a.n_units + u : a.hi + ti * a.n_units + u);
            dst[(q & 1u) * 2u] = qv[0] | (qv[1] << 8) | (qv[2] << 16) | (qv[3] << 24);
            dst[(q & 1u) * 2u + 1u] = qv[4] | (qv[5] << 8) | (qv[6] << 16) | (qv[7] << 24);
            if (q == 0)
                a.bs[ti * a.n_units + u] = (int32_t)((uint32_t)(uint16_t)(int16_t)s | ((uint32_t)(uint16_t)(int16_t)s_hi << 16));
        }
        if (lane == 0) a.d[ti * a.nblk + b] = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
    }
}

/* Segment interface for pm_gemv_warps:
 *   const uint8_t* base(m)                 first row of the CTA's tile in matrix m
 *   uint32_t ntok()                         tokens of the work unit (<= TT)
 *   const pm_block_q8K* tok(ti)             q8_K row of token ti, or
 *   const float* tok_f32(ti)                its f32 row (Seg::F32 true: quantized while staging)
 *   void epi(row, ti, const float* v)       one lane per (row, token)
 *
 * Warp-private pipelines: after the token tile is staged (one CTA barrier),
 * warp w owns stages c = w, w + 8, ... of rw rows each and streams them
 * through its own S-deep ring and mbarriers; there is no CTA-wide
 * synchronisation while rows stream, so a warp waiting on memory never
 * holds the others back.  Returns false on a wait timeout (err set). */
template <int Q, int NMAT, int TT, class Seg>
__device__ bool pm_gemv_warps(Seg &seg, uint8_t *smem, const pm_pass &ps, uint32_t nrows, uint64_t rb,
                              uint32_t n_units, const uint64_t *grid, uint32_t *err) {
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t nt = seg.ntok() < (uint32_t)TT ? seg.ntok() : (uint32_t)TT;
    const pm_block_q8K **tokrows = (const pm_block_q8K **)(smem + ps.off_tok);
    uint64_t *bars = (uint64_t *)(smem + ps.off_bar) + warp * ps.S;
    uint8_t *ring = smem + ps.off_ring + (size_t)warp * ps.S * ps.stage;
    const pm_acts acts = pm_acts_carve(smem + ps.off_acts, TT, n_units);
    if constexpr (Seg::F32) {
        if (tid < nt) ((const float **)tokrows)[tid] = seg.tok_f32(tid);
    } else {
        if (tid < nt) tokrows[tid] = seg.tok(tid);
    }
    if (lane == 0) {
        for (uint32_t i = 0; i < ps.S; i++) pm_mbar_init(bars + i, 1);
        pm_fence_barrier_init();
    }
    __syncthreads();
    if constexpr (Seg::F32)
        pm_acts_stage_f32(acts, nt, (const float *const *)tokrows, seg.n_f32);
    else
        pm_acts_stage(acts, nt, tokrows);
    __syncthreads();

    const uint32_t rw = ps.rw, lpr = ps.lpr;
    const uint32_t n_stage_all = (nrows + rw - 1) / rw;
    const uint32_t mine = n_stage_all > warp ? (n_stage_all - warp + PM_WARPS - 1) / PM_WARPS : 0u;
    const uint32_t rows_per_pass = 32u / lpr;
    const uint32_t sub = lane / lpr, sl = lane % lpr;

    auto geom = [&](uint32_t i, const uint8_t **src, uint32_t &r0, uint32_t &rows) {
        r0 = (warp + PM_WARPS * i) * rw;
        rows = nrows - r0 < rw ? nrows - r0 : rw;
#pragma unroll
        for (int m = 0; m < NMAT; m++) src[m] = seg.base(m) + (size_t)r0 * rb;
    };
    if (lane == 0) {
        const uint32_t pro = mine < ps.S ? mine : ps.S;
        for (uint32_t i = 0; i < pro; i++) {
            const uint8_t *src[NMAT];
            uint32_t r0, rows;
            geom(i, src, r0, rows);
            pm_issue_stage<NMAT>(ring + (size_t)i * ps.stage, bars + i, src, rows * (uint32_t)rb);
        }
    }
    bool ok = true;
    for (uint32_t i = 0; i < mine; i++) {
        const uint32_t st = i % ps.S;
        if (!pm_mbar_wait_sleep(bars + st, (i / ps.S) & 1u, err)) {
            ok = false;
            if (lane == 0) { /* drain this warp's copies still in flight */
                const uint32_t last = i + ps.S - 1 < mine ? i + ps.S - 1 : mine - 1;
                for (uint32_t d = i; d <= last; d++) pm_mbar_wait(bars + (d % ps.S), (d / ps.S) & 1u, nullptr);
            }
            break;
        }
        const uint8_t *src[NMAT];
        uint32_t r0, rows;
        geom(i, src, r0, rows);
        const uint8_t *stg = ring + (size_t)st * ps.stage;
        const uint8_t *rowp[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; m++) rowp[m] = pm_stage_ptr<NMAT>(stg, src, rows * (uint32_t)rb, m);
        for (uint32_t jb = 0; jb < rows; jb += rows_per_pass) {
            const uint32_t j = jb + sub;
            const bool rv = j < rows;
            float acc[NMAT][TT];
#pragma unroll
            for (int m = 0; m < NMAT; m++)
#pragma unroll
                for (int t = 0; t < TT; t++) acc[m][t] = 0.0f;
            if (rv) {
                /* a lane takes a PAIR of adjacent units (same super-block:
                 * header and packed bytes load once for both) */
                for (uint32_t u0 = 2u * sl; u0 < n_units; u0 += 2u * lpr) {
                    const bool two = u0 + 1 < n_units;
                    pm_wunit wu[NMAT][2];
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        pm_decode<Q>(rowp[m] + (size_t)j * rb, u0, grid, wu[m][0]);
                        if (two) pm_decode<Q>(rowp[m] + (size_t)j * rb, u0 + 1, grid, wu[m][1]);
                    }
#pragma unroll
                    for (int t = 0; t < TT; t++) {
                        if (t < (int)nt) {
                            const float yd = acts.d[t * acts.nblk + (u0 >> 3)];
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                if (h == 1 && !two) break;
                                const uint32_t u = u0 + h;
                                const uint4 lo = acts.lo[t * n_units + u], hi = acts.hi[t * n_units + u];
                                int32_t bp = 0;
                                if (Q == PM_QUANT_Q4_K || Q == PM_QUANT_Q2_K) bp = acts.bs[t * n_units + u];
#pragma unroll
                                for (int m = 0; m < NMAT; m++) {
                                    const pm_wunit &wv = wu[m][h];
                                    int s0 = __dp4a(wv.w[0], (int)lo.x, 0);
                                    int s1 = __dp4a(wv.w[4], (int)hi.x, 0);
                                    s0 = __dp4a(wv.w[1], (int)lo.y, s0);
                                    s1 = __dp4a(wv.w[5], (int)hi.y, s1);
                                    s0 = __dp4a(wv.w[2], (int)lo.z, s0);
                                    s1 = __dp4a(wv.w[6], (int)hi.z, s1);
                                    s0 = __dp4a(wv.w[3], (int)lo.w, s0);
                                    s1 = __dp4a(wv.w[7], (int)hi.w, s1);
                                    float cv = wv.A * (float)(s0 + s1);
                                    if (Q == PM_QUANT_Q4_K || Q == PM_QUANT_Q2_K) {
                                        const int32_t msum = wv.ma * (int32_t)(int16_t)(bp & 0xffff) +
                                                             wv.mb * (int32_t)(int16_t)((uint32_t)bp >> 16);
                                        cv -= wv.B * (float)msum;
                                    }
                                    acc[m][t] = fmaf(yd, cv, acc[m][t]);
                                }
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
                for (uint32_t t = sl; t < nt; t += lpr) { /* lane sl writes token sl */
                    float v[NMAT];
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        float pick = 0.0f;
#pragma unroll
                        for (int q = 0; q < TT; q++)
                            if (q == (int)t) pick = acc[m][q];
                        v[m] = pick;
                    }
                    seg.epi(r0 + j, t, v);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + ps.S < mine) { /* refill the stage just consumed */
            pm_fence_proxy_async();
            const uint8_t *s2[NMAT];
            uint32_t r2, rows2;
            geom(i + ps.S, s2, r2, rows2);
            pm_issue_stage<NMAT>(ring + (size_t)st * ps.stage, bars + st, s2, rows2 * (uint32_t)rb);
        }
    }
    return __syncthreads_or(!ok) == 0;
}
