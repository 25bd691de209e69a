/* pm_gemv.cuh - stream-K decode engine of the fused layer (gate/up and down).
 *
 * Work.  The layer's selection kernel lists WORK UNITS: (expert, chunk of
 * <= PM_TT tokens routed to it).  A work unit multiplies every row of the
 * expert's matrices (gate+up: F rows of each; down: H rows) with its
 * tokens.  Rows of a unit cost roughly (PM_SK_CR + nt) token-dots each
 * (decode + nt dots), so the whole launch is a line of
 *     C = sum over units of rows(unit) * (PM_SK_CR + nt(unit))
 * cost units.  The kernel is persistent: CTA b of G takes the slice
 * [b*C/G, (b+1)*C/G) of that line, cut at row boundaries (multiples of
 * PM_SK_RQ), so every CTA gets the same amount of work whatever the
 * routing skew - there is no tail of half-empty waves.  A CTA's slice is a
 * short list of SEGMENTS (unit, row range).
 *
 * Streaming.  Each warp owns every 8th stage (rw rows of all NMAT
 * matrices) of the CTA's concatenated segments and streams them through
 * its own S-deep ring of 1-D TMA bulk copies on its own mbarriers, across
 * segment boundaries, so HBM stays busy while the CTA swaps token tiles.
 * The only CTA barriers are two per segment (token tile swap).
 *
 * Math.  A lane takes PAIRS of adjacent 32-value units of a row (same
 * 256-value super-block / q8_K block): the pair's weights are decoded once
 * into int8x4 words and dotted (dp4a) against each of the nt tokens; the
 * integer sums of the pair are combined in integer arithmetic with the
 * sub-block scales and mins before one float combination per (pair,
 * token).  NT (the token count, compile time) unrolls the token loop.  The
 * per-lane partial sums of a row are reduced with a shuffle
 * reduce-scatter, which leaves each (matrix, token) total in one lane.
 * Activation tiles are stored as four 16-byte planes per unit pair
 * ([plane][token][pair]) so a quarter-warp's vector loads never collide.
 *
 * Format math (crates/kernels/cuda/pulsar_kernels.cu dot functors q4_K
 * cu:1699, q2_K cu:1625, iq2_xxs cu:1582, mxfp4 cu:2053, q8_0 cu:2174;
 * crates/quant/src/cpu_dot.rs :92 :250 :732), regrouped per unit pair:
 *   Q4_K   yd * ((d/16) * (16 sc0 S0 + sc1 S1') - dmin * (m0 B0 + m1 B1))
 *          (S1' is the high-nibble dot taken on the nibbles in place, = 16 S1)
 *   Q2_K   yd * (d * (S0 + S1) - dmin * sum m16 * B16)   (16-value scales folded)
 *   IQ2    yd * (d/8) * ((2s0+1) S0 + (2s1+1) S1)
 *   MXFP4, Q8_0  yd * (d0 S0 + d1 S1)
 */
#pragma once
#include "pm_stream.cuh"

#define PM_TT 8       /* tokens per work unit (register tile) */
#define PM_SK_CR 2u   /* per-row decode cost, in token-dot units */
#define PM_SK_RQ 8u   /* slice boundaries fall on multiples of this many rows */
#define PM_SK_MAXSEG 64u
#ifndef PM_SK_GU_WARPS
#define PM_SK_GU_WARPS 12
#endif
/* resident CTAs per SM the stream-K kernels are compiled for: gate/up (two
 * matrices, the larger register tile) runs one CTA per SM with the whole
 * register file and a deep ring; down runs two */
__host__ __device__ constexpr int pm_sk_minb(int nmat) { return nmat == 2 ? 1 : 2; }
/* warps per CTA of the stream-K kernels */
__host__ __device__ constexpr int pm_sk_warps(int nmat) { return nmat == 2 ? PM_SK_GU_WARPS : 8; }

/* ------------------------------------------------------- activations */

/* staged activations of one token tile:
 *   x  [4][PM_TT][P] uint4 : plane 0/1 = bytes 0-15/16-31 of the pair's
 *                            first unit, plane 2/3 = of its second unit
 *   bs [PM_TT][P] int4     : 16-value bsums (u0 lo, u0 hi, u1 lo, u1 hi)
 *   d  [PM_TT][NB] float   : q8_K block scale */
struct pm_acts {
    uint4 *x;
    int4 *bs;
    float *d;
    uint32_t P, NB; /* P: pair slots per token, a multiple of 4 */
};

/* slot of unit pair p in a token's planes: pair j of super-block b sits at
 * j * (P / 4) + b, so the lanes of a row, which take consecutive
 * super-blocks, read consecutive 16-byte slots (no bank conflicts) */
__host__ __device__ __forceinline__ uint32_t pm_pslot(uint32_t p, uint32_t P) { return (p & 3u) * (P >> 2) + (p >> 2); }

__host__ __device__ __forceinline__ uint32_t pm_acts_bytes(uint32_t P, uint32_t NB) {
    return PM_TT * (P * 80u + NB * 4u) + 64u;
}

__device__ __forceinline__ pm_acts pm_acts_carve(uint8_t *p, uint32_t P, uint32_t NB) {
    pm_acts a;
    a.P = P;
    a.NB = NB;
    a.x = (uint4 *)p;
    a.bs = (int4 *)(a.x + 4u * PM_TT * P);
    a.d = (float *)(a.bs + PM_TT * P);
    return a;
}

/* nt tokens' q8_K rows (n_units 32-value units each) into the planes;
 * block scales of tokens nt..PM_TT-1 are zeroed.  All threads. */
__device__ __forceinline__ void pm_acts_stage_q8(const pm_acts &a, uint32_t nt, const pm_block_q8K *const *rows,
                                                 uint32_t n_units) {
    const uint32_t words = n_units * 8u;
    for (uint32_t i = threadIdx.x; i < nt * words; i += blockDim.x) {
        const uint32_t t = i / words, wd = i % words;
        const uint32_t u = wd >> 3, k = wd & 7u;
        const int32_t v = __ldcg((const int32_t *)((const uint8_t *)(rows[t] + (u >> 3)) + 4 + 32 * (u & 7u)) + k);
        const uint32_t plane = 2u * (u & 1u) + (k >> 2);
        ((int32_t *)(a.x + (plane * PM_TT + t) * a.P + pm_pslot(u >> 1, a.P)))[k & 3u] = v;
    }
    for (uint32_t i = threadIdx.x; i < nt * n_units; i += blockDim.x) {
        const uint32_t t = i / n_units, u = i % n_units;
        const pm_block_q8K *blk = rows[t] + (u >> 3);
        const uint32_t w = (uint32_t)__ldcg((const int32_t *)((const uint8_t *)blk + 260 + 4 * (u & 7u)));
        int32_t *dst = (int32_t *)(a.bs + t * a.P + pm_pslot(u >> 1, a.P)) + 2u * (u & 1u);
        dst[0] = (int32_t)(int16_t)(w & 0xffffu);
        dst[1] = (int32_t)(int16_t)(w >> 16);
        if ((u & 7u) == 0) a.d[t * a.NB + (u >> 3)] = __ldcg(&blk->d);
    }
    for (uint32_t i = threadIdx.x; i < (PM_TT - nt) * a.NB; i += blockDim.x) a.d[nt * a.NB + i] = 0.0f;
}

/* nt f32 rows of n values quantized to q8_K exactly like the CPU lane
 * (cpu_dot.rs:26-50: d = amax/127, round half away from zero, clamp
 * +-127) straight into the planes: one warp per (token, 256-block), a lane
 * holds 8 consecutive values = a quarter of one unit.  All threads. */
__device__ __forceinline__ void pm_acts_stage_f32(const pm_acts &a, uint32_t nt, const float *const *rows,
                                                  uint32_t n) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t n_units = (n + 31u) / 32u, nblk = (n + 255u) / 256u;
    for (uint32_t job = warp; job < nt * nblk; job += nw) {
        const uint32_t t = job / nblk, b = job % nblk;
        const float *src = rows[t] + (size_t)b * 256u;
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
        s += __shfl_xor_sync(0xffffffffu, s, 1);              /* 16-value sum (lane pair) */
        const int s_hi = __shfl_down_sync(0xffffffffu, s, 2); /* the unit's second 16 */
        const uint32_t u = b * 8u + (lane >> 2);
        if (u < n_units) {
            const uint32_t q = lane & 3u; /* quarter of the unit */
            const uint32_t plane = 2u * (u & 1u) + (q >> 1);
            uint32_t *dst = (uint32_t *)(a.x + (plane * PM_TT + t) * a.P + pm_pslot(u >> 1, a.P)) + 2u * (q & 1u);
            dst[0] = qv[0] | (qv[1] << 8) | (qv[2] << 16) | (qv[3] << 24);
            dst[1] = qv[4] | (qv[5] << 8) | (qv[6] << 16) | (qv[7] << 24);
            if (q == 0) {
                int32_t *bd = (int32_t *)(a.bs + t * a.P + pm_pslot(u >> 1, a.P)) + 2u * (u & 1u);
                bd[0] = s;
                bd[1] = s_hi;
            }
        }
        if (lane == 0) a.d[t * a.NB + b] = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
    }
    for (uint32_t i = threadIdx.x; i < (PM_TT - nt) * a.NB; i += blockDim.x) a.d[nt * a.NB + i] = 0.0f;
}

/* ------------------------------------------------------ pair decode */

/* one row's unit pair (units 2p, 2p+1) of one matrix, decoded */
struct pm_wp {
    uint32_t w0[8], w1[8]; /* int8x4 weights (Q4_K: nibbles in place) */
    int32_t i0, i1;        /* integer sub-block multipliers */
    int32_t m0, m1, m2, m3;
    float d, dm;
};

__device__ __forceinline__ int pm_dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int Q>
__device__ __forceinline__ void pm_decode_pair(const uint8_t *row, uint32_t p, bool two, const uint64_t *grid,
                                               pm_wp &o) {
    if constexpr (Q == PM_QUANT_Q4_K) {
        const uint8_t *b = row + (p >> 2) * PM_Q4_K_BYTES;
        const uint32_t sp = p & 3u;
        const uint4 h = *(const uint4 *)b;
        const uint32_t hdr = h.x, sa = h.y, sb = h.z, sc = h.w;
        /* 6-bit scale/min of sub-blocks 2sp and 2sp+1 (k4 packing, cu:1699) */
        const uint32_t sh = 16u * (sp & 1u);
        const uint32_t ea = (sa >> sh) & 0xffffu, eb = (sb >> sh) & 0xffffu, ec = (sc >> sh) & 0xffffu;
        /* both sub-blocks at once, branch-free (lanes of a warp hold all four sp) */
        const uint32_t sv = sp < 2 ? (ea & 0x3f3fu) : ((ec & 0x0f0fu) | ((ea >> 2) & 0x3030u));
        const uint32_t mv = sp < 2 ? (eb & 0x3f3fu) : (((ec >> 4) & 0x0f0fu) | ((eb >> 2) & 0x3030u));
        const int32_t s0 = (int32_t)(sv & 0xffu), s1 = (int32_t)(sv >> 8);
        const int32_t n0 = (int32_t)(mv & 0xffu), n1 = (int32_t)(mv >> 8);
        const uint4 *qp = (const uint4 *)(b + 16 + 32 * sp);
        const uint4 q0 = qp[0], q1 = qp[1];
        const uint32_t raw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            o.w0[i] = raw[i] & 0x0f0f0f0fu;
            o.w1[i] = raw[i] & 0xf0f0f0f0u;
        }
        o.i0 = 16 * s0, o.i1 = s1, o.m0 = n0, o.m1 = n1;
        o.d = pm_h2f(hdr & 0xffffu) * 0.0625f;
        o.dm = pm_h2f(hdr >> 16);
    } else if constexpr (Q == PM_QUANT_Q2_K) {
        const uint8_t *b = row + (p >> 2) * PM_Q2_K_BYTES;
        const uint32_t sp = p & 3u;
        const uint32_t *q = (const uint32_t *)(b + 16 + 32 * (sp >> 1));
        const uint32_t sh0 = 4u * (sp & 1u);
        const uint32_t scw = *(const uint32_t *)(b + 4 * sp);
        const uint32_t c0 = scw & 15u, c1 = (scw >> 8) & 15u, c2 = (scw >> 16) & 15u, c3 = (scw >> 24) & 15u;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t v = q[i];
            o.w0[i] = ((v >> sh0) & 0x03030303u) * (i < 4 ? c0 : c1);
            o.w1[i] = ((v >> (sh0 + 2u)) & 0x03030303u) * (i < 4 ? c2 : c3);
        }
        o.i0 = o.i1 = 1;
        o.m0 = (int32_t)((scw >> 4) & 15u), o.m1 = (int32_t)((scw >> 12) & 15u);
        o.m2 = (int32_t)((scw >> 20) & 15u), o.m3 = (int32_t)(scw >> 28);
        const uint32_t dd = *(const uint32_t *)(b + 80);
        o.d = pm_h2f(dd & 0xffffu);
        o.dm = pm_h2f(dd >> 16);
    } else if constexpr (Q == PM_QUANT_IQ2_XXS) {
        const uint8_t *b = row + (p >> 2) * PM_IQ2_XXS_BYTES;
        const uint32_t sp = p & 3u;
        uint32_t aux[4];
        pm_lds_words<4>(b + 2 + 16 * sp, aux);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int32_t a0, a1, b0, b1;
            pm_iq2_signed(grid[(aux[0] >> (8 * k)) & 0xffu], pm_ksigns_dev((aux[1] >> (7 * k)) & 127u), a0, a1);
            pm_iq2_signed(grid[(aux[2] >> (8 * k)) & 0xffu], pm_ksigns_dev((aux[3] >> (7 * k)) & 127u), b0, b1);
            o.w0[2 * k] = (uint32_t)a0, o.w0[2 * k + 1] = (uint32_t)a1;
            o.w1[2 * k] = (uint32_t)b0, o.w1[2 * k + 1] = (uint32_t)b1;
        }
        o.i0 = (int32_t)(2u * (aux[1] >> 28) + 1u);
        o.i1 = (int32_t)(2u * (aux[3] >> 28) + 1u);
        o.d = 0.125f * pm_h2f(*(const uint16_t *)b);
        o.dm = 0.0f;
    } else if constexpr (Q == PM_QUANT_MXFP4) {
        const uint8_t *b = row + (size_t)(2u * p) * PM_MXFP4_BLOCK;
        uint32_t q[4];
        pm_lds_words<4>(b + 1, q);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            o.w0[i] = (uint32_t)pm_e2m1x4(q[i] & 0x0f0f0f0fu);
            o.w0[4 + i] = (uint32_t)pm_e2m1x4((q[i] >> 4) & 0x0f0f0f0fu);
        }
        o.d = pm_mxfp4_scale_half(b[0]);
        if (two) {
            pm_lds_words<4>(b + PM_MXFP4_BLOCK + 1, q);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                o.w1[i] = (uint32_t)pm_e2m1x4(q[i] & 0x0f0f0f0fu);
                o.w1[4 + i] = (uint32_t)pm_e2m1x4((q[i] >> 4) & 0x0f0f0f0fu);
            }
            o.dm = pm_mxfp4_scale_half(b[PM_MXFP4_BLOCK]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) o.w1[i] = 0u;
            o.dm = 0.0f;
        }
    } else if constexpr (Q == PM_QUANT_Q8_0) {
        const uint8_t *b = row + (size_t)(2u * p) * PM_Q8_0_BLOCK;
        pm_lds_words<8>(b + 2, o.w0);
        o.d = pm_h2f(*(const uint16_t *)b);
        if (two) {
            pm_lds_words<8>(b + PM_Q8_0_BLOCK + 2, o.w1);
            o.dm = pm_h2f(*(const uint16_t *)(b + PM_Q8_0_BLOCK));
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) o.w1[i] = 0u;
            o.dm = 0.0f;
        }
    }
}

/* the pair's contribution for one token (before the q8_K block scale) */
template <int Q>
__device__ __forceinline__ float pm_pair_dot(const pm_wp &w, const uint4 &A, const uint4 &B, const uint4 &C,
                                             const uint4 &D, const int4 &bs) {
    int c0, c1;
    if constexpr (Q == PM_QUANT_Q4_K) {
        c0 = pm_dp4a_us(w.w0[0], (int)A.x, 0);
        c1 = pm_dp4a_us(w.w1[0], (int)C.x, 0);
        c0 = pm_dp4a_us(w.w0[1], (int)A.y, c0);
        c1 = pm_dp4a_us(w.w1[1], (int)C.y, c1);
        c0 = pm_dp4a_us(w.w0[2], (int)A.z, c0);
        c1 = pm_dp4a_us(w.w1[2], (int)C.z, c1);
        c0 = pm_dp4a_us(w.w0[3], (int)A.w, c0);
        c1 = pm_dp4a_us(w.w1[3], (int)C.w, c1);
        c0 = pm_dp4a_us(w.w0[4], (int)B.x, c0);
        c1 = pm_dp4a_us(w.w1[4], (int)D.x, c1);
        c0 = pm_dp4a_us(w.w0[5], (int)B.y, c0);
        c1 = pm_dp4a_us(w.w1[5], (int)D.y, c1);
        c0 = pm_dp4a_us(w.w0[6], (int)B.z, c0);
        c1 = pm_dp4a_us(w.w1[6], (int)D.z, c1);
        c0 = pm_dp4a_us(w.w0[7], (int)B.w, c0);
        c1 = pm_dp4a_us(w.w1[7], (int)D.w, c1);
    } else {
        c0 = __dp4a((int)w.w0[0], (int)A.x, 0);
        c1 = __dp4a((int)w.w1[0], (int)C.x, 0);
        c0 = __dp4a((int)w.w0[1], (int)A.y, c0);
        c1 = __dp4a((int)w.w1[1], (int)C.y, c1);
        c0 = __dp4a((int)w.w0[2], (int)A.z, c0);
        c1 = __dp4a((int)w.w1[2], (int)C.z, c1);
        c0 = __dp4a((int)w.w0[3], (int)A.w, c0);
        c1 = __dp4a((int)w.w1[3], (int)C.w, c1);
        c0 = __dp4a((int)w.w0[4], (int)B.x, c0);
        c1 = __dp4a((int)w.w1[4], (int)D.x, c1);
        c0 = __dp4a((int)w.w0[5], (int)B.y, c0);
        c1 = __dp4a((int)w.w1[5], (int)D.y, c1);
        c0 = __dp4a((int)w.w0[6], (int)B.z, c0);
        c1 = __dp4a((int)w.w1[6], (int)D.z, c1);
        c0 = __dp4a((int)w.w0[7], (int)B.w, c0);
        c1 = __dp4a((int)w.w1[7], (int)D.w, c1);
    }
    if constexpr (Q == PM_QUANT_Q4_K) {
        const int32_t ms = w.m0 * (bs.x + bs.y) + w.m1 * (bs.z + bs.w);
        return w.d * (float)(w.i0 * c0 + w.i1 * c1) - w.dm * (float)ms;
    } else if constexpr (Q == PM_QUANT_Q2_K) {
        const int32_t ms = w.m0 * bs.x + w.m1 * bs.y + w.m2 * bs.z + w.m3 * bs.w;
        return w.d * (float)(c0 + c1) - w.dm * (float)ms;
    } else if constexpr (Q == PM_QUANT_IQ2_XXS) {
        return w.d * (float)(w.i0 * c0 + w.i1 * c1);
    } else {
        return w.d * (float)c0 + w.dm * (float)c1;
    }
}

/* ------------------------------------------------------ one stage */

/* what stays fixed over a segment (one work unit's rows); the stage's row
 * pointers, row count and first row are passed per call */
struct pm_rowjob {
    uint64_t rb;
    uint32_t npair, n_units, nt, act, ostride;
    pm_acts acts;
    const uint64_t *grid;
    const uint32_t *tokpair; /* (token, slot) pair id of each token of the unit */
    float *out;
    const float *b0, *b1; /* gate / up bias rows of the expert (or null) */
    const float *wts;     /* route weight per pair */
};

#define PM_TERM_V 16u /* NMAT * tokens */
#define PM_TERM_P 33u /* 32 lanes + 1 (bank skew) */

/* one unit pair's integer (or per-32-block float) contribution to the
 * super-block accumulators of one token, in the CPU lane's arithmetic:
 *   Q4_K   ia += 16 (sc0 S0 + sc1 S1)     ib += m0 B0 + m1 B1
 *   Q2_K   ia += sum sc16 S16              ib += sum m16 B16
 *   IQ2    ia += ls0 S0 + ls1 S1
 *   MXFP4  fa += d0 S0 (+ d1 S1)           (block order, no contraction)
 *   Q8_0   fa += d0 S0 (+ d1 S1), blocks whose integer sum is 0 skipped */
template <int Q>
__device__ __forceinline__ void pm_pair_acc(const pm_wp &w, const uint4 &A, const uint4 &B, const uint4 &C,
                                            const uint4 &D, const int4 &bs, bool two, int32_t &ia, int32_t &ib,
                                            float &fa) {
    int c0, c1;
    if constexpr (Q == PM_QUANT_Q4_K) {
        c0 = pm_dp4a_us(w.w0[0], (int)A.x, 0);
        c1 = pm_dp4a_us(w.w1[0], (int)C.x, 0);
        c0 = pm_dp4a_us(w.w0[1], (int)A.y, c0);
        c1 = pm_dp4a_us(w.w1[1], (int)C.y, c1);
        c0 = pm_dp4a_us(w.w0[2], (int)A.z, c0);
        c1 = pm_dp4a_us(w.w1[2], (int)C.z, c1);
        c0 = pm_dp4a_us(w.w0[3], (int)A.w, c0);
        c1 = pm_dp4a_us(w.w1[3], (int)C.w, c1);
        c0 = pm_dp4a_us(w.w0[4], (int)B.x, c0);
        c1 = pm_dp4a_us(w.w1[4], (int)D.x, c1);
        c0 = pm_dp4a_us(w.w0[5], (int)B.y, c0);
        c1 = pm_dp4a_us(w.w1[5], (int)D.y, c1);
        c0 = pm_dp4a_us(w.w0[6], (int)B.z, c0);
        c1 = pm_dp4a_us(w.w1[6], (int)D.z, c1);
        c0 = pm_dp4a_us(w.w0[7], (int)B.w, c0);
        c1 = pm_dp4a_us(w.w1[7], (int)D.w, c1);
    } else {
        c0 = __dp4a((int)w.w0[0], (int)A.x, 0);
        c1 = __dp4a((int)w.w1[0], (int)C.x, 0);
        c0 = __dp4a((int)w.w0[1], (int)A.y, c0);
        c1 = __dp4a((int)w.w1[1], (int)C.y, c1);
        c0 = __dp4a((int)w.w0[2], (int)A.z, c0);
        c1 = __dp4a((int)w.w1[2], (int)C.z, c1);
        c0 = __dp4a((int)w.w0[3], (int)A.w, c0);
        c1 = __dp4a((int)w.w1[3], (int)C.w, c1);
        c0 = __dp4a((int)w.w0[4], (int)B.x, c0);
        c1 = __dp4a((int)w.w1[4], (int)D.x, c1);
        c0 = __dp4a((int)w.w0[5], (int)B.y, c0);
        c1 = __dp4a((int)w.w1[5], (int)D.y, c1);
        c0 = __dp4a((int)w.w0[6], (int)B.z, c0);
        c1 = __dp4a((int)w.w1[6], (int)D.z, c1);
        c0 = __dp4a((int)w.w0[7], (int)B.w, c0);
        c1 = __dp4a((int)w.w1[7], (int)D.w, c1);
    }
    if constexpr (Q == PM_QUANT_Q4_K) {
        ia += w.i0 * c0 + w.i1 * c1;
        ib += w.m0 * (bs.x + bs.y) + w.m1 * (bs.z + bs.w);
    } else if constexpr (Q == PM_QUANT_Q2_K) {
        ia += c0 + c1;
        ib += w.m0 * bs.x + w.m1 * bs.y + w.m2 * bs.z + w.m3 * bs.w;
    } else if constexpr (Q == PM_QUANT_IQ2_XXS) {
        ia += w.i0 * c0 + w.i1 * c1;
    } else if constexpr (Q == PM_QUANT_MXFP4) {
        fa = __fadd_rn(fa, __fmul_rn(w.d, (float)c0));
        if (two) fa = __fadd_rn(fa, __fmul_rn(w.dm, (float)c1));
    } else {
        if (c0 != 0) fa = __fadd_rn(fa, __fmul_rn(w.d, (float)c0));
        if (two && c1 != 0) fa = __fadd_rn(fa, __fmul_rn(w.dm, (float)c1));
    }
}

/* the super-block's term of the row's dot for one token, exactly as the
 * CPU lane forms it (cpu_dot.rs:250-279 q4_K, :732-767 q2_K, :92-122
 * iq2_xxs; MXFP4 cu:2053 / Q8_0 cu:2174 as the oracle restates them): the
 * same f32 operations in the same order, no fused multiply-add */
template <int Q>
__device__ __forceinline__ float pm_sb_term(float d, float dm, float yd, int32_t ia, int32_t ib, float fa) {
    if constexpr (Q == PM_QUANT_Q4_K) /* xd yd isum - xmin yd msum (d holds xd / 16, ia 16 isum) */
        return __fsub_rn(__fmul_rn(__fmul_rn(d * 16.0f, yd), (float)(ia >> 4)), __fmul_rn(__fmul_rn(dm, yd), (float)ib));
    else if constexpr (Q == PM_QUANT_Q2_K) /* yd xd isum - yd xmin summs */
        return __fsub_rn(__fmul_rn(__fmul_rn(yd, d), (float)ia), __fmul_rn(__fmul_rn(yd, dm), (float)ib));
    else if constexpr (Q == PM_QUANT_IQ2_XXS) /* (0.125 xd) yd bsum (d holds 0.125 xd) */
        return __fmul_rn(__fmul_rn(d, yd), (float)ia);
    else /* yd sum over the blocks */
        return __fmul_rn(yd, fa);
}

/* A stage's rows, each dot formed exactly as the CPU lane forms it.  LPR
 * lanes share a row; lane l of a row takes super-blocks l, l + LPR, ...
 * (its 4 unit pairs in order), so every super-block's integer sums are
 * exact in one lane and its f32 term is the CPU lane's.  The terms then
 * meet in shared memory, round by round (LPR super-blocks per round), and
 * one lane per (row, token) adds them in super-block order - the CPU
 * lane's sequential `total +=`.  EPI 0: gate/up -> mid = glu(g + bg,
 * u + bu) * w;  EPI 1: down -> partial. */
template <int Q, int NMAT, int NT, int LPR, int EPI>
__device__ __noinline__ void pm_rows(const pm_rowjob &jb, float *tm, const uint8_t *w0, const uint8_t *w1,
                                     uint32_t rows, uint32_t row_g) {
    constexpr int RPP = 32 / LPR;
    constexpr int V = NMAT * NT;
    const uint32_t lane = threadIdx.x & 31u, sub = lane / LPR, sl = lane % LPR;
    const pm_acts &ac = jb.acts;
    const uint32_t P = ac.P;
    const uint32_t nsb = (jb.npair + 3u) / 4u, rounds = (nsb + LPR - 1u) / LPR;
    constexpr uint32_t JOBS = (uint32_t)(RPP * NT); /* (row of the pass, token) */
    for (uint32_t j0 = 0; j0 < rows; j0 += RPP) {
        const uint32_t j = j0 + sub;
        const bool rv = j < rows;
        float acc[NMAT][(JOBS + 31) / 32];
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int q = 0; q < (int)((JOBS + 31) / 32); q++) acc[m][q] = 0.0f;
        for (uint32_t rd = 0; rd < rounds; rd++) {
            const uint32_t sb = rd * LPR + sl;
            const bool live = rv && sb < nsb;
            int32_t ia[V], ib[V];
            float fa[V];
#pragma unroll
            for (int i = 0; i < V; i++) ia[i] = ib[i] = 0, fa[i] = 0.0f;
            float dd[NMAT], dmm[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; m++) dd[m] = dmm[m] = 0.0f;
            if (live) {
#pragma unroll 2
                for (uint32_t p = 4u * sb; p < 4u * sb + 4u && p < jb.npair; p++) {
                    const bool two = 2u * p + 1u < jb.n_units;
                    pm_wp W[NMAT];
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        pm_decode_pair<Q>((m == 0 ? w0 : w1) + (size_t)j * jb.rb, p, two, jb.grid, W[m]);
                        dd[m] = W[m].d, dmm[m] = W[m].dm;
                    }
                    const uint32_t ps = pm_pslot(p, P);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        const uint4 A = ac.x[(0 * PM_TT + t) * P + ps];
                        const uint4 B = ac.x[(1 * PM_TT + t) * P + ps];
                        const uint4 C = ac.x[(2 * PM_TT + t) * P + ps];
                        const uint4 D = ac.x[(3 * PM_TT + t) * P + ps];
                        int4 bs = make_int4(0, 0, 0, 0);
                        if constexpr (Q == PM_QUANT_Q4_K || Q == PM_QUANT_Q2_K) bs = ac.bs[t * P + ps];
#pragma unroll
                        for (int m = 0; m < NMAT; m++)
                            pm_pair_acc<Q>(W[m], A, B, C, D, bs, two, ia[m * NT + t], ib[m * NT + t], fa[m * NT + t]);
                        /* keep at most two tokens' activations live */
                        if ((t & 1) == 1) asm volatile("" ::: "memory");
                    }
                }
            }
            /* this round's terms, [v][lane] (skewed rows: conflict-free);
             * lanes without a super-block this round write zeros (never read) */
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float yd = live ? ac.d[t * ac.NB + sb] : 0.0f;
#pragma unroll
                for (int m = 0; m < NMAT; m++)
                    tm[(m * NT + t) * PM_TERM_P + lane] =
                        pm_sb_term<Q>(dd[m], dmm[m], yd, ia[m * NT + t], ib[m * NT + t], fa[m * NT + t]);
            }
            __syncwarp();
            /* job lanes add the round's LPR terms in super-block order */
#pragma unroll
            for (int q = 0; q < (int)((JOBS + 31) / 32); q++) {
                const uint32_t jobi = lane + 32u * q;
                if (jobi < JOBS) {
                    const uint32_t jr = jobi / NT, jt = jobi % NT;
                    const uint32_t nlim = nsb - rd * LPR < LPR ? nsb - rd * LPR : LPR;
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const float *src = tm + (m * NT + jt) * PM_TERM_P + jr * LPR;
                        float tv[LPR];
#pragma unroll
                        for (int l = 0; l < LPR; l++) tv[l] = src[l]; /* all loads first, then the ordered adds */
                        float a = acc[m][q];
#pragma unroll
                        for (int l = 0; l < LPR; l++)
                            if ((uint32_t)l < nlim) a = __fadd_rn(a, tv[l]);
                        acc[m][q] = a;
                    }
                }
            }
            __syncwarp();
        }
        /* outputs: one lane per (row, token) */
#pragma unroll
        for (int q = 0; q < (int)((JOBS + 31) / 32); q++) {
            const uint32_t jobi = lane + 32u * q;
            if (jobi >= JOBS) continue;
            const uint32_t jr = jobi / NT, jt = jobi % NT, jj = j0 + jr;
            if (jj >= rows || jt >= jb.nt) continue;
            const uint32_t row = row_g + jj, pr = jb.tokpair[jt];
            if constexpr (NMAT == 2) {
                float g = acc[0][q], up = acc[1][q];
                if (jb.b0) g = __fadd_rn(g, jb.b0[row]);
                if (jb.b1) up = __fadd_rn(up, jb.b1[row]);
                jb.out[(size_t)pr * jb.ostride + row] = __fmul_rn(pm_glu(g, up, jb.act), jb.wts[pr]);
            } else {
                jb.out[(size_t)pr * jb.ostride + row] = acc[0][q];
            }
        }
    }
}

template <int Q, int NMAT, int LPR, int EPI>
__device__ __forceinline__ void pm_rows_nt(const pm_rowjob &jb, float *tm, const uint8_t *w0, const uint8_t *w1,
                                           uint32_t rows, uint32_t row_g) {
    switch (jb.nt) {
    case 1: pm_rows<Q, NMAT, 1, LPR, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 2: pm_rows<Q, NMAT, 2, LPR, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 3: pm_rows<Q, NMAT, 3, LPR, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 4: pm_rows<Q, NMAT, 4, LPR, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 5:
    case 6: pm_rows<Q, NMAT, 6, LPR, EPI>(jb, tm, w0, w1, rows, row_g); break;
    default: pm_rows<Q, NMAT, 8, LPR, EPI>(jb, tm, w0, w1, rows, row_g); break;
    }
}

template <int Q, int NMAT, int EPI>
__device__ __forceinline__ void pm_rows_any(const pm_rowjob &jb, float *tm, uint32_t lpr, const uint8_t *w0,
                                            const uint8_t *w1, uint32_t rows, uint32_t row_g) {
    switch (lpr) {
    case 2: pm_rows_nt<Q, NMAT, 2, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 4: pm_rows_nt<Q, NMAT, 4, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 8: pm_rows_nt<Q, NMAT, 8, EPI>(jb, tm, w0, w1, rows, row_g); break;
    case 16: pm_rows_nt<Q, NMAT, 16, EPI>(jb, tm, w0, w1, rows, row_g); break;
    default: pm_rows_nt<Q, NMAT, 32, EPI>(jb, tm, w0, w1, rows, row_g); break;
    }
}

/* ------------------------------------------------------ stage copies */

/* copy one stage (rows of NMAT matrices) with 1-D bulk copies: each piece
 * is rounded out to 16-byte boundaries, so the staged byte at global
 * address g sits at dst + off(m) + (g & 15) */
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

/* ------------------------------------------------------ launch geometry */

/* per matrix kind (0 routed experts, 1 shared expert) */
struct pm_skind {
    uint64_t rb;      /* row bytes */
    uint32_t n_units; /* 32-value units per row */
    uint32_t npair;
    uint32_t lpr;     /* lanes per row: 2, 4, 8, 16 or 32 (super-block slots) */
    uint32_t rw;      /* rows per stage */
    uint32_t direct;  /* 1: rows too large for the per-warp rings, read straight from global memory */
};

/* shared-memory layout of one stream-K launch (computed on the host) */
struct pm_skp {
    pm_skind k[2];
    uint32_t S;      /* ring stages per warp */
    uint32_t stage;  /* bytes per stage */
    uint32_t P, NB;  /* activation tile geometry (max over kinds) */
    uint32_t off_bar, off_seg, off_acts, off_terms, off_ring, smem;
};

/* one segment of a CTA's slice: rows [r0, r1) of one work unit */
struct pm_segi {
    const uint8_t *base[2]; /* row 0 of each matrix */
    const uint32_t *pairs;  /* the unit's (token, slot) pair ids */
    const float *b0, *b1;   /* bias rows (gate/up) */
    uint32_t nt, r0, r1, kind;
};
