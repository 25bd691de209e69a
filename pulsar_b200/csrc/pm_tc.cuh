/* pm_tc.cuh - 5th-generation tensor core (tcgen05) building blocks for
 * sm_100a: tensor-memory allocation, UMMA shared-memory and instruction
 * descriptors, the single-thread MMA issue, its mbarrier commit, and
 * tensor-memory loads for the epilogue.
 *
 * Operand tiles are K-major with the 128-byte swizzle: a tile of R rows x
 * 64 fp16 (128 bytes per row) is stored as R/8 atoms of 1024 bytes; row r
 * of an atom sits at byte 128 (r % 8) and its 16-byte chunk c at chunk
 * position c ^ (r % 8).  Successive K = 16 slices of one 128-byte row are
 * addressed by advancing the descriptor start address by 32 bytes.
 *
 * Accumulators: M = 128 rows map to tensor-memory lanes 0..127 and N
 * columns to consecutive 32-bit columns.  Warp w of the CTA may read lanes
 * 32 (w % 4) .. 32 (w % 4) + 31.
 */
#pragma once
#include <stdint.h>

#include "pm_device.cuh"

/* ------------------------------------------------------- tensor memory */

/* one full warp: allocate ncols (power of two >= 32) columns; the base
 * address is written to *slot (shared memory) */
__device__ __forceinline__ void pm_tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pm_smem_addr(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

/* one full warp (the allocating one) */
__device__ __forceinline__ void pm_tmem_free(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void pm_tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void pm_tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

/* ------------------------------------------------------- descriptors */

/* K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart; tile base
 * 1024-byte aligned (base offset 0) */
__device__ __forceinline__ uint64_t pm_desc_sw128(const void *tile) {
    const uint64_t a = pm_smem_addr(tile);
    uint64_t d = (a >> 4) & 0x3fffull;       /* start address */
    d |= (uint64_t)1 << 16;                   /* leading byte offset (unused for swizzled K-major) */
    d |= (uint64_t)(1024 >> 4) << 32;         /* stride byte offset: next 8-row atom */
    d |= (uint64_t)1 << 46;                   /* descriptor version (sm_100) */
    d |= (uint64_t)2 << 61;                   /* layout: 128-byte swizzle */
    return d;
}

/* kind::f16 instruction descriptor: A, B fp16, D fp32, both K-major */
__host__ __device__ __forceinline__ uint32_t pm_idesc_f16(uint32_t M, uint32_t N) {
    return (1u << 4)               /* D format: f32 */
           | (0u << 7)             /* A format: f16 */
           | (0u << 10)            /* B format: f16 */
           | ((N >> 3) << 17)      /* N / 8 */
           | ((M >> 4) << 24);     /* M / 16 */
}

/* D[tmem] (+)= A * B^T for one K = 16 slice; one thread issues */
__device__ __forceinline__ void pm_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* arrive on bar once every MMA issued so far by this thread completed */
__device__ __forceinline__ void pm_mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     pm_smem_addr(bar))
                 : "memory");
}

/* 16 consecutive 32-bit columns of this thread's lane */
__device__ __forceinline__ void pm_tmem_ld16(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

/* byte offset of element (r, k) in a K-major 128-byte-swizzled tile of
 * 64-wide fp16 rows (k in 0..63) */
__device__ __forceinline__ uint32_t pm_sw128_off(uint32_t r, uint32_t k) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((((k >> 3) ^ (r & 7u)) & 7u) << 4) + (k & 7u) * 2u;
}

/* ------------------------------------------------------- operand fill */

__device__ __forceinline__ __half2 pm_u2h2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return h;
}

__device__ __forceinline__ uint32_t pm_h22u(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}

/* fp16 hi + lo pair of two f32 values: hi = rounded, lo = rounded rest */
__device__ __forceinline__ void pm_split2(float v0, float v1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(h);
    hi = pm_h22u(h);
    lo = pm_h22u(__floats2half2_rn(v0 - hf.x, v1 - hf.y));
}

/* Q4_K row -> 64 weights of chunk c (sub-blocks 2p and 2p+1 of super-block
 * c / 4, p = c % 4), w = d sc q - dmin m (k4 packing, cu:1699) evaluated in
 * f32 and returned as fp16 hi + lo parts (w = hi + lo to ~2^-22): oh[j],
 * ol[j] hold values 8 j .. 8 j + 7 (j 0-3: first sub-block, 4-7: second).
 * Nibbles become exact fp16 integers through the exponent trick
 * (0x6400 | n = 1024 + n).  HALF: 0 both sub-blocks, 1 first only, 2
 * second only.  RAW: `row` is a 16-byte aligned shared-memory copy. */
template <int HALF, bool RAW = false>
__device__ __forceinline__ void pm_tc_q4k_row(const uint8_t *row, uint32_t c, uint4 *oh, uint4 *ol) {
    const uint8_t *b = row + (c >> 2) * PM_Q4_K_BYTES;
    const uint32_t sp = c & 3u;
    const uint4 h = RAW ? *(const uint4 *)b : __ldg((const uint4 *)b);
    const uint32_t sh = 16u * (sp & 1u);
    const uint32_t ea = (h.y >> sh) & 0xffffu, eb = (h.z >> sh) & 0xffffu, ec = (h.w >> sh) & 0xffffu;
    const uint32_t sv = sp < 2 ? (ea & 0x3f3fu) : ((ec & 0x0f0fu) | ((ea >> 2) & 0x3030u));
    const uint32_t mv = sp < 2 ? (eb & 0x3f3fu) : (((ec >> 4) & 0x0f0fu) | ((eb >> 2) & 0x3030u));
    const uint32_t s0 = sv & 0xffu, s1 = sv >> 8, n0 = mv & 0xffu, n1 = mv >> 8;
    const float d = pm_h2f(h.x & 0xffffu), dm = pm_h2f(h.x >> 16);
    const float S0 = d * (float)s0, M0 = -dm * (float)n0;
    const float S1 = d * (float)s1 * 0.0625f, M1 = -dm * (float)n1; /* high nibbles come x16 */
    const uint4 *qp = (const uint4 *)(b + 16 + 32 * sp);
    const uint4 q0 = RAW ? qp[0] : __ldg(qp), q1 = RAW ? qp[1] : __ldg(qp + 1);
    const uint32_t raw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const __half2 k1024 = __float2half2_rn(1024.0f);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t t01 = __byte_perm(raw[i], 0x64646464u, 0x4140u); /* bytes 0, 1 -> fp16 high byte 0x64 */
        const uint32_t t23 = __byte_perm(raw[i], 0x64646464u, 0x4342u);
        const uint32_t o = 2 * (i & 1);
        if (HALF != 2) {
            const float2 x01 = __half22float2(__hsub2(pm_u2h2(t01 & 0xff0fff0fu), k1024));
            const float2 x23 = __half22float2(__hsub2(pm_u2h2(t23 & 0xff0fff0fu), k1024));
            uint32_t *hh = (uint32_t *)&oh[i >> 1] + o, *ll = (uint32_t *)&ol[i >> 1] + o;
            pm_split2(fmaf(x01.x, S0, M0), fmaf(x01.y, S0, M0), hh[0], ll[0]);
            pm_split2(fmaf(x23.x, S0, M0), fmaf(x23.y, S0, M0), hh[1], ll[1]);
        }
        if (HALF != 1) {
            const float2 x01 = __half22float2(__hsub2(pm_u2h2(t01 & 0xfff0fff0u), k1024));
            const float2 x23 = __half22float2(__hsub2(pm_u2h2(t23 & 0xfff0fff0u), k1024));
            uint32_t *hh = (uint32_t *)&oh[4 + (i >> 1)] + o, *ll = (uint32_t *)&ol[4 + (i >> 1)] + o;
            pm_split2(fmaf(x01.x, S1, M1), fmaf(x01.y, S1, M1), hh[0], ll[0]);
            pm_split2(fmaf(x23.x, S1, M1), fmaf(x23.y, S1, M1), hh[1], ll[1]);
        }
    }
}

/* 16 q8_K values (k0 .. k0 + 15, k0 % 16 == 0) of one token row: d * q in
 * f32 as fp16 hi + lo parts; two 16-byte chunks each */
__device__ __forceinline__ void pm_tc_q8_16(const pm_block_q8K *xr, uint32_t k0, uint4 *oh, uint4 *ol) {
    const pm_block_q8K *blk = xr + (k0 >> 8);
    const uint32_t *src = (const uint32_t *)((const uint8_t *)blk + 4 + (k0 & 255u));
    const float xd = __ldg(&blk->d);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t u = __ldg(src + i);
        uint32_t *hh = (uint32_t *)&oh[i >> 1] + 2 * (i & 1), *ll = (uint32_t *)&ol[i >> 1] + 2 * (i & 1);
        pm_split2(xd * (float)(int8_t)(u & 0xffu), xd * (float)(int8_t)((u >> 8) & 0xffu), hh[0], ll[0]);
        pm_split2(xd * (float)(int8_t)((u >> 16) & 0xffu), xd * (float)(int8_t)(u >> 24), hh[1], ll[1]);
    }
}
