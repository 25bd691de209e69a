/* pm_device.cuh - device building blocks of the expert kernels (sm_100a).
 *
 *  - 1-D TMA (cp.async.bulk) staging of contiguous weight-row ranges into
 *    shared memory, completed on an mbarrier.  Every wait is bounded: on
 *    timeout the kernel records an error code in a caller-visible word and
 *    returns, so a lost copy can never hang the GPU.  No multicast.
 *  - Per-format "unit" dots: one unit is 32 consecutive weights of one row
 *    against the matching 32 q8_K activations, integer dp4a inside, one
 *    float scale combination out.  A 256-value super-block is 8 units, so a
 *    warp covers 4 super-blocks per step with every lane busy.
 *
 * Format math: crates/kernels/cuda/pulsar_kernels.cu dot functors
 * (q4_K cu:1699, q2_K cu:1625, iq2_xxs cu:1582, mxfp4 cu:2053, q8_0
 * cu:2174) and crates/quant/src/cpu_dot.rs (:92, :250, :732), regrouped per
 * 32-value unit.
 */
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pm_format.h"

/* error word values (bitwise OR) */
#define PM_ERR_TIMEOUT 1u
#define PM_ERR_BADARG 2u

/* wait budget for one mbarrier phase: ~2^31 SM cycles (about 1 s) */
#define PM_WAIT_CYCLES (1ll << 31)

/* ------------------------------------------------------------ mbarrier */

__device__ __forceinline__ uint32_t pm_smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void pm_mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(pm_smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void pm_fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void pm_mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(pm_smem_addr(bar)), "r"(bytes)
                 : "memory");
}

/* plain arrive (count 1) */
__device__ __forceinline__ void pm_mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pm_smem_addr(bar)) : "memory");
}

/* 1-D bulk copy global -> shared, completion counted on bar.
 * dst, src 16-byte aligned; bytes a multiple of 16. */
__device__ __forceinline__ void pm_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            pm_smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(pm_smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool pm_mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(pm_smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

/* non-blocking test of phase `parity` (never suspends the thread) */
__device__ __forceinline__ bool pm_mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(pm_smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

/* bounded wait for phase `parity`; false (and err |= TIMEOUT) after
 * `budget` SM cycles.  Callers may shorten the budget of ring waits (a
 * layer descriptor's wait_cycles); waits that drain copies or MMAs still
 * in flight before a kernel exits always keep the full default budget. */
__device__ __forceinline__ bool pm_mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err,
                                             long long budget = PM_WAIT_CYCLES) {
    const bool poll = budget < PM_WAIT_CYCLES; /* a shortened budget never suspends the thread */
    if (poll ? pm_mbar_test(bar, parity) : pm_mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!(poll ? pm_mbar_test(bar, parity) : pm_mbar_try(bar, parity))) {
        if (clock64() - t0 > budget) {
            if (err) atomicOr(err, PM_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

/* try_wait that may suspend the thread up to ~1 us instead of spinning */
__device__ __forceinline__ bool pm_mbar_try_sleep(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(pm_smem_addr(bar)), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}

/* bounded wait with suspension; false (and err |= TIMEOUT) on timeout */
__device__ __forceinline__ bool pm_mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t *err,
                                                   long long budget = PM_WAIT_CYCLES) {
    /* a shortened budget polls without suspending, so it is checked at once */
    const bool poll = budget < PM_WAIT_CYCLES;
    const long long t0 = clock64();
    for (;;) {
        if (poll ? pm_mbar_test(bar, parity) : pm_mbar_try_sleep(bar, parity)) return true;
        if (clock64() - t0 > budget) {
            if (err) atomicOr(err, PM_ERR_TIMEOUT);
            return false;
        }
    }
}

/* order this thread's generic-proxy shared accesses before later
 * async-proxy (TMA) writes to the same shared memory */
__device__ __forceinline__ void pm_fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

/* ------------------------------------------------------ byte access */

/* 4-byte little-endian word at any byte alignment in shared memory */
__device__ __forceinline__ uint32_t pm_lds_u32(const uint8_t *p) {
    const uintptr_t a = (uintptr_t)p;
    const uint32_t *w = (const uint32_t *)(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    if (sh == 0) return w[0];
    return __funnelshift_r(w[0], w[1], sh);
}

/* N consecutive words starting at any byte alignment (reads only the
 * aligned words that hold at least one requested byte) */
template <int N>
__device__ __forceinline__ void pm_lds_words(const uint8_t *p, uint32_t *out) {
    const uintptr_t a = (uintptr_t)p;
    const uint32_t *w = (const uint32_t *)(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    if (sh == 0) {
#pragma unroll
        for (int i = 0; i < N; i++) out[i] = w[i];
        return;
    }
    uint32_t cur = w[0];
#pragma unroll
    for (int i = 0; i < N; i++) {
        const uint32_t nxt = w[i + 1];
        out[i] = __funnelshift_r(cur, nxt, sh);
        cur = nxt;
    }
}

__device__ __forceinline__ float pm_h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

/* ---------------------------------------------------- activations */

/* q8_K activations in the reference 292-byte block layout: 32 values of
 * block b starting at value 32*s, as 8 words, plus d and two bsums */
struct pm_q8_unit {
    int32_t a[8];
    float d;
    int32_t bs0, bs1;
};

__device__ __forceinline__ void pm_load_q8_unit(const pm_block_q8K *blk, int s, pm_q8_unit &u) {
    const int32_t *q = (const int32_t *)((const uint8_t *)blk + 4 + 32 * s);
#pragma unroll
    for (int i = 0; i < 8; i++) u.a[i] = __ldg(q + i);
    u.d = __ldg(&blk->d);
    const int32_t pair = __ldg((const int32_t *)((const uint8_t *)blk + 260 + 4 * s));
    u.bs0 = (int32_t)(int16_t)(pair & 0xffff);
    u.bs1 = (int32_t)(int16_t)((uint32_t)pair >> 16);
}

/* ------------------------------------------------------- unit dots */

/* Q4_K unit s of a super-block at sb (16-byte aligned, cu:1317 layout) */
__device__ __forceinline__ float pm_unit_q4K(const uint8_t *sb, int s, const pm_q8_unit &x) {
    const uint4 hdr = *(const uint4 *)sb; /* d, dmin, scales[0..11] */
    const uint8_t *sc = sb + 4;
    int scv, mnv;
    pm_k4_scale_min(s, sc, &scv, &mnv);
    const uint4 *qp = (const uint4 *)(sb + 16 + 32 * (s >> 1));
    const uint4 q0 = qp[0], q1 = qp[1];
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const int shift = (s & 1) * 4;
    int sumi = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) sumi = __dp4a((int)((w[i] >> shift) & 0x0f0f0f0fu), x.a[i], sumi);
    const float d = pm_h2f(hdr.x & 0xffffu), dmin = pm_h2f(hdr.x >> 16);
    return (d * x.d) * (float)(scv * sumi) - (dmin * x.d) * (float)(mnv * (x.bs0 + x.bs1));
}

/* Q2_K unit s (cu:1296 layout: scales[16], qs[64], d, dmin; 4-byte aligned) */
__device__ __forceinline__ float pm_unit_q2K(const uint8_t *sb, int s, const pm_q8_unit &x) {
    const uint32_t *q = (const uint32_t *)(sb + 16 + 32 * (s >> 2));
    const int shift = 2 * (s & 3);
    int s0 = 0, s1 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) s0 = __dp4a((int)((q[i] >> shift) & 0x03030303u), x.a[i], s0);
#pragma unroll
    for (int i = 4; i < 8; i++) s1 = __dp4a((int)((q[i] >> shift) & 0x03030303u), x.a[i], s1);
    const uint32_t scw = *(const uint16_t *)(sb + 2 * s);
    const int sc0 = scw & 0xff, sc1 = scw >> 8;
    const uint32_t dd = *(const uint32_t *)(sb + 80);
    const float xd = pm_h2f(dd & 0xffffu), xmin = pm_h2f(dd >> 16);
    const int isum = (sc0 & 15) * s0 + (sc1 & 15) * s1;
    const int summs = x.bs0 * (sc0 >> 4) + x.bs1 * (sc1 >> 4);
    return (x.d * xd) * (float)isum - (x.d * xmin) * (float)summs;
}

/* 8 signed grid bytes from a packed 64-bit grid point and 8 sign bits */
__device__ __forceinline__ void pm_iq2_signed(uint64_t g, uint32_t signs, int32_t &w0, int32_t &w1) {
    const uint32_t s4 = signs * 0x01010101u;
    const uint32_t m0 = __vcmpne4(s4 & 0x08040201u, 0u);
    const uint32_t m1 = __vcmpne4(s4 & 0x80402010u, 0u);
    w0 = (int32_t)__vsub4((uint32_t)g ^ m0, m0);
    w1 = (int32_t)__vsub4((uint32_t)(g >> 32) ^ m1, m1);
}

__device__ __forceinline__ uint32_t pm_ksigns_dev(uint32_t s7) { return s7 | ((__popc(s7) & 1u) << 7); }

/* IQ2_XXS unit g (cu:1303 layout: f16 d + 8 x (u32 grid idx, u32 signs|scale));
 * grid: 256 packed magnitudes in shared memory */
__device__ __forceinline__ float pm_unit_iq2xxs(const uint8_t *sb, int g, const pm_q8_unit &x,
                                                const uint64_t *grid) {
    const uint16_t *h = (const uint16_t *)sb; /* 2-byte aligned */
    const uint32_t aux0 = (uint32_t)h[1 + 4 * g] | ((uint32_t)h[2 + 4 * g] << 16);
    const uint32_t aux1 = (uint32_t)h[3 + 4 * g] | ((uint32_t)h[4 + 4 * g] << 16);
    int sumi = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        int32_t w0, w1;
        pm_iq2_signed(grid[(aux0 >> (8 * k)) & 0xffu], pm_ksigns_dev((aux1 >> (7 * k)) & 127u), w0, w1);
        sumi = __dp4a(w0, x.a[2 * k], sumi);
        sumi = __dp4a(w1, x.a[2 * k + 1], sumi);
    }
    const int ls = (int)(2u * (aux1 >> 28) + 1u);
    const float xd = pm_h2f(h[0]);
    return (0.125f * xd * x.d) * (float)(ls * sumi);
}

/* 4 E2M1 nibbles (one per byte, values 0..15) -> 4 signed doubled values */
__device__ __forceinline__ int32_t pm_e2m1x4(uint32_t nib) {
    /* magnitudes x2 for codes 0..7: 0 1 2 3 4 6 8 12 */
    const uint32_t sel = (nib & 0x7u) | ((nib >> 4) & 0x70u) | ((nib >> 8) & 0x700u) | ((nib >> 12) & 0x7000u);
    const uint32_t mag = __byte_perm(0x03020100u, 0x0c080604u, sel);
    const uint32_t neg = __vcmpne4(nib & 0x08080808u, 0u);
    return (int32_t)__vsub4(mag ^ neg, neg);
}

/* MXFP4 unit b: 17-byte block (E8M0 + 16 nibble bytes), any alignment */
__device__ __forceinline__ float pm_unit_mxfp4(const uint8_t *blk, const pm_q8_unit &x) {
    uint32_t q[4];
    pm_lds_words<4>(blk + 1, q);
    int sumi = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        sumi = __dp4a(pm_e2m1x4(q[i] & 0x0f0f0f0fu), x.a[i], sumi);
        sumi = __dp4a(pm_e2m1x4((q[i] >> 4) & 0x0f0f0f0fu), x.a[4 + i], sumi);
    }
    return x.d * (pm_mxfp4_scale_half(blk[0]) * (float)sumi);
}

/* Q8_0 unit b: 34-byte block (f16 d + 32 int8), 2-byte aligned */
__device__ __forceinline__ float pm_unit_q8_0(const uint8_t *blk, const pm_q8_unit &x) {
    uint32_t q[8];
    pm_lds_words<8>(blk + 2, q);
    int sumi = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) sumi = __dp4a((int)q[i], x.a[i], sumi);
    if (sumi == 0) return 0.0f;
    return x.d * (pm_h2f(*(const uint16_t *)blk) * (float)sumi);
}

/* ------------------------------------------------------ format traits */

template <int Q> struct pm_fmt;
template <> struct pm_fmt<PM_QUANT_Q4_K> {
    static constexpr uint32_t SB = PM_Q4_K_BYTES;
    static constexpr bool K = true; /* whole 256-value super-blocks only */
};
template <> struct pm_fmt<PM_QUANT_Q2_K> {
    static constexpr uint32_t SB = PM_Q2_K_BYTES;
    static constexpr bool K = true;
};
template <> struct pm_fmt<PM_QUANT_IQ2_XXS> {
    static constexpr uint32_t SB = PM_IQ2_XXS_BYTES;
    static constexpr bool K = true;
};
template <> struct pm_fmt<PM_QUANT_MXFP4> {
    static constexpr uint32_t SB = 8 * PM_MXFP4_BLOCK;
    static constexpr bool K = false;
};
template <> struct pm_fmt<PM_QUANT_Q8_0> {
    static constexpr uint32_t SB = 8 * PM_Q8_0_BLOCK;
    static constexpr bool K = false;
};

/* unit u = 8*superblock + sub of a row held in shared memory */
template <int Q>
__device__ __forceinline__ float pm_unit(const uint8_t *row, uint32_t u, const pm_q8_unit &x, const uint64_t *grid) {
    const uint32_t sb = u >> 3, s = u & 7u;
    if constexpr (Q == PM_QUANT_Q4_K) return pm_unit_q4K(row + sb * pm_fmt<Q>::SB, (int)s, x);
    if constexpr (Q == PM_QUANT_Q2_K) return pm_unit_q2K(row + sb * pm_fmt<Q>::SB, (int)s, x);
    if constexpr (Q == PM_QUANT_IQ2_XXS) return pm_unit_iq2xxs(row + sb * pm_fmt<Q>::SB, (int)s, x, grid);
    if constexpr (Q == PM_QUANT_MXFP4) return pm_unit_mxfp4(row + u * PM_MXFP4_BLOCK, x);
    if constexpr (Q == PM_QUANT_Q8_0) return pm_unit_q8_0(row + u * PM_Q8_0_BLOCK, x);
    return 0.0f;
}

/* row bytes for n values (0 = not representable) */
__host__ __device__ __forceinline__ uint64_t pm_row_bytes(uint32_t quant, uint64_t n) {
    switch (quant) {
    case PM_QUANT_Q4_K: return n % 256 ? 0 : n / 256 * PM_Q4_K_BYTES;
    case PM_QUANT_Q2_K: return n % 256 ? 0 : n / 256 * PM_Q2_K_BYTES;
    case PM_QUANT_IQ2_XXS: return n % 256 ? 0 : n / 256 * PM_IQ2_XXS_BYTES;
    case PM_QUANT_MXFP4: return n % 32 ? 0 : n / 32 * PM_MXFP4_BLOCK;
    case PM_QUANT_Q8_0: return n % 32 ? 0 : n / 32 * PM_Q8_0_BLOCK;
    default: return 0;
    }
}

__device__ __forceinline__ float pm_warp_sum(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

/* e^x rounded to binary32 from the binary64 exponential (correctly rounded
 * but for rare double-rounding cases), so the glu matches the CPU lane's
 * f32 expf (glibc, within 0.502 ulp) bit for bit in all but rare inputs */
__device__ __forceinline__ float pm_exp_f32(float x) { return (float)exp((double)x); }

/* crates/engine/src/lib.rs:2134-2159 glu (cu:124 pulsar_glu) in the CPU
 * lane's f32 operation order, without contraction: 0 silu, 1 gelu tanh,
 * 2 swiglu_oai, 3 clamped silu, 4 SiTU-GLU */
__device__ __forceinline__ float pm_glu(float g, float u, uint32_t op) {
    if (op == 2u) {
        g = fminf(g, 7.0f);
        u = fminf(fmaxf(u, -7.0f), 7.0f);
        const float e = pm_exp_f32(__fmul_rn(-1.702f, g));
        return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), __fadd_rn(u, 1.0f));
    }
    if (op == 3u) {
        g = fminf(g, 10.0f);
        u = fminf(fmaxf(u, -10.0f), 10.0f);
        return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, pm_exp_f32(-g))), u);
    }
    if (op == 4u) {
        const float a = 4.0f * tanhf(g / 4.0f) / (1.0f + pm_exp_f32(-g));
        return a * (25.0f * tanhf(u / 25.0f));
    }
    if (op == 1u) return 0.5f * g * (1.0f + tanhf(0.7978846f * (g + 0.044715f * g * g * g))) * u;
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, pm_exp_f32(-g))), u);
}

/* One warp quantizes one 256-value q8_K block exactly like the CPU lane
 * (cpu_dot.rs:26-50): d = amax/127, q = round-half-away(x * (127/amax)),
 * clamp +-127, integer bsums per 16.  src holds `valid` values (the rest
 * of the block quantizes as zero). */
__device__ __forceinline__ void pm_q8k_warp(const float *src, uint32_t valid, pm_block_q8K *y) {
    const uint32_t lane = threadIdx.x & 31u;
    float v[8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t e = lane * 8u + (uint32_t)i;
        v[i] = e < valid ? src[e] : 0.0f;
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    uint32_t qv[8];
    int s = 0;
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; i++) qv[i] = 0;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float r = roundf(__fmul_rn(v[i], inv));
            r = fminf(fmaxf(r, -127.0f), 127.0f);
            const int qi = (int)r;
            s += qi;
            qv[i] = (uint32_t)(uint8_t)(int8_t)qi;
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    uint32_t *qw = (uint32_t *)((uint8_t *)y + 4 + 8 * lane);
    qw[0] = qv[0] | (qv[1] << 8) | (qv[2] << 16) | (qv[3] << 24);
    qw[1] = qv[4] | (qv[5] << 8) | (qv[6] << 16) | (qv[7] << 24);
    if ((lane & 1u) == 0) y->bsums[lane >> 1] = (int16_t)s;
    if (lane == 0) y->d = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
}
