/* pm_format.h - block layouts, scalar decoders and the deterministic math
 * shared by the CUDA kernels (device) and the host-side code (C/C++).
 *
 * Everything here is a FORMAT contract or a bit-exact arithmetic contract:
 *
 *  - Block byte layouts follow the GGUF/ggml block formats that pulsar's
 *    crates/quant encoders write and crates/kernels/cuda/pulsar_kernels.cu
 *    reads (block_q2_K cu:1296, block_iq2_xxs cu:1303, block_q4_K cu:1317,
 *    block_mxfp4 cu:1427, q8_0_block cu:94, block_q8_K cu:1492; block sizes
 *    gguf/src/lib.rs:145-170).
 *  - The IQ2_XXS grid is stored in its packed 2-bit form (one u16 per grid
 *    point, 8 digits of 2 bits); the dot kernels expand digit d to the
 *    integer {8, 25, 43}[d] and the encoder to the odd coordinate 2d+1
 *    (crates/quant/src/iq.rs:17-52, cpu_dot_tables.rs:176).
 *  - pm_expf is this project's own single-precision exponential, built from
 *    IEEE fma / mul steps only, so that host and device produce identical
 *    bits.  The router's selection scores go through it, which is what makes
 *    the top-k indices reproducible bit-for-bit on the CPU.
 */
#ifndef PM_FORMAT_H
#define PM_FORMAT_H

#include <stdint.h>
#include <string.h>
#include <math.h>

#ifdef __CUDACC__
#define PM_HD __host__ __device__ __forceinline__
#else
#define PM_HD static inline
#endif

#define PM_QK_K 256u

/* bytes per 256-value super-block (MXFP4 / Q8_0: 8 sub-blocks of 32) */
#define PM_Q2_K_BYTES 84u
#define PM_Q4_K_BYTES 144u
#define PM_IQ2_XXS_BYTES 66u
#define PM_MXFP4_BLOCK 17u  /* 32 values */
#define PM_Q8_0_BLOCK 34u   /* 32 values */
#define PM_Q8_K_BYTES 292u  /* f32 d + i8[256] + i16 bsums[16] */

/* quant codes: the QUANT_* values of crates/kernels/src/lib.rs:55-73
 * (PULSAR_QUANT_* cu:2649-2668). Only the five formats of this path are
 * implemented; every other code is rejected with a 0 return. */
enum {
    PM_QUANT_Q2_K = 0,
    PM_QUANT_IQ2_XXS = 1,
    PM_QUANT_Q4_K = 2,
    PM_QUANT_Q8_0 = 10,
    PM_QUANT_MXFP4 = 12,
};

/* activation row block, identical to the reference GPU block_q8_K so that
 * buffers sized by the Rust engine (n_blocks * 292 bytes) stay valid */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} pm_block_q8K;

/* ---------------------------------------------------------------- f16 */

/* IEEE binary16 -> binary32, exact for every input (subnormals included) */
PM_HD float pm_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = 113; /* 127 - 15 + 1 */
            while ((man & 0x400u) == 0) {
                man <<= 1;
                e--;
            }
            bits = sign | ((uint32_t)e << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even (crates/quant/src/lib.rs:51-82) */
PM_HD uint16_t pm_f32_to_f16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    uint16_t s = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t e = (int32_t)((bits >> 23) & 0xffu);
    uint32_t m = bits & 0x7fffffu;
    if (e == 0xff) return (uint16_t)(s | 0x7c00u | (m ? 0x200u : 0u));
    int32_t e16 = e - 127 + 15;
    if (e16 >= 0x1f) return (uint16_t)(s | 0x7c00u);
    if (e16 <= 0) {
        if (e16 < -10) return s;
        uint32_t mm = m | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e16);
        uint32_t half = mm >> shift;
        uint32_t rem = mm & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        uint32_t r = half + ((rem > halfway) | ((rem == halfway) & (half & 1u)));
        return (uint16_t)(s | r);
    }
    uint32_t half = (uint32_t)s | ((uint32_t)e16 << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    return (uint16_t)(half + ((rem > 0x1000u) | ((rem == 0x1000u) & (half & 1u))));
}

PM_HD uint16_t pm_ld_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
PM_HD uint32_t pm_ld_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* ------------------------------------------------------------- Q4_K */

/* 6-bit (scale, min) pair j of the 12 packed scale bytes (ggml
 * get_scale_min_k4; cpu_dot.rs:142 k4_scale_min) */
PM_HD void pm_k4_scale_min(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* -------------------------------------------------------- IQ2_XXS grid */

/* packed grid points: digit i (bits 2i..2i+1) is coordinate i of the
 * 8-vector; ggml's kgrid_2bit_256 (iq.rs:17-34) */
#define PM_IQ2XXS_KGRID_INIT { \
        0,     2,     5,     8,    10,    17,    20,    32,    34,    40,    42,    65,    68,    80,    88,    97, \
      100,   128,   130,   138,   162,   257,   260,   272,   277,   320,   388,   408,   512,   514,   546,   642, \
     1025,  1028,  1040,  1057,  1060,  1088,  1090,  1096,  1120,  1153,  1156,  1168,  1188,  1280,  1282,  1288, \
     1312,  1350,  1385,  1408,  1425,  1545,  1552,  1600,  1668,  1700,  2048,  2053,  2056,  2068,  2088,  2113, \
     2116,  2128,  2130,  2184,  2308,  2368,  2562,  2580,  4097,  4100,  4112,  4129,  4160,  4192,  4228,  4240, \
     4245,  4352,  4360,  4384,  4432,  4442,  4480,  4644,  4677,  5120,  5128,  5152,  5157,  5193,  5248,  5400, \
     5474,  5632,  5654,  6145,  6148,  6160,  6208,  6273,  6400,  6405,  6560,  6737,  8192,  8194,  8202,  8260, \
     8289,  8320,  8322,  8489,  8520,  8704,  8706,  9217,  9220,  9232,  9280,  9302,  9472,  9537,  9572,  9872, \
    10248, 10272, 10388, 10820, 16385, 16388, 16400, 16408, 16417, 16420, 16448, 16456, 16470, 16480, 16513, 16516, \
    16528, 16640, 16672, 16737, 16768, 16773, 16897, 16912, 16968, 16982, 17000, 17408, 17416, 17440, 17536, 17561, \
    17682, 17700, 17920, 18433, 18436, 18448, 18496, 18501, 18688, 18776, 18785, 18818, 19013, 19088, 20480, 20488, \
    20497, 20505, 20512, 20608, 20616, 20740, 20802, 20900, 21137, 21648, 21650, 21770, 22017, 22100, 22528, 22545, \
    22553, 22628, 22848, 23048, 24580, 24592, 24640, 24680, 24832, 24917, 25112, 25184, 25600, 25605, 25872, 25874, \
    25988, 26690, 32768, 32770, 32778, 32833, 32898, 33028, 33048, 33088, 33297, 33793, 33796, 33808, 33813, 33856, \
    33888, 34048, 34118, 34196, 34313, 34368, 34400, 34818, 35076, 35345, 36868, 36880, 36900, 36928, 37025, 37142, \
    37248, 37445, 37888, 37922, 37956, 38225, 39041, 39200, 40962, 41040, 41093, 41225, 41472, 42008, 43088, 43268, }

/* host copy; device code keeps its own __constant__ copy (same initializer) */
static const uint16_t PM_IQ2XXS_KGRID[256] = PM_IQ2XXS_KGRID_INIT;

/* dot-side magnitude of a 2-bit grid digit */
PM_HD int pm_iq2_level(int d) { return d == 0 ? 8 : (d == 1 ? 25 : 43); }

/* the 8 magnitudes of packed grid point k, little-endian in a u64 */
PM_HD uint64_t pm_iq2xxs_expand(uint32_t k) {
    uint64_t v = 0;
    for (int i = 0; i < 8; i++) v |= (uint64_t)pm_iq2_level((k >> (2 * i)) & 3) << (8 * i);
    return v;
}

/* 7 stored sign bits -> 8-bit mask whose bit 7 keeps the parity even */
PM_HD uint32_t pm_ksigns(uint32_t s7) {
    uint32_t c = s7, p = 0;
    while (c) {
        p ^= 1u;
        c &= c - 1u;
    }
    return s7 | (p << 7);
}

/* ------------------------------------------------------------- MXFP4 */

/* E2M1 magnitudes doubled so they are integers: {0,.5,1,1.5,2,3,4,6} x 2,
 * sign in bit 3 (OCP MX; decode semantics of cu:1435-1450) */
PM_HD int pm_mxfp4_kv(int nib) {
    int m = nib & 7;
    int v = m < 4 ? m : (m == 4 ? 4 : (m == 5 ? 6 : (m == 6 ? 8 : 12)));
    return (nib & 8) ? -v : v;
}

/* 2^(e-128): the E8M0 scale with the doubled table's compensating 1/2;
 * e < 2 decodes to zero (cu:1443-1449) */
PM_HD float pm_mxfp4_scale_half(uint32_t e) {
    if (e < 2u) return 0.0f;
    uint32_t bits = (e - 1u) << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ------------------------------------------------- deterministic math */

/* exp(x) for binary32 x in binary32 arithmetic only (the GPUs this runs on
 * have a slow binary64 pipe).  Method: Cody-Waite reduction x = k ln2 + r,
 * k = nearest(x log2 e), with ln2 split into a head of 16 significant bits
 * (k * head exact) and a tail, both applied with fma, so |r| <= ln2/2 to
 * within an ulp of r; then the degree-7 Taylor series of exp(r) in Horner
 * form with fma (truncation < 1e-8 relative); then 2^k as two exact powers
 * of two built from the exponent field (one rounding, into the subnormal
 * range for k < -126).  Only IEEE fma / mul / div steps: a C host and a CUDA
 * device produce identical bits.  Error vs the true value: within 1 ulp
 * (checked against libm exp in the tests). */
PM_HD float pm_pow2i(int k) { /* 2^k for k in [-126, 127] */
    const uint32_t bits = (uint32_t)(k + 127) << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

PM_HD float pm_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const float k = rintf(x * 1.44269504088896340736f);
    float r = fmaf(-k, 0.693145751953125f, x);   /* head of ln 2: 16 significant bits */
    r = fmaf(-k, 1.428606765330187045e-06f, r);  /* ln 2 - head */
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ki = (int)k, k1 = ki / 2, k2 = ki - k1; /* both within the normal exponent range */
    return (p * pm_pow2i(k1)) * pm_pow2i(k2);
}

/* router probability, same branch structure as the reference router
 * (cu:913-920) so large |x| stays accurate */
PM_HD float pm_sigmoid(float x) {
    if (x >= 0.0f) {
        const float e = pm_expf(-x);
        return 1.0f / (1.0f + e);
    }
    const float e = pm_expf(x);
    return e / (1.0f + e);
}

#endif /* PM_FORMAT_H */
