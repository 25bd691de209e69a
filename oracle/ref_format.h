/* ref_format.h - block layouts and scalar helpers of the parity oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  The oracle keeps its own statement of every
 * format detail it needs, written from the reference sources, so that a
 * mistake in the product's headers (pulsar_b200/csrc) cannot repeat itself
 * on both sides of a parity check.  Sources (pulsar repo):
 *   block sizes, quant codes   crates/kernels/src/lib.rs:55-73,
 *                              crates/quant/src/lib.rs (block structs)
 *   f16 <-> f32                crates/quant/src/lib.rs:51-82 (RNE encode)
 *   Q4_K scale / min pairs     crates/quant/src/cpu_dot.rs:142
 *   IQ2_XXS grid and signs     crates/quant/src/iq.rs:17-52, :496
 *   MXFP4 decode               crates/kernels/cuda/pulsar_kernels.cu:1435-1450
 * The exponential used for router scores is this project's documented
 * binary32 method (Cody-Waite reduction, degree-7 Taylor, exact 2^k), the
 * contract the CUDA router keeps; it is restated here from that method. */
#ifndef ORF_FORMAT_H
#define ORF_FORMAT_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORF_Q2_K 0
#define ORF_IQ2_XXS 1
#define ORF_Q4_K 2
#define ORF_Q8_0 10
#define ORF_MXFP4 12

#define ORF_Q2_K_BYTES 84u   /* scales[16] qs[64] d dmin */
#define ORF_Q4_K_BYTES 144u  /* d dmin scales[12] qs[128] */
#define ORF_IQ2_XXS_BYTES 66u /* d, 8 x (u32 grid idx, u32 signs|scale) */
#define ORF_MXFP4_BLOCK 17u  /* e8m0 + 16 nibble bytes, 32 values */
#define ORF_Q8_0_BLOCK 34u   /* f16 d + 32 int8 */

/* q8_K activation block: f32 d, 256 int8, 16 int16 sums (292 bytes) */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} orf_q8k;

static inline float orf_bits_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
static inline uint32_t orf_f32_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

/* binary16 -> binary32: the value (-1)^s 2^(e-15) (1 + m/1024), or
 * 2^-14 m/1024 for e = 0; every binary16 value is exact in binary32 */
static inline float orf_f16(uint16_t h) {
    const int e = (h >> 10) & 31, m = h & 1023;
    const float sgn = (h & 0x8000u) ? -1.0f : 1.0f;
    if (e == 31) return m ? NAN : sgn * INFINITY;
    if (e == 0) return sgn * ldexpf((float)m, -24);
    return sgn * ldexpf((float)(1024 + m), e - 25);
}

/* binary32 -> binary16, round half to even (overflow to infinity) */
static inline uint16_t orf_to_f16(float x) {
    const uint32_t b = orf_f32_bits(x);
    const uint16_t s = (uint16_t)((b >> 16) & 0x8000u);
    if ((b & 0x7fffffffu) >= 0x7f800000u) return (uint16_t)(s | 0x7c00u | ((b & 0x7fffffu) ? 0x200u : 0u));
    const double a = fabs((double)x);
    if (a >= 65520.0) return (uint16_t)(s | 0x7c00u);       /* rounds past the largest finite */
    if (a < ldexp(1.0, -14)) {                              /* subnormal range: units of 2^-24 */
        const double q = a * 16777216.0;
        double r = floor(q);
        const double f = q - r;
        if (f > 0.5 || (f == 0.5 && fmod(r, 2.0) == 1.0)) r += 1.0;
        return (uint16_t)(s | (uint16_t)r);                 /* r = 1024 becomes the smallest normal */
    }
    int ex;
    const double fr = frexp(a, &ex);                        /* a = fr 2^ex, fr in [0.5, 1) */
    const double q = fr * 2048.0;                           /* 11 significant bits */
    double r = floor(q);
    const double f = q - r;
    if (f > 0.5 || (f == 0.5 && fmod(r, 2.0) == 1.0)) r += 1.0;
    if (r == 2048.0) {
        r = 1024.0;
        ex += 1;
    }
    const int e16 = ex - 1 + 15;
    if (e16 >= 31) return (uint16_t)(s | 0x7c00u);
    return (uint16_t)(s | (uint16_t)(e16 << 10) | (uint16_t)((int)r - 1024));
}

static inline uint16_t orf_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t orf_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Q4_K: sub-block j (0..7) takes a 6-bit scale and min from the 12 packed
 * bytes: j < 4 from the low 6 bits of bytes j and j + 4; j >= 4 from the
 * nibbles of byte j + 4 and the top 2 bits of bytes j - 4 and j */
static inline void orf_k4_pair(int j, const uint8_t *sc12, int *scale, int *min) {
    if (j < 4) {
        *scale = sc12[j] & 0x3f;
        *min = sc12[4 + j] & 0x3f;
        return;
    }
    *scale = (sc12[4 + j] & 0x0f) + 16 * (sc12[j - 4] >> 6);
    *min = (sc12[4 + j] >> 4) + 16 * (sc12[j] >> 6);
}

/* IQ2_XXS: the 256 grid points of iq.rs:17-34 (KGRID_2BIT_256), each a
 * base-4 number whose digit i is coordinate i: 0 -> 8, 1 -> 25, 2 -> 43 */
static const uint16_t ORF_KGRID[256] = {
    0, 2, 5, 8, 10, 17, 20, 32, 34, 40, 42, 65, 68, 80, 88, 97, 100, 128, 130, 138, 162, 257, 260, 272, 277, 320,
    388, 408, 512, 514, 546, 642, 1025, 1028, 1040, 1057, 1060, 1088, 1090, 1096, 1120, 1153, 1156, 1168, 1188,
    1280, 1282, 1288, 1312, 1350, 1385, 1408, 1425, 1545, 1552, 1600, 1668, 1700, 2048, 2053, 2056, 2068, 2088,
    2113, 2116, 2128, 2130, 2184, 2308, 2368, 2562, 2580, 4097, 4100, 4112, 4129, 4160, 4192, 4228, 4240, 4245,
    4352, 4360, 4384, 4432, 4442, 4480, 4644, 4677, 5120, 5128, 5152, 5157, 5193, 5248, 5400, 5474, 5632, 5654,
    6145, 6148, 6160, 6208, 6273, 6400, 6405, 6560, 6737, 8192, 8194, 8202, 8260, 8289, 8320, 8322, 8489, 8520,
    8704, 8706, 9217, 9220, 9232, 9280, 9302, 9472, 9537, 9572, 9872, 10248, 10272, 10388, 10820, 16385, 16388,
    16400, 16408, 16417, 16420, 16448, 16456, 16470, 16480, 16513, 16516, 16528, 16640, 16672, 16737, 16768,
    16773, 16897, 16912, 16968, 16982, 17000, 17408, 17416, 17440, 17536, 17561, 17682, 17700, 17920, 18433,
    18436, 18448, 18496, 18501, 18688, 18776, 18785, 18818, 19013, 19088, 20480, 20488, 20497, 20505, 20512,
    20608, 20616, 20740, 20802, 20900, 21137, 21648, 21650, 21770, 22017, 22100, 22528, 22545, 22553, 22628,
    22848, 23048, 24580, 24592, 24640, 24680, 24832, 24917, 25112, 25184, 25600, 25605, 25872, 25874, 25988,
    26690, 32768, 32770, 32778, 32833, 32898, 33028, 33048, 33088, 33297, 33793, 33796, 33808, 33813, 33856,
    33888, 34048, 34118, 34196, 34313, 34368, 34400, 34818, 35076, 35345, 36868, 36880, 36900, 36928, 37025,
    37142, 37248, 37445, 37888, 37922, 37956, 38225, 39041, 39200, 40962, 41040, 41093, 41225, 41472, 42008,
    43088, 43268};

/* the 8 magnitudes of grid point k as bytes of a u64 (byte i = coordinate i) */
static inline uint64_t orf_grid8(uint32_t k) {
    static const uint8_t level[3] = {8, 25, 43};
    uint64_t v = 0;
    for (int i = 7; i >= 0; i--) v = (v << 8) | level[(k >> (2 * i)) & 3u];
    return v;
}

/* 7 stored sign bits plus an 8th that makes the count of set bits even */
static inline uint32_t orf_signs8(uint32_t s7) {
    uint32_t n = 0;
    for (int i = 0; i < 7; i++) n += (s7 >> i) & 1u;
    return s7 | ((n & 1u) << 7);
}

/* MXFP4: E2M1 code -> twice its value {0, 0.5, 1, 1.5, 2, 3, 4, 6}, so
 * the decode stays integral; the sign is bit 3 */
static inline int orf_e2m1x2(int code) {
    static const int twice[8] = {0, 1, 2, 3, 4, 6, 8, 12};
    const int v = twice[code & 7];
    return (code & 8) ? -v : v;
}

/* E8M0 scale 2^(e-127), halved to undo the doubled codes: 2^(e-128);
 * exponent bytes 0 and 1 decode to zero (cu:1443-1449) */
static inline float orf_e8m0_half(uint32_t e) { return e < 2u ? 0.0f : ldexpf(1.0f, (int)e - 128); }

/* router exponential (binary32 steps only): x = k ln2 + r with k the
 * nearest integer to x log2(e) and ln2 split as 0.693145751953125 +
 * 1.428606765330187e-06 (both fma), exp(r) by its degree-7 Taylor
 * polynomial in Horner form (fma), scaled by 2^k in two exact halves */
static inline float orf_expf(float x) {
    if (isnan(x)) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const float k = rintf(x * 1.44269504088896340736f);
    const float r = fmaf(-k, 1.428606765330187045e-06f, fmaf(-k, 0.693145751953125f, x));
    static const float inv_fact[8] = {1.0f / 5040.0f, 1.0f / 720.0f, 1.0f / 120.0f, 1.0f / 24.0f,
                                      1.0f / 6.0f,    0.5f,          1.0f,          1.0f};
    float p = inv_fact[0];
    for (int i = 1; i < 8; i++) p = fmaf(p, r, inv_fact[i]);
    const int ki = (int)k, k1 = ki / 2, k2 = ki - k1;
    return (p * orf_bits_f32((uint32_t)(k1 + 127) << 23)) * orf_bits_f32((uint32_t)(k2 + 127) << 23);
}

/* sigmoid with the reference router's branches (cu:913-920) */
static inline float orf_sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + orf_expf(-x));
    const float e = orf_expf(x);
    return e / (1.0f + e);
}

#endif /* ORF_FORMAT_H */
