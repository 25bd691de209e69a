/* encode.cu - GPU block encoders: f32 rows -> Q8_0 / Q2_K / Q4_K / IQ2_XXS
 * / MXFP4 bytes, byte-identical to the CPU encoders of crates/quant.
 *
 * Each thread encodes one block with the reference's sequential f32
 * arithmetic (this file is compiled with -fmad=false so no multiply-add
 * is contracted, matching the Rust originals), so the output bytes equal
 * the host encoders' bytes for the same input.
 *   q8_0     crates/quant/src/lib.rs:251-265
 *   q2_K     crates/quant/src/lib.rs:271-342 (make_qkx2_quants :163-246)
 *   q4_K     crates/quant/src/lib.rs:486-585
 *   iq2_xxs  crates/quant/src/iq.rs:52-405 (grid map and neighbour lists
 *            built once on the host and copied to device symbols)
 *   mxfp4    OCP MX: E8M0 = floor(log2 amax) - 2 + 127, E2M1 ties-to-even
 *            (no reference encoder; decode per cu:2053)
 * Used to build model weights from seeded f32 tensors on the device.
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/pulsar_moe.h"
#include "pm_format.h"
#include "pm_host.h"

__device__ __forceinline__ int pe_nearest(float x) { return (int)roundf(x); }
__device__ __forceinline__ int pe_clamp(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ------------------------------------------------------------ q8_0 */

__device__ void pe_q8_0(const float *x, uint32_t len, uint8_t *out) {
    float amax = 0.0f;
    for (uint32_t i = 0; i < len; i++) amax = fmaxf(amax, fabsf(x[i]));
    const float d = amax / 127.0f;
    const float id = d > 0.0f ? 1.0f / d : 0.0f;
    const uint16_t h = pm_f32_to_f16(d);
    out[0] = (uint8_t)h;
    out[1] = (uint8_t)(h >> 8);
    for (uint32_t i = 0; i < 32; i++) {
        const float v = i < len ? x[i] : 0.0f;
        out[2 + i] = (uint8_t)(int8_t)pe_clamp(pe_nearest(v * id), -127, 127);
    }
}

/* ------------------------------------------------ make_qkx2_quants */

__device__ float pe_qkx2(int n, int nmax, const float *x, const float *weights, uint8_t *ls, float *the_min,
                         uint8_t *laux, float rmin, float rdelta, int nstep, bool use_mad) {
    float mn = x[0], mx = x[0];
    float sum_w = weights[0];
    float sum_x = sum_w * x[0];
    for (int i = 1; i < n; i++) {
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
        const float w = weights[i];
        sum_w += w;
        sum_x += w * x[i];
    }
    if (mn > 0.0f) mn = 0.0f;
    if (mx == mn) {
        for (int i = 0; i < n; i++) ls[i] = 0;
        *the_min = -mn;
        return 0.0f;
    }
    float iscale = (float)nmax / (mx - mn);
    float scale = 1.0f / iscale;
    float best_mad = 0.0f;
    for (int i = 0; i < n; i++) {
        const int l = pe_clamp(pe_nearest(iscale * (x[i] - mn)), 0, nmax);
        ls[i] = (uint8_t)l;
        float diff = scale * (float)l + mn - x[i];
        diff = use_mad ? fabsf(diff) : diff * diff;
        best_mad += weights[i] * diff;
    }
    if (nstep < 1) {
        *the_min = -mn;
        return scale;
    }
    for (int is = 0; is <= nstep; is++) {
        iscale = (rmin + rdelta * (float)is + (float)nmax) / (mx - mn);
        float sum_l = 0.0f, sum_l2 = 0.0f, sum_xl = 0.0f;
        for (int i = 0; i < n; i++) {
            const int l = pe_clamp(pe_nearest(iscale * (x[i] - mn)), 0, nmax);
            laux[i] = (uint8_t)l;
            const float w = weights[i];
            sum_l += w * (float)l;
            sum_l2 += w * (float)(l * l);
            sum_xl += w * (float)l * x[i];
        }
        const float D = sum_w * sum_l2 - sum_l * sum_l;
        if (D > 0.0f) {
            float this_scale = (sum_w * sum_xl - sum_x * sum_l) / D;
            float this_min = (sum_l2 * sum_x - sum_l * sum_xl) / D;
            if (this_min > 0.0f) {
                this_min = 0.0f;
                this_scale = sum_l2 > 0.0f ? sum_xl / sum_l2 : 0.0f;
            }
            float mad = 0.0f;
            for (int i = 0; i < n; i++) {
                float diff = this_scale * (float)laux[i] + this_min - x[i];
                diff = use_mad ? fabsf(diff) : diff * diff;
                mad += weights[i] * diff;
            }
            if (mad < best_mad) {
                for (int i = 0; i < n; i++) ls[i] = laux[i];
                best_mad = mad;
                scale = this_scale;
                mn = this_min;
            }
        }
    }
    *the_min = -mn;
    return scale;
}

/* ------------------------------------------------------------ q2_K */

__device__ void pe_q2_k(const float *blk, uint8_t *out) {
    uint8_t ls[16], laux[16], lall[256];
    float weights[16], scales[16], mins[16];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 16; j++) {
        const float *xs = blk + 16 * j;
        for (int l = 0; l < 16; l++) weights[l] = fabsf(xs[l]);
        float m = 0.0f;
        const float s = pe_qkx2(16, 3, xs, weights, ls, &m, laux, -0.5f, 0.1f, 15, true);
        for (int l = 0; l < 16; l++) lall[16 * j + l] = ls[l];
        scales[j] = s;
        mins[j] = m;
        max_scale = fmaxf(max_scale, s);
        max_min = fmaxf(max_min, m);
    }
    uint8_t sc[16];
    for (int j = 0; j < 16; j++) sc[j] = 0;
    float d = 0.0f, dmin = 0.0f;
    if (max_scale > 0.0f) {
        const float iscale = 15.0f / max_scale;
        for (int j = 0; j < 16; j++) sc[j] = (uint8_t)pe_clamp(pe_nearest(iscale * scales[j]), 0, 15);
        d = max_scale / 15.0f;
    }
    if (max_min > 0.0f) {
        const float iscale = 15.0f / max_min;
        for (int j = 0; j < 16; j++) sc[j] |= (uint8_t)(pe_clamp(pe_nearest(iscale * mins[j]), 0, 15) << 4);
        dmin = max_min / 15.0f;
    }
    for (int j = 0; j < 16; j++) {
        const float dj = d * (float)(sc[j] & 0xf);
        if (dj == 0.0f) {
            for (int l = 0; l < 16; l++) lall[16 * j + l] = 0;
            continue;
        }
        const float mj = dmin * (float)(sc[j] >> 4);
        for (int l = 0; l < 16; l++)
            lall[16 * j + l] = (uint8_t)pe_clamp(pe_nearest((blk[16 * j + l] + mj) / dj), 0, 3);
    }
    for (int j = 0; j < 16; j++) out[j] = sc[j];
    for (int h = 0; h < 2; h++)
        for (int j = 0; j < 32; j++) {
            const int b = 128 * h + j;
            out[16 + 32 * h + j] =
                (uint8_t)(lall[b] | (lall[b + 32] << 2) | (lall[b + 64] << 4) | (lall[b + 96] << 6));
        }
    const uint16_t hd = pm_f32_to_f16(d), hm = pm_f32_to_f16(dmin);
    out[80] = (uint8_t)hd;
    out[81] = (uint8_t)(hd >> 8);
    out[82] = (uint8_t)hm;
    out[83] = (uint8_t)(hm >> 8);
}

/* ------------------------------------------------------------ q4_K */

__device__ void pe_q4_k(const float *blk, uint8_t *out) {
    uint8_t lall[256], ls[32], laux[32];
    float weights[32], scales[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
        const float *xs = blk + 32 * j;
        float sum_x2 = 0.0f;
        for (int i = 0; i < 32; i++) sum_x2 += xs[i] * xs[i];
        const float av_x = sqrtf(sum_x2 / 32.0f);
        for (int i = 0; i < 32; i++) weights[i] = av_x + fabsf(xs[i]);
        float m = 0.0f;
        const float s = pe_qkx2(32, 15, xs, weights, ls, &m, laux, -1.0f, 0.1f, 20, false);
        for (int i = 0; i < 32; i++) lall[32 * j + i] = ls[i];
        scales[j] = s;
        mins[j] = m;
        max_scale = fmaxf(max_scale, s);
        max_min = fmaxf(max_min, m);
    }
    const float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    const float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    uint8_t sc_q[8], mn_q[8];
    for (int j = 0; j < 8; j++) {
        sc_q[j] = (uint8_t)pe_clamp(pe_nearest(inv_scale * scales[j]), 0, 63);
        mn_q[j] = (uint8_t)pe_clamp(pe_nearest(inv_min * mins[j]), 0, 63);
    }
    const float d = max_scale > 0.0f ? max_scale / 63.0f : 0.0f;
    const float dmin = max_min > 0.0f ? max_min / 63.0f : 0.0f;
    const float dq = pm_f16_to_f32(pm_f32_to_f16(d));
    const float mq = pm_f16_to_f32(pm_f32_to_f16(dmin));
    for (int j = 0; j < 8; j++) {
        const float dj = dq * (float)sc_q[j];
        if (dj == 0.0f) {
            for (int l = 0; l < 32; l++) lall[32 * j + l] = 0;
            continue;
        }
        const float mj = mq * (float)mn_q[j];
        for (int l = 0; l < 32; l++)
            lall[32 * j + l] = (uint8_t)pe_clamp(pe_nearest((blk[32 * j + l] + mj) / dj), 0, 15);
    }
    const uint16_t hd = pm_f32_to_f16(d), hm = pm_f32_to_f16(dmin);
    out[0] = (uint8_t)hd;
    out[1] = (uint8_t)(hd >> 8);
    out[2] = (uint8_t)hm;
    out[3] = (uint8_t)(hm >> 8);
    uint8_t *s = out + 4;
    for (int j = 0; j < 12; j++) s[j] = 0;
    for (int j = 0; j < 8; j++) { /* pack 6-bit (scale, min) pairs (lib.rs:494-509) */
        if (j < 4) {
            s[j] = sc_q[j];
            s[j + 4] = mn_q[j];
        } else {
            s[j + 4] = (uint8_t)((sc_q[j] & 0xf) | ((mn_q[j] & 0xf) << 4));
            s[j - 4] |= (uint8_t)((sc_q[j] >> 4) << 6);
            s[j] |= (uint8_t)((mn_q[j] >> 4) << 6);
        }
    }
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) out[16 + 32 * g + l] = (uint8_t)(lall[64 * g + l] | (lall[64 * g + 32 + l] << 4));
}

/* ----------------------------------------------------------- mxfp4 */

__device__ __forceinline__ int pe_e2m1(float a) {
    if (a <= 0.25f) return 0;
    if (a < 0.75f) return 1;
    if (a <= 1.25f) return 2;
    if (a < 1.75f) return 3;
    if (a <= 2.5f) return 4;
    if (a < 3.5f) return 5;
    if (a <= 5.0f) return 6;
    return 7;
}

__device__ void pe_mxfp4(const float *x, uint32_t len, uint8_t *out) {
    float amax = 0.0f;
    for (uint32_t i = 0; i < len; i++) amax = fmaxf(amax, fabsf(x[i]));
    int e = 0;
    if (amax > 0.0f) {
        int ex;
        (void)frexpf(amax, &ex);
        e = pe_clamp(ex - 1 - 2 + 127, 0, 254);
    }
    out[0] = (uint8_t)e;
    const float inv = ldexpf(1.0f, 127 - e);
    for (int i = 0; i < 16; i++) {
        int c[2];
        for (int h = 0; h < 2; h++) {
            const uint32_t idx = (uint32_t)i + 16u * (uint32_t)h;
            const float v = idx < len ? x[idx] : 0.0f;
            int code = e == 0 ? 0 : pe_e2m1(fabsf(v) * inv);
            if (code != 0 && v < 0.0f) code |= 8;
            c[h] = code;
        }
        out[1 + i] = (uint8_t)(c[0] | (c[1] << 4));
    }
}

/* --------------------------------------------------------- iq2_xxs */

#define PE_KMAP 43692
#define PE_NEIGH_MAX (1u << 19)
__device__ int32_t pe_kmap[PE_KMAP];
__device__ uint16_t pe_neigh[PE_NEIGH_MAX];
__device__ static const uint16_t pe_kgrid[256] = PM_IQ2XXS_KGRID_INIT;

/* grid coordinate i of point g in encoder units (2 * digit + 1) */
__device__ __forceinline__ int pe_g(int g, int i) { return 2 * ((pe_kgrid[g] >> (2 * i)) & 3) + 1; }

static int pe_tables_ready[64];

/* packed-index -> grid map and neighbour lists (iq.rs:52-116), host-built */
static int pe_iq2_tables_upload() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && pe_tables_ready[dev]) return 1;
    int32_t *kmap = (int32_t *)malloc(PE_KMAP * sizeof(int32_t));
    uint16_t *nb = (uint16_t *)malloc(PE_NEIGH_MAX * sizeof(uint16_t));
    if (!kmap || !nb) {
        free(kmap);
        free(nb);
        return 0;
    }
    int grid[256][8];
    for (int g = 0; g < 256; g++)
        for (int i = 0; i < 8; i++) grid[g][i] = 2 * ((PM_IQ2XXS_KGRID[g] >> (2 * i)) & 3) + 1;
    for (int i = 0; i < PE_KMAP; i++) kmap[i] = -1;
    for (int g = 0; g < 256; g++) {
        uint32_t idx = 0;
        for (int i = 0; i < 8; i++) idx |= (uint32_t)((grid[g][i] - 1) / 2) << (2 * i);
        kmap[idx] = g;
    }
    size_t len = 0;
    int ok = 1;
    for (int p = 0; p < PE_KMAP && ok; p++) {
        if (kmap[p] >= 0) continue;
        int pos[8];
        for (int i = 0; i < 8; i++) pos[i] = 2 * ((p >> (2 * i)) & 3) + 1;
        int d2s[256];
        for (int g = 0; g < 256; g++) {
            int d2 = 0;
            for (int i = 0; i < 8; i++) d2 += (grid[g][i] - pos[i]) * (grid[g][i] - pos[i]);
            d2s[g] = d2;
        }
        /* the two smallest distinct distances, all points at them, by index */
        int m1 = 1 << 30, m2 = 1 << 30;
        for (int g = 0; g < 256; g++) m1 = d2s[g] < m1 ? d2s[g] : m1;
        for (int g = 0; g < 256; g++) m2 = d2s[g] > m1 && d2s[g] < m2 ? d2s[g] : m2;
        const size_t start = len;
        if (len + 258 > PE_NEIGH_MAX) {
            ok = 0;
            break;
        }
        nb[len++] = 0;
        uint16_t n = 0;
        for (int pass = 0; pass < 2; pass++)
            for (int g = 0; g < 256; g++)
                if (d2s[g] == (pass ? m2 : m1)) {
                    nb[len++] = (uint16_t)g;
                    n++;
                }
        nb[start] = n;
        kmap[p] = -(int32_t)(start + 1);
    }
    ok = ok && pm_ok(cudaMemcpyToSymbol(pe_kmap, kmap, PE_KMAP * sizeof(int32_t)), "iq2 kmap upload") &&
         pm_ok(cudaMemcpyToSymbol(pe_neigh, nb, len * sizeof(uint16_t)), "iq2 neighbours upload");
    free(kmap);
    free(nb);
    if (ok && dev < 64) pe_tables_ready[dev] = 1;
    return ok;
}

__device__ float pe_qp(int n, int nmax, const float *x, uint8_t *ls, const float *qw) {
    float mx = 0.0f;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
    if (mx < 1e-30f) {
        for (int i = 0; i < n; i++) ls[i] = 0;
        return 0.0f;
    }
    float iscale = (float)nmax / mx;
    const float scale = 1.0f / iscale;
    float best_mse = 0.0f;
    for (int i = 0; i < n; i++) {
        int l = pe_nearest(iscale * x[i]);
        if (l > nmax) l = nmax;
        const float diff = x[i] - scale * (float)l;
        best_mse += qw[i] * diff * diff;
    }
    for (int is = -4; is <= 4; is++) {
        if (is == 0) continue;
        const float iscale_is = (0.1f * (float)is + (float)nmax) / mx;
        const float scale_is = 1.0f / iscale_is;
        float mse = 0.0f;
        for (int i = 0; i < n; i++) {
            int l = pe_nearest(iscale_is * x[i]);
            if (l > nmax) l = nmax;
            const float diff = x[i] - scale_is * (float)l;
            mse += qw[i] * diff * diff;
        }
        if (mse < best_mse) {
            best_mse = mse;
            iscale = iscale_is;
        }
    }
    float sumlx = 0.0f, suml2 = 0.0f;
    for (int i = 0; i < n; i++) {
        int l = pe_nearest(iscale * x[i]);
        if (l > nmax) l = nmax;
        ls[i] = (uint8_t)l;
        sumlx += qw[i] * x[i] * (float)l;
        suml2 += qw[i] * (float)(l * l);
    }
    for (int it = 0; it < 5; it++) {
        int changed = 0;
        for (int i = 0; i < n; i++) {
            const float w = qw[i];
            const float slx = sumlx - w * x[i] * (float)ls[i];
            const float sl2 = suml2 - w * (float)((int)ls[i] * (int)ls[i]);
            if (slx > 0.0f && sl2 > 0.0f) {
                int nl = pe_nearest(x[i] * sl2 / slx);
                if (nl > nmax) nl = nmax;
                if (nl != (int)ls[i]) {
                    const float slx2 = slx + w * x[i] * (float)nl;
                    const float sl22 = sl2 + w * (float)(nl * nl);
                    if (slx2 * slx2 * suml2 > sumlx * sumlx * sl22) {
                        ls[i] = (uint8_t)nl;
                        sumlx = slx2;
                        suml2 = sl22;
                        changed++;
                    }
                }
            }
        }
        if (!changed) break;
    }
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

__device__ int pe_best_neighbour(uint32_t noff, const float *xval, const float *waux, float scale, int8_t *ls) {
    const int count = pe_neigh[noff];
    float best_d2 = 3.40282347e+38f;
    int gi = -1;
    for (int q = 0; q < count; q++) {
        const int j = pe_neigh[noff + 1 + q];
        float d2 = 0.0f;
        for (int i = 0; i < 8; i++) {
            const float diff = scale * (float)pe_g(j, i) - xval[i];
            d2 += waux[i] * diff * diff;
        }
        if (d2 < best_d2) {
            best_d2 = d2;
            gi = j;
        }
    }
    for (int i = 0; i < 8; i++) ls[i] = (int8_t)((pe_g(gi, i) - 1) / 2);
    return gi;
}

/* one 256-value block; ls persists across sub-blocks like the Rust */
__device__ void pe_iq2_xxs(const float *xbl, const float *qwbl, uint8_t *out) {
    const int KQ = 3;
    float weight[32], waux[32], xval[32], scales[8];
    int8_t ls[32], laux[32];
    uint8_t signs[4];
    uint32_t q2[16];
    for (int i = 0; i < 32; i++) ls[i] = 0, laux[i] = 0;
    for (int i = 0; i < 16; i++) q2[i] = 0;
    float max_scale = 0.0f, sigma2 = 0.0f;
    for (int i = 0; i < 256; i++) sigma2 += xbl[i] * xbl[i];
    sigma2 = sigma2 / 256.0f;
    for (int ib = 0; ib < 8; ib++) {
        const float *xb = xbl + 32 * ib;
        for (int i = 0; i < 32; i++) {
            const float q = qwbl ? qwbl[32 * ib + i] : 1.0f;
            weight[i] = q * sqrtf(sigma2 + xb[i] * xb[i]);
            waux[i] = sqrtf(weight[i]);
        }
        for (int k = 0; k < 4; k++) {
            int nflip = 0;
            uint8_t s = 0;
            for (int i = 0; i < 8; i++) {
                if (xb[8 * k + i] >= 0.0f) {
                    xval[8 * k + i] = xb[8 * k + i];
                } else {
                    xval[8 * k + i] = -xb[8 * k + i];
                    nflip++;
                    s |= (uint8_t)(1u << i);
                }
            }
            if (nflip % 2 == 1) {
                int imin = 0;
                float mn = weight[8 * k] * xb[8 * k] * xb[8 * k];
                for (int i = 1; i < 8; i++) {
                    const float ax = weight[8 * k + i] * xb[8 * k + i] * xb[8 * k + i];
                    if (ax < mn) {
                        mn = ax;
                        imin = i;
                    }
                }
                xval[8 * k + imin] = -xval[8 * k + imin];
                s ^= (uint8_t)(1u << imin);
            }
            signs[k] = s & 127;
        }
        float mx = xval[0];
        for (int i = 0; i < 32; i++) mx = fmaxf(mx, xval[i]);
        if (mx < 1e-30f) {
            scales[ib] = 0.0f;
            continue;
        }
        uint8_t lsu8[32];
        float scale = pe_qp(32, KQ + 1, xval, lsu8, weight);
        const float eff_max = scale * (float)KQ;
        if (eff_max <= 0.0f) {
            scales[ib] = 0.0f;
            continue;
        }
        float best = 0.0f;
        for (int is = -6; is <= 6; is++) {
            const float id = (2.0f * (float)KQ - 1.0f + (float)is * 0.1f) / eff_max;
            const float this_scale = 1.0f / id;
            for (int k = 0; k < 4; k++) {
                uint32_t u = 0;
                for (int i = 0; i < 8; i++) {
                    const int l = pe_clamp(pe_nearest(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, KQ - 1);
                    laux[8 * k + i] = (int8_t)l;
                    u |= (uint32_t)l << (2 * i);
                }
                const int gi = pe_kmap[u];
                if (gi < 0)
                    pe_best_neighbour((uint32_t)(-gi - 1), xval + 8 * k, waux + 8 * k, this_scale, laux + 8 * k);
            }
            float sumqx = 0.0f, sumq2 = 0.0f;
            for (int i = 0; i < 32; i++) {
                const float q = (float)(2 * laux[i] + 1);
                sumqx += weight[i] * xval[i] * q;
                sumq2 += weight[i] * q * q;
            }
            if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                scale = sumqx / sumq2;
                best = scale * sumqx;
                for (int i = 0; i < 32; i++) ls[i] = laux[i];
            }
        }
        if (scale > 0.0f) {
            const float id = 1.0f / scale;
            for (int k = 0; k < 4; k++) {
                uint32_t u = 0;
                for (int i = 0; i < 8; i++) {
                    const int l = pe_clamp(pe_nearest(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, KQ - 1);
                    u |= (uint32_t)l << (2 * i);
                }
                int gi = pe_kmap[u];
                if (gi < 0) gi = pe_best_neighbour((uint32_t)(-gi - 1), xval + 8 * k, waux + 8 * k, scale, ls + 8 * k);
                for (int i = 0; i < 8; i++) ls[8 * k + i] = (int8_t)((pe_g(gi, i) - 1) / 2);
            }
            float sumqx = 0.0f, sumq2 = 0.0f;
            for (int i = 0; i < 32; i++) {
                const float q = (float)(2 * ls[i] + 1);
                sumqx += weight[i] * xval[i] * q;
                sumq2 += weight[i] * q * q;
            }
            if (sumq2 > 0.0f) scale = sumqx / sumq2;
        }
        if (scale < 0.0f) {
            scale = -scale;
            for (int k = 0; k < 4; k++) signs[k] = (uint8_t)(~signs[k] & 127);
        }
        for (int k = 0; k < 4; k++) {
            uint32_t u = 0;
            for (int i = 0; i < 8; i++) u |= (uint32_t)ls[8 * k + i] << (2 * i);
            const int gi = pe_kmap[u]; /* on-grid by construction */
            q2[2 * ib] |= (uint32_t)(gi < 0 ? 0 : gi) << (8 * k);
            q2[2 * ib + 1] |= (uint32_t)signs[k] << (7 * k);
        }
        scales[ib] = scale;
        max_scale = fmaxf(max_scale, scale);
    }
    if (max_scale == 0.0f) {
        for (int i = 0; i < 66; i++) out[i] = 0;
        return;
    }
    const float d = max_scale / 31.0f;
    const float id = 1.0f / d;
    for (int ib = 0; ib < 8; ib++) {
        const int l = pe_clamp(pe_nearest(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
        q2[2 * ib + 1] |= (uint32_t)l << 28;
    }
    const uint16_t hd = pm_f32_to_f16(d);
    out[0] = (uint8_t)hd;
    out[1] = (uint8_t)(hd >> 8);
    for (int i = 0; i < 16; i++) {
        out[2 + 4 * i] = (uint8_t)q2[i];
        out[3 + 4 * i] = (uint8_t)(q2[i] >> 8);
        out[4 + 4 * i] = (uint8_t)(q2[i] >> 16);
        out[5 + 4 * i] = (uint8_t)(q2[i] >> 24);
    }
}

/* ---------------------------------------------------------- kernels */

/* one thread per block: 256 values (K-quants, iq2_xxs) or 32 (q8_0, mxfp4) */
__global__ void pe_encode_kernel(uint8_t *out, const float *x, const float *qw, uint32_t quant, uint64_t rows,
                                 uint32_t n, uint64_t rb, uint32_t bvals, uint32_t bbytes) {
    const uint32_t nblk = (n + bvals - 1) / bvals;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nblk) return;
    const uint64_t r = gid / nblk;
    const uint32_t b = (uint32_t)(gid % nblk);
    const float *xb = x + r * n + (uint64_t)b * bvals;
    uint8_t *ob = out + r * rb + (uint64_t)b * bbytes;
    const uint32_t len = n - b * bvals < bvals ? n - b * bvals : bvals;
    switch (quant) {
    case PM_QUANT_Q8_0: pe_q8_0(xb, len, ob); break;
    case PM_QUANT_MXFP4: pe_mxfp4(xb, len, ob); break;
    case PM_QUANT_Q2_K: pe_q2_k(xb, ob); break;
    case PM_QUANT_Q4_K: pe_q4_k(xb, ob); break;
    case PM_QUANT_IQ2_XXS: pe_iq2_xxs(xb, qw ? qw + (uint64_t)b * 256u : nullptr, ob); break;
    }
}

extern "C" uint64_t pulsar_row_bytes(uint32_t quant, uint32_t n) {
    switch (quant) {
    case PM_QUANT_Q4_K: return n % 256 ? 0 : (uint64_t)n / 256 * PM_Q4_K_BYTES;
    case PM_QUANT_Q2_K: return n % 256 ? 0 : (uint64_t)n / 256 * PM_Q2_K_BYTES;
    case PM_QUANT_IQ2_XXS: return n % 256 ? 0 : (uint64_t)n / 256 * PM_IQ2_XXS_BYTES;
    case PM_QUANT_MXFP4: return n % 32 ? 0 : (uint64_t)n / 32 * PM_MXFP4_BLOCK;
    case PM_QUANT_Q8_0: return n % 32 ? 0 : (uint64_t)n / 32 * PM_Q8_0_BLOCK;
    default: return 0;
    }
}

/* x f32 [rows][n] -> out [rows][row_bytes]; qw: per-column importance [n]
 * for iq2_xxs (NULL = uniform 1.0) */
extern "C" int pulsar_quantize_rows(void *out, const void *x, const void *qw, uint32_t quant, uint64_t rows,
                                    uint32_t n, void *stream) {
    const uint64_t rb = pulsar_row_bytes(quant, n);
    if (!out || !x || !rows || !rb) return 0;
    if (quant == PM_QUANT_IQ2_XXS && !pe_iq2_tables_upload()) return 0;
    const bool small = quant == PM_QUANT_Q8_0 || quant == PM_QUANT_MXFP4;
    const uint32_t bvals = small ? 32u : 256u;
    const uint32_t bbytes = quant == PM_QUANT_Q8_0 ? PM_Q8_0_BLOCK
                            : quant == PM_QUANT_MXFP4 ? PM_MXFP4_BLOCK
                            : (uint32_t)(rb / (n / 256u));
    const uint64_t threads = rows * ((n + bvals - 1) / bvals);
    const uint32_t tpb = small ? 256u : 64u;
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    pe_encode_kernel<<<(uint32_t)((threads + tpb - 1) / tpb), tpb, 0, st>>>(
        (uint8_t *)out, (const float *)x, (const float *)qw, quant, rows, n, rb, bvals, bbytes);
    return pm_ok(cudaGetLastError(), "quantize rows launch");
}
