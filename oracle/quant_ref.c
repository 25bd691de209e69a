/* quant_ref.c - CPU restatement of pulsar's block encoders, the q8_K
 * activation quantizer and the per-format integer dots.
 *
 * TEST INFRASTRUCTURE ONLY (the parity oracle; see oracle.h).
 *
 * Float semantics follow the Rust originals: f32 arithmetic in source
 * order, no FMA contraction (built with -ffp-contract=off), round() =
 * half away from zero (roundf), sequential left-fold sums.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"
#include "ref_format.h"

static int nearest_int(float x) { return (int)roundf(x); }
static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ------------------------------------------------------------------ q8_0 */

/* crates/quant/src/lib.rs:251-265 quantize_row_q8_0 */
size_t orc_quantize_row_q8_0(const float *x, size_t n, uint8_t *out) {
    size_t o = 0;
    for (size_t b0 = 0; b0 < n; b0 += 32) {
        size_t len = n - b0 < 32 ? n - b0 : 32;
        float amax = 0.0f;
        for (size_t i = 0; i < len; i++) amax = fmaxf(amax, fabsf(x[b0 + i]));
        float d = amax / 127.0f;
        float id = d > 0.0f ? 1.0f / d : 0.0f;
        uint16_t h = orf_to_f16(d);
        out[o++] = (uint8_t)(h & 0xff);
        out[o++] = (uint8_t)(h >> 8);
        for (size_t i = 0; i < 32; i++) {
            float v = i < len ? x[b0 + i] : 0.0f;
            out[o++] = (uint8_t)(int8_t)clampi(nearest_int(v * id), -127, 127);
        }
    }
    return o;
}

/* ------------------------------------------------ make_qkx2_quants (ggml) */

/* crates/quant/src/lib.rs:163-246 */
static float make_qkx2_quants(int n, int nmax, const float *x, const float *weights, uint8_t *ls,
                              float *the_min, uint8_t *laux, float rmin, float rdelta, int nstep,
                              int use_mad) {
    float min = x[0], max = x[0];
    float sum_w = weights[0];
    float sum_x = sum_w * x[0];
    for (int i = 1; i < n; i++) {
        min = fminf(min, x[i]);
        max = fmaxf(max, x[i]);
        float w = weights[i];
        sum_w += w;
        sum_x += w * x[i];
    }
    if (min > 0.0f) min = 0.0f;
    if (max == min) {
        for (int i = 0; i < n; i++) ls[i] = 0;
        *the_min = -min;
        return 0.0f;
    }
    float iscale = (float)nmax / (max - min);
    float scale = 1.0f / iscale;
    float best_mad = 0.0f;
    for (int i = 0; i < n; i++) {
        int l = clampi(nearest_int(iscale * (x[i] - min)), 0, nmax);
        ls[i] = (uint8_t)l;
        float diff = scale * (float)l + min - x[i];
        diff = use_mad ? fabsf(diff) : diff * diff;
        best_mad += weights[i] * diff;
    }
    if (nstep < 1) {
        *the_min = -min;
        return scale;
    }
    for (int is = 0; is <= nstep; is++) {
        iscale = (rmin + rdelta * (float)is + (float)nmax) / (max - min);
        float sum_l = 0.0f, sum_l2 = 0.0f, sum_xl = 0.0f;
        for (int i = 0; i < n; i++) {
            int l = clampi(nearest_int(iscale * (x[i] - min)), 0, nmax);
            laux[i] = (uint8_t)l;
            float w = weights[i];
            sum_l += w * (float)l;
            sum_l2 += w * (float)(l * l);
            sum_xl += w * (float)l * x[i];
        }
        float D = sum_w * sum_l2 - sum_l * sum_l;
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
                memcpy(ls, laux, (size_t)n);
                best_mad = mad;
                scale = this_scale;
                min = this_min;
            }
        }
    }
    *the_min = -min;
    return scale;
}

/* ------------------------------------------------------------------ q2_K */

/* crates/quant/src/lib.rs:271-342 quantize_row_q2_k */
size_t orc_quantize_row_q2_k(const float *x, size_t n, uint8_t *out) {
    size_t o = 0;
    uint8_t ls[16], laux[16], lall[256];
    float weights[16];
    for (size_t b0 = 0; b0 + 256 <= n; b0 += 256) {
        const float *blk = x + b0;
        float scales[16], mins[16];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 16; j++) {
            const float *xs = blk + 16 * j;
            for (int l = 0; l < 16; l++) weights[l] = fabsf(xs[l]);
            float m = 0.0f;
            float s = make_qkx2_quants(16, 3, xs, weights, ls, &m, laux, -0.5f, 0.1f, 15, 1);
            memcpy(lall + 16 * j, ls, 16);
            scales[j] = s;
            mins[j] = m;
            max_scale = fmaxf(max_scale, s);
            max_min = fmaxf(max_min, m);
        }
        uint8_t sc[16] = {0};
        float d = 0.0f, dmin = 0.0f;
        if (max_scale > 0.0f) {
            float iscale = 15.0f / max_scale;
            for (int j = 0; j < 16; j++) sc[j] = (uint8_t)clampi(nearest_int(iscale * scales[j]), 0, 15);
            d = max_scale / 15.0f;
        }
        if (max_min > 0.0f) {
            float iscale = 15.0f / max_min;
            for (int j = 0; j < 16; j++)
                sc[j] |= (uint8_t)(clampi(nearest_int(iscale * mins[j]), 0, 15) << 4);
            dmin = max_min / 15.0f;
        }
        for (int j = 0; j < 16; j++) {
            float dj = d * (float)(sc[j] & 0xf);
            if (dj == 0.0f) {
                memset(lall + 16 * j, 0, 16);
                continue;
            }
            float mj = dmin * (float)(sc[j] >> 4);
            for (int l = 0; l < 16; l++)
                lall[16 * j + l] = (uint8_t)clampi(nearest_int((blk[16 * j + l] + mj) / dj), 0, 3);
        }
        memcpy(out + o, sc, 16);
        o += 16;
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 32; j++) {
                int base = 128 * h + j;
                out[o++] = (uint8_t)(lall[base] | (lall[base + 32] << 2) | (lall[base + 64] << 4) |
                                     (lall[base + 96] << 6));
            }
        uint16_t hd = orf_to_f16(d), hm = orf_to_f16(dmin);
        out[o++] = (uint8_t)(hd & 0xff);
        out[o++] = (uint8_t)(hd >> 8);
        out[o++] = (uint8_t)(hm & 0xff);
        out[o++] = (uint8_t)(hm >> 8);
    }
    return o;
}

/* ------------------------------------------------------------------ q4_K */

/* crates/quant/src/lib.rs:486-492 */
static void qkx_weights_av(const float *xs, int n, float *weights) {
    float sum_x2 = 0.0f;
    for (int i = 0; i < n; i++) sum_x2 += xs[i] * xs[i];
    float av_x = sqrtf(sum_x2 / (float)n);
    for (int i = 0; i < n; i++) weights[i] = av_x + fabsf(xs[i]);
}

/* crates/quant/src/lib.rs:494-509 */
static void pack_scale_min_k4(const uint8_t *sc_q, const uint8_t *mn_q, uint8_t *s) {
    memset(s, 0, 12);
    for (int j = 0; j < 8; j++) {
        uint8_t ls = sc_q[j], lm = mn_q[j];
        if (j < 4) {
            s[j] = ls;
            s[j + 4] = lm;
        } else {
            s[j + 4] = (uint8_t)((ls & 0xf) | ((lm & 0xf) << 4));
            s[j - 4] |= (uint8_t)((ls >> 4) << 6);
            s[j] |= (uint8_t)((lm >> 4) << 6);
        }
    }
}

/* crates/quant/src/lib.rs:570-585 quantize_row_q4_k (with qkx2_block_scales
 * :511-548 and requant_sub32 :550-568 inlined) */
size_t orc_quantize_row_q4_k(const float *x, size_t n, uint8_t *out) {
    size_t o = 0;
    uint8_t lall[256];
    for (size_t b0 = 0; b0 + 256 <= n; b0 += 256) {
        const float *blk = x + b0;
        float scales[8], mins[8];
        uint8_t ls[32], laux[32];
        float weights[32];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; j++) {
            const float *xs = blk + 32 * j;
            qkx_weights_av(xs, 32, weights);
            float m = 0.0f;
            float s = make_qkx2_quants(32, 15, xs, weights, ls, &m, laux, -1.0f, 0.1f, 20, 0);
            memcpy(lall + 32 * j, ls, 32);
            scales[j] = s;
            mins[j] = m;
            max_scale = fmaxf(max_scale, s);
            max_min = fmaxf(max_min, m);
        }
        float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
        float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
        uint8_t sc_q[8], mn_q[8];
        for (int j = 0; j < 8; j++) {
            sc_q[j] = (uint8_t)clampi(nearest_int(inv_scale * scales[j]), 0, 63);
            mn_q[j] = (uint8_t)clampi(nearest_int(inv_min * mins[j]), 0, 63);
        }
        float d = max_scale > 0.0f ? max_scale / 63.0f : 0.0f;
        float dmin = max_min > 0.0f ? max_min / 63.0f : 0.0f;
        /* requant with the f16-rounded scales */
        float dq = orf_f16(orf_to_f16(d));
        float mq = orf_f16(orf_to_f16(dmin));
        for (int j = 0; j < 8; j++) {
            float dj = dq * (float)sc_q[j];
            if (dj == 0.0f) {
                memset(lall + 32 * j, 0, 32);
                continue;
            }
            float mj = mq * (float)mn_q[j];
            for (int l = 0; l < 32; l++)
                lall[32 * j + l] = (uint8_t)clampi(nearest_int((blk[32 * j + l] + mj) / dj), 0, 15);
        }
        uint16_t hd = orf_to_f16(d), hm = orf_to_f16(dmin);
        out[o++] = (uint8_t)(hd & 0xff);
        out[o++] = (uint8_t)(hd >> 8);
        out[o++] = (uint8_t)(hm & 0xff);
        out[o++] = (uint8_t)(hm >> 8);
        pack_scale_min_k4(sc_q, mn_q, out + o);
        o += 12;
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) out[o++] = (uint8_t)(lall[64 * g + l] | (lall[64 * g + 32 + l] << 4));
    }
    return o;
}

/* --------------------------------------------------------------- iq2_xxs */

/* encoder tables (crates/quant/src/iq.rs:52-116): the grid in encoder
 * units 2l+1, the packed-index -> grid map, and the neighbour lists */
#define KMAP_SIZE 43692
typedef struct {
    int8_t grid[256][8];
    int32_t kmap[KMAP_SIZE];
    uint16_t *neigh;
    size_t n_neigh;
} iq2_tables;

static iq2_tables *g_iq2 = NULL;

typedef struct {
    int d2;
    int j;
} dist_ent;
static int dist_cmp(const void *a, const void *b) {
    const dist_ent *x = (const dist_ent *)a, *y = (const dist_ent *)b;
    if (x->d2 != y->d2) return x->d2 < y->d2 ? -1 : 1;
    return x->j < y->j ? -1 : (x->j > y->j);
}

static const iq2_tables *iq2_get(void) {
    if (g_iq2) return g_iq2;
    iq2_tables *t = (iq2_tables *)calloc(1, sizeof(iq2_tables));
    for (int i = 0; i < 256; i++)
        for (int k = 0; k < 8; k++) t->grid[i][k] = (int8_t)(2 * ((ORF_KGRID[i] >> (2 * k)) & 3) + 1);
    for (int i = 0; i < KMAP_SIZE; i++) t->kmap[i] = -1;
    for (int i = 0; i < 256; i++) {
        uint32_t index = 0;
        for (int k = 0; k < 8; k++) index |= (uint32_t)((t->grid[i][k] - 1) / 2) << (2 * k);
        t->kmap[index] = i;
    }
    size_t cap = 1u << 20, len = 0;
    uint16_t *nb = (uint16_t *)malloc(cap * sizeof(uint16_t));
    dist_ent dist[256];
    for (int i = 0; i < KMAP_SIZE; i++) {
        if (t->kmap[i] >= 0) continue;
        int pos[8];
        for (int k = 0; k < 8; k++) pos[k] = 2 * ((i >> (2 * k)) & 3) + 1;
        for (int j = 0; j < 256; j++) {
            int d2 = 0;
            for (int k = 0; k < 8; k++) {
                int df = t->grid[j][k] - pos[k];
                d2 += df * df;
            }
            dist[j].d2 = d2;
            dist[j].j = j;
        }
        qsort(dist, 256, sizeof(dist_ent), dist_cmp);
        if (len + 300 > cap) {
            cap *= 2;
            nb = (uint16_t *)realloc(nb, cap * sizeof(uint16_t));
        }
        size_t start = len;
        nb[len++] = 0;
        int n = 0, d2 = dist[0].d2, nhave = 1;
        for (int q = 0; q < 256; q++) {
            if (dist[q].d2 > d2) {
                if (nhave == 2) break;
                d2 = dist[q].d2;
                nhave++;
            }
            nb[len++] = (uint16_t)dist[q].j;
            n++;
        }
        nb[start] = (uint16_t)n;
        t->kmap[i] = -(int32_t)(start + 1);
    }
    t->neigh = nb;
    t->n_neigh = len;
    g_iq2 = t;
    return t;
}

/* crates/quant/src/iq.rs:122-186 make_qp_quants */
static float make_qp_quants(int n, int nmax, const float *x, uint8_t *ls, const float *qw) {
    float max = 0.0f;
    for (int i = 0; i < n; i++) max = fmaxf(max, x[i]);
    if (max < 1e-30f) {
        memset(ls, 0, (size_t)n);
        return 0.0f;
    }
    float iscale = (float)nmax / max;
    float scale = 1.0f / iscale;
    float best_mse = 0.0f;
    for (int i = 0; i < n; i++) {
        int l = nearest_int(iscale * x[i]);
        if (l > nmax) l = nmax;
        float diff = x[i] - scale * (float)l;
        best_mse += qw[i] * diff * diff;
    }
    for (int is = -4; is <= 4; is++) {
        if (is == 0) continue;
        float iscale_is = (0.1f * (float)is + (float)nmax) / max;
        float scale_is = 1.0f / iscale_is;
        float mse = 0.0f;
        for (int i = 0; i < n; i++) {
            int l = nearest_int(iscale_is * x[i]);
            if (l > nmax) l = nmax;
            float diff = x[i] - scale_is * (float)l;
            mse += qw[i] * diff * diff;
        }
        if (mse < best_mse) {
            best_mse = mse;
            iscale = iscale_is;
        }
    }
    float sumlx = 0.0f, suml2 = 0.0f;
    for (int i = 0; i < n; i++) {
        int l = nearest_int(iscale * x[i]);
        if (l > nmax) l = nmax;
        ls[i] = (uint8_t)l;
        sumlx += qw[i] * x[i] * (float)l;
        suml2 += qw[i] * (float)(l * l);
    }
    for (int it = 0; it < 5; it++) {
        int n_changed = 0;
        for (int i = 0; i < n; i++) {
            float w = qw[i];
            float slx = sumlx - w * x[i] * (float)ls[i];
            float sl2 = suml2 - w * (float)((int)ls[i] * (int)ls[i]);
            if (slx > 0.0f && sl2 > 0.0f) {
                int new_l = nearest_int(x[i] * sl2 / slx);
                if (new_l > nmax) new_l = nmax;
                if (new_l != (int)ls[i]) {
                    float slx2 = slx + w * x[i] * (float)new_l;
                    float sl22 = sl2 + w * (float)(new_l * new_l);
                    if (slx2 * slx2 * suml2 > sumlx * sumlx * sl22) {
                        ls[i] = (uint8_t)new_l;
                        sumlx = slx2;
                        suml2 = sl22;
                        n_changed++;
                    }
                }
            }
        }
        if (n_changed == 0) break;
    }
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

/* crates/quant/src/iq.rs:188-218 find_best_neighbour */
static int find_best_neighbour(const iq2_tables *t, size_t noff, const float *xval, const float *waux,
                               float scale, int8_t *ls) {
    int count = t->neigh[noff];
    float best_d2 = 3.40282347e+38f;
    int grid_index = -1;
    for (int q = 0; q < count; q++) {
        int j = t->neigh[noff + 1 + q];
        float d2 = 0.0f;
        for (int i = 0; i < 8; i++) {
            float diff = scale * (float)t->grid[j][i] - xval[i];
            d2 += waux[i] * diff * diff;
        }
        if (d2 < best_d2) {
            best_d2 = d2;
            grid_index = j;
        }
    }
    for (int i = 0; i < 8; i++) ls[i] = (int8_t)((t->grid[grid_index][i] - 1) / 2);
    return grid_index;
}

/* crates/quant/src/iq.rs:221-405 quantize_row_iq2_xxs */
size_t orc_quantize_row_iq2_xxs(const float *x, const float *qw, size_t n, uint8_t *out) {
    const iq2_tables *t = iq2_get();
    const int KMAXQ = 3;
    float weight[32], waux[32], xval[32];
    int8_t ls[32] = {0}, laux[32] = {0};
    uint8_t block_signs[4];
    size_t o = 0;
    for (size_t b0 = 0; b0 + 256 <= n; b0 += 256) {
        const float *xbl = x + b0;
        const float *qwbl = qw ? qw + b0 : NULL;
        uint32_t q2[16] = {0};
        float scales[8] = {0};
        float max_scale = 0.0f;
        float sigma2 = 0.0f;
        for (int i = 0; i < 256; i++) sigma2 += xbl[i] * xbl[i];
        sigma2 = sigma2 / 256.0f;
        for (int ib = 0; ib < 8; ib++) {
            const float *xb = xbl + 32 * ib;
            for (int i = 0; i < 32; i++) {
                float q = qwbl ? qwbl[32 * ib + i] : 1.0f;
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
                        float ax = weight[8 * k + i] * xb[8 * k + i] * xb[8 * k + i];
                        if (ax < mn) {
                            mn = ax;
                            imin = i;
                        }
                    }
                    xval[8 * k + imin] = -xval[8 * k + imin];
                    s ^= (uint8_t)(1u << imin);
                }
                block_signs[k] = s & 127;
            }
            float max = xval[0];
            for (int i = 0; i < 32; i++) max = fmaxf(max, xval[i]);
            if (max < 1e-30f) {
                scales[ib] = 0.0f;
                continue;
            }
            uint8_t lsu8[32];
            float scale = make_qp_quants(32, KMAXQ + 1, xval, lsu8, weight);
            float eff_max = scale * (float)KMAXQ;
            if (eff_max <= 0.0f) {
                scales[ib] = 0.0f;
                continue;
            }
            float best = 0.0f;
            /* ls holds the best candidate so far (the Rust keeps it across
             * sub-blocks; a fresh sub-block always improves on best = 0 when
             * any candidate has sumq2 > 0) */
            for (int is = -6; is <= 6; is++) {
                float id = (2.0f * (float)KMAXQ - 1.0f + (float)is * 0.1f) / eff_max;
                float this_scale = 1.0f / id;
                for (int k = 0; k < 4; k++) {
                    for (int i = 0; i < 8; i++) {
                        int l = clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, KMAXQ - 1);
                        laux[8 * k + i] = (int8_t)l;
                    }
                    uint32_t u = 0;
                    for (int i = 0; i < 8; i++) u |= (uint32_t)laux[8 * k + i] << (2 * i);
                    int gi = t->kmap[u];
                    if (gi < 0)
                        find_best_neighbour(t, (size_t)(-gi - 1), xval + 8 * k, waux + 8 * k, this_scale,
                                            laux + 8 * k);
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 32; i++) {
                    float q = (float)(2 * laux[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                    scale = sumqx / sumq2;
                    best = scale * sumqx;
                    memcpy(ls, laux, 32);
                }
            }
            if (scale > 0.0f) {
                float id = 1.0f / scale;
                for (int k = 0; k < 4; k++) {
                    uint32_t u = 0;
                    for (int i = 0; i < 8; i++) {
                        int l = clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, KMAXQ - 1);
                        u |= (uint32_t)l << (2 * i);
                    }
                    int gi = t->kmap[u];
                    int grid_index = gi;
                    if (gi < 0)
                        grid_index = find_best_neighbour(t, (size_t)(-gi - 1), xval + 8 * k, waux + 8 * k, scale,
                                                         ls + 8 * k);
                    for (int i = 0; i < 8; i++) ls[8 * k + i] = (int8_t)((t->grid[grid_index][i] - 1) / 2);
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 32; i++) {
                    float q = (float)(2 * ls[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f) scale = sumqx / sumq2;
            }
            if (scale < 0.0f) {
                scale = -scale;
                for (int k = 0; k < 4; k++) block_signs[k] = (uint8_t)(~block_signs[k] & 127);
            }
            for (int k = 0; k < 4; k++) {
                uint32_t u = 0;
                for (int i = 0; i < 8; i++) u |= (uint32_t)ls[8 * k + i] << (2 * i);
                int gi = t->kmap[u];
                if (gi < 0) abort(); /* off-grid point after the final requant */
                q2[2 * ib] |= (uint32_t)gi << (8 * k);
                q2[2 * ib + 1] |= (uint32_t)block_signs[k] << (7 * k);
            }
            scales[ib] = scale;
            max_scale = fmaxf(max_scale, scale);
        }
        if (max_scale == 0.0f) {
            memset(out + o, 0, 66);
            o += 66;
            continue;
        }
        float d = max_scale / 31.0f;
        float id = 1.0f / d;
        for (int ib = 0; ib < 8; ib++) {
            int l = clampi(nearest_int(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
            q2[2 * ib + 1] |= (uint32_t)l << 28;
        }
        uint16_t hd = orf_to_f16(d);
        out[o++] = (uint8_t)(hd & 0xff);
        out[o++] = (uint8_t)(hd >> 8);
        for (int i = 0; i < 16; i++) {
            out[o++] = (uint8_t)(q2[i] & 0xff);
            out[o++] = (uint8_t)((q2[i] >> 8) & 0xff);
            out[o++] = (uint8_t)((q2[i] >> 16) & 0xff);
            out[o++] = (uint8_t)(q2[i] >> 24);
        }
    }
    return o;
}

/* ----------------------------------------------------------------- MXFP4 */

/* OCP MX encoder (no reference encoder exists; decode pinned by cu:2053).
 * Per 32-block: shared exponent e = floor(log2(amax)) - 2 + 127, clamped
 * to [0, 254]; each value x / 2^(e-127) rounds to the nearest E2M1
 * magnitude {0, .5, 1, 1.5, 2, 3, 4, 6} with ties to the even code and
 * saturation at 6.  Byte i = code(elem i) | code(elem i+16) << 4. */
static int e2m1_code(float a) {
    /* a >= 0, already scaled; thresholds are the midpoints, ties to even */
    if (a <= 0.25f) return 0;
    if (a < 0.75f) return 1;
    if (a <= 1.25f) return 2;
    if (a < 1.75f) return 3;
    if (a <= 2.5f) return 4;
    if (a < 3.5f) return 5;
    if (a <= 5.0f) return 6;
    return 7;
}

size_t orc_quantize_row_mxfp4(const float *x, size_t n, uint8_t *out) {
    size_t o = 0;
    for (size_t b0 = 0; b0 < n; b0 += 32) {
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(b0 + i < n ? x[b0 + i] : 0.0f));
        int e = 0;
        if (amax > 0.0f) {
            int ex;
            (void)frexpf(amax, &ex); /* amax = m * 2^ex, m in [0.5, 1) */
            e = clampi(ex - 1 - 2 + 127, 0, 254);
        }
        out[o] = (uint8_t)e;
        /* 2^(127-e) as an exact power of two (e in [0,254]) */
        float inv = ldexpf(1.0f, 127 - e);
        for (int i = 0; i < 16; i++) {
            int c[2];
            for (int h = 0; h < 2; h++) {
                size_t idx = b0 + (size_t)i + 16u * (size_t)h;
                float v = idx < n ? x[idx] : 0.0f;
                int code = e == 0 ? 0 : e2m1_code(fabsf(v) * inv);
                if (code != 0 && v < 0.0f) code |= 8;
                c[h] = code;
            }
            out[o + 1 + i] = (uint8_t)(c[0] | (c[1] << 4));
        }
        o += 17;
    }
    return o;
}

/* --------------------------------------------------------- dispatch / rows */

uint64_t orc_row_bytes(int quant, uint64_t n) {
    switch (quant) {
    case ORF_Q2_K: return n / 256 * ORF_Q2_K_BYTES;
    case ORF_Q4_K: return n / 256 * ORF_Q4_K_BYTES;
    case ORF_IQ2_XXS: return n / 256 * ORF_IQ2_XXS_BYTES;
    case ORF_Q8_0: return (n + 31) / 32 * ORF_Q8_0_BLOCK;
    case ORF_MXFP4: return (n + 31) / 32 * ORF_MXFP4_BLOCK;
    default: return 0;
    }
}

int orc_quantize_rows(int quant, const float *x, size_t rows, size_t n, const float *qw, uint8_t *out) {
    uint64_t rb = orc_row_bytes(quant, n);
    if (!rb) return 0;
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * n;
        uint8_t *o = out + r * rb;
        switch (quant) {
        case ORF_Q2_K: orc_quantize_row_q2_k(xr, n, o); break;
        case ORF_Q4_K: orc_quantize_row_q4_k(xr, n, o); break;
        case ORF_IQ2_XXS: orc_quantize_row_iq2_xxs(xr, qw ? qw : NULL, n, o); break;
        case ORF_Q8_0: orc_quantize_row_q8_0(xr, n, o); break;
        case ORF_MXFP4: orc_quantize_row_mxfp4(xr, n, o); break;
        default: return 0;
        }
    }
    return 1;
}

/* --------------------------------------------------------------- dequant */

int orc_dequant_row(int quant, const uint8_t *row, size_t n, float *out) {
    switch (quant) {
    case ORF_Q4_K: /* cpu_dot.rs:224-240 dequant_q4_k */
        for (size_t ib = 0; ib < n / 256; ib++) {
            const uint8_t *b = row + ib * ORF_Q4_K_BYTES;
            float d = orf_f16(orf_u16(b)), dmin = orf_f16(orf_u16(b + 2));
            for (int j = 0; j < 4; j++) {
                int sc1, m1, sc2, m2;
                orf_k4_pair(2 * j, b + 4, &sc1, &m1);
                orf_k4_pair(2 * j + 1, b + 4, &sc2, &m2);
                for (int i = 0; i < 32; i++)
                    out[ib * 256 + 64 * j + i] = d * (float)sc1 * (float)(b[16 + 32 * j + i] & 15) - dmin * (float)m1;
                for (int i = 0; i < 32; i++)
                    out[ib * 256 + 64 * j + 32 + i] = d * (float)sc2 * (float)(b[16 + 32 * j + i] >> 4) - dmin * (float)m2;
            }
        }
        return 1;
    case ORF_Q2_K: /* cpu_dot.rs:870-890 (test-side dequant_q2_k) */
        for (size_t ib = 0; ib < n / 256; ib++) {
            const uint8_t *b = row + ib * ORF_Q2_K_BYTES;
            float d = orf_f16(orf_u16(b + 80)), dmin = orf_f16(orf_u16(b + 82));
            for (int c = 0; c < 16; c++) {
                int k = c / 8, js = (c % 8) / 2, half = c % 2;
                for (int i = 0; i < 16; i++) {
                    int q = (b[16 + 32 * k + 16 * half + i] >> (2 * js)) & 3;
                    out[ib * 256 + 16 * c + i] = d * (float)(b[c] & 15) * (float)q - dmin * (float)(b[c] >> 4);
                }
            }
        }
        return 1;
    case ORF_IQ2_XXS: /* cpu_dot.rs:785-806 dequant_row_iq2_xxs */
        for (size_t ib = 0; ib < n / 256; ib++) {
            const uint8_t *b = row + ib * ORF_IQ2_XXS_BYTES;
            float d = orf_f16(orf_u16(b));
            for (int g = 0; g < 8; g++) {
                uint32_t a0 = orf_u32(b + 2 + 8 * g), a1 = orf_u32(b + 6 + 8 * g);
                float db = 0.125f * d * (float)(2 * (a1 >> 28) + 1);
                for (int k = 0; k < 4; k++) {
                    uint64_t gv = orf_grid8(ORF_KGRID[(a0 >> (8 * k)) & 255]);
                    uint32_t sm = orf_signs8((a1 >> (7 * k)) & 127);
                    for (int i = 0; i < 8; i++) {
                        float v = db * (float)(int8_t)((gv >> (8 * i)) & 255);
                        out[ib * 256 + 32 * g + 8 * k + i] = ((sm >> i) & 1) ? -v : v;
                    }
                }
            }
        }
        return 1;
    case ORF_MXFP4:
        for (size_t b0 = 0; b0 < n; b0 += 32) {
            const uint8_t *b = row + (b0 / 32) * ORF_MXFP4_BLOCK;
            float s = orf_e8m0_half(b[0]);
            for (int i = 0; i < 16; i++) {
                if (b0 + i < n) out[b0 + i] = s * (float)orf_e2m1x2(b[1 + i] & 15);
                if (b0 + 16 + i < n) out[b0 + 16 + i] = s * (float)orf_e2m1x2(b[1 + i] >> 4);
            }
        }
        return 1;
    case ORF_Q8_0: /* cpu_dot.rs:206-216 dequant_q8_0 */
        for (size_t b0 = 0; b0 < n; b0 += 32) {
            const uint8_t *b = row + (b0 / 32) * ORF_Q8_0_BLOCK;
            float d = orf_f16(orf_u16(b));
            for (int i = 0; i < 32 && b0 + i < n; i++) out[b0 + i] = (float)(int8_t)b[2 + i] * d;
        }
        return 1;
    default: return 0;
    }
}

/* ------------------------------------------------------------------ q8_K */

/* crates/quant/src/cpu_dot.rs:26-50 quantize_row_q8_k, on 292-byte blocks;
 * a partial tail block quantizes as if zero-padded (cu:1499-1505) */
void orc_quantize_q8k(const float *x, size_t n, void *out_blocks) {
    orf_q8k *out = (orf_q8k *)out_blocks;
    size_t nb = (n + 255) / 256;
    for (size_t b = 0; b < nb; b++) {
        float v[256];
        for (int i = 0; i < 256; i++) v[i] = b * 256 + i < n ? x[b * 256 + i] : 0.0f;
        orf_q8k *y = out + b;
        float amax = 0.0f;
        for (int i = 0; i < 256; i++) amax = fmaxf(amax, fabsf(v[i]));
        if (amax == 0.0f) {
            memset(y, 0, sizeof(*y));
            continue;
        }
        float scale = amax / 127.0f;
        float inv = 127.0f / amax;
        y->d = scale;
        for (int i = 0; i < 256; i++) {
            float q = roundf(v[i] * inv);
            q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
            y->qs[i] = (int8_t)q;
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += y->qs[16 * g + i];
            y->bsums[g] = (int16_t)s;
        }
    }
}

void orc_quantize_q8k_rows(const float *x, size_t n, size_t rows, void *out_blocks) {
    size_t nb = (n + 255) / 256;
    for (size_t r = 0; r < rows; r++) orc_quantize_q8k(x + r * n, n, (orf_q8k *)out_blocks + r * nb);
}

/* ------------------------------------------------------------------ dots */

/* cpu_dot.rs:250-279 vec_dot_q4_k_q8_k_scalar */
static float dot_q4_k(const uint8_t *row, const orf_q8k *x, size_t nb) {
    float total = 0.0f;
    for (size_t ib = 0; ib < nb; ib++) {
        const uint8_t *b = row + ib * ORF_Q4_K_BYTES;
        float xd = orf_f16(orf_u16(b)), xmin = orf_f16(orf_u16(b + 2));
        const uint8_t *q4 = b + 16;
        const int8_t *q8 = x[ib].qs;
        const int16_t *bs = x[ib].bsums;
        int isum = 0, msum = 0;
        for (int j = 0; j < 4; j++) {
            int sc1, m1, sc2, m2;
            orf_k4_pair(2 * j, b + 4, &sc1, &m1);
            orf_k4_pair(2 * j + 1, b + 4, &sc2, &m2);
            int s1 = 0, s2 = 0;
            for (int i = 0; i < 32; i++) {
                uint8_t v = q4[32 * j + i];
                s1 += (v & 15) * q8[64 * j + i];
                s2 += (v >> 4) * q8[64 * j + 32 + i];
            }
            isum += sc1 * s1 + sc2 * s2;
            msum += m1 * (bs[4 * j] + bs[4 * j + 1]) + m2 * (bs[4 * j + 2] + bs[4 * j + 3]);
        }
        total += xd * x[ib].d * (float)isum - xmin * x[ib].d * (float)msum;
    }
    return total;
}

/* cpu_dot.rs:732-767 vec_dot_q2_k_q8_k_scalar */
static float dot_q2_k(const uint8_t *row, const orf_q8k *x, size_t nb) {
    float total = 0.0f;
    for (size_t ib = 0; ib < nb; ib++) {
        const uint8_t *b = row + ib * ORF_Q2_K_BYTES;
        const uint8_t *sc = b, *q2 = b + 16;
        float xd = orf_f16(orf_u16(b + 80)), xmin = orf_f16(orf_u16(b + 82));
        const int8_t *q8 = x[ib].qs;
        const int16_t *bs = x[ib].bsums;
        int summs = 0;
        for (int j = 0; j < 16; j++) summs += bs[j] * (sc[j] >> 4);
        int isum = 0, is = 0;
        for (int k = 0; k < 2; k++)
            for (int shift = 0; shift < 8; shift += 2)
                for (int half = 0; half < 2; half++) {
                    int d = sc[is++] & 15;
                    int sumi = 0;
                    for (int i = 0; i < 16; i++) {
                        int q = (q2[32 * k + 16 * half + i] >> shift) & 3;
                        sumi += q * q8[128 * k + 32 * (shift / 2) + 16 * half + i];
                    }
                    isum += d * sumi;
                }
        total += x[ib].d * xd * (float)isum - x[ib].d * xmin * (float)summs;
    }
    return total;
}

/* cpu_dot.rs:92-122 vec_dot_iq2_xxs_q8_k_scalar */
static float dot_iq2_xxs(const uint8_t *row, const orf_q8k *x, size_t nb) {
    float total = 0.0f;
    for (size_t ib = 0; ib < nb; ib++) {
        const uint8_t *b = row + ib * ORF_IQ2_XXS_BYTES;
        float xd = orf_f16(orf_u16(b));
        const int8_t *q8 = x[ib].qs;
        int bsum = 0;
        for (int g = 0; g < 8; g++) {
            uint32_t a0 = orf_u32(b + 2 + 8 * g), a1 = orf_u32(b + 6 + 8 * g);
            int ls = (int)(2 * (a1 >> 28) + 1);
            int sumi = 0;
            for (int k = 0; k < 4; k++) {
                uint64_t gv = orf_grid8(ORF_KGRID[(a0 >> (8 * k)) & 255]);
                uint32_t sm = orf_signs8((a1 >> (7 * k)) & 127);
                for (int i = 0; i < 8; i++) {
                    int w = (int)((gv >> (8 * i)) & 255);
                    if ((sm >> i) & 1) w = -w;
                    sumi += w * q8[32 * g + 8 * k + i];
                }
            }
            bsum += sumi * ls;
        }
        total += 0.125f * xd * x[ib].d * (float)bsum;
    }
    return total;
}

/* MXFP4 x q8_K, the reference GPU math (cu:2053-2073; host mirror
 * cu:5715-5741): per 32-block integer sum of doubled E2M1 values times
 * q8, scaled by 2^(e-128); per super-block yd * sum.  A partial tail
 * super-block only visits its real 32-blocks (the q8 tail is zero, so the
 * reference's extra blocks add exactly 0). */
static float dot_mxfp4(const uint8_t *row, const orf_q8k *x, size_t n) {
    float total = 0.0f;
    size_t nblk = (n + 31) / 32;
    for (size_t ib = 0; ib < (n + 255) / 256; ib++) {
        const int8_t *q8 = x[ib].qs;
        float sumf = 0.0f;
        for (size_t b = 0; b < 8 && ib * 8 + b < nblk; b++) {
            const uint8_t *bp = row + (ib * 8 + b) * ORF_MXFP4_BLOCK;
            int sumi = 0;
            for (int i = 0; i < 16; i++) {
                sumi += orf_e2m1x2(bp[1 + i] & 15) * q8[b * 32 + i];
                sumi += orf_e2m1x2(bp[1 + i] >> 4) * q8[b * 32 + 16 + i];
            }
            sumf += orf_e8m0_half(bp[0]) * (float)sumi;
        }
        total += x[ib].d * sumf;
    }
    return total;
}

/* Q8_0 x q8_K, the reference GPU math (cu:2174-2190): a zero integer sum
 * skips its block scale */
static float dot_q8_0(const uint8_t *row, const orf_q8k *x, size_t n) {
    float total = 0.0f;
    size_t nblk = (n + 31) / 32;
    for (size_t ib = 0; ib < (n + 255) / 256; ib++) {
        const int8_t *q8 = x[ib].qs;
        float sumf = 0.0f;
        for (size_t b = 0; b < 8 && ib * 8 + b < nblk; b++) {
            const uint8_t *bp = row + (ib * 8 + b) * ORF_Q8_0_BLOCK;
            int sumi = 0;
            for (int i = 0; i < 32; i++) sumi += (int8_t)bp[2 + i] * q8[b * 32 + i];
            if (sumi != 0) sumf += orf_f16(orf_u16(bp)) * (float)sumi;
        }
        total += x[ib].d * sumf;
    }
    return total;
}

float orc_vec_dot(int quant, const uint8_t *row, const void *xq_blocks, size_t n) {
    const orf_q8k *x = (const orf_q8k *)xq_blocks;
    switch (quant) {
    case ORF_Q4_K: return dot_q4_k(row, x, n / 256);
    case ORF_Q2_K: return dot_q2_k(row, x, n / 256);
    case ORF_IQ2_XXS: return dot_iq2_xxs(row, x, n / 256);
    case ORF_MXFP4: return dot_mxfp4(row, x, n);
    case ORF_Q8_0: return dot_q8_0(row, x, n);
    default: return NAN;
    }
}

float orc_expf(float x) { return orf_expf(x); }
float orc_sigmoid(float x) { return orf_sigmoid(x); }
uint64_t orc_iq2xxs_grid(int i) { return orf_grid8(ORF_KGRID[i & 255]); }
