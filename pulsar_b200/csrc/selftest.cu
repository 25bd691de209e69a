/* selftest.cu - pulsar_router_selftest / pulsar_moe_selftest, the
 * device-vs-host self checks that crates/kernels/tests/selftests.rs runs
 * (reference cu:1271 and cu:6421).
 *
 * Router: the reference's shapes and its host reference (full softmax or
 * sigmoid over all experts, top-k, renormalise; cu:1140-1180), indices
 * exact and weights within 1e-5.  MoE: per expert format, random weights
 * encoded on the GPU, pair -> q8_K -> down on the GPU, and a binary64 host
 * mirror built from the decoded blocks; mid and out within
 * 1e-3 * max(max|ref|, 1) (cu:6318-6319), one NULL slot included.
 * These entry points allocate device memory; they are test entries, not
 * part of the inference path.
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/pulsar_moe.h"
#include "pm_format.h"
#include "pm_host.h"

static uint32_t st_rng = 0x1234567u;
static float st_randf(void) { /* u32 LCG in [-1, 1) */
    st_rng = st_rng * 1664525u + 1013904223u;
    return ((float)(st_rng >> 8) / (float)(1u << 24)) * 2.0f - 1.0f;
}
static float st_normal(void) { /* sum of 4 uniforms, unit variance */
    float s = 0.0f;
    for (int i = 0; i < 4; i++) s += st_randf();
    return s * 0.8660254f;
}

struct st_buf {
    void *p = nullptr;
    ~st_buf() {
        if (p) cudaFree(p);
    }
    bool alloc(size_t n) { return cudaMalloc(&p, n) == cudaSuccess; }
};

/* ---------------------------------------------------------------- router */

static int st_router_one(uint32_t E, uint32_t k, float scale, uint32_t T, uint32_t softmax) {
    const size_t nl = (size_t)T * E;
    float *logits = (float *)malloc(nl * 4), *bias = (float *)malloc(E * 4), *prob = (float *)malloc(E * 8);
    double *score = (double *)malloc(E * 8);
    int32_t *sel_ref = (int32_t *)malloc(T * k * 4), *sel = (int32_t *)malloc(T * k * 4);
    float *w = (float *)malloc(T * k * 4);
    double *w_ref = (double *)malloc(T * k * 8);
    for (size_t i = 0; i < nl; i++) logits[i] = st_randf() * 4.0f;
    for (uint32_t e = 0; e < E; e++) bias[e] = softmax ? 0.0f : st_randf();
    for (uint32_t t = 0; t < T; t++) {
        const float *lg = logits + (size_t)t * E;
        double mx = -INFINITY, sum = 0.0;
        if (softmax) {
            for (uint32_t e = 0; e < E; e++) mx = fmax(mx, lg[e]);
            for (uint32_t e = 0; e < E; e++) sum += exp((double)lg[e] - mx);
        }
        double *p = (double *)prob;
        for (uint32_t e = 0; e < E; e++) {
            p[e] = softmax ? exp((double)lg[e] - mx) / sum : 1.0 / (1.0 + exp(-(double)lg[e]));
            score[e] = p[e] + bias[e];
        }
        double ws = 0.0;
        for (uint32_t j = 0; j < k; j++) {
            uint32_t b = 0;
            for (uint32_t e = 1; e < E; e++)
                if (score[e] > score[b]) b = e;
            sel_ref[t * k + j] = (int32_t)b;
            w_ref[t * k + j] = p[b];
            ws += p[b];
            score[b] = -INFINITY;
        }
        ws = fmax(ws, 6.103515625e-5);
        for (uint32_t j = 0; j < k; j++) w_ref[t * k + j] = w_ref[t * k + j] / ws * scale;
    }
    st_buf dl, db, ds, dw;
    int ok = dl.alloc(nl * 4) && db.alloc(E * 4) && ds.alloc(T * k * 4) && dw.alloc(T * k * 4) &&
             cudaMemcpy(dl.p, logits, nl * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(db.p, bias, E * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             pulsar_router_select(ds.p, dw.p, dl.p, db.p, E, k, scale, T, softmax, 0) &&
             cudaDeviceSynchronize() == cudaSuccess &&
             cudaMemcpy(sel, ds.p, T * k * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
             cudaMemcpy(w, dw.p, T * k * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    uint32_t bad = 0;
    double maxd = 0.0;
    if (ok)
        for (uint32_t i = 0; i < T * k; i++) {
            bad += sel[i] != sel_ref[i];
            maxd = fmax(maxd, fabs((double)w[i] - w_ref[i]));
        }
    ok = ok && bad == 0 && maxd <= 1e-5;
    fprintf(stderr, "pulsar-b200 router-selftest E=%u k=%u%s: %s (idx mismatches %u, max w diff %.2e)\n", E, k,
            softmax ? " softmax" : "", ok ? "PASS" : "FAIL", bad, maxd);
    free(logits), free(bias), free(prob), free(score), free(sel_ref), free(sel), free(w), free(w_ref);
    return ok;
}

extern "C" int pulsar_router_selftest(void) {
    st_rng = 0x1234567u;
    return st_router_one(64, 8, 2.5f, 7, 0) && st_router_one(256, 8, 1.0f, 5, 0) && st_router_one(96, 6, 1.5f, 1, 0) &&
           st_router_one(128, 8, 1.0f, 6, 1) && st_router_one(384, 8, 1.0f, 3, 1) &&
           st_router_one(896, 16, 1.0f, 3, 0) && st_router_one(896, 16, 1.0f, 2, 1);
}

/* ------------------------------------------------------------------ moe */

/* decode n values of one row (host mirror of the block formats) */
static void st_dequant(uint32_t q, const uint8_t *row, uint32_t n, double *out) {
    for (uint32_t b0 = 0; b0 < n; b0 += 256) {
        const uint32_t sb = b0 / 256;
        if (q == PM_QUANT_Q4_K) {
            const uint8_t *b = row + sb * PM_Q4_K_BYTES;
            const double d = pm_f16_to_f32(pm_ld_u16(b)), dm = pm_f16_to_f32(pm_ld_u16(b + 2));
            for (int j = 0; j < 8; j++) {
                int sc, mn;
                pm_k4_scale_min(j, b + 4, &sc, &mn);
                for (int i = 0; i < 32; i++) {
                    const uint8_t v = b[16 + 32 * (j / 2) + i];
                    out[b0 + 32 * j + i] = d * sc * ((j & 1) ? (v >> 4) : (v & 15)) - dm * mn;
                }
            }
        } else if (q == PM_QUANT_Q2_K) {
            const uint8_t *b = row + sb * PM_Q2_K_BYTES;
            const double d = pm_f16_to_f32(pm_ld_u16(b + 80)), dm = pm_f16_to_f32(pm_ld_u16(b + 82));
            for (int c = 0; c < 16; c++)
                for (int i = 0; i < 16; i++) {
                    const int qv = (b[16 + 32 * (c / 8) + 16 * (c % 2) + i] >> (2 * ((c % 8) / 2))) & 3;
                    out[b0 + 16 * c + i] = d * (b[c] & 15) * qv - dm * (b[c] >> 4);
                }
        } else if (q == PM_QUANT_IQ2_XXS) {
            const uint8_t *b = row + sb * PM_IQ2_XXS_BYTES;
            const double d = pm_f16_to_f32(pm_ld_u16(b));
            for (int g = 0; g < 8; g++) {
                const uint32_t a0 = pm_ld_u32(b + 2 + 8 * g), a1 = pm_ld_u32(b + 6 + 8 * g);
                const double db = 0.125 * d * (2 * (a1 >> 28) + 1);
                for (int k = 0; k < 4; k++) {
                    const uint64_t gv = pm_iq2xxs_expand(PM_IQ2XXS_KGRID[(a0 >> (8 * k)) & 255]);
                    const uint32_t sm = pm_ksigns((a1 >> (7 * k)) & 127);
                    for (int i = 0; i < 8; i++)
                        out[b0 + 32 * g + 8 * k + i] = db * (double)((gv >> (8 * i)) & 255) * (((sm >> i) & 1) ? -1 : 1);
                }
            }
        } else {
            for (uint32_t bi = 0; bi < 8 && b0 + 32 * bi < n; bi++) {
                const uint32_t blk = b0 / 32 + bi;
                if (q == PM_QUANT_MXFP4) {
                    const uint8_t *b = row + blk * PM_MXFP4_BLOCK;
                    const double s = pm_mxfp4_scale_half(b[0]);
                    for (int i = 0; i < 16; i++) {
                        out[32 * blk + i] = s * pm_mxfp4_kv(b[1 + i] & 15);
                        out[32 * blk + 16 + i] = s * pm_mxfp4_kv(b[1 + i] >> 4);
                    }
                } else {
                    const uint8_t *b = row + blk * PM_Q8_0_BLOCK;
                    const double d = pm_f16_to_f32(pm_ld_u16(b));
                    for (int i = 0; i < 32; i++) out[32 * blk + i] = d * (int8_t)b[2 + i];
                }
            }
        }
    }
}

/* q8_K row -> values */
static void st_deq8k(const uint8_t *blocks, uint32_t n, double *out) {
    for (uint32_t i = 0; i < n; i++) {
        const pm_block_q8K *b = (const pm_block_q8K *)(blocks + (i / 256) * PM_Q8_K_BYTES);
        out[i] = (double)b->d * b->qs[i % 256];
    }
}

static double st_glu(double g, double u, uint32_t op) {
    if (op == 2) {
        g = fmin(g, 7.0);
        u = fmin(fmax(u, -7.0), 7.0);
        return g / (1.0 + exp(-1.702 * g)) * (u + 1.0);
    }
    return g / (1.0 + exp(-g)) * u;
}

static int st_moe_one(uint32_t quant, uint32_t H, uint32_t F, uint32_t act) {
    const uint32_t E = 8, k = 4, T = 3;
    const uint64_t rbg = pulsar_row_bytes(quant, H), rbd = pulsar_row_bytes(quant, F);
    const size_t gbytes = (size_t)E * F * rbg, dbytes = (size_t)E * H * rbd;
    const size_t nw = (size_t)E * F * H;
    float *wf = (float *)malloc(nw * 4 * 3), *x = (float *)malloc((size_t)T * H * 4);
    for (size_t i = 0; i < nw * 3; i++) wf[i] = 0.02f * st_normal();
    for (size_t i = 0; i < (size_t)T * H; i++) x[i] = st_normal();
    int32_t sel[12];
    float w[12];
    for (uint32_t i = 0; i < T * k; i++) {
        sel[i] = (int32_t)((i * 5 + 1) % E);
        w[i] = 0.1f + 0.05f * (float)i;
    }
    uint8_t *gh = (uint8_t *)malloc(gbytes), *uh = (uint8_t *)malloc(gbytes), *dh = (uint8_t *)malloc(dbytes);
    const size_t xqb = (size_t)T * ((H + 255) / 256) * PM_Q8_K_BYTES, mqb = (size_t)T * k * ((F + 255) / 256) * PM_Q8_K_BYTES;
    uint8_t *xqh = (uint8_t *)malloc(xqb), *mqh = (uint8_t *)malloc(mqb);
    float *mid = (float *)malloc((size_t)T * k * F * 4), *out = (float *)malloc((size_t)T * H * 4);
    st_buf dwf, dg, du, dd, dx, dxq, dmid, dmq, dout, dptr, dwt;
    int ok = dwf.alloc(nw * 4 * 3) && dg.alloc(gbytes + 256) && du.alloc(gbytes + 256) && dd.alloc(dbytes + 256) &&
             dx.alloc((size_t)T * H * 4) && dxq.alloc(xqb) && dmid.alloc((size_t)T * k * F * 4) && dmq.alloc(mqb) &&
             dout.alloc((size_t)T * H * 4) && dptr.alloc(T * k * sizeof(pulsar_expert_ptrs)) && dwt.alloc(T * k * 4);
    ok = ok && cudaMemcpy(dwf.p, wf, nw * 12, cudaMemcpyHostToDevice) == cudaSuccess &&
         pulsar_quantize_rows(dg.p, dwf.p, nullptr, quant, (uint64_t)E * F, H, nullptr) &&
         pulsar_quantize_rows(du.p, (float *)dwf.p + nw, nullptr, quant, (uint64_t)E * F, H, nullptr) &&
         pulsar_quantize_rows(dd.p, (float *)dwf.p + 2 * nw, nullptr, quant, (uint64_t)E * H, F, nullptr);
    pulsar_expert_ptrs ptrs[12];
    for (uint32_t i = 0; i < T * k; i++) {
        const uint32_t e = (uint32_t)sel[i];
        ptrs[i].gate = (uint8_t *)dg.p + e * F * rbg;
        ptrs[i].up = (uint8_t *)du.p + e * F * rbg;
        ptrs[i].down = (uint8_t *)dd.p + e * H * rbd;
        ptrs[i].gate_b = ptrs[i].up_b = ptrs[i].down_b = nullptr;
    }
    memset(&ptrs[5], 0, sizeof(ptrs[5])); /* one NULL slot */
    ok = ok && cudaMemcpy(dptr.p, ptrs, sizeof(ptrs[0]) * T * k, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(dwt.p, w, T * k * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(dx.p, x, (size_t)T * H * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         pulsar_quantize_q8_K(dxq.p, dx.p, H, T) &&
         pulsar_moe_pair_swiglu(dmid.p, dptr.p, dwt.p, dxq.p, H, F, k, T, rbg, quant, act) &&
         pulsar_quantize_q8_K(dmq.p, dmid.p, F, T * k) &&
         pulsar_moe_down(dout.p, dptr.p, dmq.p, F, H, k, T, rbd, quant) && cudaDeviceSynchronize() == cudaSuccess &&
         cudaMemcpy(gh, dg.p, gbytes, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(uh, du.p, gbytes, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(dh, dd.p, dbytes, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(xqh, dxq.p, xqb, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(mqh, dmq.p, mqb, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(mid, dmid.p, (size_t)T * k * F * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(out, dout.p, (size_t)T * H * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    double dm = 0, mm = 1, dout_max = 0, om = 1;
    if (ok) {
        double *xa = (double *)malloc(H * 8), *wr = (double *)malloc((H > F ? H : F) * 8), *ma = (double *)malloc(F * 8);
        for (uint32_t t = 0; t < T; t++) {
            st_deq8k(xqh + (size_t)t * ((H + 255) / 256) * PM_Q8_K_BYTES, H, xa);
            for (uint32_t s = 0; s < k; s++) {
                const uint32_t i = t * k + s, e = (uint32_t)sel[i];
                for (uint32_t r = 0; r < F; r++) {
                    double ref = 0.0;
                    if (i != 5) {
                        double g = 0.0, u = 0.0;
                        st_dequant(quant, gh + ((size_t)e * F + r) * rbg, H, wr);
                        for (uint32_t c = 0; c < H; c++) g += wr[c] * xa[c];
                        st_dequant(quant, uh + ((size_t)e * F + r) * rbg, H, wr);
                        for (uint32_t c = 0; c < H; c++) u += wr[c] * xa[c];
                        ref = st_glu(g, u, act) * w[i];
                    }
                    dm = fmax(dm, fabs(ref - mid[(size_t)i * F + r]));
                    mm = fmax(mm, fabs(ref));
                }
            }
            for (uint32_t r = 0; r < H; r++) {
                double ref = 0.0;
                for (uint32_t s = 0; s < k; s++) {
                    const uint32_t i = t * k + s;
                    if (i == 5) continue;
                    st_deq8k(mqh + (size_t)i * ((F + 255) / 256) * PM_Q8_K_BYTES, F, ma);
                    st_dequant(quant, dh + ((size_t)sel[i] * H + r) * rbd, F, wr);
                    for (uint32_t c = 0; c < F; c++) ref += wr[c] * ma[c];
                }
                dout_max = fmax(dout_max, fabs(ref - out[(size_t)t * H + r]));
                om = fmax(om, fabs(ref));
            }
        }
        free(xa), free(wr), free(ma);
        ok = dm <= 1e-3 * mm && dout_max <= 1e-3 * om;
    }
    fprintf(stderr, "pulsar-b200 moe-selftest quant=%u in=%u mid=%u: %s (mid %.2e, out %.2e)\n", quant, H, F,
            ok ? "PASS" : "FAIL", dm / mm, dout_max / om);
    free(wf), free(x), free(gh), free(uh), free(dh), free(xqh), free(mqh), free(mid), free(out);
    return ok;
}

extern "C" int pulsar_moe_selftest(void) {
    st_rng = 0x7654321u;
    return st_moe_one(PM_QUANT_Q4_K, 512, 512, 0) && st_moe_one(PM_QUANT_Q2_K, 512, 256, 0) &&
           st_moe_one(PM_QUANT_IQ2_XXS, 512, 256, 0) && st_moe_one(PM_QUANT_MXFP4, 704, 704, 2) &&
           st_moe_one(PM_QUANT_Q8_0, 704, 512, 0);
}

/* ------------------------------------------------- bounded-wait check */

#include "pm_device.cuh"

/* One thread waits, with the kernels' bounded wait, on an mbarrier phase
 * that nothing completes (count 1, no arrival): the wait runs out after
 * `cycles` SM cycles, records PM_ERR_TIMEOUT in the error word and
 * returns.  No copy is in flight and nothing is left waiting. */
__global__ void pm_wait_selftest_kernel(uint32_t *err, long long cycles) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    pm_mbar_init(&bar, 1);
    pm_fence_barrier_init();
    const bool ok = pm_mbar_wait_sleep(&bar, 0, err, cycles);
    if (ok) atomicOr(err, 0x80000000u); /* completed: must not happen */
}

extern "C" uint32_t pulsar_wait_selftest(uint64_t cycles) {
    if (cycles == 0 || cycles > (1ull << 31)) return 0xffffffffu;
    uint32_t *err = nullptr, host = 0xffffffffu;
    if (!pm_ok(cudaMalloc(&err, 4), "wait selftest alloc")) return 0xffffffffu;
    if (pm_ok(cudaMemset(err, 0, 4), "wait selftest clear")) {
        pm_wait_selftest_kernel<<<1, 32>>>(err, (long long)cycles);
        if (pm_ok(cudaGetLastError(), "wait selftest launch") && pm_ok(cudaDeviceSynchronize(), "wait selftest"))
            cudaMemcpy(&host, err, 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(err);
    return host;
}
