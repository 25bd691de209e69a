/* lane_ref.c - CPU restatement of the router and of pulsar's CPU expert
 * lane (the expert FFN), threaded like the reference lane.
 *
 * TEST INFRASTRUCTURE ONLY (the parity oracle; see oracle.h).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "oracle.h"
#include "ref_format.h"

/* ---------------------------------------------------------------- glu */

/* crates/engine/src/lib.rs:2134-2159 glu (cu:124 pulsar_glu): 0 silu,
 * 1 gelu tanh, 2 swiglu_oai, 3 clamped silu, 4 SiTU-GLU */
float orc_glu(float g, float u, uint32_t op) {
    switch (op) {
    case 1: return 0.5f * g * (1.0f + tanhf(0.7978846f * (g + 0.044715f * g * g * g))) * u;
    case 2:
        g = fminf(g, 7.0f);
        u = fminf(fmaxf(u, -7.0f), 7.0f);
        return g / (1.0f + expf(-1.702f * g)) * (u + 1.0f);
    case 3:
        g = fminf(g, 10.0f);
        u = fminf(fmaxf(u, -10.0f), 10.0f);
        return g / (1.0f + expf(-g)) * u;
    case 4: {
        float a = 4.0f * tanhf(g / 4.0f) / (1.0f + expf(-g));
        return a * (25.0f * tanhf(u / 25.0f));
    }
    default: return g / (1.0f + expf(-g)) * u;
    }
}

/* ------------------------------------------------------------- router */

/* Router logits, the contract the CUDA router keeps bit-for-bit:
 * logit[t][e] = S(t, e) + logit_bias[e], where S is the f32 dot of the f32
 * router row with the f32 hidden row in a fixed order: 32 partial sums p_L
 * (L = 0..31) over the indices i = 128 j + 4 L + c (j ascending, then
 * c = 0..3), each step one fused multiply-add, followed by the butterfly
 * p_L += p_(L^m) for m = 16, 8, 4, 2, 1.  The reference computes the same dot
 * in f32 with a 256-way tree (cu:6504-6524); the fixed order is this
 * project's choice so that top-k ties resolve identically on host and
 * device. */
void orc_router_logits(float *logits, const float *w, const float *x, const float *logit_bias,
                       uint32_t n_expert, uint32_t in_dim, uint32_t n_tok) {
    const uint32_t nj = (in_dim + 127) / 128;
    for (uint32_t t = 0; t < n_tok; t++) {
        const float *xr = x + (size_t)t * in_dim;
        for (uint32_t e = 0; e < n_expert; e++) {
            const float *wr = w + (size_t)e * in_dim;
            float p[32];
            for (int L = 0; L < 32; L++) {
                float s = 0.0f;
                for (uint32_t j = 0; j < nj; j++)
                    for (int c = 0; c < 4; c++) {
                        uint32_t i = 128 * j + 4 * (uint32_t)L + (uint32_t)c;
                        if (i < in_dim) s = fmaf(wr[i], xr[i], s);
                    }
                p[L] = s;
            }
            for (int m = 16; m >= 1; m >>= 1) {
                float q[32];
                for (int L = 0; L < 32; L++) q[L] = p[L] + p[L ^ m];
                memcpy(p, q, sizeof(p));
            }
            float l = p[0];
            if (logit_bias) l = l + logit_bias[e];
            logits[(size_t)t * n_expert + e] = l;
        }
    }
}

static int better(float av, uint32_t ai, float bv, uint32_t bi) { return av > bv || (av == bv && ai < bi); }

/* Top-k selection and route weights, router_select_kernel semantics
 * (cu:939-1050):
 *   mode 0  p = sigmoid(l), score = p + bias, w = p / max(sum p, 2^-14) * scale
 *   mode 1  score = l + bias, w = softmax over the selected raw logits * scale
 *   mode 2  sink: mode-0 selection, shared logits appended as slots
 *           k..k+n_shexp, w = softmax(logsigmoid(raw)) * scale
 * ties go to the lower expert index.  Group-limited selection (n_group > 1,
 * no counterpart in the reference; DeepSeek-V3 rule): the group score is
 * the sum of the two highest scores in each of n_group equal groups, the
 * topk_group best groups stay (ties -> lower group), all other experts
 * leave the candidate set, then top-k runs as above. */
int orc_router_select(int32_t *selected, float *weights, const float *logits, const float *bias,
                      uint32_t n_expert, uint32_t k_used, float weight_scale, uint32_t n_tok,
                      uint32_t softmax_mode, uint32_t n_shexp, uint32_t n_group, uint32_t topk_group) {
    if (n_expert == 0 || k_used == 0 || k_used > n_expert || n_tok == 0) return 0;
    const uint32_t sink = softmax_mode == 2 ? n_shexp : 0;
    const uint32_t n_logit = n_expert + sink, n_slot = k_used + sink;
    float *prob = (float *)malloc(n_expert * sizeof(float));
    float *score = (float *)malloc(n_expert * sizeof(float));
    for (uint32_t t = 0; t < n_tok; t++) {
        const float *lg = logits + (size_t)t * n_logit;
        int32_t *sel = selected + (size_t)t * n_slot;
        float *w = weights + (size_t)t * n_slot;
        for (uint32_t e = 0; e < n_expert; e++) {
            float raw = lg[e];
            float p = softmax_mode == 1 ? raw : orf_sigmoid(raw);
            prob[e] = softmax_mode == 2 ? raw : p;
            score[e] = p + (bias ? bias[e] : 0.0f);
        }
        if (n_group > 1 && topk_group < n_group) {
            uint32_t gs = n_expert / n_group;
            float gscore[64];
            for (uint32_t g = 0; g < n_group; g++) {
                float b1 = -INFINITY, b2 = -INFINITY;
                uint32_t i1 = UINT32_MAX;
                for (uint32_t e = g * gs; e < (g + 1) * gs; e++)
                    if (better(score[e], e, b1, i1)) {
                        b1 = score[e];
                        i1 = e;
                    }
                uint32_t i2 = UINT32_MAX;
                for (uint32_t e = g * gs; e < (g + 1) * gs; e++)
                    if (e != i1 && better(score[e], e, b2, i2)) {
                        b2 = score[e];
                        i2 = e;
                    }
                gscore[g] = b1 + b2;
            }
            uint8_t keep[64] = {0};
            for (uint32_t r = 0; r < topk_group; r++) {
                uint32_t bg = UINT32_MAX;
                float bv = -INFINITY;
                for (uint32_t g = 0; g < n_group; g++)
                    if (!keep[g] && better(gscore[g], g, bv, bg)) {
                        bv = gscore[g];
                        bg = g;
                    }
                keep[bg] = 1;
            }
            for (uint32_t e = 0; e < n_expert; e++)
                if (!keep[e / gs]) score[e] = -INFINITY;
        }
        float sum = 0.0f;
        for (uint32_t k = 0; k < k_used; k++) {
            uint32_t best = UINT32_MAX;
            float bs = -INFINITY, bp = 0.0f;
            for (uint32_t e = 0; e < n_expert; e++)
                if (better(score[e], e, bs, best)) {
                    bs = score[e];
                    bp = prob[e];
                    best = e;
                }
            /* only NaN scores left: the slot stays unrouted (-1, weight 0) */
            sel[k] = best == UINT32_MAX ? -1 : (int32_t)best;
            w[k] = bp;
            sum += bp;
            if (best != UINT32_MAX) score[best] = -INFINITY;
        }
        if (softmax_mode == 2) {
            for (uint32_t s = 0; s < sink; s++) {
                sel[k_used + s] = (int32_t)(n_expert + s);
                w[k_used + s] = lg[n_expert + s];
            }
            float m = -INFINITY;
            for (uint32_t k = 0; k < n_slot; k++) {
                float xv = w[k];
                w[k] = xv < 0.0f ? xv - log1pf(orf_expf(xv)) : -log1pf(orf_expf(-xv));
                m = fmaxf(m, w[k]);
            }
            float es = 0.0f;
            for (uint32_t k = 0; k < n_slot; k++) {
                w[k] = orf_expf(w[k] - m);
                es += w[k];
            }
            for (uint32_t k = 0; k < n_slot; k++) w[k] = w[k] / es * weight_scale;
        } else if (softmax_mode == 1) {
            float m = -INFINITY;
            for (uint32_t k = 0; k < k_used; k++) m = fmaxf(m, w[k]);
            float es = 0.0f;
            for (uint32_t k = 0; k < k_used; k++) {
                w[k] = orf_expf(w[k] - m);
                es += w[k];
            }
            for (uint32_t k = 0; k < k_used; k++) w[k] = w[k] / es * weight_scale;
        } else {
            sum = fmaxf(sum, 6.103515625e-5f);
            for (uint32_t k = 0; k < k_used; k++) w[k] = w[k] / sum * weight_scale;
        }
    }
    free(prob);
    free(score);
    return 1;
}

/* ------------------------------------------------------------ lane FFN */

typedef struct {
    /* shared read-only state */
    const orc_expert_ptrs *ptrs;
    const float *w;
    const orf_q8k *xq;  /* [n_tok][H blocks] */
    orf_q8k *midq;      /* [n_tok*n_slot][F blocks] */
    float *mid;              /* [n_tok*n_slot][Fmax] */
    float *out;
    uint32_t H, n_tok, n_slot, n_routed, Fmax;
    uint32_t F[2], quant[2];
    uint64_t rb_gu[2], rb_down[2];
    uint32_t act_op;
    /* job queue */
    int stage;
    uint32_t n_jobs;
    uint32_t next;
    pthread_mutex_t mu;
} lane_ctx;

static int slot_class(const lane_ctx *c, uint32_t s) { return s < c->n_routed ? 0 : 1; }

/* stage A: one job = (pair, 256-row chunk of F): mid = glu(g + gb, u + ub) * w
 * (elib:2038-2052; biases per cu:2604-2609) */
static void job_a(lane_ctx *c, uint32_t job) {
    const uint32_t per_pair = (c->Fmax + 255) / 256;
    uint32_t pair = job / per_pair, chunk = job % per_pair;
    uint32_t t = pair / c->n_slot, s = pair % c->n_slot;
    int cl = slot_class(c, s);
    uint32_t F = c->F[cl];
    uint32_t lo = chunk * 256, hi = lo + 256 < F ? lo + 256 : F;
    const orc_expert_ptrs *p = &c->ptrs[pair];
    float *mid = c->mid + (size_t)pair * c->Fmax;
    const orf_q8k *xq = c->xq + (size_t)t * ((c->H + 255) / 256);
    for (uint32_t j = lo; j < hi; j++) {
        if (!p->gate || !p->up) {
            mid[j] = 0.0f;
            continue;
        }
        float g = orc_vec_dot((int)c->quant[cl], p->gate + (size_t)j * c->rb_gu[cl], xq, c->H);
        float u = orc_vec_dot((int)c->quant[cl], p->up + (size_t)j * c->rb_gu[cl], xq, c->H);
        if (p->gate_b) g += p->gate_b[j];
        if (p->up_b) u += p->up_b[j];
        mid[j] = orc_glu(g, u, c->act_op) * c->w[pair];
    }
}

/* finish: one job = (token, 512-row chunk of H): out = sum over slots in
 * slot order of down . q8_K(mid) (elib:2076-2098), then the down bias
 * sum_s w_s * b_s added once (cu:3601-3620) */
static void job_b(lane_ctx *c, uint32_t job) {
    const uint32_t per_tok = (c->H + 511) / 512;
    uint32_t t = job / per_tok, chunk = job % per_tok;
    uint32_t lo = chunk * 512, hi = lo + 512 < c->H ? lo + 512 : c->H;
    const uint32_t fb = (c->Fmax + 255) / 256;
    for (uint32_t r = lo; r < hi; r++) {
        float sum = 0.0f;
        for (uint32_t s = 0; s < c->n_slot; s++) {
            const orc_expert_ptrs *p = &c->ptrs[(size_t)t * c->n_slot + s];
            if (!p->down) continue;
            int cl = slot_class(c, s);
            const orf_q8k *mq = c->midq + ((size_t)t * c->n_slot + s) * fb;
            sum += orc_vec_dot((int)c->quant[cl], p->down + (size_t)r * c->rb_down[cl], mq, c->F[cl]);
        }
        float b = 0.0f;
        for (uint32_t s = 0; s < c->n_slot; s++) {
            const orc_expert_ptrs *p = &c->ptrs[(size_t)t * c->n_slot + s];
            if (p->down_b) b += c->w[(size_t)t * c->n_slot + s] * p->down_b[r];
        }
        if (b != 0.0f) sum += b;
        c->out[(size_t)t * c->H + r] = sum;
    }
}

static void *worker(void *arg) {
    lane_ctx *c = (lane_ctx *)arg;
    for (;;) {
        pthread_mutex_lock(&c->mu);
        uint32_t j = c->next++;
        pthread_mutex_unlock(&c->mu);
        if (j >= c->n_jobs) return NULL;
        if (c->stage == 0)
            job_a(c, j);
        else
            job_b(c, j);
    }
}

static void run_stage(lane_ctx *c, int stage, uint32_t n_jobs, int n_threads) {
    c->stage = stage;
    c->n_jobs = n_jobs;
    c->next = 0;
    if (n_threads <= 1) {
        worker(c);
        return;
    }
    pthread_t th[256];
    int nt = n_threads > 256 ? 256 : n_threads;
    for (int i = 0; i < nt; i++) pthread_create(&th[i], NULL, worker, c);
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
}

int orc_moe_ffn(float *out, float *mid_out, const orc_expert_ptrs *ptrs, const float *w,
                const float *x, uint32_t H, uint32_t n_tok, uint32_t n_slot, uint32_t n_routed,
                uint32_t F_r, uint32_t quant_r, uint64_t rb_gu_r, uint64_t rb_down_r,
                uint32_t F_s, uint32_t quant_s, uint64_t rb_gu_s, uint64_t rb_down_s,
                uint32_t act_op, int n_threads) {
    if (!out || !ptrs || !w || !x || H == 0 || n_tok == 0 || n_slot == 0) return 0;
    lane_ctx c;
    memset(&c, 0, sizeof(c));
    c.ptrs = ptrs;
    c.w = w;
    c.H = H;
    c.n_tok = n_tok;
    c.n_slot = n_slot;
    c.n_routed = n_routed;
    c.F[0] = F_r;
    c.F[1] = F_s;
    c.quant[0] = quant_r;
    c.quant[1] = quant_s;
    c.rb_gu[0] = rb_gu_r;
    c.rb_gu[1] = rb_gu_s;
    c.rb_down[0] = rb_down_r;
    c.rb_down[1] = rb_down_s;
    c.act_op = act_op;
    c.Fmax = n_routed < n_slot && F_s > F_r ? F_s : F_r;
    c.out = out;
    pthread_mutex_init(&c.mu, NULL);
    if (n_threads <= 0) n_threads = (int)sysconf(_SC_NPROCESSORS_ONLN);

    const uint32_t hb = (H + 255) / 256, fb = (c.Fmax + 255) / 256;
    orf_q8k *xq = (orf_q8k *)malloc((size_t)n_tok * hb * sizeof(orf_q8k));
    float *mid = (float *)calloc((size_t)n_tok * n_slot * c.Fmax, sizeof(float));
    orf_q8k *midq = (orf_q8k *)calloc((size_t)n_tok * n_slot * fb, sizeof(orf_q8k));
    for (uint32_t t = 0; t < n_tok; t++) orc_quantize_q8k(x + (size_t)t * H, H, xq + (size_t)t * hb);
    c.xq = xq;
    c.mid = mid;
    c.midq = midq;
    run_stage(&c, 0, n_tok * n_slot * ((c.Fmax + 255) / 256), n_threads);
    for (uint32_t p = 0; p < n_tok * n_slot; p++) {
        uint32_t F = c.F[slot_class(&c, p % n_slot)];
        orc_quantize_q8k(mid + (size_t)p * c.Fmax, F, midq + (size_t)p * fb);
    }
    run_stage(&c, 1, n_tok * ((H + 511) / 512), n_threads);
    if (mid_out) memcpy(mid_out, mid, (size_t)n_tok * n_slot * c.Fmax * sizeof(float));
    free(xq);
    free(mid);
    free(midq);
    pthread_mutex_destroy(&c.mu);
    return 1;
}
