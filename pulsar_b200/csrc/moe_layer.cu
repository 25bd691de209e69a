/* moe_layer.cu - one routed-expert MoE layer as a single call, with the
 * expert resolve on the device.
 *
 * The reference engine (crates/engine/src/lib.rs:7537-8705, Ffn::Moe arm)
 * runs the router on the GPU, syncs, reads the selected ids back, builds
 * the per-(token, slot) pointer array on the host, writes it back and then
 * launches pair / q8_K / down.  Here the whole layer stays on the device:
 *
 *   1 router logits (binary64 fixed-order GEMV) ........ router_q8k.cu
 *   2 q8_K of the hidden rows ........................... router_q8k.cu
 *   3 top-k per token (warp per token); the last CTA to finish groups the
 *     (token, slot) pairs by expert into a CSR work list (ascending expert
 *     id, pairs in (token, slot) order) and appends the shared experts
 *   4 gate/up: one CTA per (expert work item, row tile) streams the
 *     expert's rows once through a TMA ring and serves every token routed
 *     to it; glu * route weight -> mid (f32)
 *   5 down: one CTA per (expert work item, tile of output rows), the same
 *     engine; it quantizes its tokens' mid rows to q8_K (CPU-lane math)
 *     while staging them and writes one partial row per (token, slot)
 *   6 combine: per (token, row) the partials in slot order, + the down
 *     bias (sum_s w_s b_s, cu:3601) + the residual (deterministic)
 * Both expert kernels stage each token tile's q8_K rows in shared memory
 * and decode every weight unit once for the whole tile (pm_gemv.cuh).
 *
 * Nothing is allocated; all state lives in the caller's workspace and the
 * call is capturable into a CUDA graph.
 */
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/pulsar_moe.h"
#include "pm_host.h"
#include "pm_router.cuh"
#include "pm_gemv.cuh"

int pm_launch_q8k(void *out, const float *x, uint32_t in_dim, uint32_t n_rows, cudaStream_t st);
int pm_launch_router_logits(float *logits, const float *w, const float *x, const float *lbias, uint32_t n_expert,
                            uint32_t in_dim, uint32_t n_tok, cudaStream_t st);
int pm_router_args_ok(uint32_t n_expert, uint32_t k_used, uint32_t n_tok, uint32_t mode, uint32_t n_shexp,
                      uint32_t n_group, uint32_t topk_group);

__device__ static const uint16_t pm_kgrid_layer[256] = PM_IQ2XXS_KGRID_INIT;

#define PM_TT 8 /* tokens per register tile = tokens per work unit */

/* ------------------------------------------------------------ layout */

struct pm_layout {
    uint32_t T, E, k, S, n_slot, H, Fr, Fs, Fmax, hb, fb, max_items;
    uint32_t max_work;
    size_t logits, sel, w, xq, n_items, item_expert, item_start, work_item, work_t0, pairs, mid, partial,
        sel_done, err, total;
};

static size_t pm_al(size_t v) { return (v + 255) & ~(size_t)255; }

static pm_layout pm_make_layout(const pulsar_moe_layer_desc *d, uint32_t T) {
    pm_layout L;
    L.T = T;
    L.E = d->n_expert;
    L.k = d->n_used;
    L.S = d->n_shared;
    L.n_slot = L.k + L.S;
    L.H = d->n_embd;
    L.Fr = d->n_ff;
    L.Fs = L.S ? d->shared_n_ff : 0;
    L.Fmax = L.Fr > L.Fs ? L.Fr : L.Fs;
    L.hb = (L.H + 255) / 256;
    L.fb = (L.Fmax + 255) / 256;
    const uint64_t routed = (uint64_t)T * L.k;
    L.max_items = (uint32_t)((routed < L.E ? routed : L.E) + L.S);
    size_t o = 0;
    L.logits = o, o = pm_al(o + (size_t)T * L.E * 4);
    L.sel = o, o = pm_al(o + (size_t)T * L.n_slot * 4);
    L.w = o, o = pm_al(o + (size_t)T * L.n_slot * 4);
    L.xq = o, o = pm_al(o + (size_t)T * L.hb * PM_Q8_K_BYTES);
    L.n_items = o, o = pm_al(o + 16);
    L.item_expert = o, o = pm_al(o + (size_t)L.max_items * 4);
    L.item_start = o, o = pm_al(o + (size_t)(L.max_items + 1) * 4);
    L.max_work = L.max_items + (uint32_t)(((uint64_t)T * L.n_slot + PM_TT - 1) / PM_TT);
    L.work_item = o, o = pm_al(o + (size_t)L.max_work * 4);
    L.work_t0 = o, o = pm_al(o + (size_t)L.max_work * 4);
    L.pairs = o, o = pm_al(o + (size_t)T * L.n_slot * 4);
    L.mid = o, o = pm_al(o + (size_t)T * L.n_slot * L.Fmax * 4);
    L.partial = o, o = pm_al(o + (size_t)T * L.n_slot * L.H * 4);
    L.sel_done = o, o = pm_al(o + 4);
    L.err = o, o = pm_al(o + 4);
    L.total = o;
    return L;
}

/* device-side view of the descriptor + workspace */
struct pm_layer_args {
    /* geometry */
    uint32_t T, E, k, S, n_slot, H, Fr, Fs, Fmax, hb, fb, max_items;
    uint32_t lo, hi, act, mode, n_group, topk_group;
    float scale;
    uint64_t rb_gu_r, rb_dn_r, st_gu_r, st_dn_r, rb_gu_s, rb_dn_s;
    const uint8_t *gate, *up, *down, *sgate, *sup, *sdown;
    const float *gate_b, *up_b, *down_b, *router_sel_b;
    /* workspace */
    float *logits;
    int32_t *sel;
    float *w;
    pm_block_q8K *xq;
    uint32_t *n_items; /* [0] all items, [1] routed items, [2] work units */
    uint32_t *item_expert, *item_start, *pairs;
    uint32_t *work_item, *work_t0; /* work unit = (item, first token of its chunk of <= PM_TT) */
    float *mid;
    float *partial; /* [T * n_slot][H] down outputs before the combine */
    uint32_t *sel_done, *err;
    /* io */
    float *out;
    const float *residual;
    uint32_t gu_rows, dn_rows; /* rows per CTA */
};

/* ============================================ 3: select + CSR build */

__global__ void __launch_bounds__(128) pm_layer_select_kernel(const __grid_constant__ pm_layer_args a) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ uint32_t is_last, tot_pairs, tot_items, tot_work;
    const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    const uint32_t token = blockIdx.x * 4u + wid;
    if (token < a.T) {
        float *score = (float *)sm + (size_t)wid * 2 * a.E;
        pm_select_token(a.sel, a.w, a.logits, a.router_sel_b, a.E, a.k, a.scale, token, a.mode, 0, a.n_group,
                        a.topk_group, score, score + a.E, a.n_slot);
        if (lane < a.S) { /* shared experts: always-on slots k.., ids E + s, weight 1 */
            a.sel[token * a.n_slot + a.k + lane] = (int32_t)(a.E + lane);
            a.w[token * a.n_slot + a.k + lane] = 1.0f;
        }
    }
    __threadfence(); /* every thread publishes its own selection writes */
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(a.sel_done, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    /* ---- the last CTA: CSR by expert over routed pairs in [lo, hi) ---- */
    uint32_t *cnt = (uint32_t *)sm; /* [E] counts, then fill cursors */
    for (uint32_t e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const uint32_t n_routed = a.T * a.k;
    for (uint32_t q = threadIdx.x; q < n_routed; q += blockDim.x) {
        const uint32_t e = (uint32_t)__ldcg(a.sel + (q / a.k) * a.n_slot + q % a.k);
        if (e >= a.lo && e < a.hi) atomicAdd(&cnt[e], 1u);
    }
    __syncthreads();
    if (wid == 0) {
        /* exclusive scans over experts: pair offsets, item indices, work units */
        uint32_t carry_p = 0, carry_i = 0, carry_w = 0;
        for (uint32_t c = 0; c < a.E; c += 32u) {
            const uint32_t e = c + lane;
            const uint32_t v = e < a.E ? cnt[e] : 0u;
            const uint32_t nw = (v + PM_TT - 1) / PM_TT;
            uint32_t ip = v, ii = v ? 1u : 0u, iw = nw;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t up = __shfl_up_sync(0xffffffffu, ip, o);
                const uint32_t ui = __shfl_up_sync(0xffffffffu, ii, o);
                const uint32_t uw = __shfl_up_sync(0xffffffffu, iw, o);
                if (lane >= (uint32_t)o) ip += up, ii += ui, iw += uw;
            }
            const uint32_t start = carry_p + ip - v, item = carry_i + ii - (v ? 1u : 0u), w0 = carry_w + iw - nw;
            if (e < a.E) {
                cnt[e] = start;
                if (v) {
                    a.item_expert[item] = e;
                    a.item_start[item] = start;
                    for (uint32_t j = 0; j < nw; j++) {
                        a.work_item[w0 + j] = item;
                        a.work_t0[w0 + j] = j * PM_TT;
                    }
                }
            }
            carry_p += __shfl_sync(0xffffffffu, ip, 31);
            carry_i += __shfl_sync(0xffffffffu, ii, 31);
            carry_w += __shfl_sync(0xffffffffu, iw, 31);
        }
        if (lane == 0) tot_pairs = carry_p, tot_items = carry_i, tot_work = carry_w;
    }
    __syncthreads();
    if (wid == 0) {
        /* stable fill: entries in (token, slot) order, ranks via match_any */
        for (uint32_t c = 0; c < n_routed; c += 32u) {
            const uint32_t q = c + lane;
            uint32_t e = UINT32_MAX, pair = 0;
            if (q < n_routed) {
                pair = (q / a.k) * a.n_slot + q % a.k;
                const uint32_t v = (uint32_t)__ldcg(a.sel + pair);
                if (v >= a.lo && v < a.hi) e = v;
            }
            const uint32_t peers = __match_any_sync(0xffffffffu, e);
            const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
            if (e != UINT32_MAX) a.pairs[cnt[e] + rank] = pair;
            __syncwarp();
            if (e != UINT32_MAX && rank == 0) cnt[e] += __popc(peers);
            __syncwarp();
        }
    }
    __syncthreads();
    /* shared experts (computed on the shard that owns expert 0): one item
     * each over all tokens, appended after the routed items */
    const uint32_t n_sh = a.lo == 0 ? a.S : 0u;
    const uint32_t sh_chunks = (a.T + PM_TT - 1) / PM_TT;
    for (uint32_t s = 0; s < n_sh; s++) {
        const uint32_t item = tot_items + s, base = tot_pairs + s * a.T, w0 = tot_work + s * sh_chunks;
        if (threadIdx.x == 0) {
            a.item_expert[item] = a.E + s;
            a.item_start[item] = base;
        }
        for (uint32_t t = threadIdx.x; t < a.T; t += blockDim.x) a.pairs[base + t] = t * a.n_slot + a.k + s;
        for (uint32_t j = threadIdx.x; j < sh_chunks; j += blockDim.x) {
            a.work_item[w0 + j] = item;
            a.work_t0[w0 + j] = j * PM_TT;
        }
    }
    if (threadIdx.x == 0) {
        a.item_start[tot_items + n_sh] = tot_pairs + n_sh * a.T;
        a.n_items[0] = tot_items + n_sh;
        a.n_items[1] = tot_items;
        a.n_items[2] = tot_work + n_sh * sh_chunks;
        *a.sel_done = 0;
    }
}

/* ====================================================== 4: gate / up */

struct pm_seg_gu2 {
    static constexpr bool F32 = false;
    uint32_t n_f32;
    const uint8_t *g, *u;
    const uint32_t *pairs;
    uint32_t n, row0;
    const pm_layer_args *a;
    const float *gb, *ub;
    __device__ const uint8_t *base(int m) const { return m == 0 ? g : u; }
    __device__ uint32_t ntok() const { return n; }
    __device__ const pm_block_q8K *tok(uint32_t ti) const {
        return a->xq + (uint64_t)(__ldcg(pairs + ti) / a->n_slot) * a->hb;
    }
    __device__ void epi(uint32_t row, uint32_t ti, const float *v) const {
        const uint32_t p = __ldcg(pairs + ti);
        float x0 = v[0], x1 = v[1];
        if (gb) x0 += gb[row0 + row];
        if (ub) x1 += ub[row0 + row];
        a->mid[(uint64_t)p * a->Fmax + row0 + row] = pm_glu(x0, x1, a->act) * a->w[p];
    }
};

/* the IQ2_XXS magnitude grid, expanded into shared memory (all threads) */
__device__ __forceinline__ const uint64_t *pm_grid_fill(uint8_t *smem, bool need) {
    uint64_t *g = (uint64_t *)smem;
    if (need)
        for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) {
            const uint32_t k = pm_kgrid_layer[i];
            uint64_t v = 0;
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const uint32_t d = (k >> (2 * q)) & 3u;
                v |= (uint64_t)(d == 0 ? 8u : (d == 1 ? 25u : 43u)) << (8 * q);
            }
            g[i] = v;
        }
    return g; /* the first __syncthreads of the engine publishes it */
}

template <int Q>
__device__ bool pm_layer_gu_item(const pm_layer_args &a, uint8_t *smem, uint32_t item, uint32_t t0, uint32_t e,
                                 uint32_t row0, uint32_t nrows, const pm_pass &ps) {
    const bool routed = e < a.E;
    const uint64_t rb = routed ? a.rb_gu_r : a.rb_gu_s;
    const uint64_t *grid = pm_grid_fill(smem, Q == PM_QUANT_IQ2_XXS);
    pm_seg_gu2 seg;
    seg.g = (routed ? a.gate + (uint64_t)e * a.st_gu_r : a.sgate) + (uint64_t)row0 * rb;
    seg.u = (routed ? a.up + (uint64_t)e * a.st_gu_r : a.sup) + (uint64_t)row0 * rb;
    const uint32_t s0 = __ldcg(a.item_start + item), s1 = __ldcg(a.item_start + item + 1);
    seg.pairs = a.pairs + s0 + t0;
    seg.n = s1 - s0 - t0 < PM_TT ? s1 - s0 - t0 : PM_TT;
    seg.row0 = row0;
    seg.a = &a;
    seg.gb = routed && a.gate_b ? a.gate_b + (uint64_t)e * a.Fr : nullptr;
    seg.ub = routed && a.up_b ? a.up_b + (uint64_t)e * a.Fr : nullptr;
    return pm_gemv_warps<Q, 2, PM_TT>(seg, smem, ps, nrows, rb, a.H / 32u, grid, a.err);
}

template <int QR, int QS>
__global__ void __launch_bounds__(PM_THREADS, 2)
    pm_layer_gu_kernel(const __grid_constant__ pm_layer_args a, pm_pass pr, pm_pass psh) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t wk = blockIdx.x;
    if (wk >= __ldcg(a.n_items + 2)) return;
    const uint32_t item = __ldcg(a.work_item + wk), t0 = __ldcg(a.work_t0 + wk);
    const uint32_t e = __ldcg(a.item_expert + item);
    const bool routed = e < a.E;
    const uint32_t F = routed ? a.Fr : a.Fs;
    const uint32_t row0 = blockIdx.y * a.gu_rows;
    if (row0 >= F) return;
    const uint32_t nrows = F - row0 < a.gu_rows ? F - row0 : a.gu_rows;
    const bool ok = routed ? pm_layer_gu_item<QR>(a, smem, item, t0, e, row0, nrows, pr)
                           : pm_layer_gu_item<QS>(a, smem, item, t0, e, row0, nrows, psh);
    if (ok) return;
    (void)ok; /* a timeout is recorded in the error word; the layer output is then undefined */
}

/* ======================================================= 5: down */

struct pm_seg_dn2 {
    static constexpr bool F32 = true; /* mid rows are quantized to q8_K while staging */
    uint32_t n_f32;
    const uint8_t *d;
    const uint32_t *pairs;
    uint32_t n, row0;
    const pm_layer_args *a;
    __device__ const uint8_t *base(int) const { return d; }
    __device__ uint32_t ntok() const { return n; }
    __device__ const pm_block_q8K *tok(uint32_t) const { return nullptr; }
    __device__ const float *tok_f32(uint32_t ti) const { return a->mid + (uint64_t)__ldcg(pairs + ti) * a->Fmax; }
    __device__ void epi(uint32_t row, uint32_t ti, const float *v) const {
        a->partial[(uint64_t)__ldcg(pairs + ti) * a->H + row0 + row] = v[0];
    }
};

template <int Q>
__device__ void pm_layer_dn_item(const pm_layer_args &a, uint8_t *smem, uint32_t item, uint32_t t0, uint32_t e,
                                 uint32_t row0, uint32_t nrows, const pm_pass &ps) {
    const bool routed = e < a.E;
    const uint64_t rb = routed ? a.rb_dn_r : a.rb_dn_s;
    const uint64_t *grid = pm_grid_fill(smem, Q == PM_QUANT_IQ2_XXS);
    pm_seg_dn2 seg;
    seg.d = (routed ? a.down + (uint64_t)e * a.st_dn_r : a.sdown) + (uint64_t)row0 * rb;
    const uint32_t s0 = __ldcg(a.item_start + item), s1 = __ldcg(a.item_start + item + 1);
    seg.pairs = a.pairs + s0 + t0;
    seg.n = s1 - s0 - t0 < PM_TT ? s1 - s0 - t0 : PM_TT;
    seg.row0 = row0;
    seg.a = &a;
    const uint32_t F = routed ? a.Fr : a.Fs;
    seg.n_f32 = F;
    pm_gemv_warps<Q, 1, PM_TT>(seg, smem, ps, nrows, rb, (F + 31u) / 32u, grid, a.err);
}

template <int QR, int QS>
__global__ void __launch_bounds__(PM_THREADS, 2)
    pm_layer_dn_kernel(const __grid_constant__ pm_layer_args a, pm_pass pr, pm_pass psh) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t wk = blockIdx.x;
    if (wk >= __ldcg(a.n_items + 2)) return;
    const uint32_t item = __ldcg(a.work_item + wk), t0 = __ldcg(a.work_t0 + wk);
    const uint32_t e = __ldcg(a.item_expert + item);
    const uint32_t row0 = blockIdx.y * a.dn_rows;
    const uint32_t nrows = a.H - row0 < a.dn_rows ? a.H - row0 : a.dn_rows;
    if (e < a.E)
        pm_layer_dn_item<QR>(a, smem, item, t0, e, row0, nrows, pr);
    else
        pm_layer_dn_item<QS>(a, smem, item, t0, e, row0, nrows, psh);
}

/* ================================================= 6: combine */

/* out[t][r] = sum over the token's local slots (slot order) of the down
 * partials + down bias (sum_s w_s b_s, cu:3601-3620) + residual */
__global__ void pm_layer_combine_kernel(const __grid_constant__ pm_layer_args a) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (uint64_t)a.T * a.H) return;
    const uint32_t t = (uint32_t)(gid / a.H), r = (uint32_t)(gid % a.H);
    float v = 0.0f, b = 0.0f;
    for (uint32_t s = 0; s < a.k; s++) {
        const uint32_t e = (uint32_t)a.sel[t * a.n_slot + s];
        if (e >= a.lo && e < a.hi) {
            v += a.partial[(uint64_t)(t * a.n_slot + s) * a.H + r];
            if (a.down_b) b += a.w[t * a.n_slot + s] * a.down_b[(uint64_t)e * a.H + r];
        }
    }
    if (a.lo == 0)
        for (uint32_t s = a.k; s < a.n_slot; s++) v += a.partial[(uint64_t)(t * a.n_slot + s) * a.H + r];
    if (b != 0.0f) v += b;
    if (a.residual) v += a.residual[gid];
    a.out[gid] = v;
}

/* ============================================================= host */

static bool pm_fmt_ok(uint32_t q, uint32_t n) { return pm_row_bytes(q, n) != 0; }

static int pm_desc_ok(const pulsar_moe_layer_desc *d) {
    if (!d || !d->n_embd || !d->n_ff || !d->n_expert || !d->n_used || d->n_used > d->n_expert) return 0;
    if (!d->gate || !d->up || !d->down || !d->router_w) return 0;
    if (!pm_fmt_ok(d->quant, d->n_embd) || !pm_fmt_ok(d->quant, d->n_ff)) return 0;
    if (d->row_bytes_gu < pm_row_bytes(d->quant, d->n_embd) || d->row_bytes_down < pm_row_bytes(d->quant, d->n_ff))
        return 0;
    if (d->n_shared > 1) return 0;
    if (d->n_shared) {
        if (!d->shared_gate || !d->shared_up || !d->shared_down || !d->shared_n_ff) return 0;
        if (!pm_fmt_ok(d->shared_quant, d->n_embd) || !pm_fmt_ok(d->shared_quant, d->shared_n_ff)) return 0;
        if (d->shared_row_bytes_gu < pm_row_bytes(d->shared_quant, d->n_embd) ||
            d->shared_row_bytes_down < pm_row_bytes(d->shared_quant, d->shared_n_ff))
            return 0;
    }
    if (d->router_mode > 1) return 0;
    if (d->expert_hi && (d->expert_lo >= d->expert_hi || d->expert_hi > d->n_expert)) return 0;
    return 1;
}

extern "C" size_t pulsar_moe_layer_workspace(const pulsar_moe_layer_desc *d, uint32_t max_tok) {
    if (!pm_desc_ok(d) || max_tok == 0) return 0;
    return pm_make_layout(d, max_tok).total;
}

extern "C" int pulsar_moe_layer_ws_view(const pulsar_moe_layer_desc *d, uint32_t n_tok, void *ws,
                                        pulsar_moe_ws_view *v) {
    if (!pm_desc_ok(d) || !ws || !v || n_tok == 0) return 0;
    const pm_layout L = pm_make_layout(d, n_tok);
    uint8_t *b = (uint8_t *)ws;
    v->logits = (float *)(b + L.logits);
    v->selected = (int32_t *)(b + L.sel);
    v->weights = (float *)(b + L.w);
    v->xq = b + L.xq;
    v->mid = (float *)(b + L.mid);
    v->err = (uint32_t *)(b + L.err);
    v->n_items = (uint32_t *)(b + L.n_items);
    v->item_expert = (uint32_t *)(b + L.item_expert);
    v->item_start = (uint32_t *)(b + L.item_start);
    v->pairs = (uint32_t *)(b + L.pairs);
    v->work_item = (uint32_t *)(b + L.work_item);
    v->work_t0 = (uint32_t *)(b + L.work_t0);
    v->partial = (float *)(b + L.partial);
    v->n_slot = L.n_slot;
    v->f_max = L.Fmax;
    return 1;
}

/* largest power-of-two row count in [lo, hi] that still gives ~2 waves */
static uint32_t pm_pow2_rows(uint64_t nrows_total, uint64_t ctas_other, uint32_t lo, uint32_t hi) {
    uint32_t r = hi;
    while (r > lo && ((nrows_total + r - 1) / r) * ctas_other < 2ull * 148ull) r >>= 1;
    return r;
}

/* pass geometry: lanes per row (one lane per pair of units), rows per
 * stage (~6 KB, whole passes of the warp), per-warp ring depth within a
 * ~100 KB budget (two CTAs per SM), and the shared-memory layout */
static pm_pass pm_pass_for(uint32_t nmat, uint64_t rb, uint32_t n_units, uint32_t rows_cta, bool grid) {
    pm_pass p;
    const uint32_t pairs = (n_units + 1) / 2;
    p.lpr = pairs >= 32 ? 32u : (pairs >= 16 ? 16u : (pairs >= 8 ? 8u : (pairs >= 4 ? 4u : 2u)));
    const uint32_t rpp = 32u / p.lpr;
    uint64_t rw = 6144u / (nmat * rb);
    rw = (rw / rpp) * rpp;
    if (rw < rpp) rw = rpp;
    const uint32_t per_warp = (rows_cta + PM_WARPS - 1) / PM_WARPS;
    if (rw > per_warp) rw = ((per_warp + rpp - 1) / rpp) * rpp;
    p.rw = (uint32_t)rw;
    p.stage = pm_stage_bytes(nmat, rb, p.rw);
    p.off_bar = grid ? 2048u : 0u;
    p.off_tok = p.off_bar + 512u;
    p.off_acts = p.off_tok + 128u;
    const uint32_t ring0 = (p.off_acts + pm_acts_bytes(PM_TT, n_units) + 127u) & ~127u;
    const uint32_t budget = 100u * 1024u;
    uint32_t S = budget > ring0 ? (budget - ring0) / (PM_WARPS * p.stage) : 2u;
    p.S = S < 2 ? 2 : (S > 8 ? 8 : S);
    p.off_ring = ring0;
    p.smem = ring0 + PM_WARPS * p.S * p.stage;
    return p;
}

static inline void pm_ev(void *const *ev, int i, cudaStream_t st) {
    if (ev && ev[i]) cudaEventRecord((cudaEvent_t)ev[i], st);
}

template <int QR, int QS>
static int pm_layer_launch(pm_layer_args a, const pm_layout &L, cudaStream_t st, void *const *ev) {
    static uint64_t done_gu = 0, done_dn = 0;
    /* 4: gate/up (+ q8_K of mid) */
    const uint32_t hu = a.H / 32u;
    const pm_pass gr = pm_pass_for(2, a.rb_gu_r, hu, a.gu_rows, QR == PM_QUANT_IQ2_XXS);
    const pm_pass gs = a.S ? pm_pass_for(2, a.rb_gu_s, hu, a.gu_rows, QS == PM_QUANT_IQ2_XXS) : gr;
    uint32_t smem_gu = gr.smem > gs.smem ? gr.smem : gs.smem;
    if (!pm_smem_attr(pm_layer_gu_kernel<QR, QS>, smem_gu, &done_gu)) return 0;
    dim3 ggrid(L.max_work, (L.Fmax + a.gu_rows - 1) / a.gu_rows);
    pm_layer_gu_kernel<QR, QS><<<ggrid, PM_THREADS, smem_gu, st>>>(a, gr, gs);
    if (!pm_ok(cudaGetLastError(), "moe layer gate/up launch")) return 0;
    pm_ev(ev, 4, st);
    /* 5: down -> partial rows */
    const uint32_t fr = (a.Fr + 31u) / 32u, fs = a.S ? (a.Fs + 31u) / 32u : fr;
    const pm_pass dr = pm_pass_for(1, a.rb_dn_r, fr, a.dn_rows, QR == PM_QUANT_IQ2_XXS);
    const pm_pass ds = a.S ? pm_pass_for(1, a.rb_dn_s, fs, a.dn_rows, QS == PM_QUANT_IQ2_XXS) : dr;
    const uint32_t smem_dn = dr.smem > ds.smem ? dr.smem : ds.smem;
    if (!pm_smem_attr(pm_layer_dn_kernel<QR, QS>, smem_dn, &done_dn)) return 0;
    dim3 dgrid(L.max_work, (a.H + a.dn_rows - 1) / a.dn_rows);
    pm_layer_dn_kernel<QR, QS><<<dgrid, PM_THREADS, smem_dn, st>>>(a, dr, ds);
    if (!pm_ok(cudaGetLastError(), "moe layer down launch")) return 0;
    /* 6: combine */
    const uint64_t tot = (uint64_t)a.T * a.H;
    pm_layer_combine_kernel<<<(uint32_t)((tot + 255) / 256), 256, 0, st>>>(a);
    if (!pm_ok(cudaGetLastError(), "moe layer combine launch")) return 0;
    pm_ev(ev, 5, st);
    return 1;
}

#define PM_Q2(QR)                                                                          \
    switch (qs) {                                                                          \
    case PM_QUANT_Q4_K: return pm_layer_launch<QR, PM_QUANT_Q4_K>(a, L, st, ev);           \
    case PM_QUANT_Q2_K: return pm_layer_launch<QR, PM_QUANT_Q2_K>(a, L, st, ev);           \
    case PM_QUANT_IQ2_XXS: return pm_layer_launch<QR, PM_QUANT_IQ2_XXS>(a, L, st, ev);     \
    case PM_QUANT_MXFP4: return pm_layer_launch<QR, PM_QUANT_MXFP4>(a, L, st, ev);         \
    case PM_QUANT_Q8_0: return pm_layer_launch<QR, PM_QUANT_Q8_0>(a, L, st, ev);           \
    default: return 0;                                                                     \
    }

static int pm_layer_dispatch(uint32_t qr, uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st,
                             void *const *ev) {
    switch (qr) {
    case PM_QUANT_Q4_K: PM_Q2(PM_QUANT_Q4_K)
    case PM_QUANT_Q2_K: PM_Q2(PM_QUANT_Q2_K)
    case PM_QUANT_IQ2_XXS: PM_Q2(PM_QUANT_IQ2_XXS)
    case PM_QUANT_MXFP4: PM_Q2(PM_QUANT_MXFP4)
    case PM_QUANT_Q8_0: PM_Q2(PM_QUANT_Q8_0)
    default: return 0;
    }
}

static int pm_moe_layer_impl(const pulsar_moe_layer_desc *d, float *out, const float *x, const float *residual,
                             uint32_t n_tok, void *ws, size_t ws_bytes, void *stream, void *const *ev) {
    if (!pm_desc_ok(d) || !out || !x || !ws || n_tok == 0) return 0;
    if (!pm_router_args_ok(d->n_expert, d->n_used, n_tok, d->router_mode, 0, d->n_group, d->topk_group)) return 0;
    const pm_layout L = pm_make_layout(d, n_tok);
    if (L.total > ws_bytes) return 0;
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    uint8_t *b = (uint8_t *)ws;
    pm_layer_args a;
    memset(&a, 0, sizeof(a));
    a.T = L.T, a.E = L.E, a.k = L.k, a.S = L.S, a.n_slot = L.n_slot, a.H = L.H, a.Fr = L.Fr, a.Fs = L.Fs;
    a.Fmax = L.Fmax, a.hb = L.hb, a.fb = L.fb, a.max_items = L.max_items;
    a.lo = d->expert_hi ? d->expert_lo : 0;
    a.hi = d->expert_hi ? d->expert_hi : d->n_expert;
    a.act = d->act_op, a.mode = d->router_mode, a.n_group = d->n_group, a.topk_group = d->topk_group;
    a.scale = d->weight_scale;
    a.rb_gu_r = d->row_bytes_gu, a.rb_dn_r = d->row_bytes_down;
    a.st_gu_r = d->expert_stride_gu ? d->expert_stride_gu : (uint64_t)d->n_ff * d->row_bytes_gu;
    a.st_dn_r = d->expert_stride_down ? d->expert_stride_down : (uint64_t)d->n_embd * d->row_bytes_down;
    a.rb_gu_s = d->shared_row_bytes_gu, a.rb_dn_s = d->shared_row_bytes_down;
    a.gate = (const uint8_t *)d->gate, a.up = (const uint8_t *)d->up, a.down = (const uint8_t *)d->down;
    a.sgate = (const uint8_t *)d->shared_gate, a.sup = (const uint8_t *)d->shared_up;
    a.sdown = (const uint8_t *)d->shared_down;
    a.gate_b = d->gate_b, a.up_b = d->up_b, a.down_b = d->down_b, a.router_sel_b = d->router_select_b;
    a.logits = (float *)(b + L.logits);
    a.sel = (int32_t *)(b + L.sel);
    a.w = (float *)(b + L.w);
    a.xq = (pm_block_q8K *)(b + L.xq);
    a.n_items = (uint32_t *)(b + L.n_items);
    a.item_expert = (uint32_t *)(b + L.item_expert);
    a.item_start = (uint32_t *)(b + L.item_start);
    a.pairs = (uint32_t *)(b + L.pairs);
    a.work_item = (uint32_t *)(b + L.work_item);
    a.work_t0 = (uint32_t *)(b + L.work_t0);
    a.mid = (float *)(b + L.mid);
    a.partial = (float *)(b + L.partial);
    a.sel_done = (uint32_t *)(b + L.sel_done);
    a.err = (uint32_t *)(b + L.err);
    a.out = out;
    a.residual = residual;
    a.gu_rows = pm_pow2_rows(L.Fmax, L.max_items, 8, 256);
    a.dn_rows = pm_pow2_rows(L.H, L.max_items, 16, 512);

    /* 1, 2: logits and q8_K(x) */
    pm_ev(ev, 0, st);
    if (!pm_launch_router_logits(a.logits, d->router_w, x, d->router_logit_b, L.E, L.H, L.T, st)) return 0;
    pm_ev(ev, 1, st);
    if (!pm_launch_q8k(a.xq, x, L.H, L.T, st)) return 0;
    pm_ev(ev, 2, st);
    /* 3: select + CSR */
    const uint32_t smem_sel = 4u * 2u * L.E * 4u;
    static uint64_t done_sel = 0;
    if (!pm_smem_attr(pm_layer_select_kernel, smem_sel, &done_sel)) return 0;
    pm_layer_select_kernel<<<(L.T + 3u) / 4u, 128, smem_sel, st>>>(a);
    if (!pm_ok(cudaGetLastError(), "moe layer select launch")) return 0;
    pm_ev(ev, 3, st);
    return pm_layer_dispatch(d->quant, d->n_shared ? d->shared_quant : d->quant, a, L, st, ev);
}

extern "C" int pulsar_moe_layer(const pulsar_moe_layer_desc *d, float *out, const float *x, const float *residual,
                                uint32_t n_tok, void *ws, size_t ws_bytes, void *stream) {
    return pm_moe_layer_impl(d, out, x, residual, n_tok, ws, ws_bytes, stream, nullptr);
}

extern "C" int pulsar_moe_layer_profiled(const pulsar_moe_layer_desc *d, float *out, const float *x,
                                         const float *residual, uint32_t n_tok, void *ws, size_t ws_bytes,
                                         void *stream, void *const *events) {
    return pm_moe_layer_impl(d, out, x, residual, n_tok, ws, ws_bytes, stream, events);
}

/* ============================================ allocation-free variant */

/* Some callers cannot call cudaMalloc: a plugin loaded into a host process
 * that owns every byte of device memory through its own pool, or code that
 * must not allocate (or synchronize the device) while it runs.  For them,
 * pulsar_moe_layer_noalloc keeps the layer's workspace in this fixed
 * array, which every GPU that loads the library holds until the process
 * exits.  In host code `pm_noalloc_scratch` only names the symbol; the
 * device address is resolved per device with cudaGetSymbolAddress. */
#define PM_NOALLOC_SCRATCH_BYTES (32u << 20) /* 32 MiB */
static __device__ __align__(256) uint8_t pm_noalloc_scratch[PM_NOALLOC_SCRATCH_BYTES];

static std::mutex pm_noalloc_mu;
static void *pm_noalloc_addr[64];

extern "C" int pulsar_moe_layer_noalloc(const pulsar_moe_layer_desc *d, float *out, const float *x,
                                        const float *residual, uint32_t n_tok, void *stream) {
    if (!pm_desc_ok(d) || !out || !x || n_tok == 0) return 0;
    const pm_layout L = pm_make_layout(d, n_tok);
    if (L.total > PM_NOALLOC_SCRATCH_BYTES) {
        fprintf(stderr,
                "pulsar-b200: pulsar_moe_layer_noalloc: %u tokens need %zu bytes of scratch, more than the "
                "built-in %u; use fewer tokens per call or pulsar_moe_layer with your own workspace\n",
                n_tok, L.total, PM_NOALLOC_SCRATCH_BYTES);
        return 0;
    }
    int dev = 0;
    if (!pm_ok(cudaGetDevice(&dev), "noalloc: current device") || dev < 0 || dev >= 64) return 0;
    void *ws = nullptr;
    {
        /* first call on a device: resolve the array's device address there */
        std::lock_guard<std::mutex> lock(pm_noalloc_mu);
        if (!pm_noalloc_addr[dev]) {
            void *p = nullptr;
            if (!pm_ok(cudaGetSymbolAddress(&p, pm_noalloc_scratch), "noalloc: scratch address")) return 0;
            pm_noalloc_addr[dev] = p;
        }
        ws = pm_noalloc_addr[dev];
    }
    /* the array keeps the previous call's contents: clear the words that
     * must start at zero (selection arrival counter, error word) */
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    if (!pm_ok(cudaMemsetAsync((uint8_t *)ws + L.sel_done, 0, 4, st), "noalloc: clear counter") ||
        !pm_ok(cudaMemsetAsync((uint8_t *)ws + L.err, 0, 4, st), "noalloc: clear error word"))
        return 0;
    return pm_moe_layer_impl(d, out, x, residual, n_tok, ws, PM_NOALLOC_SCRATCH_BYTES, stream, nullptr);
}
