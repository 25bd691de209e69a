/* moe_layer.cu - one routed-expert MoE layer as a single call, with the
 * expert resolve on the device.
 *
 * The reference engine (crates/engine/src/lib.rs:7537-8705, Ffn::Moe arm)
 * runs the router on the GPU, syncs, reads the selected ids back, builds
 * the per-(token, slot) pointer array on the host, writes it back and then
 * launches pair / q8_K / down.  Here the whole layer stays on the device:
 *
 *   1 router logits (f32 fixed-order GEMV) + q8_K(x) ... router_q8k.cu
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

#include <nccl.h>

#include "pm_layer.cuh"

int pm_launch_q8k(void *out, const float *x, uint32_t in_dim, uint32_t n_rows, cudaStream_t st);
int pm_launch_router_logits_q8(float *logits, const float *w, const float *x, const float *lbias, uint32_t n_expert,
                               uint32_t in_dim, uint32_t n_tok, void *xq, uint32_t *ctl, cudaStream_t st);
int pm_router_args_ok(uint32_t n_expert, uint32_t k_used, uint32_t n_tok, uint32_t mode, uint32_t n_shexp,
                      uint32_t n_group, uint32_t topk_group);

static int pm_sm_count() {
    static int sms[64];
    const int dev = pm_cur_device();
    if (dev < 0 || dev >= 64) return 148;
    if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        (void)cudaGetLastError();
        return 148;
    }
    return sms[dev];
}


/* ------------------------------------------------------------ layout */
static size_t pm_al(size_t v) { return (v + 255) & ~(size_t)255; }

/* routed Q2_K experts on the integer tensor cores (pm_tci8.cuh): whole
 * super-blocks, the select kernel's 20-bit cost / 12-bit tile packing, and
 * at least one routed token per expert on average (T k >= E) for the tiles
 * to pay for their fixed per-super-block cost; below that the dp4a engine
 * streams the weights faster (measured on B200 at config 4's shapes: T 32,
 * T k = 2 E, integer passes 0.32 ms per layer against 0.45 ms; T 8 even;
 * T 1 dp4a ahead).  PULSAR_LAYER_NO_I8 / PULSAR_LAYER_FORCE_I8 override. */
static bool pm_i8_on(const pulsar_moe_layer_desc *d, uint32_t T) {
    const uint64_t routed = (uint64_t)T * d->n_used;
    const bool fits = d->quant == PM_QUANT_Q2_K && d->gate_tiles && d->up_tiles && d->down_tiles &&
                      d->n_embd % 256u == 0 && d->n_ff % 256u == 0 &&
                      routed < (1u << 19) && routed / PM_I8_N + d->n_expert < 4000u;
    if (!fits || (d->path_flags & PULSAR_LAYER_NO_I8)) return false;
    return (d->path_flags & PULSAR_LAYER_FORCE_I8) || routed >= (uint64_t)d->n_expert;
}

/* tensor-core path available for the routed / shared experts */
static bool pm_tc_on_r(const pulsar_moe_layer_desc *d, uint32_t T) {
    return pm_tc_fmt(d->quant) && d->n_embd % 64 == 0 && d->n_ff % 64 == 0 && !pm_i8_on(d, T);
}
static bool pm_tc_on_s(const pulsar_moe_layer_desc *d) {
    return d->n_shared && pm_tc_fmt(d->shared_quant) && d->n_embd % 64 == 0 && d->shared_n_ff % 64 == 0;
}

static pm_layout pm_make_layout(const pulsar_moe_layer_desc *d, uint32_t T, bool ep = false) {
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
    L.n_items = o, o = pm_al(o + 32);
    L.item_expert = o, o = pm_al(o + (size_t)L.max_items * 4);
    L.item_start = o, o = pm_al(o + (size_t)(L.max_items + 1) * 4);
    L.max_work = L.max_items + (uint32_t)(((uint64_t)T * L.n_slot + PM_TT - 1) / PM_TT);
    L.work_item = o, o = pm_al(o + (size_t)L.max_work * 4);
    L.work_t0 = o, o = pm_al(o + (size_t)L.max_work * 4);
    L.wd = o, o = pm_al(o + (size_t)L.max_work * 16);
    L.sk_c = o, o = pm_al(o + (size_t)(L.max_work + 1) * 4);
    /* tensor-core tiles: experts with >= PM_TC_MIN tokens, in tiles of PM_TC_N */
    L.max_tc = (uint32_t)(routed / PM_TC_MIN + (routed + PM_TC_N - 1) / PM_TC_N + 1 +
                          (uint64_t)L.S * ((T + PM_TC_N - 1) / PM_TC_N));
    L.tc_tile = o, o = pm_al(o + (size_t)L.max_tc * 8);
    L.tc_ord = o, o = pm_al(o + (size_t)L.max_tc * 4);
    L.tc_first = o, o = pm_al(o + (size_t)L.max_tc * 4);
    /* integer tensor-core tiles: every routed expert's tokens in chunks of PM_I8_N */
    L.max_i8 = (uint32_t)((routed < L.E ? routed : L.E) + routed / PM_I8_N + 1);
    L.i8_tile = o, o = pm_al(o + (pm_i8_on(d, T) ? (size_t)L.max_i8 * 8 : 0));
    /* tensor-core operand images: token images of every tile, expanded
     * weight images of up to tc_slots experts at a time */
    {
        const bool tr = pm_tc_on_r(d, T), ts = pm_tc_on_s(d);
        const uint64_t n_r = tr ? (routed / PM_TC_MIN < L.E ? routed / PM_TC_MIN : L.E) : 0;
        const uint64_t n_items = T >= PM_TC_MIN ? n_r + (ts ? L.S : 0u) : 0;
        uint64_t sb = 0;
        if (tr) sb = pm_tc_img_bytes(L.H, L.Fr, 2) > pm_tc_img_bytes(L.H, L.Fr, 1) ? pm_tc_img_bytes(L.H, L.Fr, 2)
                                                                                     : pm_tc_img_bytes(L.H, L.Fr, 1);
        if (ts) {
            const uint64_t s2 = pm_tc_img_bytes(L.H, L.Fs, 2), s1 = pm_tc_img_bytes(L.H, L.Fs, 1);
            sb = sb > s2 ? sb : s2;
            sb = sb > s1 ? sb : s1;
        }
        L.tc_slot_bytes = sb;
        L.tc_slots = L.tc_waves = 0;
        size_t nb = 0, nx = 0;
        if (n_items && sb) {
            uint64_t ew = PM_TC_SCRATCH_CAP / sb;
            ew = ew < 1 ? 1 : ew;
            L.tc_slots = (uint32_t)(n_items < ew ? n_items : ew);
            L.tc_waves = (uint32_t)((n_items + L.tc_slots - 1) / L.tc_slots);
            const uint32_t kmax = L.H > L.Fmax ? L.H : L.Fmax;
            nb = (size_t)(kmax / 64u) * 2u * L.max_tc * PM_TC_BIMG;
            nx = (size_t)L.tc_slots * sb;
        }
        L.tcb = o, o = pm_al(o + nb);
        L.tcx = o, o = pm_al(o + nx);
        L.tclo = o, o = pm_al(o + (sb ? nx / (2u * PM_TC_IMG) : 0));
    }
    L.pairs = o, o = pm_al(o + (size_t)T * L.n_slot * 4);
    L.mid = o, o = pm_al(o + (size_t)T * L.n_slot * L.Fmax * 4);
    L.midq = o, o = pm_al(o + (size_t)T * L.n_slot * L.fb * PM_Q8_K_BYTES);
    /* split-K partial sums of the tensor-core gate/up tiles: [ks][pair][gate|up][Fmax] */
    {
        const uint64_t per = (uint64_t)T * L.n_slot * 2 * L.Fmax * 4;
        uint64_t ks = per ? (64ull << 20) / per : 1;
        L.ks_max = (uint32_t)(ks < 1 ? 1 : (ks > 8 ? 8 : ks));
        L.tcp = o, o = pm_al(o + (size_t)L.ks_max * per);
    }
    L.partial = o, o = pm_al(o + (size_t)T * L.n_slot * L.H * 4);
    L.shg = o, o = pm_al(o + (d->shared_gate_w && L.S ? (size_t)T * 4 : 0)); /* shared-expert gate logits */
    /* control words: [0] selection arrival counter, [1] error word; both
     * cleared by the first kernel of every call */
    L.ctl = o, o = pm_al(o + 8);
    /* expert parallel: per-token sums over this rank's experts, before the
     * combine (last, so every other region sits where a single-GPU call of
     * the same T has it) */
    L.epo = o, o = pm_al(o + (ep ? (size_t)T * L.H * 4 : 0));
    L.total = o;
    return L;
}


/* ============================================ 3: select + CSR build */

#define PM_SEL_STAGE 16384u /* routed pairs staged in shared memory (u16 each) */
#define PM_SEL_WARPS 8u      /* tokens per CTA (one warp each) */
#define PM_SEL_MASK_T 448u   /* batches up to this size fill pairs from token masks */

/* uint4 component-wise sum */
__device__ __forceinline__ uint4 pm_add4(uint4 x, uint4 y) {
    return make_uint4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
}

/* Phase 1: one warp per token picks its top-k (pm_select_token).  Phase 2
 * (the last CTA to arrive): group the routed (token, slot) pairs of this
 * shard by expert.  Per expert e with v pairs: one item, ceil(v / PM_TT)
 * work units, and the stream-K cost (PM_SK_CR * units + v); a block-wide
 * exclusive scan over experts places everything.  Pairs are filled in
 * (token, slot) order: a token selects an expert at most once, so the
 * rank of pair (t, s) in its expert's list is the number of earlier tokens
 * that chose the same expert - a popcount over a per-expert token mask. */
__global__ void __launch_bounds__(256) pm_layer_select_kernel(const __grid_constant__ pm_layer_args a) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ uint32_t is_last;
    __shared__ uint4 wsum[PM_SEL_WARPS], carry;
    const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    if (a.phase != 2u) {
        const uint32_t token = a.sel_t0 + blockIdx.x * PM_SEL_WARPS + wid;
        if (token < a.sel_t0 + a.sel_nt) {
            float *score = (float *)sm + (size_t)wid * 2 * (a.E > 256u ? a.E : 256u);
            if (a.E <= 256u && a.k <= 32u && a.mode <= 1u && (a.n_group <= 1u || a.topk_group >= a.n_group))
                pm_select_fast(a.sel, a.w, a.logits, a.router_sel_b, a.E, a.k, a.scale, token, a.mode, score,
                               score + 256, a.n_slot);
            else
                pm_select_token(a.sel, a.w, a.logits, a.router_sel_b, a.E, a.k, a.scale, token, a.mode, 0,
                                a.n_group, a.topk_group, score, score + a.E, a.n_slot);
            if (lane < a.S) { /* shared experts: always-on slots k.., ids E + s, weight 1 */
                a.sel[token * a.n_slot + a.k + lane] = (int32_t)(a.E + lane);
                a.w[token * a.n_slot + a.k + lane] = 1.0f;
            }
        }
        if (a.phase == 1u) return;
        __threadfence(); /* every thread publishes its own selection writes */
        __syncthreads();
        if (threadIdx.x == 0) is_last = atomicAdd(a.sel_done, 1u) == gridDim.x - 1u;
        __syncthreads();
        if (!is_last) return;
        __threadfence();
    }

    /* ---- the last CTA: CSR by expert over routed pairs in [lo, hi) ---- */
    const uint32_t n_routed = a.T * a.k;
    uint32_t *cnt = (uint32_t *)sm; /* [E] counts, then start offsets */
    const uint32_t mw = (a.T + 31u) / 32u;
    uint32_t *mask = cnt + a.E; /* [E][mw] token masks (small batches) */
    const bool masks = a.T <= PM_SEL_MASK_T;
    /* the selections, read once with independent loads (u16; 0xffff = not in this shard) */
    uint16_t *ss = (uint16_t *)(sm + (size_t)PM_SEL_WARPS * 2 * (a.E > 256u ? a.E : 256u) * 4);
    const bool staged = n_routed <= PM_SEL_STAGE && a.E < 65535u;
    auto sel_at = [&](uint32_t q) -> uint32_t {
        uint32_t e;
        if (staged) {
            e = ss[q];
            return e == 0xffffu ? UINT32_MAX : e;
        }
        e = (uint32_t)__ldcg(a.sel + (q / a.k) * a.n_slot + q % a.k);
        return e >= a.lo && e < a.hi ? e : UINT32_MAX;
    };
    for (uint32_t e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;
    if (masks)
        for (uint32_t i = threadIdx.x; i < a.E * mw; i += blockDim.x) mask[i] = 0;
    if (staged) {
#pragma unroll 4
        for (uint32_t q = threadIdx.x; q < n_routed; q += blockDim.x) {
            const uint32_t e = (uint32_t)__ldcg(a.sel + (q / a.k) * a.n_slot + q % a.k);
            ss[q] = (uint16_t)(e >= a.lo && e < a.hi ? e : 0xffffu);
        }
    }
    if (threadIdx.x == 0) carry = make_uint4(0, 0, 0, 0);
    __syncthreads();
    for (uint32_t q = threadIdx.x; q < n_routed; q += blockDim.x) {
        const uint32_t e = sel_at(q);
        if (e == UINT32_MAX) continue;
        atomicAdd(&cnt[e], 1u);
        if (masks) {
            const uint32_t t = q / a.k;
            atomicOr(&mask[e * mw + t / 32u], 1u << (t % 32u));
        }
    }
    __syncthreads();
    /* exclusive scan over experts of (pairs, items, work units, cost) */
#pragma unroll 1
    for (uint32_t c0 = 0; c0 < a.E; c0 += blockDim.x) {
        const uint32_t e = c0 + threadIdx.x;
        const uint32_t v = e < a.E ? cnt[e] : 0u;
        const bool tcq = a.tc_r && v >= PM_TC_MIN; /* this expert's tokens go to tensor-core tiles */
        const bool i8q = !tcq && a.i8 && v;       /* ... or to integer tensor-core tiles of <= 32 */
        const uint32_t nw = tcq || i8q ? 0u : (v + PM_TT - 1) / PM_TT;
        const uint32_t nti = tcq ? (v + PM_TC_N - 1) / PM_TC_N : 0u;
        const uint32_t ni8 = i8q ? (v + PM_I8_N - 1) / PM_I8_N : 0u;
        /* .y packs items (high 16 bits) and tensor-core tiles (low 16 bits); .w packs the
         * stream-K cost (low 20 bits) and the integer tiles (high 12 bits) */
        const uint4 own = make_uint4(v, ((v ? 1u : 0u) << 16) | nti, nw,
                                     PM_SK_CR * nw + (tcq || i8q ? 0u : v) + (ni8 << 20));
        uint4 x = own;
#pragma unroll 1
        for (uint32_t o = 1; o < 32u; o <<= 1) {
            const uint4 y = make_uint4(__shfl_up_sync(0xffffffffu, x.x, o), __shfl_up_sync(0xffffffffu, x.y, o),
                                       __shfl_up_sync(0xffffffffu, x.z, o), __shfl_up_sync(0xffffffffu, x.w, o));
            if (lane >= o) x = pm_add4(x, y);
        }
        if (lane == 31u) wsum[wid] = x;
        __syncthreads();
        uint4 pre = carry;
#pragma unroll 1
        for (uint32_t w2 = 0; w2 < wid; w2++) pre = pm_add4(pre, wsum[w2]);
        const uint4 incl = pm_add4(pre, x);
        const uint32_t start = incl.x - own.x, item = (incl.y >> 16) - (own.y >> 16);
        const uint32_t tt0 = (incl.y & 0xffffu) - nti, w0 = incl.z - own.z;
        const uint32_t cst = (incl.w & 0xfffffu) - (own.w & 0xfffffu), i80 = (incl.w >> 20) - ni8;
        if (e < a.E) {
            cnt[e] = start;
            if (v) {
                a.item_expert[item] = e;
                a.item_start[item] = start;
#pragma unroll 1
                for (uint32_t j = 0; j < nw; j++) {
                    const uint32_t nt = v - j * PM_TT < PM_TT ? v - j * PM_TT : PM_TT;
                    a.work_item[w0 + j] = item;
                    a.work_t0[w0 + j] = j * PM_TT;
                    a.wd[w0 + j] = make_uint4(e, start + j * PM_TT, nt, 0u);
                    a.sk_c[w0 + j] = cst + j * (PM_SK_CR + PM_TT);
                }
#pragma unroll 1
                for (uint32_t j = 0; j < nti; j++) a.tc_tile[tt0 + j] = make_uint2(item, j * PM_TC_N);
#pragma unroll 1
                for (uint32_t j = 0; j < ni8; j++) a.i8_tile[i80 + j] = make_uint2(item, j * PM_I8_N);
            }
        }
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1u) carry = incl;
        __syncthreads();
    }
    const uint32_t tot_pairs = carry.x, tot_items = carry.y >> 16, tot_tc = carry.y & 0xffffu;
    const uint32_t tot_work = carry.z, tot_cost = carry.w & 0xfffffu, tot_i8 = carry.w >> 20;
    /* fill the pair lists in (token, slot) order */
    if (masks) {
        for (uint32_t q = threadIdx.x; q < n_routed; q += blockDim.x) {
            const uint32_t e = sel_at(q);
            if (e == UINT32_MAX) continue;
            const uint32_t t = q / a.k;
            const uint32_t *m = mask + e * mw;
            uint32_t rank = __popc(m[t / 32u] & ((1u << (t % 32u)) - 1u));
            for (uint32_t i = 0; i < t / 32u; i++) rank += __popc(m[i]);
            a.pairs[cnt[e] + rank] = t * a.n_slot + q % a.k;
        }
    } else if (wid == 0) {
        /* large batches: one warp in order, ranks via match_any */
        for (uint32_t c = 0; c < n_routed; c += 32u) {
            const uint32_t q = c + lane;
            uint32_t e = UINT32_MAX, pair = 0;
            if (q < n_routed) {
                pair = (q / a.k) * a.n_slot + q % a.k;
                e = sel_at(q);
            }
            const uint32_t peers = __match_any_sync(0xffffffffu, e);
            const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
            if (e != UINT32_MAX) a.pairs[cnt[e] + rank] = pair;
            __syncwarp();
            if (e != UINT32_MAX && rank == 0) cnt[e] += __popc(peers);
            __syncwarp();
        }
    }
    /* shared experts: one item each over the tokens [sh_t0, sh_t0 + sh_nt)
     * they serve here, appended after the routed items */
    const uint32_t n_sh = a.sh_nt ? a.S : 0u, snt = a.sh_nt;
    const bool sh_tc = a.tc_s && snt >= PM_TC_MIN; /* shared experts on the tensor-core path */
    const uint32_t sh_chunks = sh_tc ? 0u : (snt + PM_TT - 1) / PM_TT;
    const uint32_t sh_cost = sh_tc ? 0u : PM_SK_CR * sh_chunks + snt;
    const uint32_t sh_tiles = sh_tc ? (snt + PM_TC_N - 1) / PM_TC_N : 0u;
    for (uint32_t s = 0; s < n_sh; s++) {
        const uint32_t item = tot_items + s, base = tot_pairs + s * snt, w0 = tot_work + s * sh_chunks;
        const uint32_t c0 = tot_cost + s * sh_cost;
        if (threadIdx.x == 0) {
            a.item_expert[item] = a.E + s;
            a.item_start[item] = base;
        }
        for (uint32_t t = threadIdx.x; t < snt; t += blockDim.x) a.pairs[base + t] = (a.sh_t0 + t) * a.n_slot + a.k + s;
        for (uint32_t j = threadIdx.x; j < sh_chunks; j += blockDim.x) {
            const uint32_t nt = snt - j * PM_TT < PM_TT ? snt - j * PM_TT : PM_TT;
            a.work_item[w0 + j] = item;
            a.work_t0[w0 + j] = j * PM_TT;
            a.wd[w0 + j] = make_uint4(a.E + s, base + j * PM_TT, nt, 0u);
            a.sk_c[w0 + j] = c0 + j * (PM_SK_CR + PM_TT);
        }
        for (uint32_t j = threadIdx.x; j < sh_tiles; j += blockDim.x)
            a.tc_tile[tot_tc + s * sh_tiles + j] = make_uint2(item, j * PM_TC_N);
    }
    /* tensor-core items: dense ordinals (expand slots) and MMA groups */
    const uint32_t n_tc = tot_tc + n_sh * sh_tiles;
    uint32_t n_ti = 0, n_grp = 0;
    {
        __shared__ uint32_t s_cnt[2][32];
        __syncthreads(); /* tile writes of this block are visible */
        const uint32_t nwarp = blockDim.x >> 5;
#pragma unroll 1
        for (uint32_t c0 = 0; c0 < n_tc; c0 += blockDim.x) {
            const uint32_t j = c0 + threadIdx.x;
            const uint32_t ty = j < n_tc ? a.tc_tile[j].y : 1u;
            const uint32_t bf = __ballot_sync(0xffffffffu, j < n_tc && ty == 0u);
            const uint32_t bg = __ballot_sync(0xffffffffu, j < n_tc && ty % (PM_TC_G * PM_TC_N) == 0u);
            if (lane == 0) {
                s_cnt[0][wid] = __popc(bf);
                s_cnt[1][wid] = __popc(bg);
            }
            __syncthreads();
            uint32_t pre = n_ti, tf = 0, tg = 0;
            for (uint32_t w2 = 0; w2 < nwarp; w2++) {
                if (w2 < wid) pre += s_cnt[0][w2];
                tf += s_cnt[0][w2];
                tg += s_cnt[1][w2];
            }
            if (j < n_tc) {
                const uint32_t ord = pre + __popc(bf & ((2u << lane) - 1u)) - 1u;
                a.tc_ord[j] = ord;
                if (ty == 0u) a.tc_first[ord] = j;
            }
            __syncthreads();
            n_ti += tf;
            n_grp += tg;
        }
    }
    if (threadIdx.x == 0) {
        /* K splits of the tensor-core gate/up pass: about one unit per SM,
         * and no split left without chunks */
        const uint32_t units = n_grp * 2u * ((a.Fmax + 127u) / 128u);
        uint32_t ks = units ? (a.n_sm + units - 1) / units : 1u;
        const uint32_t ks_cap = a.ks_max < a.H / 64u ? a.ks_max : a.H / 64u;
        ks = ks < 1u ? 1u : (ks > ks_cap ? ks_cap : ks);
        const uint32_t cps = (a.H / 64u + ks - 1) / ks;
        ks = (a.H / 64u + cps - 1) / cps;
        a.n_items[6] = n_ti;
        a.item_start[tot_items + n_sh] = tot_pairs + n_sh * snt;
        a.n_items[0] = tot_items + n_sh;
        a.n_items[1] = tot_items;
        a.n_items[2] = tot_work + n_sh * sh_chunks;
        a.n_items[3] = tot_work;
        a.n_items[4] = n_tc;
        a.n_items[5] = ks;
        a.n_items[7] = tot_i8;
        a.sk_c[tot_work + n_sh * sh_chunks] = tot_cost + n_sh * sh_cost;
        *a.sel_done = 0;
    }
}

/* mid rows of tensor-core pairs: the K-split gate/up sums (fixed order),
 * biases, glu, route weight -> mid (f32), then q8_K of each 256-block with
 * the CPU-lane quantizer -> midq (the tensor-core down pass's input).
 * Block (tile, 256-row block, group of 8 tokens), a thread per row: the
 * split sums of all 8 tokens are loaded together. */
#define PM_TC_MID_TG 8u
__global__ void __launch_bounds__(256) pm_tc_mid_kernel(const __grid_constant__ pm_layer_args a) {
    __shared__ float s_v[PM_TC_MID_TG][256];
    const uint32_t n_tiles = __ldcg(a.n_items + 4);
    const uint32_t ngrp = PM_TC_N / PM_TC_MID_TG;
    const uint32_t tile = blockIdx.x / ngrp, grp = blockIdx.x % ngrp;
    if (tile >= n_tiles) return;
    const uint32_t KS = __ldcg(a.n_items + 5);
    const uint2 tt = __ldcg(a.tc_tile + tile);
    const uint32_t item = tt.x, e = __ldcg(a.item_expert + item);
    const uint32_t s0 = __ldcg(a.item_start + item), cnt = __ldcg(a.item_start + item + 1) - s0;
    const uint32_t t0 = tt.y + grp * PM_TC_MID_TG;
    if (t0 >= cnt) return;
    const uint32_t nt = cnt - t0 < PM_TC_MID_TG ? cnt - t0 : PM_TC_MID_TG;
    const bool routed = e < a.E;
    const uint32_t F = routed ? a.Fr : a.Fs;
    const uint32_t b = blockIdx.y, row = b * 256u + threadIdx.x;
    if (b * 256u >= F) return;
    const float gb = routed && a.gate_b && row < F ? a.gate_b[(uint64_t)e * a.Fr + row] : 0.0f;
    const float ub = routed && a.up_b && row < F ? a.up_b[(uint64_t)e * a.Fr + row] : 0.0f;
    const uint64_t NP = (uint64_t)a.T * a.n_slot;
    uint32_t p[PM_TC_MID_TG];
    float g[PM_TC_MID_TG], u[PM_TC_MID_TG];
#pragma unroll
    for (uint32_t t = 0; t < PM_TC_MID_TG; t++) {
        p[t] = t < nt ? __ldcg(a.pairs + s0 + t0 + t) : 0u;
        g[t] = u[t] = 0.0f;
    }
    for (uint32_t ks = 0; ks < KS; ks++) {
#pragma unroll
        for (uint32_t t = 0; t < PM_TC_MID_TG; t++) {
            if (t < nt && row < F) {
                const float *src = a.tcp + ((ks * NP + p[t]) * 2u) * a.Fmax + row;
                g[t] += __ldcg(src);
                u[t] += __ldcg(src + a.Fmax);
            }
        }
    }
#pragma unroll
    for (uint32_t t = 0; t < PM_TC_MID_TG; t++) {
        if (t < nt) {
            const float v = row < F ? pm_glu(g[t] + gb, u[t] + ub, a.act) * __ldcg(a.w + p[t]) : 0.0f;
            if (row < F) a.mid[(uint64_t)p[t] * a.Fmax + row] = v;
            s_v[t][threadIdx.x] = v;
        }
    }
    __syncthreads();
    /* q8_K of each token's 256-block: warp t */
    const uint32_t warp = threadIdx.x >> 5;
    if (warp < nt) {
        const uint32_t bn = F - b * 256u < 256u ? F - b * 256u : 256u;
        pm_q8k_warp(s_v[warp], bn, a.midq + (uint64_t)p[warp] * a.fb + b);
    }
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
            if (a.down_b) b = __fadd_rn(b, __fmul_rn(a.w[t * a.n_slot + s], a.down_b[(uint64_t)e * a.H + r]));
        }
    }
    if (t - a.sh_t0 < a.sh_nt) { /* unsigned: t >= sh_t0 and t < sh_t0 + sh_nt */
        /* qwen35: shared output x sigmoid(gate logit), 1 / (1 + e^-s) as the reference forms it */
        const float g = a.shg ? __fdiv_rn(1.0f, __fadd_rn(1.0f, pm_exp_f32(-a.shg[t]))) : 1.0f;
        for (uint32_t s = a.k; s < a.n_slot; s++) {
            const float p = a.partial[(uint64_t)(t * a.n_slot + s) * a.H + r];
            v += a.shg ? __fmul_rn(p, g) : p;
        }
    }
    if (b != 0.0f) v += b;
    if (a.residual && t - a.res_t0 < a.res_nt) v += a.residual[(uint64_t)(t - a.res_t0) * a.H + r];
    a.out[gid] = v;
}

int pm_launch_tc_mid(const pm_layer_args &a, const pm_layout &L, cudaStream_t st) {
    dim3 gm(L.max_tc * (PM_TC_N / PM_TC_MID_TG), (L.Fmax + 255u) / 256u);
    pm_tc_mid_kernel<<<gm, 256, 0, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer tensor-core mid launch");
}

int pm_launch_combine(const pm_layer_args &a, cudaStream_t st) {
    const uint64_t tot = (uint64_t)a.T * a.H;
    pm_layer_combine_kernel<<<(uint32_t)((tot + 255) / 256), 256, 0, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer combine launch");
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

static void *pm_noalloc_ws();

/* GGUF Q2_K rows -> tile planes (layout above); thread per (chunk, row) */
static __global__ void pm_q2k_tiles_kernel(uint8_t *dst, const uint8_t *src, uint32_t n_mat, uint32_t rows,
                                           uint32_t nsb, uint64_t row_bytes, uint64_t mat_stride) {
    const uint32_t nrb = rows / 128u;
    const uint64_t n = (uint64_t)n_mat * nrb * nsb * 128u;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(i % 128u);
        const uint64_t chunk = i / 128u; /* (e nrb + b) nsb + sb */
        const uint32_t sb = (uint32_t)(chunk % nsb);
        const uint64_t eb = chunk / nsb;
        const uint32_t b = (uint32_t)(eb % nrb), e = (uint32_t)(eb / nrb);
        const uint32_t *blk = (const uint32_t *)(src + e * mat_stride + (uint64_t)(b * 128u + r) * row_bytes +
                                                 (uint64_t)sb * PM_Q2_K_BYTES);
        uint32_t w[21];
#pragma unroll
        for (int k = 0; k < 21; k++) w[k] = blk[k]; /* scales 0-3, qs 4-19, d dmin 20 */
        uint8_t *c = dst + chunk * PM_I8_CHUNK;
#pragma unroll
        for (uint32_t j = 0; j < 4; j++)
            *(uint4 *)(c + (j * 128u + r) * 16u) = make_uint4(w[4 + 4 * j], w[5 + 4 * j], w[6 + 4 * j], w[7 + 4 * j]);
        *(uint4 *)(c + 8192u + 16u * r) = make_uint4(w[0], w[1], w[2], w[3]);
        *(uint32_t *)(c + 10240u + 4u * r) = w[20];
    }
}

extern "C" int pulsar_repack_q2k_tiles(void *dst, const void *src, uint32_t n_mat, uint32_t rows, uint32_t cols,
                                       uint64_t row_bytes, uint64_t mat_stride, void *stream) {
    if (!dst || !src || !n_mat || !rows || rows % 128u || !cols || cols % 256u) return 0;
    if (row_bytes < pm_row_bytes(PM_QUANT_Q2_K, cols) || row_bytes % 4u || mat_stride % 4u ||
        (uintptr_t)src % 4u || (uintptr_t)dst % 16u)
        return 0;
    if (n_mat > 1 && mat_stride < (uint64_t)rows * row_bytes) return 0;
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    const uint64_t n = (uint64_t)n_mat * rows * (cols / 256u);
    const uint32_t grid = (uint32_t)((n + 255u) / 256u < 65536u ? (n + 255u) / 256u : 65536u);
    pm_q2k_tiles_kernel<<<grid, 256, 0, st>>>((uint8_t *)dst, (const uint8_t *)src, n_mat, rows, cols / 256u,
                                               row_bytes, mat_stride);
    return pm_ok(cudaGetLastError(), "q2_K tile-plane repack launch");
}

extern "C" int pulsar_moe_layer_ws_view(const pulsar_moe_layer_desc *d, uint32_t n_tok, void *ws,
                                        pulsar_moe_ws_view *v) {
    if (!ws) ws = pm_noalloc_ws(); /* the built-in array of pulsar_moe_layer_noalloc on this device */
    if (!pm_desc_ok(d) || !ws || !v || n_tok == 0) return 0;
    const pm_layout L = pm_make_layout(d, n_tok);
    uint8_t *b = (uint8_t *)ws;
    v->logits = (float *)(b + L.logits);
    v->selected = (int32_t *)(b + L.sel);
    v->weights = (float *)(b + L.w);
    v->xq = b + L.xq;
    v->mid = (float *)(b + L.mid);
    v->err = (uint32_t *)(b + L.ctl) + 1;
    v->n_items = (uint32_t *)(b + L.n_items);
    v->item_expert = (uint32_t *)(b + L.item_expert);
    v->item_start = (uint32_t *)(b + L.item_start);
    v->pairs = (uint32_t *)(b + L.pairs);
    v->work_item = (uint32_t *)(b + L.work_item);
    v->work_t0 = (uint32_t *)(b + L.work_t0);
    v->partial = (float *)(b + L.partial);
    v->tc_tile = (uint32_t *)(b + L.tc_tile);
    v->n_slot = L.n_slot;
    v->f_max = L.Fmax;
    v->tc_img = b + L.tcx;
    v->tc_lo = b + L.tclo;
    v->tc_slot_bytes = L.tc_slot_bytes;
    v->tc_slots = L.tc_slots;
    v->max_tc = L.max_tc;
    return 1;
}

static int pm_layer_dispatch(uint32_t qr, uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st,
                             void *const *ev) {
    switch (qr) {
    case PM_QUANT_Q4_K: return pm_layer_q4k(qs, a, L, st, ev);
    case PM_QUANT_Q2_K: return pm_layer_q2k(qs, a, L, st, ev);
    case PM_QUANT_IQ2_XXS: return pm_layer_iq2xxs(qs, a, L, st, ev);
    case PM_QUANT_MXFP4: return pm_layer_mxfp4(qs, a, L, st, ev);
    case PM_QUANT_Q8_0: return pm_layer_q80(qs, a, L, st, ev);
    default: return 0;
    }
}

/* expert-parallel context of a call (world 1 = a plain single-GPU call) */
struct pm_ep {
    ncclComm_t comm;
    uint32_t rank, world;
};

static int pm_nccl_ok(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return 1;
    fprintf(stderr, "pulsar-b200: %s: %s\n", what, ncclGetErrorString(r));
    return 0;
}

/* the argument block of a call over T tokens in workspace ws */
static void pm_fill_args(pm_layer_args &a, const pulsar_moe_layer_desc *d, const pm_layout &L, uint8_t *b) {
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
    a.gate_t = (const uint8_t *)d->gate_tiles, a.up_t = (const uint8_t *)d->up_tiles;
    a.down_t = (const uint8_t *)d->down_tiles;
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
    a.wd = (uint4 *)(b + L.wd);
    a.sk_c = (uint32_t *)(b + L.sk_c);
    a.tc_tile = (uint2 *)(b + L.tc_tile);
    a.tc_ord = (uint32_t *)(b + L.tc_ord);
    a.tc_first = (uint32_t *)(b + L.tc_first);
    a.tcb = b + L.tcb;
    a.tcx = b + L.tcx;
    a.tclo = b + L.tclo;
    a.tc_slot_bytes = L.tc_slot_bytes;
    a.tc_slots = L.tc_slots;
    a.max_tc = L.max_tc;
    a.midq = (pm_block_q8K *)(b + L.midq);
    a.tcp = (float *)(b + L.tcp);
    a.ks_max = L.ks_max;
    a.tc_r = pm_tc_on_r(d, L.T);
    a.i8 = pm_i8_on(d, L.T) ? 1u : 0u;
    a.i8_tile = (uint2 *)(b + L.i8_tile);
    a.max_i8 = L.max_i8;
    a.tc_s = pm_tc_on_s(d);
    a.n_sm = (uint32_t)pm_sm_count();
    a.mid = (float *)(b + L.mid);
    a.partial = (float *)(b + L.partial);
    a.sel_done = (uint32_t *)(b + L.ctl);
    a.err = a.sel_done + 1;
    a.wait = d->wait_cycles ? (long long)(d->wait_cycles < (uint64_t)PM_WAIT_CYCLES ? d->wait_cycles
                                                                                  : (uint64_t)PM_WAIT_CYCLES)
                            : PM_WAIT_CYCLES;
    /* single GPU: every token is this call's, the shared expert serves all
     * of them (on the shard that owns expert 0 when the experts are split) */
    a.shg = d->shared_gate_w && L.S ? (const float *)(b + L.shg) : nullptr;
    a.sel_t0 = 0, a.sel_nt = L.T;
    a.sh_t0 = 0, a.sh_nt = a.lo == 0 ? L.T : 0u;
    a.res_t0 = 0, a.res_nt = L.T;
    a.phase = 0;
}

static int pm_select_launch(const pm_layer_args &a, const pm_layout &L, uint32_t grid, cudaStream_t st) {
    const uint32_t n_routed = L.T * L.k;
    const uint32_t per_warp = 2u * (L.E > 256u ? L.E : 256u) * 4u; /* scores + probabilities */
    const uint32_t smem_sel = PM_SEL_WARPS * per_warp + (n_routed <= PM_SEL_STAGE ? 2u * n_routed : 0u);
    static uint64_t done_sel = 0;
    if (!pm_smem_attr(pm_layer_select_kernel, smem_sel, &done_sel)) return 0;
    pm_layer_select_kernel<<<grid, PM_SEL_WARPS * 32u, smem_sel, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer select launch");
}

/* One layer call.  ep.world > 1: this rank's n_tok tokens are routed here,
 * the (q8_K rows, ids, weights) of every rank's tokens are all-gathered,
 * this rank's experts [lo, hi) run for every token that chose them and its
 * shared expert for its own tokens, and the per-token sums are
 * reduce-scattered back to the token owners. */
static int pm_moe_layer_run(const pulsar_moe_layer_desc *d, const pm_ep &ep, float *out, const float *x,
                            const float *residual, uint32_t n_tok, void *ws, size_t ws_bytes, void *stream,
                            void *const *ev) {
    if (!pm_desc_ok(d) || !out || !x || !ws || n_tok == 0) return 0;
    if (ep.world > 1 && (!d->expert_hi || ep.rank >= ep.world || (uint64_t)n_tok * ep.world > 0xffffffffull))
        return 0;
    if (!pm_router_args_ok(d->n_expert, d->n_used, n_tok * ep.world, d->router_mode, 0, d->n_group, d->topk_group))
        return 0;
    const pm_layout L = pm_make_layout(d, n_tok * ep.world, ep.world > 1);
    if (L.total > ws_bytes) return 0;
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    uint8_t *b = (uint8_t *)ws;
    pm_layer_args a;
    pm_fill_args(a, d, L, b);
    const uint32_t t0 = ep.rank * n_tok; /* this rank's tokens in the gathered order */
    if (ep.world > 1) {
        a.sel_t0 = t0, a.sel_nt = n_tok;
        a.sh_t0 = t0, a.sh_nt = d->n_shared ? n_tok : 0u;
        a.res_t0 = t0, a.res_nt = residual ? n_tok : 0u;
        a.out = (float *)(b + L.epo);
    } else {
        a.out = out;
    }
    a.residual = residual;

    /* 1, 2: logits and q8_K(x) of this call's own tokens */
    pm_ev(ev, 0, st);
    if (!pm_launch_router_logits_q8(a.logits + (uint64_t)t0 * L.E, d->router_w, x, d->router_logit_b, L.E, L.H,
                                    n_tok, a.xq + (uint64_t)t0 * L.hb, a.sel_done, st))
        return 0;
    if (a.shg && !pm_launch_router_logits_q8((float *)a.shg + t0, d->shared_gate_w, x, nullptr, 1u, L.H, n_tok,
                                             nullptr, nullptr, st))
        return 0;
    pm_ev(ev, 1, st);
    pm_ev(ev, 2, st); /* q8_K of x is written by the router kernel */
    /* 3: select + CSR */
    const uint32_t sel_grid = (n_tok + PM_SEL_WARPS - 1) / PM_SEL_WARPS;
    if (ep.world == 1) {
        if (!pm_select_launch(a, L, sel_grid, st)) return 0;
    } else {
        a.phase = 1;
        if (!pm_select_launch(a, L, sel_grid, st)) return 0;
        /* dispatch: every rank's q8_K rows, ids and weights (in place) */
        const size_t xq_b = (size_t)n_tok * L.hb * PM_Q8_K_BYTES, nsl = (size_t)n_tok * L.n_slot;
        if (!pm_nccl_ok(ncclGroupStart(), "ep dispatch") ||
            !pm_nccl_ok(ncclAllGather((uint8_t *)a.xq + (size_t)ep.rank * xq_b, a.xq, xq_b, ncclUint8, ep.comm, st),
                        "ep dispatch q8_K rows") ||
            !pm_nccl_ok(ncclAllGather(a.sel + (size_t)ep.rank * nsl, a.sel, nsl, ncclInt32, ep.comm, st),
                        "ep dispatch ids") ||
            !pm_nccl_ok(ncclAllGather(a.w + (size_t)ep.rank * nsl, a.w, nsl, ncclFloat32, ep.comm, st),
                        "ep dispatch weights") ||
            !pm_nccl_ok(ncclGroupEnd(), "ep dispatch"))
            return 0;
        a.phase = 2;
        if (!pm_select_launch(a, L, 1, st)) return 0;
    }
    pm_ev(ev, 3, st);
    if (!pm_layer_dispatch(d->quant, d->n_shared ? d->shared_quant : d->quant, a, L, st, ev)) return 0;
    if (ep.world > 1) /* combine: this rank's tokens summed over every rank's experts */
        if (!pm_nccl_ok(ncclReduceScatter(a.out, out, (size_t)n_tok * L.H, ncclFloat32, ncclSum, ep.comm, st),
                        "ep combine"))
            return 0;
    return 1;
}

static int pm_moe_layer_impl(const pulsar_moe_layer_desc *d, float *out, const float *x, const float *residual,
                             uint32_t n_tok, void *ws, size_t ws_bytes, void *stream, void *const *ev) {
    const pm_ep one = {nullptr, 0u, 1u};
    return pm_moe_layer_run(d, one, out, x, residual, n_tok, ws, ws_bytes, stream, ev);
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

/* the array's device address on the current device.  Resolved on every
 * call (cudaGetSymbolAddress allocates nothing and is cheap once the module
 * is loaded on the device), so it stays right across a device reset. */
static void *pm_noalloc_ws() {
    void *p = nullptr;
    if (!pm_ok(cudaGetSymbolAddress(&p, pm_noalloc_scratch), "noalloc: scratch address")) return nullptr;
    return p;
}

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
    /* the first call on a device loads the module there and resolves the
     * address; the array keeps the previous call's contents, and the words
     * that must start at zero (selection counter, error word) are cleared
     * by the call's first kernel, as for every pulsar_moe_layer call */
    void *ws = pm_noalloc_ws();
    if (!ws) return 0;
    return pm_moe_layer_impl(d, out, x, residual, n_tok, ws, PM_NOALLOC_SCRATCH_BYTES, stream, nullptr);
}


/* ============================================ expert parallel (NCCL) */

extern "C" size_t pulsar_moe_layer_ep_workspace(const pulsar_moe_layer_desc *d, uint32_t world, uint32_t max_tok) {
    if (!pm_desc_ok(d) || max_tok == 0 || world == 0 || (uint64_t)max_tok * world > 0xffffffffull) return 0;
    return pm_make_layout(d, max_tok * world, world > 1).total;
}

extern "C" int pulsar_moe_layer_ep(const pulsar_moe_layer_desc *d, void *nccl_comm, uint32_t rank, uint32_t world,
                                   float *out, const float *x, const float *residual, uint32_t n_tok, void *ws,
                                   size_t ws_bytes, void *stream) {
    if (world == 0 || (world > 1 && !nccl_comm)) return 0;
    const pm_ep ep = {(ncclComm_t)nccl_comm, rank, world};
    return pm_moe_layer_run(d, ep, out, x, residual, n_tok, ws, ws_bytes, stream, nullptr);
}

extern "C" int pulsar_ep_unique_id(void *id) {
    if (!id) return 0;
    ncclUniqueId u;
    if (!pm_nccl_ok(ncclGetUniqueId(&u), "ep unique id")) return 0;
    memcpy(id, &u, sizeof(u));
    return 1;
}

extern "C" int pulsar_ep_comm_init(void **comm, const void *id, uint32_t world, uint32_t rank) {
    if (!comm || !id || world == 0 || rank >= world) return 0;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    if (!pm_nccl_ok(ncclCommInitRank(&c, (int)world, u, (int)rank), "ep communicator")) return 0;
    *comm = (void *)c;
    return 1;
}

extern "C" int pulsar_ep_comm_destroy(void *comm) {
    if (!comm) return 0;
    return pm_nccl_ok(ncclCommDestroy((ncclComm_t)comm), "ep communicator destroy");
}
