/* pm_layer.cuh - the expert kernels of the fused MoE layer call and their
 * launch helpers, shared by moe_layer.cu (layout, selection, combine, entry
 * points) and the moe_layer_<format>.cu files, which each instantiate the
 * gate/up and down passes of one routed-expert format (split so the format
 * instantiations compile in parallel).
 *
 * Kernels here:
 *  - pm_layer_sk_kernel: the persistent stream-K dp4a pass (gate/up + glu
 *    -> mid, or down -> partial rows);
 *  - pm_tc_expand_kernel / pm_tc_pack_kernel / pm_tc_gemm_kernel: the
 *    tcgen05 tiles of experts with many tokens.
 */
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/pulsar_moe.h"
#include "pm_host.h"
#include "pm_router.cuh"
#include "pm_gemv.cuh"
#include "pm_tc.cuh"

__device__ static const uint16_t pm_kgrid_layer[256] = PM_IQ2XXS_KGRID_INIT;

#define PM_TC_N 64u  /* tokens per tensor-core tile (MMA N) */
#define PM_TC_MIN 192u /* experts with at least this many tokens take the tensor-core path: below it the
                        * once-per-call expand costs more than the dp4a units it replaces */
#define PM_TC_G 4u                   /* tiles per MMA group */
#define PM_TC_IMG 16384u             /* one 128 x 64 fp16 operand image */
#define PM_TC_BIMG (PM_TC_N * 128u)  /* one 64-token x 64 fp16 image */
#define PM_TC_XP 276u                /* largest raw row pitch of the expand kernel */
#define PM_TC_SCRATCH_CAP (4ull << 30) /* bound of the expanded-image region of the workspace */

/* per item kind: operand rows, 128-row blocks, 64-wide K chunks, matrices */
struct pm_tcgeo {
    uint32_t rows, rt_n, nch, nm;
};
__host__ __device__ __forceinline__ pm_tcgeo pm_tc_geo(uint32_t H, uint32_t F, int nmat) {
    pm_tcgeo g;
    g.rows = nmat == 2 ? F : H;
    g.rt_n = (g.rows + 127u) / 128u;
    g.nch = (nmat == 2 ? H : F) / 64u;
    g.nm = (uint32_t)nmat;
    return g;
}
/* bytes of one expert's images (hi + lo) for a pass */
__host__ __device__ __forceinline__ uint64_t pm_tc_img_bytes(uint32_t H, uint32_t F, int nmat) {
    const pm_tcgeo g = pm_tc_geo(H, F, nmat);
    return (uint64_t)g.nm * g.rt_n * g.nch * 2u * PM_TC_IMG;
}
/* raw row pitch of the expand kernel: room for the span and the bytes
 * below it to the word boundary.  Q4_K (read with 16-byte loads, rows
 * 16-byte aligned) keeps 144 = 9 x 16: eight threads of a quarter warp hit
 * distinct bank quads.  The others (byte, 2- and 4-byte loads) use an odd
 * number of words, so the 32 rows of a warp fall in 32 distinct banks. */
__host__ __device__ constexpr uint32_t pm_tc_xpitch(int q) {
    return q == PM_QUANT_Q4_K ? 144u
           : q == PM_QUANT_Q2_K ? 92u
           : q == PM_QUANT_IQ2_XXS ? 76u
           : q == PM_QUANT_MXFP4 ? 140u : 276u;
}
/* bytes of 256 weights of a row (a super-block; 8 blocks of 32) */
__host__ __device__ constexpr uint32_t pm_tc_sb_bytes(int q) {
    return q == PM_QUANT_Q4_K ? PM_Q4_K_BYTES
           : q == PM_QUANT_Q2_K ? PM_Q2_K_BYTES
           : q == PM_QUANT_IQ2_XXS ? PM_IQ2_XXS_BYTES
           : q == PM_QUANT_MXFP4 ? 8u * PM_MXFP4_BLOCK : 8u * PM_Q8_0_BLOCK;
}

/* formats with a tensor-core (fp16 dequant) path */
static bool pm_tc_fmt(uint32_t q) {
    return q == PM_QUANT_Q4_K || q == PM_QUANT_Q2_K || q == PM_QUANT_IQ2_XXS || q == PM_QUANT_MXFP4 ||
           q == PM_QUANT_Q8_0;
}



struct pm_layout {
    uint32_t T, E, k, S, n_slot, H, Fr, Fs, Fmax, hb, fb, max_items;
    uint32_t max_work;
    uint32_t max_tc, ks_max, tc_slots, tc_waves, max_i8;
    uint64_t tc_slot_bytes;
    size_t tc_ord, tc_first, tcb, tcx, tclo, i8_tile;
    size_t logits, sel, w, xq, n_items, item_expert, item_start, work_item, work_t0, wd, sk_c, tc_tile, pairs, mid,
        midq, tcp, partial, epo, shg, ctl, total;
};


/* device-side view of the descriptor + workspace */
struct pm_layer_args {
    /* geometry */
    uint32_t T, E, k, S, n_slot, H, Fr, Fs, Fmax, hb, fb, max_items;
    uint32_t lo, hi, act, mode, n_group, topk_group;
    float scale;
    uint64_t rb_gu_r, rb_dn_r, st_gu_r, st_dn_r, rb_gu_s, rb_dn_s;
    const uint8_t *gate, *up, *down, *sgate, *sup, *sdown;
    const uint8_t *gate_t, *up_t, *down_t; /* Q2_K tile-plane images (integer tensor-core passes) */
    const float *gate_b, *up_b, *down_b, *router_sel_b;
    /* workspace */
    float *logits;
    int32_t *sel;
    float *w;
    pm_block_q8K *xq;
    uint32_t *n_items; /* [0] all items, [1] routed items, [2] work units, [3] routed work units,
                        * [4] tensor-core tiles, [5] their gate/up K splits, [6] tensor-core items */
    uint32_t *item_expert, *item_start, *pairs;
    uint32_t *work_item, *work_t0; /* work unit = (item, first token of its chunk of <= PM_TT) */
    uint4 *wd;      /* per work unit: expert id (E + s for shared s), first pair, token count */
    uint2 *tc_tile; /* tensor-core tiles: (item, first token) */
    uint32_t *tc_ord;   /* per tile: dense ordinal of its item among the tensor-core items */
    uint32_t *tc_first; /* per ordinal: the item's first tile */
    uint8_t *tcb;       /* token images ((chunk * 2 + hl) * max_tc + tile) */
    uint8_t *tcx;       /* expanded weight images of the current wave, tc_slot_bytes per item */
    uint8_t *tclo;      /* per image pair: 1 if its lo image is written (nonzero), 0 if all lo parts are 0 */
    uint64_t tc_slot_bytes;
    uint32_t tc_slots, max_tc;
    pm_block_q8K *midq; /* q8_K of the mid rows of tensor-core pairs */
    float *tcp;     /* [ks][pair][2][Fmax] split-K gate/up sums of tensor-core tiles */
    uint32_t ks_max, tc_r, tc_s, n_sm; /* split bound; tensor-core path on for routed / shared */
    uint32_t *sk_c; /* [n_work + 1] prefix of per-row costs (PM_SK_CR + nt) over work units */
    float *mid;
    float *partial; /* [T * n_slot][H] down outputs before the combine */
    uint32_t *sel_done, *err;
    long long wait; /* budget of ring / accumulator waits in SM cycles */
    /* token ranges (expert parallel: the T tokens are every rank's, gathered)
     *  sel_t0, sel_nt  tokens whose top-k this call computes (selection phase)
     *  sh_t0, sh_nt    tokens the shared expert serves here
     *  res_t0, res_nt  tokens whose residual rows this call adds
     * phase: 0 selection then CSR in one launch, 1 selection only, 2 CSR only */
    uint32_t sel_t0, sel_nt, sh_t0, sh_nt, res_t0, res_nt, phase;
    uint2 *i8_tile;           /* integer tensor-core tiles (item, first token); count n_items[7] */
    uint32_t i8, max_i8;      /* routed experts on the integer tensor cores */
    const float *shg; /* [T] shared-expert gate logits (qwen35), or null */
    /* io */
    float *out;
    const float *residual;
};

#include "pm_tci8.cuh"

/* launchers of the kernels defined in moe_layer.cu */
int pm_launch_tc_mid(const pm_layer_args &a, const pm_layout &L, cudaStream_t st);
int pm_launch_combine(const pm_layer_args &a, cudaStream_t st);

/* ========================================= 4, 5: gate/up and down */

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
    return g; /* the first __syncthreads of the kernel publishes it */
}

/* matrix rows of a work unit: gate/up F (routed or shared), down H */
template <int EPI>
__device__ __forceinline__ uint32_t pm_unit_rows(const pm_layer_args &a, uint32_t e) {
    if (EPI == 1) return a.H;
    return e < a.E ? a.Fr : a.Fs;
}

/* position of work unit w on the cost line (rows x per-row cost) */
template <int EPI>
__device__ __forceinline__ uint64_t pm_line(const pm_layer_args &a, uint32_t w, uint32_t n_rw, uint64_t c_rw) {
    const uint64_t c = __ldcg(a.sk_c + w);
    if (EPI == 1) return c * a.H;
    return w <= n_rw ? c * a.Fr : c_rw * a.Fr + (c - c_rw) * a.Fs;
}

template <int EPI>
__device__ __forceinline__ pm_segi pm_seg_load(const pm_layer_args &a, uint32_t w, uint32_t r0, uint32_t r1) {
    const uint4 d = __ldcg(a.wd + w);
    const uint32_t e = d.x;
    pm_segi s;
    s.kind = e < a.E ? 0u : 1u;
    s.nt = d.z;
    s.r0 = r0;
    s.r1 = r1;
    s.pairs = a.pairs + d.y;
    s.b0 = s.b1 = nullptr;
    if (EPI == 0) {
        s.base[0] = s.kind == 0 ? a.gate + (uint64_t)e * a.st_gu_r : a.sgate;
        s.base[1] = s.kind == 0 ? a.up + (uint64_t)e * a.st_gu_r : a.sup;
        if (s.kind == 0 && a.gate_b) s.b0 = a.gate_b + (uint64_t)e * a.Fr;
        if (s.kind == 0 && a.up_b) s.b1 = a.up_b + (uint64_t)e * a.Fr;
    } else {
        s.base[0] = s.kind == 0 ? a.down + (uint64_t)e * a.st_dn_r : a.sdown;
        s.base[1] = nullptr;
    }
    return s;
}

/* the CTA's slice of the cost line as segments k = 0 .. n_seg-1 */
struct pm_slice {
    uint32_t w_lo, r_lo, w_hi, r_hi, n_seg;
};

template <int EPI>
__device__ __forceinline__ pm_segi pm_seg_get(const pm_layer_args &a, const pm_segi *tab, const pm_slice &sl,
                                              uint32_t k) {
    if (k < PM_SK_MAXSEG) return tab[k];
    const uint32_t w = sl.w_lo + k;
    const uint32_t r1 = w == sl.w_hi ? sl.r_hi : pm_unit_rows<EPI>(a, __ldcg(a.wd + w).x);
    return pm_seg_load<EPI>(a, w, 0u, r1);
}

/* a warp's walk over its stages g = warp, warp + 8, ... of the CTA's
 * concatenated segments (segment k holds stages [g0, g0 + nst)) */
struct pm_it {
    uint32_t k, g0, nst, g;
};

template <int EPI>
__device__ __forceinline__ void pm_it_norm(pm_it &it, const pm_layer_args &a, const pm_segi *tab,
                                           const pm_slice &sl, const pm_skp &P) {
    while (it.k < sl.n_seg && it.g >= it.g0 + it.nst) {
        it.g0 += it.nst;
        it.k++;
        if (it.k < sl.n_seg) {
            const pm_segi s = pm_seg_get<EPI>(a, tab, sl, it.k);
            const uint32_t rw = P.k[s.kind].rw;
            it.nst = (s.r1 - s.r0 + rw - 1) / rw;
        }
    }
}

template <int NMAT>
__device__ __forceinline__ void pm_stage_src(const pm_segi &s, const pm_skind &kd, const pm_it &it,
                                             const uint8_t **src, uint32_t &r, uint32_t &rows) {
    r = s.r0 + (it.g - it.g0) * kd.rw;
    rows = s.r1 - r < kd.rw ? s.r1 - r : kd.rw;
#pragma unroll
    for (int m = 0; m < NMAT; m++) src[m] = s.base[m] + (uint64_t)r * kd.rb;
}

/* Persistent stream-K pass (pm_gemv.cuh).  EPI 0: gate+up of every work
 * unit, glu * route weight -> mid.  EPI 1: down of every work unit (mid
 * rows quantized to q8_K while staging) -> one partial row per pair. */
template <int QR, int QS, int NMAT, int EPI>
__global__ void __launch_bounds__(32 * pm_sk_warps(NMAT), pm_sk_minb(NMAT))
    pm_layer_sk_kernel(const __grid_constant__ pm_layer_args a, const __grid_constant__ pm_skp P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t s_cnt[2], s_lim[4], s_tok[PM_TT];
    __shared__ pm_rowjob s_jb;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint64_t *grid = pm_grid_fill(smem, QR == PM_QUANT_IQ2_XXS || QS == PM_QUANT_IQ2_XXS);
    uint64_t *bars = (uint64_t *)(smem + P.off_bar) + warp * P.S;
    pm_segi *tab = (pm_segi *)(smem + P.off_seg);
    uint8_t *ring = smem + P.off_ring + (size_t)warp * P.S * P.stage;
    const pm_acts acts = pm_acts_carve(smem + P.off_acts, P.P, P.NB);
    if (lane == 0) {
        for (uint32_t i = 0; i < P.S; i++) pm_mbar_init(bars + i, 1);
        pm_fence_barrier_init();
    }
    if (tid < 2) s_cnt[tid] = 0;
    __syncthreads();

    /* ---- this CTA's slice [lo, hi) of the cost line ---- */
    const uint32_t n_work = __ldcg(a.n_items + 2), n_rw = __ldcg(a.n_items + 3);
    const uint64_t c_rw = __ldcg(a.sk_c + n_rw);
    const uint64_t C = pm_line<EPI>(a, n_work, n_rw, c_rw);
    const uint64_t lo = C * blockIdx.x / gridDim.x, hi = C * (blockIdx.x + 1) / gridDim.x;
    {
        uint32_t c0 = 0, c1 = 0; /* units that start at or before lo / hi */
        for (uint32_t i = tid + 1; i <= n_work; i += blockDim.x) {
            const uint64_t v = pm_line<EPI>(a, i, n_rw, c_rw);
            c0 += v <= lo;
            c1 += v <= hi;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            c0 += __shfl_xor_sync(0xffffffffu, c0, o);
            c1 += __shfl_xor_sync(0xffffffffu, c1, o);
        }
        if (lane == 0) {
            atomicAdd(&s_cnt[0], c0);
            atomicAdd(&s_cnt[1], c1);
        }
    }
    __syncthreads();
    if (tid < 2) { /* (unit, row) of a position, rows rounded up to PM_SK_RQ */
        const uint64_t pos = tid ? hi : lo;
        uint32_t w = s_cnt[tid], r = 0;
        if (w < n_work) {
            const uint4 d = __ldcg(a.wd + w);
            const uint32_t rows = pm_unit_rows<EPI>(a, d.x);
            const uint64_t off = (pos - pm_line<EPI>(a, w, n_rw, c_rw)) / (PM_SK_CR + d.z);
            const uint64_t rq = (off + PM_SK_RQ - 1) / PM_SK_RQ * PM_SK_RQ;
            if (rq >= rows)
                w++;
            else
                r = (uint32_t)rq;
        }
        s_lim[2 * tid] = w;
        s_lim[2 * tid + 1] = r;
    }
    __syncthreads();
    pm_slice sl;
    sl.w_lo = s_lim[0], sl.r_lo = s_lim[1], sl.w_hi = s_lim[2], sl.r_hi = s_lim[3];
    sl.n_seg = sl.w_hi >= sl.w_lo ? sl.w_hi - sl.w_lo + (sl.r_hi ? 1u : 0u) : 0u;
    for (uint32_t k = tid; k < sl.n_seg && k < PM_SK_MAXSEG; k += blockDim.x) {
        const uint32_t w = sl.w_lo + k;
        const uint32_t r1 = w == sl.w_hi ? sl.r_hi : pm_unit_rows<EPI>(a, __ldcg(a.wd + w).x);
        tab[k] = pm_seg_load<EPI>(a, w, k == 0 ? sl.r_lo : 0u, r1);
    }
    __syncthreads();
    if (sl.n_seg == 0) return;

    /* ---- warp-private rings: the prologue fills S stages ---- */
    auto it_init = [&]() {
        pm_it it;
        it.k = 0, it.g0 = 0, it.g = warp;
        const pm_segi s = tab[0];
        it.nst = (s.r1 - s.r0 + P.k[s.kind].rw - 1) / P.k[s.kind].rw;
        pm_it_norm<EPI>(it, a, tab, sl, P);
        return it;
    };
    /* stages of "direct" kinds (rows too large for the ring) are read from
     * global memory by the consumer: the issue walk steps over them */
    auto skip_direct = [&](pm_it &it) {
        while (it.k < sl.n_seg) {
            const uint32_t kind = it.k < PM_SK_MAXSEG ? tab[it.k].kind : pm_seg_get<EPI>(a, tab, sl, it.k).kind;
            if (!P.k[kind].direct) break;
            const uint32_t end = it.g0 + it.nst, W = (uint32_t)pm_sk_warps(NMAT);
            it.g += (end - it.g + W - 1) / W * W;
            pm_it_norm<EPI>(it, a, tab, sl, P);
        }
    };
    pm_it iti = it_init(), itc = iti;
    skip_direct(iti);
    uint32_t ni = 0, ci = 0;
    auto issue = [&](uint32_t slot) { /* lane 0: the stage iti points at */
        const uint8_t *src[NMAT];
        uint32_t r, rows, kind;
        if (iti.k < PM_SK_MAXSEG) { /* the fields it needs, straight from the table */
            const pm_segi *t = tab + iti.k;
            kind = t->kind;
            const pm_skind &kd = P.k[kind];
            r = t->r0 + (iti.g - iti.g0) * kd.rw;
            rows = t->r1 - r < kd.rw ? t->r1 - r : kd.rw;
#pragma unroll
            for (int m = 0; m < NMAT; m++) src[m] = t->base[m] + (uint64_t)r * kd.rb;
        } else {
            const pm_segi sg = pm_seg_get<EPI>(a, tab, sl, iti.k);
            kind = sg.kind;
            pm_stage_src<NMAT>(sg, P.k[kind], iti, src, r, rows);
        }
        pm_issue_stage<NMAT>(ring + (size_t)slot * P.stage, bars + slot, src, rows * (uint32_t)P.k[kind].rb);
    };
    while (ni < P.S && iti.k < sl.n_seg) {
        if (lane == 0) issue(ni);
        ni++;
        iti.g += (uint32_t)pm_sk_warps(NMAT);
        pm_it_norm<EPI>(iti, a, tab, sl, P);
        skip_direct(iti);
    }

    /* ---- segments: swap the token tile, then consume this warp's stages ---- */
    bool fail = false;
    for (uint32_t k = 0; k < sl.n_seg; k++) {
        if (k > 0 && __syncthreads_or(fail)) break;
        const pm_segi s = pm_seg_get<EPI>(a, tab, sl, k);
        const pm_skind &kd = P.k[s.kind];
        if (EPI == 0) {
            const pm_block_q8K *rows[PM_TT];
#pragma unroll
            for (uint32_t t = 0; t < PM_TT; t++)
                rows[t] = t < s.nt ? a.xq + (uint64_t)(__ldcg(s.pairs + t) / a.n_slot) * a.hb : nullptr;
            pm_acts_stage_q8(acts, s.nt, rows, kd.n_units);
        } else {
            const float *rows[PM_TT];
#pragma unroll
            for (uint32_t t = 0; t < PM_TT; t++)
                rows[t] = t < s.nt ? a.mid + (uint64_t)__ldcg(s.pairs + t) * a.Fmax : nullptr;
            pm_acts_stage_f32(acts, s.nt, rows, s.kind == 0 ? a.Fr : a.Fs);
        }
        if (tid < s.nt) s_tok[tid] = __ldcg(s.pairs + tid);
        if (tid == 0) { /* the segment's fixed job fields, in shared memory (read by every warp) */
            s_jb.rb = kd.rb;
            s_jb.npair = kd.npair;
            s_jb.n_units = kd.n_units;
            s_jb.nt = s.nt;
            s_jb.act = a.act;
            s_jb.ostride = EPI == 0 ? a.Fmax : a.H;
            s_jb.acts = acts;
            s_jb.grid = grid;
            s_jb.tokpair = s_tok;
            s_jb.out = EPI == 0 ? a.mid : a.partial;
            s_jb.b0 = s.b0;
            s_jb.b1 = s.b1;
            s_jb.wts = a.w;
        }
        __syncthreads();
        const pm_rowjob &jb = s_jb;
        float *const terms = (float *)(smem + P.off_terms) + warp * (PM_TERM_V * PM_TERM_P);
        const uint32_t bytes_row = (uint32_t)kd.rb;
        if (kd.direct) { /* rows straight from global memory, no ring stage */
            while (itc.k == k) {
                const uint8_t *src[NMAT];
                uint32_t r, rows;
                pm_stage_src<NMAT>(s, kd, itc, src, r, rows);
                if (s.kind == 0)
                    pm_rows_any<QR, NMAT, EPI>(jb, terms, kd.lpr, src[0], NMAT == 2 ? src[1] : nullptr, rows, r);
                else
                    pm_rows_any<QS, NMAT, EPI>(jb, terms, kd.lpr, src[0], NMAT == 2 ? src[1] : nullptr, rows, r);
                itc.g += (uint32_t)pm_sk_warps(NMAT);
                pm_it_norm<EPI>(itc, a, tab, sl, P);
            }
            continue;
        }
        while (itc.k == k) {
            const uint32_t slot = ci % P.S;
            if (!pm_mbar_wait_sleep(bars + slot, (ci / P.S) & 1u, a.err, a.wait)) {
                fail = true;
                break;
            }
            const uint8_t *src[NMAT];
            uint32_t r, rows;
            pm_stage_src<NMAT>(s, kd, itc, src, r, rows);
            const uint8_t *stg = ring + (size_t)slot * P.stage;
            const uint8_t *w0 = pm_stage_ptr<NMAT>(stg, src, rows * bytes_row, 0);
            const uint8_t *w1 = NMAT == 2 ? pm_stage_ptr<NMAT>(stg, src, rows * bytes_row, 1) : nullptr;
            if (s.kind == 0)
                pm_rows_any<QR, NMAT, EPI>(jb, terms, kd.lpr, w0, w1, rows, r);
            else
                pm_rows_any<QS, NMAT, EPI>(jb, terms, kd.lpr, w0, w1, rows, r);
            __syncwarp();
            if (iti.k < sl.n_seg) { /* refill the slot just consumed */
                if (lane == 0) {
                    pm_fence_proxy_async();
                    issue(slot);
                }
                ni++;
                iti.g += (uint32_t)pm_sk_warps(NMAT);
                pm_it_norm<EPI>(iti, a, tab, sl, P);
                skip_direct(iti);
            }
            ci++;
            itc.g += (uint32_t)pm_sk_warps(NMAT);
            pm_it_norm<EPI>(itc, a, tab, sl, P);
        }
    }
    if (__syncthreads_or(fail) && lane == 0) /* drain this warp's copies still in flight */
        for (uint32_t d = ci; d < ni; d++) pm_mbar_wait(bars + (d % P.S), (d / P.S) & 1u, nullptr);
}

/* ============================== 4b, 5b: tensor-core expert tiles */

/* Experts with >= PM_TC_MIN tokens (prefill, large batches) run on tcgen05
 * in three kernels per pass (gate/up, then down):
 *  - expand: every tensor-core expert's weights are dequantized ONCE per
 *    layer call into fp16 hi + lo operand images (w = hi + lo to ~2^-22, the
 *    exact f32 value of the block formula), each a 128-row x 64-K tile in the
 *    128-byte-swizzled K-major layout the MMA descriptors read.  Raw rows are
 *    staged through shared memory with coalesced 4-byte loads, 256 weights of
 *    every row at a time.  The images of up to tc_slots experts live in the
 *    workspace at once; more experts run in waves of that many.
 *  - pack: the q8_K token rows of every tile (x for gate/up, q8_K(mid) for
 *    down) become fp16 hi + lo images of 64 tokens x 64 K, stored so that
 *    the consecutive tiles of one expert are adjacent: a group of up to
 *    PM_TC_G tiles is one MMA operand of N = 64 x tiles (<= 256).
 *  - gemm: a persistent warp-specialized kernel.  One thread streams the
 *    images of each (group, matrix, 128-row block, K split) unit into a
 *    two-stage shared-memory ring with 1-D bulk copies, one thread issues
 *    the MMAs (w x = wh xh + wh xl + wl xh per K-16 slice, fp32 in tensor
 *    memory), and four warps drain the accumulators (double-buffered in
 *    tensor memory, so the next unit's MMAs overlap the epilogue) into the
 *    split-K gate/up sums or the down partial rows. */

/* 8 weights of a row, values 64 c + 8 j .. + 7, in f32 (exact products of
 * the block's integers and scales, as the dot functors use them: Q8_0 cu:2174,
 * MXFP4 cu:2053 doubled e2m1 x 2^(e-128), Q2_K cu:1625, IQ2_XXS cu:1582).
 * Rows of these formats are only 2- (Q8_0, IQ2_XXS), 4- (Q2_K) or 1-byte
 * (MXFP4) aligned, so the loads are of that width.  RAW: `row` points into
 * a shared-memory copy of the row's bytes (plain loads), else to global
 * memory (read-only loads). */
template <bool RAW, class T>
__device__ __forceinline__ T pm_ldw(const T *p) {
    if constexpr (RAW) return *p;
    else return __ldg(p);
}

template <int Q, bool RAW>
__device__ __forceinline__ void pm_tc_group(const uint8_t *row, uint32_t c, uint32_t j, float *v) {
    if constexpr (Q == PM_QUANT_Q8_0) {
        const uint8_t *b = row + (size_t)(2u * c + (j >> 2)) * PM_Q8_0_BLOCK;
        const float d = pm_h2f(pm_ldw<RAW>((const uint16_t *)b));
        const uint16_t *q = (const uint16_t *)(b + 2 + 8u * (j & 3u));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t w = pm_ldw<RAW>(q + i);
            v[2 * i] = d * (float)(int8_t)(w & 0xffu);
            v[2 * i + 1] = d * (float)(int8_t)(w >> 8);
        }
    } else if constexpr (Q == PM_QUANT_MXFP4) {
        const uint8_t *b = row + (size_t)(2u * c + (j >> 2)) * PM_MXFP4_BLOCK;
        const float sc = pm_mxfp4_scale_half(pm_ldw<RAW>(b));
        const uint32_t e0 = 8u * (j & 3u); /* element of the block: low nibbles 0-15, high 16-31 */
        const uint32_t sh = e0 < 16u ? 0u : 4u;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t code = (pm_ldw<RAW>(b + 1 + ((e0 + (uint32_t)i) & 15u)) >> sh) & 15u;
            /* doubled e2m1 magnitudes {0, 1, 2, 3, 4, 6, 8, 12} as nibbles; the sign is bit 3 */
            const float mag = (float)((0xC8643210u >> (4u * (code & 7u))) & 15u);
            v[i] = __uint_as_float(__float_as_uint(mag * sc) ^ ((code & 8u) << 28));
        }
    } else if constexpr (Q == PM_QUANT_Q2_K) {
        const uint8_t *b = row + (size_t)(c >> 2) * PM_Q2_K_BYTES;
        const uint32_t i0 = 64u * (c & 3u) + 8u * j; /* element in the super-block */
        const uint32_t n = i0 >> 7, sft = 2u * ((i0 & 127u) >> 5), jj = i0 & 31u;
        const uint32_t scb = pm_ldw<RAW>(b + (i0 >> 4));
        const uint32_t dd = pm_ldw<RAW>((const uint32_t *)(b + 80));
        const float dsc = pm_h2f(dd & 0xffffu) * (float)(scb & 15u);
        const float dmn = pm_h2f(dd >> 16) * (float)(scb >> 4);
        const uint32_t *q = (const uint32_t *)(b + 16 + 32u * n + jj);
        const uint32_t q0 = pm_ldw<RAW>(q), q1 = pm_ldw<RAW>(q + 1);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t byte = ((i < 4 ? q0 : q1) >> (8 * (i & 3))) & 0xffu;
            v[i] = dsc * (float)((byte >> sft) & 3u) - dmn;
        }
    } else if constexpr (Q == PM_QUANT_IQ2_XXS) {
        const uint8_t *b = row + (size_t)(c >> 2) * PM_IQ2_XXS_BYTES;
        const uint32_t i0 = 64u * (c & 3u) + 8u * j, sb = i0 >> 5, g = (i0 & 31u) >> 3;
        const uint16_t *h = (const uint16_t *)b;
        const uint32_t aux0 = (uint32_t)pm_ldw<RAW>(h + 1 + 4 * sb) | ((uint32_t)pm_ldw<RAW>(h + 2 + 4 * sb) << 16);
        const uint32_t aux1 = (uint32_t)pm_ldw<RAW>(h + 3 + 4 * sb) | ((uint32_t)pm_ldw<RAW>(h + 4 + 4 * sb) << 16);
        const float dl = 0.125f * pm_h2f(pm_ldw<RAW>(h)) * (float)(2u * (aux1 >> 28) + 1u);
        const uint32_t grid = pm_kgrid_layer[(aux0 >> (8 * g)) & 0xffu];
        const uint32_t signs = pm_ksigns_dev((aux1 >> (7 * g)) & 127u);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t dg = (grid >> (2 * i)) & 3u;
            const float m = (float)(dg == 0 ? 8u : (dg == 1 ? 25u : 43u));
            v[i] = dl * ((signs >> i) & 1u ? -m : m);
        }
    }
}

template <int Q, int HALF, bool RAW>
__device__ __forceinline__ void pm_tc_weights(const uint8_t *row, uint32_t c, uint4 *oh, uint4 *ol) {
    if constexpr (Q == PM_QUANT_Q4_K) {
        pm_tc_q4k_row<HALF, RAW>(row, c, oh, ol);
    } else {
#pragma unroll
        for (uint32_t j = 0; j < 8; j++) {
            if ((HALF == 1 && j >= 4) || (HALF == 2 && j < 4)) continue;
            float v[8];
            pm_tc_group<Q, RAW>(row, c, j, v);
            uint32_t *hh = (uint32_t *)&oh[j], *ll = (uint32_t *)&ol[j];
#pragma unroll
            for (int i = 0; i < 4; i++) pm_split2(v[2 * i], v[2 * i + 1], hh[i], ll[i]);
        }
    }
}

/* Expand: block (slot, (matrix, 128-row block, 256-weight span)); thread r
 * owns row 128 rt + r.  The span's raw bytes of all 128 rows are copied to
 * shared memory (a warp per row at a time, 4-byte words from the word
 * boundary below the span), then each thread writes the hi + lo images of
 * the span's (up to) four 64-wide chunks of its row.  Rows past the end are
 * written as zeros. */
template <int Q, int NM>
__device__ __forceinline__ void pm_tc_expand_span(const pm_layer_args &a, uint8_t *sraw, const uint8_t *mat,
                                                  uint64_t rb, const pm_tcgeo &g, uint32_t K, uint32_t m,
                                                  uint32_t rt, uint32_t sp, uint8_t *img, uint8_t *lo) {
    constexpr uint32_t SB = pm_tc_sb_bytes(Q), XP = pm_tc_xpitch(Q);
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint64_t sb0 = (uint64_t)sp * SB;
    const uint32_t bytes = rb - sb0 < SB ? (uint32_t)(rb - sb0) : SB;
    /* word i of the flattened (row, word) copy: batches of 8 loads in flight per thread */
    constexpr uint32_t NW = XP / 4u, NI = NW; /* 128 threads x NW iterations = 128 rows x NW words */
    (void)lane;
    (void)warp;
#pragma unroll 1
    for (uint32_t i0 = 0; i0 < NI; i0 += 8u) {
        uint32_t v[8];
        bool ok[8];
#pragma unroll
        for (uint32_t k = 0; k < 8; k++) {
            const uint32_t idx = tid + 128u * (i0 + k), r = idx / NW, w = idx % NW, grow = rt * 128u + r;
            const uintptr_t src = (uintptr_t)(mat + (uint64_t)grow * rb + sb0);
            const uintptr_t a0 = src & ~(uintptr_t)3;
            ok[k] = i0 + k < NI && grow < g.rows && 4u * w < (uint32_t)(src + bytes - a0);
            v[k] = ok[k] ? __ldg((const uint32_t *)(a0 + 4u * w)) : 0u;
        }
#pragma unroll
        for (uint32_t k = 0; k < 8; k++) {
            const uint32_t idx = tid + 128u * (i0 + k);
            if (ok[k]) *(uint32_t *)(sraw + (idx / NW) * XP + 4u * (idx % NW)) = v[k];
        }
    }
    __syncthreads();
    const uint32_t r = tid, grow = rt * 128u + r;
    const uint32_t c_end = 4u * sp + 4u < g.nch ? 4u * sp + 4u : g.nch;
    const uint8_t *rowp = nullptr;
    if (grow < g.rows) {
        const uint32_t mis = (uint32_t)((uintptr_t)(mat + (uint64_t)grow * rb + sb0) & 3u);
        rowp = sraw + r * XP + mis - sb0;
    }
    (void)K;
    for (uint32_t c = 4u * sp; c < c_end; c++) {
        uint4 vh[8], vl[8];
        if (rowp) {
            pm_tc_weights<Q, 0, true>(rowp, c, vh, vl);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) vh[j] = vl[j] = make_uint4(0, 0, 0, 0);
        }
        const uint32_t pi = (m * g.rt_n + rt) * g.nch + c; /* image pair */
        uint8_t *ih = img + (uint64_t)pi * 2u * PM_TC_IMG + (r >> 3) * 1024u + (r & 7u) * 128u;
        uint32_t nz = 0;
#pragma unroll
        for (uint32_t j = 0; j < 8; j++) {
            const uint32_t off = (j ^ (r & 7u)) << 4;
            *(uint4 *)(ih + off) = vh[j];
            nz |= (vl[j].x | vl[j].y | vl[j].z | vl[j].w) & 0x7fff7fffu; /* -0 parts count as 0 */
        }
        /* the lo image is written only when some lo part of the tile is nonzero */
        if (__syncthreads_or(nz != 0)) {
#pragma unroll
            for (uint32_t j = 0; j < 8; j++) *(uint4 *)(ih + PM_TC_IMG + (((j ^ (r & 7u)) << 4))) = vl[j];
            if (r == 0) lo[pi] = 1;
        } else if (r == 0) {
            lo[pi] = 0;
        }
    }
}

template <int QR, int QS, int NM>
__global__ void __launch_bounds__(128) pm_tc_expand_kernel(const __grid_constant__ pm_layer_args a, uint32_t wave) {
    __shared__ __align__(16) uint8_t sraw[128u * PM_TC_XP];
    const uint32_t o = wave * a.tc_slots + blockIdx.y;
    if (blockIdx.y >= a.tc_slots || o >= __ldcg(a.n_items + 6)) return;
    const uint32_t item = __ldcg(&a.tc_tile[__ldcg(a.tc_first + o)].x);
    const uint32_t e = __ldcg(a.item_expert + item);
    const bool routed = e < a.E;
    const uint32_t F = routed ? a.Fr : a.Fs;
    const pm_tcgeo g = pm_tc_geo(a.H, F, NM);
    const uint32_t K = NM == 2 ? a.H : F, nsp = (K + 255u) / 256u;
    const uint32_t bx = blockIdx.x;
    if (bx >= g.nm * g.rt_n * nsp) return;
    const uint32_t sp = bx % nsp, rt = (bx / nsp) % g.rt_n, m = bx / (nsp * g.rt_n);
    const uint8_t *mat;
    uint64_t rb;
    if (NM == 2) {
        mat = m == 0 ? (routed ? a.gate + (uint64_t)e * a.st_gu_r : a.sgate)
                     : (routed ? a.up + (uint64_t)e * a.st_gu_r : a.sup);
        rb = routed ? a.rb_gu_r : a.rb_gu_s;
    } else {
        mat = routed ? a.down + (uint64_t)e * a.st_dn_r : a.sdown;
        rb = routed ? a.rb_dn_r : a.rb_dn_s;
    }
    const uint64_t slot = o - wave * a.tc_slots;
    uint8_t *img = a.tcx + slot * a.tc_slot_bytes;
    uint8_t *lo = a.tclo + slot * (a.tc_slot_bytes / (2u * PM_TC_IMG));
    if (routed)
        pm_tc_expand_span<QR, NM>(a, sraw, mat, rb, g, K, m, rt, sp, img, lo);
    else
        pm_tc_expand_span<QS, NM>(a, sraw, mat, rb, g, K, m, rt, sp, img, lo);
}

/* Pack: block (64-wide K chunk, tile); thread (token tok = tid / 4, quarter
 * q = tid % 4) converts 16 q8_K values to fp16 hi + lo.  Image (chunk c,
 * part hl, tile j) sits at ((c * 2 + hl) * max_tc + j) * PM_TC_BIMG. */
template <int NM>
__global__ void __launch_bounds__(256) pm_tc_pack_kernel(const __grid_constant__ pm_layer_args a) {
    const uint32_t tile = blockIdx.y, c = blockIdx.x;
    if (tile >= __ldcg(a.n_items + 4)) return;
    const uint2 tt = __ldcg(a.tc_tile + tile);
    const uint32_t item = tt.x, t0 = tt.y, e = __ldcg(a.item_expert + item);
    const uint32_t s0 = __ldcg(a.item_start + item), cnt = __ldcg(a.item_start + item + 1) - s0;
    const uint32_t nt = cnt - t0 < PM_TC_N ? cnt - t0 : PM_TC_N;
    const uint32_t K = NM == 2 ? a.H : (e < a.E ? a.Fr : a.Fs);
    if (c * 64u >= K) return;
    const uint32_t tok = threadIdx.x >> 2, bq = threadIdx.x & 3u;
    uint4 vh[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, vl[2] = {vh[0], vh[1]};
    if (tok < nt) {
        const uint32_t p = __ldcg(a.pairs + s0 + t0 + tok);
        const pm_block_q8K *src = NM == 2 ? a.xq + (uint64_t)(p / a.n_slot) * a.hb : a.midq + (uint64_t)p * a.fb;
        pm_tc_q8_16(src, 64u * c + 16u * bq, vh, vl);
    }
    uint8_t *bh = a.tcb + ((uint64_t)(c * 2u) * a.max_tc + tile) * PM_TC_BIMG + (tok >> 3) * 1024u + (tok & 7u) * 128u;
    uint8_t *bl = bh + (uint64_t)a.max_tc * PM_TC_BIMG;
#pragma unroll
    for (uint32_t j = 0; j < 2; j++) {
        const uint32_t off = ((2u * bq + j) ^ (tok & 7u)) << 4;
        *(uint4 *)(bh + off) = vh[j];
        *(uint4 *)(bl + off) = vl[j];
    }
}

/* one gemm unit: (group of tiles, matrix, 128-row block, K split) */
struct pm_tcu {
    uint32_t tile, item, s0, t0, ng, ntile, m, rt, ks, c0, c1, rows, rt_n, nch, slot;
};

template <int NM>
__device__ __forceinline__ bool pm_tc_unit(const pm_layer_args &a, uint32_t u, uint32_t wave, uint32_t rt_max,
                                           uint32_t KS, pm_tcu &x) {
    const uint32_t per = NM * rt_max * KS;
    x.tile = u / per;
    const uint32_t rem = u % per;
    x.m = rem / (rt_max * KS);
    x.rt = (rem % (rt_max * KS)) / KS;
    x.ks = rem % KS;
    const uint2 tt = __ldcg(a.tc_tile + x.tile);
    if (tt.y % (PM_TC_G * PM_TC_N)) return false; /* not the first tile of a group */
    const uint32_t ord = __ldcg(a.tc_ord + x.tile);
    if (ord / a.tc_slots != wave) return false;
    x.slot = ord % a.tc_slots;
    x.item = tt.x;
    x.t0 = tt.y;
    const uint32_t e = __ldcg(a.item_expert + x.item);
    x.s0 = __ldcg(a.item_start + x.item);
    const uint32_t cnt = __ldcg(a.item_start + x.item + 1) - x.s0;
    x.ng = cnt - x.t0 < PM_TC_G * PM_TC_N ? cnt - x.t0 : PM_TC_G * PM_TC_N;
    x.ntile = (x.ng + PM_TC_N - 1) / PM_TC_N;
    const pm_tcgeo g = pm_tc_geo(a.H, e < a.E ? a.Fr : a.Fs, NM);
    if (x.rt >= g.rt_n) return false;
    x.rows = g.rows, x.rt_n = g.rt_n, x.nch = g.nch;
    const uint32_t cps = (g.nch + KS - 1) / KS;
    x.c0 = x.ks * cps;
    x.c1 = x.c0 + cps < g.nch ? x.c0 + cps : g.nch;
    return x.c0 < x.c1;
}

#define PM_TCG_S 2u
#define PM_TCG_BMAX (PM_TC_G * PM_TC_BIMG)               /* one token operand (hi or lo) of a group */
#define PM_TCG_STAGE (2u * PM_TC_IMG + 2u * PM_TCG_BMAX) /* A hi, A lo, B hi, B lo */
#define PM_TCG_SMEM (1024u + PM_TCG_S * PM_TCG_STAGE)
#define PM_TCG_COLS 512u /* two accumulator buffers of up to 256 columns */

template <int NM>
__global__ void __launch_bounds__(192, 1) pm_tc_gemm_kernel(const __grid_constant__ pm_layer_args a, uint32_t wave) {
    extern __shared__ uint8_t smem_raw[];
    constexpr uint32_t S = PM_TCG_S;
    __shared__ uint64_t full[S], empty[S], accf[2], acce[2], fin;
    __shared__ uint32_t tslot;
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023u) & ~(uintptr_t)1023u);
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t n_tiles = __ldcg(a.n_items + 4);
    const uint32_t KS = NM == 2 ? __ldcg(a.n_items + 5) : 1u;
    const uint32_t rt_max = ((NM == 2 ? a.Fmax : a.H) + 127u) / 128u;
    const uint32_t units = n_tiles * NM * rt_max * KS;
    if (blockIdx.x >= units) return;
    if (warp == 0) pm_tmem_alloc(&tslot, PM_TCG_COLS);
    if (tid == 0) {
        for (uint32_t i = 0; i < S; i++) {
            pm_mbar_init(&full[i], 1);
            pm_mbar_init(&empty[i], 1);
        }
        for (uint32_t i = 0; i < 2; i++) {
            pm_mbar_init(&accf[i], 1);
            pm_mbar_init(&acce[i], 4);
        }
        pm_mbar_init(&fin, 1);
        pm_fence_barrier_init();
    }
    pm_tc_fence_before();
    __syncthreads();
    pm_tc_fence_after();
    const uint32_t tmem = tslot;
    const uint64_t NP = (uint64_t)a.T * a.n_slot;
    if (warp == 0) {
        if (lane == 0) { /* producer */
            uint32_t it = 0;
            pm_tcu x;
            for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
                if (!pm_tc_unit<NM>(a, u, wave, rt_max, KS, x)) continue;
                const uint32_t pi0 = (x.m * x.rt_n + x.rt) * x.nch;
                const uint8_t *ab = a.tcx + (uint64_t)x.slot * a.tc_slot_bytes + (uint64_t)pi0 * 2u * PM_TC_IMG;
                const uint8_t *lo = a.tclo + (uint64_t)x.slot * (a.tc_slot_bytes / (2u * PM_TC_IMG)) + pi0;
                const uint32_t bb = x.ntile * PM_TC_BIMG;
                bool ok = true;
                for (uint32_t c = x.c0; c < x.c1; c++, it++) {
                    const uint32_t st = it % S;
                    if (it >= S && !pm_mbar_wait(&empty[st], ((it / S) + 1u) & 1u, a.err, a.wait)) {
                        ok = false;
                        break;
                    }
                    uint8_t *stage = sm + st * PM_TCG_STAGE;
                    const uint8_t *bsrc = a.tcb + ((uint64_t)(c * 2u) * a.max_tc + x.tile) * PM_TC_BIMG;
                    const uint32_t na = __ldcg(lo + c) ? 2u * PM_TC_IMG : PM_TC_IMG; /* A hi (+ A lo) */
                    pm_mbar_expect_tx(&full[st], na + 2u * bb);
                    pm_bulk_g2s(stage, ab + (uint64_t)c * 2u * PM_TC_IMG, na, &full[st]);
                    pm_bulk_g2s(stage + 2u * PM_TC_IMG, bsrc, bb, &full[st]);
                    pm_bulk_g2s(stage + 2u * PM_TC_IMG + PM_TCG_BMAX, bsrc + (uint64_t)a.max_tc * PM_TC_BIMG, bb,
                                &full[st]);
                }
                if (!ok) break;
            }
            /* the copies still in flight land before the CTA leaves */
            for (uint32_t d = it > S ? it - S : 0u; d < it; d++) pm_mbar_wait(&full[d % S], (d / S) & 1u, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) { /* MMA issue */
            uint32_t it = 0, nu = 0;
            pm_tcu x;
            bool ok = true;
            for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
                if (!pm_tc_unit<NM>(a, u, wave, rt_max, KS, x)) continue;
                const uint32_t b = nu & 1u;
                if (nu >= 2 && !pm_mbar_wait(&acce[b], ((nu / 2u) + 1u) & 1u, a.err, a.wait)) break;
                pm_tc_fence_after();
                const uint32_t idesc = pm_idesc_f16(128, x.ntile * PM_TC_N);
                const uint32_t d = tmem + b * 256u;
                const uint8_t *lo = a.tclo + (uint64_t)x.slot * (a.tc_slot_bytes / (2u * PM_TC_IMG)) +
                                    (x.m * x.rt_n + x.rt) * x.nch;
                for (uint32_t c = x.c0; c < x.c1; c++, it++) {
                    const uint32_t st = it % S;
                    if (!pm_mbar_wait(&full[st], (it / S) & 1u, a.err, a.wait)) {
                        ok = false;
                        break;
                    }
                    pm_tc_fence_after();
                    const bool wl = __ldcg(lo + c) != 0;
                    uint8_t *stage = sm + st * PM_TCG_STAGE;
                    const uint64_t ah = pm_desc_sw128(stage), al = pm_desc_sw128(stage + PM_TC_IMG);
                    const uint64_t bh = pm_desc_sw128(stage + 2u * PM_TC_IMG);
                    const uint64_t bl = pm_desc_sw128(stage + 2u * PM_TC_IMG + PM_TCG_BMAX);
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; kk++) {
                        /* w x = wh xh + wh xl + wl xh (+ wl xl, below fp32 rounding) */
                        pm_mma_f16(d, ah + 2 * kk, bh + 2 * kk, idesc, (c > x.c0 || kk > 0) ? 1u : 0u);
                        pm_mma_f16(d, ah + 2 * kk, bl + 2 * kk, idesc, 1u);
                        if (wl) pm_mma_f16(d, al + 2 * kk, bh + 2 * kk, idesc, 1u);
                    }
                    pm_mma_commit(&empty[st]);
                }
                if (!ok) break;
                pm_mma_commit(&accf[b]);
                nu++;
            }
            /* every MMA issued has completed before tensor memory is released */
            pm_mma_commit(&fin);
            pm_mbar_wait(&fin, 0, a.err);
        }
    } else { /* epilogue: warps 2-5 read tensor-memory lanes 32 (warp % 4) .. + 31 */
        const uint32_t lq = warp & 3u;
        uint32_t nu = 0;
        pm_tcu x;
        for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
            if (!pm_tc_unit<NM>(a, u, wave, rt_max, KS, x)) continue;
            const uint32_t b = nu & 1u;
            if (!pm_mbar_wait(&accf[b], (nu / 2u) & 1u, a.err, a.wait)) break;
            pm_tc_fence_after();
            const uint32_t row = x.rt * 128u + lq * 32u + lane;
            for (uint32_t h = 0; h < x.ntile * (PM_TC_N / 16u); h++) {
                float v[16];
                pm_tmem_ld16(tmem + ((lq * 32u) << 16) + b * 256u + h * 16u, v);
                if (row < x.rows) {
#pragma unroll
                    for (uint32_t i = 0; i < 16; i++) {
                        const uint32_t t = h * 16u + i;
                        if (t < x.ng) {
                            const uint32_t p = __ldcg(a.pairs + x.s0 + x.t0 + t);
                            if (NM == 2)
                                a.tcp[((x.ks * NP + p) * 2u + x.m) * a.Fmax + row] = v[i];
                            else
                                a.partial[(uint64_t)p * a.H + row] = v[i];
                        }
                    }
                }
            }
            pm_tc_fence_before();
            __syncwarp();
            if (lane == 0) pm_mbar_arrive(&acce[b]);
            nu++;
        }
    }
    pm_tc_fence_before();
    __syncthreads();
    pm_tc_fence_after();
    if (warp == 0) {
        __syncwarp();
        pm_tmem_free(tmem, PM_TCG_COLS);
    }
}


/* ============================================================= host */

/* geometry of one matrix kind: 16 lanes per row when a row has at least
 * 32 unit pairs (2+ pairs per lane), else 4; a stage holds whole passes
 * of the warp (32 / lpr rows) */
/* rows per stage: whole passes of the warp (rpp rows each), ~9 KB stages
 * where one CTA holds the SM (fewer stage hand-offs per row), ~4.5 KB
 * otherwise */
static uint32_t pm_kind_rw(uint32_t nmat, uint64_t rb, uint32_t rpp) {
    const uint32_t target = pm_sk_minb((int)nmat) == 1 && pm_sk_warps((int)nmat) <= 8 ? 9216u : 4608u;
    uint64_t passes = target / (nmat * rb * rpp);
    if (passes < 1) passes = 1;
    return (uint32_t)(rpp * passes);
}

static pm_skind pm_kind_for(uint32_t nmat, uint64_t rb, uint32_t n) {
    pm_skind k;
    k.rb = rb;
    k.n_units = (n + 31u) / 32u;
    k.npair = (k.n_units + 1u) / 2u;
    /* lanes per row: the super-block slots of a row (a power of two up to
     * 16, at least 2) */
    const uint32_t nsb = (k.npair + 3u) / 4u;
    k.lpr = 2u;
    while (k.lpr * 2u <= nsb && k.lpr < 16u) k.lpr *= 2u;
    k.rw = pm_kind_rw(nmat, rb, 32u / k.lpr);
    k.direct = 0;
    return k;
}

/* shared-memory layout: IQ2 grid | segment table | token tile | per-warp
 * super-block terms | mbarriers | per-warp rings; ring depth from the
 * budget of the CTAs per SM the kernel is built for */
static pm_skp pm_skp_for(uint32_t nmat, const pm_skind &r, const pm_skind &s, bool grid) {
    pm_skp P;
    P.k[0] = r;
    P.k[1] = s;
    const uint32_t W = (uint32_t)pm_sk_warps((int)nmat);
    const uint32_t budget = pm_sk_minb(nmat) == 1 ? 200u * 1024u : 110u * 1024u;
    P.P = ((r.npair > s.npair ? r.npair : s.npair) + 3u) & ~3u; /* pair slots: whole super-blocks */
    const uint32_t nb0 = (r.n_units + 7u) / 8u, nb1 = (s.n_units + 7u) / 8u;
    P.NB = nb0 > nb1 ? nb0 : nb1;
    uint32_t off = grid ? 2048u : 0u;
    P.off_seg = off;
    off += PM_SK_MAXSEG * (uint32_t)sizeof(pm_segi);
    P.off_acts = (off + 15u) & ~15u;
    off = P.off_acts + pm_acts_bytes(P.P, P.NB);
    P.off_terms = (off + 15u) & ~15u;
    off = P.off_terms + W * PM_TERM_V * PM_TERM_P * 4u;
    P.off_bar = (off + 15u) & ~15u;
    P.off_ring = (P.off_bar + W * 8u * 8u + 127u) & ~127u;
    /* a kind whose two-deep rings do not fit next to the token tile takes a
     * whole warp per row (one row per stage); if that still does not fit,
     * it reads its rows from global memory (e.g. Q8_0 rows of 7168 values) */
    P.stage = 16u;
    for (int i = 0; i < 2; i++) {
        pm_skind &k = P.k[i];
        auto fits = [&](const pm_skind &kk) {
            const uint32_t sti = (pm_stage_bytes(nmat, kk.rb, kk.rw) + 15u) & ~15u;
            return (uint64_t)P.off_ring + (uint64_t)W * 2u * sti <= budget;
        };
        if (!fits(k) && k.lpr < 32u) {
            k.lpr = 32u;
            k.rw = pm_kind_rw(nmat, k.rb, 1u);
        }
        k.direct = fits(k) ? 0u : 1u;
        const uint32_t sti = (pm_stage_bytes(nmat, k.rb, k.rw) + 15u) & ~15u;
        if (!k.direct && sti > P.stage) P.stage = sti;
    }
    uint32_t S = budget > P.off_ring ? (budget - P.off_ring) / (W * P.stage) : 2u;
    P.S = S < 2 ? 2 : (S > 8 ? 8 : S);
    P.smem = P.off_ring + W * P.S * P.stage;
    return P;
}

/* persistent grid: resident CTAs per SM x SMs, cached per device */
template <class K>
static uint32_t pm_sk_grid(K kernel, uint32_t smem, int *occ, uint32_t *occ_smem, uint32_t threads = PM_THREADS) {
    static int sms[64];
    const int dev = pm_cur_device();
    if (dev < 0 || dev >= 64) return 0;
    if (!sms[dev] && !pm_ok(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev), "SM count"))
        return 0;
    if (occ_smem[dev] != smem || occ[dev] <= 0) {
        int n = 0;
        if (!pm_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, (int)threads, smem), "occupancy"))
            return 0;
        occ[dev] = n;
        occ_smem[dev] = smem;
    }
    return (uint32_t)(occ[dev] > 0 ? occ[dev] : 1) * (uint32_t)sms[dev];
}

static inline void pm_ev(void *const *ev, int i, cudaStream_t st) {
    if (ev && ev[i]) cudaEventRecord((cudaEvent_t)ev[i], st);
}

/* one tensor-core pass: token images, then per wave the expanded weight
 * images and the MMA units of that wave's items */
template <int QR, int QS, int NM>
static int pm_tc_launch(const pm_layer_args &a, const pm_layout &L, cudaStream_t st) {
    static uint64_t done = 0;
    static int occ[64];
    static uint32_t occ_smem[64];
    const uint32_t kmax = NM == 2 ? L.H : L.Fmax;
    pm_tc_pack_kernel<NM><<<dim3(kmax / 64u, L.max_tc), 256, 0, st>>>(a);
    if (!pm_ok(cudaGetLastError(), "moe layer tensor-core pack launch")) return 0;
    const uint32_t nx = NM == 2 ? 2u * ((L.Fmax + 127u) / 128u) * ((L.H + 255u) / 256u)
                                : ((L.H + 127u) / 128u) * ((L.Fmax + 255u) / 256u);
    auto kg = pm_tc_gemm_kernel<NM>;
    if (!pm_smem_attr(kg, PM_TCG_SMEM, &done)) return 0;
    const uint32_t g = pm_sk_grid(kg, PM_TCG_SMEM, occ, occ_smem, 192u);
    if (!g) return 0;
    for (uint32_t w = 0; w < L.tc_waves; w++) {
        pm_tc_expand_kernel<QR, QS, NM><<<dim3(nx, L.tc_slots), 128, 0, st>>>(a, w);
        if (!pm_ok(cudaGetLastError(), "moe layer tensor-core expand launch")) return 0;
        kg<<<g, 192, PM_TCG_SMEM, st>>>(a, w);
        if (!pm_ok(cudaGetLastError(), "moe layer tensor-core gemm launch")) return 0;
    }
    return 1;
}

template <int QR, int QS>
static int pm_layer_launch(pm_layer_args a, const pm_layout &L, cudaStream_t st, void *const *ev) {
    static uint64_t done_gu = 0, done_dn = 0;
    static int occ_gu[64], occ_dn[64];
    static uint32_t sm_gu[64], sm_dn[64];
    const bool grid = QR == PM_QUANT_IQ2_XXS || QS == PM_QUANT_IQ2_XXS;
    constexpr bool TC = true; /* every supported format has a tensor-core fill */
    const bool tc = TC && (a.tc_r || a.tc_s) && L.T >= PM_TC_MIN; /* an expert can reach the threshold */
    /* 4: gate/up -> tensor-core split-K sums, dp4a work units -> mid */
    if constexpr (TC)
        if (tc && !pm_tc_launch<QR, QS, 2>(a, L, st)) return 0;
    if constexpr (QR == PM_QUANT_Q2_K) /* routed Q2_K experts on the integer tensor cores */
        if (a.i8 && !pm_i8_launch<QR, 2>(a, st)) return 0;
    const pm_skind gr = pm_kind_for(2, a.rb_gu_r, a.H);
    const pm_skp pg = pm_skp_for(2, gr, a.S ? pm_kind_for(2, a.rb_gu_s, a.H) : gr, grid);
    auto kgu = pm_layer_sk_kernel<QR, QS, 2, 0>;
    if (!pm_smem_attr(kgu, pg.smem, &done_gu)) return 0;
    const uint32_t g_gu = pm_sk_grid(kgu, pg.smem, occ_gu, sm_gu, 32u * pm_sk_warps(2));
    if (!g_gu) return 0;
    kgu<<<g_gu, 32u * pm_sk_warps(2), pg.smem, st>>>(a, pg);
    if (!pm_ok(cudaGetLastError(), "moe layer gate/up launch")) return 0;
    pm_ev(ev, 4, st); /* the gate/up weight passes end here (mid of their pairs written) */
    if (tc) { /* tensor-core pairs: mid and its q8_K */
        if (!pm_launch_tc_mid(a, L, st)) return 0;
    }
    if constexpr (QR == PM_QUANT_Q2_K)
        if (a.i8 && !pm_i8_midq_launch(a, st)) return 0;
    /* 5: down -> partial rows */
    if constexpr (TC)
        if (tc && !pm_tc_launch<QR, QS, 1>(a, L, st)) return 0;
    if constexpr (QR == PM_QUANT_Q2_K)
        if (a.i8 && !pm_i8_launch<QR, 1>(a, st)) return 0;
    const pm_skind dr = pm_kind_for(1, a.rb_dn_r, a.Fr);
    const pm_skp pd = pm_skp_for(1, dr, a.S ? pm_kind_for(1, a.rb_dn_s, a.Fs) : dr, grid);
    auto kdn = pm_layer_sk_kernel<QR, QS, 1, 1>;
    if (!pm_smem_attr(kdn, pd.smem, &done_dn)) return 0;
    const uint32_t g_dn = pm_sk_grid(kdn, pd.smem, occ_dn, sm_dn, 32u * pm_sk_warps(1));
    if (!g_dn) return 0;
    kdn<<<g_dn, 32u * pm_sk_warps(1), pd.smem, st>>>(a, pd);
    if (!pm_ok(cudaGetLastError(), "moe layer down launch")) return 0;
    /* 6: combine */
    if (!pm_launch_combine(a, st)) return 0;
    pm_ev(ev, 5, st);
    return 1;
}


/* the layer's expert passes for routed format QR and shared format qs
 * (one moe_layer_<format>.cu each) */
#define PM_LAYER_FOR_QR(NAME, QR)                                                                              \
    int NAME(uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st, void *const *ev) {      \
        switch (qs) {                                                                                          \
        case PM_QUANT_Q4_K: return pm_layer_launch<QR, PM_QUANT_Q4_K>(a, L, st, ev);                           \
        case PM_QUANT_Q2_K: return pm_layer_launch<QR, PM_QUANT_Q2_K>(a, L, st, ev);                           \
        case PM_QUANT_IQ2_XXS: return pm_layer_launch<QR, PM_QUANT_IQ2_XXS>(a, L, st, ev);                     \
        case PM_QUANT_MXFP4: return pm_layer_launch<QR, PM_QUANT_MXFP4>(a, L, st, ev);                         \
        case PM_QUANT_Q8_0: return pm_layer_launch<QR, PM_QUANT_Q8_0>(a, L, st, ev);                           \
        default: return 0;                                                                                     \
        }                                                                                                      \
    }
int pm_layer_q4k(uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st, void *const *ev);
int pm_layer_q2k(uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st, void *const *ev);
int pm_layer_iq2xxs(uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st, void *const *ev);
int pm_layer_mxfp4(uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st, void *const *ev);
int pm_layer_q80(uint32_t qs, const pm_layer_args &a, const pm_layout &L, cudaStream_t st, void *const *ev);
