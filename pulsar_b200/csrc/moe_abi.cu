/* moe_abi.cu - the reference's MoE kernel entry points, re-implemented
 * for sm_100a on the streaming GEMV engine (pm_stream.cuh).
 *
 * Signatures, argument meaning and the 1/0 return convention are those of
 * crates/kernels/cuda/pulsar_kernels.cu (declared for Rust at
 * crates/kernels/src/lib.rs:116-131).  Launches go to the calling
 * thread's default stream (built with --default-stream=per-thread, as
 * crates/kernels/build.rs:42-48), so the calls stay graph-capturable.
 */
#include <cuda_runtime.h>
#include <stdint.h>

#include "pm_host.h"
#include "pm_stream.cuh"

__device__ static const uint16_t pm_kgrid_dev[256] = PM_IQ2XXS_KGRID_INIT;
__device__ uint32_t pm_err_word_abi;

uint32_t *pm_global_err_word() {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, pm_err_word_abi) != cudaSuccess) return nullptr;
    return (uint32_t *)p;
}

/* the reference's expert pointer record (cu:2555-2563, klib:21-48) */
struct pm_expert_ptrs {
    const void *gate, *up, *down;
    const float *gate_b, *up_b, *down_b;
};

/* --------------------------------------------------------- geometry */

struct pm_geom {
    uint32_t rows_cta; /* rows per CTA */
    uint32_t rc;       /* rows per pipeline chunk */
    uint32_t S;        /* ring stages */
    uint32_t stage;    /* bytes per stage */
    uint32_t smem;     /* dynamic shared memory */
};

static pm_geom pm_pick(uint32_t nmat, uint64_t rb, uint32_t nrows, uint32_t rows_cta, bool grid) {
    pm_geom g;
    g.rows_cta = rows_cta < nrows ? rows_cta : nrows;
    uint64_t rc = 16384u / (nmat * rb);
    if (rc < 1) rc = 1;
    if (rc > g.rows_cta) rc = g.rows_cta;
    while (g.rows_cta % rc) rc--;
    g.rc = (uint32_t)rc;
    g.stage = pm_stage_bytes(nmat, rb, g.rc);
    uint32_t S = 65536u / g.stage;
    g.S = S < 2 ? 2 : (S > 8 ? 8 : S);
    g.smem = pm_ring_offset(grid) + g.S * g.stage;
    return g;
}

static inline bool pm_quant_ok(uint32_t q) {
    return q == PM_QUANT_Q4_K || q == PM_QUANT_Q2_K || q == PM_QUANT_IQ2_XXS || q == PM_QUANT_MXFP4 ||
           q == PM_QUANT_Q8_0;
}

/* 32-value units of an in_dim-wide row (K-quants need whole super-blocks) */
static inline uint32_t pm_units(uint32_t quant, uint32_t in_dim) {
    if (quant == PM_QUANT_MXFP4 || quant == PM_QUANT_Q8_0) return in_dim % 32 ? 0 : in_dim / 32;
    return in_dim % 256 ? 0 : in_dim / 32;
}

/* rows per CTA so that a launch of `ctas_other` x tiles fills ~2 waves */
static uint32_t pm_rows_for(uint32_t nrows, uint64_t ctas_other, uint32_t lo, uint32_t hi) {
    const uint64_t want = 2ull * 148ull;
    uint64_t tiles = (want + ctas_other - 1) / ctas_other;
    uint64_t r = (nrows + tiles - 1) / (tiles ? tiles : 1);
    r = (r + 7) & ~7ull;
    if (r < lo) r = lo;
    if (r > hi) r = hi;
    return (uint32_t)r;
}

#define PM_SWITCH(quant, FN, ...)                                            \
    switch (quant) {                                                         \
    case PM_QUANT_Q4_K: return FN<PM_QUANT_Q4_K>(__VA_ARGS__);               \
    case PM_QUANT_Q2_K: return FN<PM_QUANT_Q2_K>(__VA_ARGS__);               \
    case PM_QUANT_IQ2_XXS: return FN<PM_QUANT_IQ2_XXS>(__VA_ARGS__);         \
    case PM_QUANT_MXFP4: return FN<PM_QUANT_MXFP4>(__VA_ARGS__);             \
    case PM_QUANT_Q8_0: return FN<PM_QUANT_Q8_0>(__VA_ARGS__);               \
    default: return 0;                                                       \
    }

/* ================================================= pair (gate/up + glu) */

struct pm_seg_pair {
    const uint8_t *g, *u;
    uint64_t rb;
    uint32_t nrows, n_units;
    const pm_block_q8K *xt;
    float *mid; /* mid row of this (token, slot), offset to the tile */
    const float *gb, *ub;
    float w;
    uint32_t act;
    __device__ uint32_t count() const { return 1; }
    __device__ const uint8_t *base(uint32_t, int m) const { return m == 0 ? g : u; }
    __device__ uint32_t ntok(uint32_t) const { return 1; }
    __device__ const pm_block_q8K *tok(uint32_t, uint32_t) const { return xt; }
    __device__ void epi(uint32_t, uint32_t row, uint32_t, const float *v) const {
        float a = v[0], b = v[1];
        if (gb) a += gb[row];
        if (ub) b += ub[row];
        mid[row] = pm_glu(a, b, act) * w;
    }
    __device__ void skip(uint32_t, uint32_t, uint32_t) const {}
};

template <int Q>
__global__ void __launch_bounds__(PM_THREADS)
    pm_pair_kernel(float *mid, const pm_expert_ptrs *ptrs, const float *weights, const pm_block_q8K *xq,
                   uint32_t in_blocks, uint32_t n_units, uint32_t mid_dim, uint32_t n_used, uint64_t rb,
                   uint32_t act_op, pm_geom geo, uint32_t *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t slot = blockIdx.y, token = blockIdx.z;
    const uint32_t row0 = blockIdx.x * geo.rows_cta;
    const uint64_t so = (uint64_t)token * n_used + slot;
    const pm_expert_ptrs p = ptrs[so];
    float *mrow = mid + so * mid_dim + row0;
    const uint32_t nrows = mid_dim - row0 < geo.rows_cta ? mid_dim - row0 : geo.rows_cta;
    if (!p.gate || !p.up) { /* not routed: the mid rows are zero (cu:2584-2588) */
        for (uint32_t j = threadIdx.x; j < nrows; j += blockDim.x) mrow[j] = 0.0f;
        return;
    }
    uint64_t *grid;
    pm_ring ring = pm_ring_setup(smem, geo.S, geo.stage, Q == PM_QUANT_IQ2_XXS, pm_kgrid_dev, &grid);
    pm_seg_pair seg;
    seg.g = (const uint8_t *)p.gate + (uint64_t)row0 * rb;
    seg.u = (const uint8_t *)p.up + (uint64_t)row0 * rb;
    seg.rb = rb;
    seg.nrows = nrows;
    seg.n_units = n_units;
    seg.xt = xq + (uint64_t)token * in_blocks;
    seg.mid = mrow;
    seg.gb = p.gate_b ? p.gate_b + row0 : nullptr;
    seg.ub = p.up_b ? p.up_b + row0 : nullptr;
    seg.w = weights[so];
    seg.act = act_op;
    pm_stream_segments<Q, 2>(seg, ring, geo.rc, grid, err);
}

template <int Q>
static int pm_pair_launch(float *mid, const pm_expert_ptrs *ptrs, const float *w, const pm_block_q8K *xq,
                          uint32_t in_dim, uint32_t mid_dim, uint32_t n_used, uint32_t n_tok, uint64_t rb,
                          uint32_t act) {
    static uint64_t done = 0;
    const uint32_t rows = pm_rows_for(mid_dim, (uint64_t)n_used * n_tok, 8, 64);
    const pm_geom geo = pm_pick(2, rb, mid_dim, rows, Q == PM_QUANT_IQ2_XXS);
    if (!pm_smem_attr(pm_pair_kernel<Q>, geo.smem, &done)) return 0;
    dim3 grid((mid_dim + geo.rows_cta - 1) / geo.rows_cta, n_used, n_tok);
    pm_pair_kernel<Q><<<grid, PM_THREADS, geo.smem>>>(mid, ptrs, w, xq, (in_dim + 255u) / 256u,
                                                      pm_units(Q, in_dim), mid_dim, n_used, rb, act, geo,
                                                      pm_global_err_word());
    return pm_ok(cudaGetLastError(), "moe pair swiglu launch");
}

/* cu:5149 pulsar_moe_pair_swiglu: mid[t][s][r] = glu(gate_r.x + gb, up_r.x + ub) * w[t][s] */
extern "C" int pulsar_moe_pair_swiglu(void *mid_dev, const void *ptrs_dev, const void *weights_dev, const void *xq_dev,
                                      uint32_t in_dim, uint32_t mid_dim, uint32_t n_used, uint32_t n_tok,
                                      uint64_t row_bytes, uint32_t quant, uint32_t act_op) {
    if (!mid_dev || !ptrs_dev || !weights_dev || !xq_dev || in_dim == 0 || mid_dim == 0 || n_used == 0 ||
        n_tok == 0 || row_bytes == 0 || !pm_quant_ok(quant) || !pm_units(quant, in_dim) ||
        row_bytes < pm_row_bytes(quant, in_dim))
        return 0;
    PM_SWITCH(quant, pm_pair_launch, (float *)mid_dev, (const pm_expert_ptrs *)ptrs_dev, (const float *)weights_dev,
              (const pm_block_q8K *)xq_dev, in_dim, mid_dim, n_used, n_tok, row_bytes, act_op)
}

/* ======================================================== down (slot sum) */

struct pm_seg_down {
    const pm_expert_ptrs *ptrs; /* this token's n_used records */
    uint32_t row0;
    uint64_t rb;
    uint32_t nrows, n_units;
    const pm_block_q8K *midq; /* this token's [n_used][mid_blocks] */
    uint32_t mid_blocks;
    uint32_t n_used;
    float *acc; /* shared [nrows] */
    __device__ uint32_t count() const { return n_used; }
    __device__ const uint8_t *base(uint32_t s, int) const {
        const void *d = ptrs[s].down;
        return d ? (const uint8_t *)d + (uint64_t)row0 * rb : nullptr;
    }
    __device__ uint32_t ntok(uint32_t) const { return 1; }
    __device__ const pm_block_q8K *tok(uint32_t s, uint32_t) const { return midq + (uint64_t)s * mid_blocks; }
    __device__ void epi(uint32_t, uint32_t row, uint32_t, const float *v) const { acc[row] += v[0]; }
    __device__ void skip(uint32_t, uint32_t, uint32_t) const {}
};

template <int Q>
__global__ void __launch_bounds__(PM_THREADS)
    pm_down_kernel(float *out, const pm_expert_ptrs *ptrs, const pm_block_q8K *midq, uint32_t mid_blocks,
                   uint32_t n_units, uint32_t out_dim, uint32_t n_used, uint64_t rb, pm_geom geo, uint32_t *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t token = blockIdx.y;
    const uint32_t row0 = blockIdx.x * geo.rows_cta;
    const uint32_t nrows = out_dim - row0 < geo.rows_cta ? out_dim - row0 : geo.rows_cta;
    uint64_t *grid;
    pm_ring ring = pm_ring_setup(smem, geo.S, geo.stage, Q == PM_QUANT_IQ2_XXS, pm_kgrid_dev, &grid);
    float *acc = (float *)(ring.buf + (size_t)geo.S * geo.stage);
    for (uint32_t j = threadIdx.x; j < nrows; j += blockDim.x) acc[j] = 0.0f;
    __syncthreads();
    pm_seg_down seg;
    seg.ptrs = ptrs + (uint64_t)token * n_used;
    seg.row0 = row0;
    seg.rb = rb;
    seg.nrows = nrows;
    seg.n_units = n_units;
    seg.midq = midq + (uint64_t)token * n_used * mid_blocks;
    seg.mid_blocks = mid_blocks;
    seg.n_used = n_used;
    seg.acc = acc;
    if (!pm_stream_segments<Q, 1>(seg, ring, geo.rc, grid, err)) return;
    for (uint32_t j = threadIdx.x; j < nrows; j += blockDim.x) out[(uint64_t)token * out_dim + row0 + j] = acc[j];
}

template <int Q>
static int pm_down_launch(float *out, const pm_expert_ptrs *ptrs, const pm_block_q8K *midq, uint32_t mid_dim,
                          uint32_t out_dim, uint32_t n_used, uint32_t n_tok, uint64_t rb) {
    static uint64_t done = 0;
    const uint32_t rows = pm_rows_for(out_dim, n_tok, 8, 64);
    pm_geom geo = pm_pick(1, rb, out_dim, rows, Q == PM_QUANT_IQ2_XXS);
    const uint32_t smem = geo.smem + geo.rows_cta * 4u;
    if (!pm_smem_attr(pm_down_kernel<Q>, smem, &done)) return 0;
    dim3 grid((out_dim + geo.rows_cta - 1) / geo.rows_cta, n_tok);
    pm_down_kernel<Q><<<grid, PM_THREADS, smem>>>(out, ptrs, midq, (mid_dim + 255u) / 256u, pm_units(Q, mid_dim),
                                                  out_dim, n_used, rb, geo, pm_global_err_word());
    return pm_ok(cudaGetLastError(), "moe down launch");
}

/* cu:5289 pulsar_moe_down: out[t][r] = sum over slots (in order) of down_r . midq[t][s] */
extern "C" int pulsar_moe_down(void *out_dev, const void *ptrs_dev, const void *midq_dev, uint32_t mid_dim,
                               uint32_t out_dim, uint32_t n_used, uint32_t n_tok, uint64_t row_bytes,
                               uint32_t quant) {
    if (!out_dev || !ptrs_dev || !midq_dev || mid_dim == 0 || out_dim == 0 || n_used == 0 || n_tok == 0 ||
        row_bytes == 0 || !pm_quant_ok(quant) || !pm_units(quant, mid_dim) ||
        row_bytes < pm_row_bytes(quant, mid_dim))
        return 0;
    PM_SWITCH(quant, pm_down_launch, (float *)out_dev, (const pm_expert_ptrs *)ptrs_dev,
              (const pm_block_q8K *)midq_dev, mid_dim, out_dim, n_used, n_tok, row_bytes)
}

/* ============================================== grouped (CSR by expert) */

/* one group: rows of its expert streamed once, every (token, slot) pair of
 * the group dotted against the staged rows (cu:2690-2790 semantics) */
struct pm_seg_gpair {
    const uint8_t *g, *u;
    uint32_t row0;
    uint64_t rb;
    uint32_t nrows, n_units;
    const uint32_t *pairs; /* token << 4 | slot */
    uint32_t n;
    const pm_block_q8K *xq;
    uint32_t in_blocks, n_used, mid_dim;
    float *mid;
    const float *weights, *gb, *ub;
    uint32_t act;
    __device__ uint32_t count() const { return 1; }
    __device__ const uint8_t *base(uint32_t, int m) const { return m == 0 ? g : u; }
    __device__ uint32_t ntok(uint32_t) const { return n; }
    __device__ const pm_block_q8K *tok(uint32_t, uint32_t ti) const {
        return xq + (uint64_t)(pairs[ti] >> 4) * in_blocks;
    }
    __device__ void epi(uint32_t, uint32_t row, uint32_t ti, const float *v) const {
        const uint32_t pr = pairs[ti], t = pr >> 4, s = pr & 15u;
        float a = v[0], b = v[1];
        if (gb) a += gb[row0 + row];
        if (ub) b += ub[row0 + row];
        const uint64_t so = (uint64_t)t * n_used + s;
        mid[so * mid_dim + row0 + row] = pm_glu(a, b, act) * weights[so];
    }
    __device__ void skip(uint32_t, uint32_t, uint32_t) const {}
};

template <int Q>
__global__ void __launch_bounds__(PM_THREADS)
    pm_gpair_kernel(float *mid, const pm_expert_ptrs *gptrs, const uint32_t *starts, const uint32_t *pairs,
                    const float *weights, const pm_block_q8K *xq, uint32_t in_blocks, uint32_t n_units,
                    uint32_t mid_dim, uint32_t n_used, uint64_t rb, uint32_t act, pm_geom geo, uint32_t *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t group = blockIdx.y, row0 = blockIdx.x * geo.rows_cta;
    const pm_expert_ptrs p = gptrs[group];
    if (!p.gate || !p.up) return;
    const uint32_t s0 = starts[group], s1 = starts[group + 1];
    if (s1 <= s0) return;
    uint64_t *grid;
    pm_ring ring = pm_ring_setup(smem, geo.S, geo.stage, Q == PM_QUANT_IQ2_XXS, pm_kgrid_dev, &grid);
    pm_seg_gpair seg;
    seg.g = (const uint8_t *)p.gate + (uint64_t)row0 * rb;
    seg.u = (const uint8_t *)p.up + (uint64_t)row0 * rb;
    seg.row0 = row0;
    seg.rb = rb;
    seg.nrows = mid_dim - row0 < geo.rows_cta ? mid_dim - row0 : geo.rows_cta;
    seg.n_units = n_units;
    seg.pairs = pairs + s0;
    seg.n = s1 - s0;
    seg.xq = xq;
    seg.in_blocks = in_blocks;
    seg.n_used = n_used;
    seg.mid_dim = mid_dim;
    seg.mid = mid;
    seg.weights = weights;
    seg.gb = p.gate_b;
    seg.ub = p.up_b;
    seg.act = act;
    pm_stream_segments<Q, 2>(seg, ring, geo.rc, grid, err);
}

template <int Q>
static int pm_gpair_launch(float *mid, const pm_expert_ptrs *gptrs, const uint32_t *starts, const uint32_t *pairs,
                           const float *w, const pm_block_q8K *xq, uint32_t in_dim, uint32_t mid_dim,
                           uint32_t n_used, uint32_t n_group, uint64_t rb, uint32_t act) {
    static uint64_t done = 0;
    const uint32_t rows = pm_rows_for(mid_dim, n_group, 8, 64);
    const pm_geom geo = pm_pick(2, rb, mid_dim, rows, Q == PM_QUANT_IQ2_XXS);
    if (!pm_smem_attr(pm_gpair_kernel<Q>, geo.smem, &done)) return 0;
    dim3 grid((mid_dim + geo.rows_cta - 1) / geo.rows_cta, n_group);
    pm_gpair_kernel<Q><<<grid, PM_THREADS, geo.smem>>>(mid, gptrs, starts, pairs, w, xq, (in_dim + 255u) / 256u,
                                                       pm_units(Q, in_dim), mid_dim, n_used, rb, act, geo,
                                                       pm_global_err_word());
    return pm_ok(cudaGetLastError(), "moe pair grouped launch");
}

/* cu:3483 pulsar_moe_pair_swiglu_grouped */
extern "C" int pulsar_moe_pair_swiglu_grouped(void *mid_dev, const void *gptrs_dev, const void *starts_dev,
                                              const void *pairs_dev, const void *weights_dev, const void *xq_dev,
                                              uint32_t in_dim, uint32_t mid_dim, uint32_t n_used, uint32_t n_group,
                                              uint64_t row_bytes, uint32_t quant, uint32_t act_op) {
    if (!mid_dev || !gptrs_dev || !starts_dev || !pairs_dev || !weights_dev || !xq_dev || in_dim == 0 ||
        mid_dim == 0 || n_used == 0 || n_used > 16 || n_group == 0 || row_bytes == 0 || !pm_quant_ok(quant) ||
        !pm_units(quant, in_dim) || row_bytes < pm_row_bytes(quant, in_dim))
        return 0;
    PM_SWITCH(quant, pm_gpair_launch, (float *)mid_dev, (const pm_expert_ptrs *)gptrs_dev,
              (const uint32_t *)starts_dev, (const uint32_t *)pairs_dev, (const float *)weights_dev,
              (const pm_block_q8K *)xq_dev, in_dim, mid_dim, n_used, n_group, row_bytes, act_op)
}

struct pm_seg_gdown {
    const uint8_t *d;
    uint32_t row0;
    uint64_t rb;
    uint32_t nrows, n_units;
    const uint32_t *pairs;
    uint32_t n;
    const pm_block_q8K *midq;
    uint32_t mid_blocks, n_used, out_dim;
    float *partial;
    __device__ uint32_t count() const { return 1; }
    __device__ const uint8_t *base(uint32_t, int) const { return d; }
    __device__ uint32_t ntok(uint32_t) const { return n; }
    __device__ const pm_block_q8K *tok(uint32_t, uint32_t ti) const {
        const uint32_t pr = pairs[ti];
        return midq + ((uint64_t)(pr >> 4) * n_used + (pr & 15u)) * mid_blocks;
    }
    __device__ void epi(uint32_t, uint32_t row, uint32_t ti, const float *v) const {
        const uint32_t pr = pairs[ti];
        partial[((uint64_t)(pr >> 4) * n_used + (pr & 15u)) * out_dim + row0 + row] = v[0];
    }
    __device__ void skip(uint32_t, uint32_t, uint32_t) const {}
};

template <int Q>
__global__ void __launch_bounds__(PM_THREADS)
    pm_gdown_kernel(float *partial, const pm_expert_ptrs *gptrs, const uint32_t *starts, const uint32_t *pairs,
                    const pm_block_q8K *midq, uint32_t mid_blocks, uint32_t n_units, uint32_t out_dim,
                    uint32_t n_used, uint64_t rb, pm_geom geo, uint32_t *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t group = blockIdx.y, row0 = blockIdx.x * geo.rows_cta;
    const pm_expert_ptrs p = gptrs[group];
    if (!p.down) return;
    const uint32_t s0 = starts[group], s1 = starts[group + 1];
    if (s1 <= s0) return;
    uint64_t *grid;
    pm_ring ring = pm_ring_setup(smem, geo.S, geo.stage, Q == PM_QUANT_IQ2_XXS, pm_kgrid_dev, &grid);
    pm_seg_gdown seg;
    seg.d = (const uint8_t *)p.down + (uint64_t)row0 * rb;
    seg.row0 = row0;
    seg.rb = rb;
    seg.nrows = out_dim - row0 < geo.rows_cta ? out_dim - row0 : geo.rows_cta;
    seg.n_units = n_units;
    seg.pairs = pairs + s0;
    seg.n = s1 - s0;
    seg.midq = midq;
    seg.mid_blocks = mid_blocks;
    seg.n_used = n_used;
    seg.out_dim = out_dim;
    seg.partial = partial;
    pm_stream_segments<Q, 1>(seg, ring, geo.rc, grid, err);
}

template <int Q>
static int pm_gdown_launch(float *partial, const pm_expert_ptrs *gptrs, const uint32_t *starts,
                           const uint32_t *pairs, const pm_block_q8K *midq, uint32_t mid_dim, uint32_t out_dim,
                           uint32_t n_used, uint32_t n_group, uint64_t rb) {
    static uint64_t done = 0;
    const uint32_t rows = pm_rows_for(out_dim, n_group, 8, 64);
    const pm_geom geo = pm_pick(1, rb, out_dim, rows, Q == PM_QUANT_IQ2_XXS);
    if (!pm_smem_attr(pm_gdown_kernel<Q>, geo.smem, &done)) return 0;
    dim3 grid((out_dim + geo.rows_cta - 1) / geo.rows_cta, n_group);
    pm_gdown_kernel<Q><<<grid, PM_THREADS, geo.smem>>>(partial, gptrs, starts, pairs, midq, (mid_dim + 255u) / 256u,
                                                       pm_units(Q, mid_dim), out_dim, n_used, rb, geo,
                                                       pm_global_err_word());
    return pm_ok(cudaGetLastError(), "moe down grouped launch");
}

/* cu:3537 pulsar_moe_down_grouped: partial[t][s][r] for the group's pairs */
extern "C" int pulsar_moe_down_grouped(void *partial_dev, const void *gptrs_dev, const void *starts_dev,
                                       const void *pairs_dev, const void *midq_dev, uint32_t mid_dim,
                                       uint32_t out_dim, uint32_t n_used, uint32_t n_group, uint64_t row_bytes,
                                       uint32_t quant) {
    if (!partial_dev || !gptrs_dev || !starts_dev || !pairs_dev || !midq_dev || mid_dim == 0 || out_dim == 0 ||
        n_used == 0 || n_used > 16 || n_group == 0 || row_bytes == 0 || !pm_quant_ok(quant) ||
        !pm_units(quant, mid_dim) || row_bytes < pm_row_bytes(quant, mid_dim))
        return 0;
    PM_SWITCH(quant, pm_gdown_launch, (float *)partial_dev, (const pm_expert_ptrs *)gptrs_dev,
              (const uint32_t *)starts_dev, (const uint32_t *)pairs_dev, (const pm_block_q8K *)midq_dev, mid_dim,
              out_dim, n_used, n_group, row_bytes)
}

/* ==================================================== elementwise ops */

__global__ void pm_slot_sum_kernel(float *out, const float *partial, uint32_t out_dim, uint32_t n_used,
                                   uint32_t n_tok) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (uint64_t)n_tok * out_dim) return;
    const uint64_t t = gid / out_dim, r = gid % out_dim;
    float acc = 0.0f;
    for (uint32_t s = 0; s < n_used; s++) acc += partial[(t * n_used + s) * out_dim + r];
    out[gid] = acc;
}

/* cu:3651 pulsar_moe_slot_sum: out[t][r] = sum_s partial[t][s][r], slot order */
extern "C" int pulsar_moe_slot_sum(void *out_dev, const void *partial_dev, uint32_t out_dim, uint32_t n_used,
                                   uint32_t n_tok) {
    if (!out_dev || !partial_dev || out_dim == 0 || n_used == 0 || n_tok == 0) return 0;
    const uint64_t total = (uint64_t)n_tok * out_dim;
    pm_slot_sum_kernel<<<(uint32_t)((total + 255) / 256), 256>>>((float *)out_dev, (const float *)partial_dev,
                                                                  out_dim, n_used, n_tok);
    return pm_ok(cudaGetLastError(), "moe slot sum launch");
}

__global__ void pm_down_bias_kernel(float *out, const pm_expert_ptrs *ptrs, const float *weights, uint32_t out_dim,
                                    uint32_t n_used, uint32_t n_tok) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (uint64_t)n_tok * out_dim) return;
    const uint64_t t = gid / out_dim, r = gid % out_dim;
    float b = 0.0f;
    for (uint32_t s = 0; s < n_used; s++) {
        const pm_expert_ptrs p = ptrs[t * n_used + s];
        if (p.down_b) b += weights[t * n_used + s] * p.down_b[r];
    }
    if (b != 0.0f) out[gid] += b;
}

/* cu:3640 pulsar_moe_down_bias: out[t][r] += sum_s w_s * down_b_s[r] */
extern "C" int pulsar_moe_down_bias(void *out_dev, const void *ptrs_dev, const void *weights_dev, uint32_t out_dim,
                                    uint32_t n_used, uint32_t n_tok) {
    if (!out_dev || !ptrs_dev || !weights_dev || out_dim == 0 || n_used == 0 || n_tok == 0) return 0;
    const uint64_t total = (uint64_t)n_tok * out_dim;
    pm_down_bias_kernel<<<(uint32_t)((total + 255) / 256), 256>>>(
        (float *)out_dev, (const pm_expert_ptrs *)ptrs_dev, (const float *)weights_dev, out_dim, n_used, n_tok);
    return pm_ok(cudaGetLastError(), "moe down bias launch");
}

__global__ void pm_add_bias_rows_kernel(float *x, const float *bias, uint32_t dim, uint32_t rows) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (uint64_t)rows * dim) return;
    x[gid] += bias[gid % dim];
}

/* cu:3631 pulsar_add_bias_rows: x[r][i] += bias[i] */
extern "C" int pulsar_add_bias_rows(void *x_dev, const void *bias_dev, uint32_t dim, uint32_t rows) {
    if (!x_dev || !bias_dev || dim == 0 || rows == 0) return 0;
    const uint64_t total = (uint64_t)rows * dim;
    pm_add_bias_rows_kernel<<<(uint32_t)((total + 255) / 256), 256>>>((float *)x_dev, (const float *)bias_dev, dim,
                                                                       rows);
    return pm_ok(cudaGetLastError(), "add bias rows launch");
}

__global__ void pm_swiglu_kernel(float *out, const float *gate, const float *up, uint32_t n, float clamp,
                                 float weight, uint32_t act) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float g = gate[i], u = up[i];
    if (clamp > 1.0e-6f) {
        g = fminf(g, clamp);
        u = fminf(fmaxf(u, -clamp), clamp);
    }
    out[i] = pm_glu(g, u, act) * weight;
}

/* cu:6551 pulsar_swiglu */
extern "C" int pulsar_swiglu(void *out_dev, const void *gate_dev, const void *up_dev, uint32_t n, float clamp,
                             float weight, uint32_t act_op) {
    if (!out_dev || !gate_dev || !up_dev || n == 0) return 0;
    pm_swiglu_kernel<<<(n + 255) / 256, 256>>>((float *)out_dev, (const float *)gate_dev, (const float *)up_dev, n,
                                               clamp, weight, act_op);
    return pm_ok(cudaGetLastError(), "swiglu launch");
}

__global__ void pm_add_kernel(float *out, const float *a, const float *b, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] + b[i];
}

/* cu:6754 pulsar_add */
extern "C" int pulsar_add(void *out_dev, const void *a_dev, const void *b_dev, uint32_t n) {
    if (!out_dev || !a_dev || !b_dev || n == 0) return 0;
    pm_add_kernel<<<(n + 255) / 256, 256>>>((float *)out_dev, (const float *)a_dev, (const float *)b_dev, n);
    return pm_ok(cudaGetLastError(), "add launch");
}

/* kernel timeout / bad-argument word of the reference-ABI kernels: reads
 * it back (synchronously) and clears it; 0 = no error recorded */
extern "C" uint32_t pulsar_b200_abi_error(void) {
    uint32_t v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, pm_err_word_abi, 4) != cudaSuccess) return 0xffffffffu;
    cudaMemcpyToSymbol(pm_err_word_abi, &z, 4);
    return v;
}

/* ============================================================ rms norm */

/* out[r][i] = x[r][i] / sqrt(mean_i x[r][i]^2 + eps) * w[i] (w NULL = 1):
 * the normalisation the engine applies to a layer's FFN input
 * (cu:6469-6502 semantics).  One CTA per row, warp-shuffle reduction. */
__global__ void pm_rms_norm_kernel(float *out, const float *x, const float *w, uint32_t n, float eps) {
    __shared__ float part[32];
    const float *xr = x + (uint64_t)blockIdx.x * n;
    float *orow = out + (uint64_t)blockIdx.x * n;
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) s += xr[i] * xr[i];
    s = pm_warp_sum(s);
    if ((threadIdx.x & 31u) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
        v = pm_warp_sum(v);
        if (threadIdx.x == 0) part[0] = rsqrtf(v / (float)n + eps);
    }
    __syncthreads();
    const float scale = part[0];
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) orow[i] = xr[i] * scale * (w ? w[i] : 1.0f);
}

/* replaces cu:6494 pulsar_rms_norm (klib:88) */
extern "C" int pulsar_rms_norm(void *out_dev, const void *x_dev, const void *w_dev, uint32_t n, uint32_t rows,
                               float eps) {
    if (!out_dev || !x_dev || n == 0 || rows == 0) return 0;
    pm_rms_norm_kernel<<<rows, 256>>>((float *)out_dev, (const float *)x_dev, (const float *)w_dev, n, eps);
    return pm_ok(cudaGetLastError(), "rms norm launch");
}

/* the same on an explicit stream (cudaStream_t, NULL = per-thread default) */
extern "C" int pulsar_rms_norm_stream(void *out_dev, const void *x_dev, const void *w_dev, uint32_t n, uint32_t rows,
                                      float eps, void *stream) {
    if (!out_dev || !x_dev || n == 0 || rows == 0) return 0;
    cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamPerThread;
    pm_rms_norm_kernel<<<rows, 256, 0, st>>>((float *)out_dev, (const float *)x_dev, (const float *)w_dev, n, eps);
    return pm_ok(cudaGetLastError(), "rms norm launch");
}
