/* pm_stream.cuh - the CTA-level weight-row streaming GEMV engine.
 *
 * A CTA walks a list of SEGMENTS.  A segment is one row range [row0,
 * row0 + nrows) of up to NMAT weight matrices with identical geometry
 * (gate and up of one expert, or one down slab) plus the set of tokens
 * whose q8_K activations multiply those rows.  Rows of a segment are
 * contiguous bytes in HBM, so each pipeline chunk (rc rows of every
 * matrix) is one 1-D TMA bulk copy per matrix into an S-stage shared
 * memory ring.  All warps consume: each (row, token) pair of a chunk is a
 * warp-cooperative dot over 32-value units (all 32 lanes busy), and the
 * segment's epilogue receives the NMAT finished dots from lane 0.
 *
 * Ordering: chunks are consumed strictly in order with a CTA barrier
 * between them, and within a chunk each (row, token) pair belongs to one
 * warp, so any accumulation an epilogue does across segments happens in
 * segment order - results are deterministic run to run.
 */
#pragma once
#include "pm_device.cuh"

#define PM_THREADS 256
#define PM_WARPS 8

struct pm_ring {
    uint8_t *buf;       /* S * stage_bytes, 16-byte aligned */
    uint64_t *full;     /* S mbarriers */
    uint32_t stage_bytes;
    uint32_t S;
};

/* bytes the ring needs for one chunk of `rows` rows of NMAT matrices */
__host__ __device__ __forceinline__ uint32_t pm_stage_bytes(uint32_t nmat, uint64_t rb, uint32_t rows) {
    /* each piece: rounded to 16 at both ends, plus a 16-byte tail guard */
    return (uint32_t)(nmat * (((rb * rows + 15u) & ~15ull) + 32u));
}

/* Segment provider interface (duck-typed):
 *   uint32_t count()                         number of segments
 *   const uint8_t* base(seg, m)              row 0 of matrix m (nullptr = skip)
 *   uint32_t ntok(seg)                       tokens of the segment
 *   const pm_block_q8K* tok(seg, ti)         token ti's q8_K row
 *   void epi(seg, row, ti, const float* v)   lane 0 only, v[NMAT]
 * plus the shared geometry rb (row bytes), nrows, n_units (32-value units). */

template <int NMAT>
__device__ __forceinline__ void pm_issue_chunk(const pm_ring &ring, uint32_t c, const uint8_t *const *src,
                                               uint32_t bytes) {
    uint8_t *dst = ring.buf + (size_t)(c % ring.S) * ring.stage_bytes;
    uint64_t *bar = ring.full + (c % ring.S);
    uint32_t total = 0;
    uint32_t len[NMAT];
    const uint8_t *a0[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        if (!src[m]) {
            len[m] = 0;
            a0[m] = nullptr;
            continue;
        }
        const uintptr_t s = (uintptr_t)src[m];
        const uintptr_t lo = s & ~(uintptr_t)15;
        const uintptr_t hi = (s + bytes + 15u) & ~(uintptr_t)15;
        a0[m] = (const uint8_t *)lo;
        len[m] = (uint32_t)(hi - lo);
        total += len[m];
    }
    pm_mbar_expect_tx(bar, total);
    uint32_t off = 0;
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        if (len[m]) pm_bulk_g2s(dst + off, a0[m], len[m], bar);
        off += len[m] + 16u;
    }
}

/* shared-memory address of the first byte of matrix m's rows in stage c */
template <int NMAT>
__device__ __forceinline__ const uint8_t *pm_chunk_ptr(const pm_ring &ring, uint32_t c, const uint8_t *const *src,
                                                       uint32_t bytes, int m) {
    const uint8_t *p = ring.buf + (size_t)(c % ring.S) * ring.stage_bytes;
    uint32_t off = 0;
#pragma unroll
    for (int i = 0; i < NMAT; i++) {
        if (i == m) break;
        if (src[i]) {
            const uintptr_t s = (uintptr_t)src[i];
            off += (uint32_t)(((s + bytes + 15u) & ~(uintptr_t)15) - (s & ~(uintptr_t)15)) + 16u;
        } else {
            off += 16u;
        }
    }
    return p + off + ((uintptr_t)src[m] & 15u);
}

/* Run all segments.  rc = rows per chunk.  Returns false on a wait
 * timeout (error word set; copies in flight drained with bounded waits). */
template <int Q, int NMAT, class Seg>
__device__ bool pm_stream_segments(Seg &seg, const pm_ring &ring, uint32_t rc, const uint64_t *grid,
                                   uint32_t *err) {
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t nrows = seg.nrows, rb = (uint32_t)seg.rb;
    const uint32_t cps = (nrows + rc - 1) / rc; /* chunks per segment */
    const uint32_t nseg = seg.count();
    const uint32_t nchunk = nseg * cps;
    const uint32_t n_units = seg.n_units;

    /* chunk c -> (segment, first row, rows, sources) */
    auto geom = [&](uint32_t c, const uint8_t **src, uint32_t &r0, uint32_t &rows, uint32_t &sg) {
        sg = c / cps;
        r0 = (c % cps) * rc;
        rows = nrows - r0 < rc ? nrows - r0 : rc;
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            const uint8_t *b = seg.base(sg, m);
            src[m] = b ? b + (size_t)r0 * rb : nullptr;
        }
    };

    if (tid == 0) {
        const uint32_t pro = nchunk < ring.S - 1 ? nchunk : ring.S - 1;
        for (uint32_t c = 0; c < pro; c++) {
            const uint8_t *src[NMAT];
            uint32_t r0, rows, sg;
            geom(c, src, r0, rows, sg);
            pm_issue_chunk<NMAT>(ring, c, src, rows * rb);
        }
    }
    for (uint32_t c = 0; c < nchunk; c++) {
        if (tid == 0 && c + ring.S - 1 < nchunk) {
            const uint8_t *src[NMAT];
            uint32_t r0, rows, sg;
            geom(c + ring.S - 1, src, r0, rows, sg);
            pm_issue_chunk<NMAT>(ring, c + ring.S - 1, src, rows * rb);
        }
        const bool ok = pm_mbar_wait(ring.full + (c % ring.S), (c / ring.S) & 1u, err);
        if (__syncthreads_or(!ok)) {
            /* drain: wait (bounded) for every chunk issued after c */
            if (tid == 0) {
                const uint32_t last = c + ring.S - 1 < nchunk ? c + ring.S - 1 : nchunk - 1;
                for (uint32_t d = c; d <= last; d++) pm_mbar_wait(ring.full + (d % ring.S), (d / ring.S) & 1u, nullptr);
            }
            __syncthreads();
            return false;
        }
        const uint8_t *src[NMAT];
        uint32_t r0, rows, sg;
        geom(c, src, r0, rows, sg);
        const uint8_t *rowp[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; m++) rowp[m] = src[m] ? pm_chunk_ptr<NMAT>(ring, c, src, rows * rb, m) : nullptr;
        const uint32_t nt = seg.ntok(sg);
        const bool live = NMAT == 1 ? rowp[0] != nullptr : (rowp[0] != nullptr && rowp[NMAT - 1] != nullptr);
        if (live) {
            const uint32_t work = rows * nt;
            for (uint32_t w = warp; w < work; w += PM_WARPS) {
                const uint32_t ti = w / rows, j = w % rows;
                const pm_block_q8K *xt = seg.tok(sg, ti);
                float acc[NMAT];
#pragma unroll
                for (int m = 0; m < NMAT; m++) acc[m] = 0.0f;
                for (uint32_t u = lane; u < n_units; u += 32u) {
                    pm_q8_unit xu;
                    pm_load_q8_unit(xt + (u >> 3), (int)(u & 7u), xu);
#pragma unroll
                    for (int m = 0; m < NMAT; m++) acc[m] += pm_unit<Q>(rowp[m] + (size_t)j * rb, u, xu, grid);
                }
#pragma unroll
                for (int m = 0; m < NMAT; m++) acc[m] = pm_warp_sum(acc[m]);
                if (lane == 0) seg.epi(sg, r0 + j, ti, acc);
            }
        } else if (tid == 0) {
            seg.skip(sg, r0, rows);
        }
        __syncthreads();
    }
    return true;
}

/* ring + grid table setup in dynamic shared memory; call from all threads.
 * Layout: [S mbarriers][iq2 grid 2 KB if needed][stages...][extra] */
__device__ __forceinline__ pm_ring pm_ring_setup(uint8_t *smem, uint32_t S, uint32_t stage_bytes, bool need_grid,
                                                 const uint16_t *kgrid, uint64_t **grid_out) {
    pm_ring r;
    r.full = (uint64_t *)smem;
    uint32_t off = 128; /* room for up to 16 barriers */
    uint64_t *grid = (uint64_t *)(smem + off);
    if (need_grid) {
        for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) {
            const uint32_t k = kgrid[i];
            uint64_t v = 0;
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const uint32_t d = (k >> (2 * q)) & 3u;
                v |= (uint64_t)(d == 0 ? 8u : (d == 1 ? 25u : 43u)) << (8 * q);
            }
            grid[i] = v;
        }
        off += 2048;
    }
    *grid_out = grid;
    r.buf = smem + off;
    r.stage_bytes = stage_bytes;
    r.S = S;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < S; i++) pm_mbar_init(r.full + i, 1);
        pm_fence_barrier_init();
    }
    __syncthreads();
    return r;
}

/* invalidate the ring's barriers so the shared memory can be reused (or
 * the ring set up again); call from all threads after the last chunk */
__device__ __forceinline__ void pm_ring_teardown(const pm_ring &r) {
    __syncthreads();
    if (threadIdx.x == 0)
        for (uint32_t i = 0; i < r.S; i++)
            asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(pm_smem_addr(r.full + i)) : "memory");
    __syncthreads();
}

__host__ __device__ __forceinline__ uint32_t pm_ring_offset(bool need_grid) { return 128u + (need_grid ? 2048u : 0u); }
