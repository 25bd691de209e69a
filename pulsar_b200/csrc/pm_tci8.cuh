/* pm_tci8.cuh - Q2_K expert passes on the tcgen05 integer tensor cores
 * (kind::i8, s32 accumulators in tensor memory), exact in the CPU lane's
 * arithmetic.
 *
 * Why.  A Q2_K weight is d sc q - dmin m with q in 0..3 and 4-bit sc, m
 * per 16 values (crates/quant/src/cpu_dot.rs:732-767).  q sc is at most 45,
 * so the whole super-block's integer sum  isum = sum q sc x  (x the q8_K
 * activations) is an int8 x int8 dot: one MMA chain over K = 256 per
 * super-block, exact in s32.  The CPU lane's f32 arithmetic then happens
 * once per (row, token, super-block):
 *     total += yd xd isum - yd xmin msum,   msum = sum_j m_j bsum_j
 * in super-block order - here in the epilogue, per tensor-memory lane (one
 * weight row) and token, in the same order, so the result is the CPU
 * lane's bit for bit.  The decode per weight (shift, mask, times sc) is
 * the only per-weight work; the tokens of a tile cost the tensor cores and
 * a few f32 operations per super-block, where the dp4a path spends ~27
 * instructions per 64 weights per token.
 *
 * Work.  A tile is up to 32 tokens of one routed expert (the selection
 * kernel lists them); a task is (tile, 128-row block of the pass's
 * matrices).  Persistent CTAs take tasks round-robin and stream their
 * super-blocks through four pipelines:
 *   raw     every decode thread copies exactly the bytes it later reads
 *           (its row's 84 bytes of a matrix per super-block, a quarter of a
 *           token's q8 values, the token's scale and bsums) in 16-byte
 *           asynchronous copies (rounded out) into a 2-deep ring, one copy
 *           group per super-block, waited on by the thread itself: no
 *           cross-thread hand-off on the weight stream (the bulk-copy engine
 *           would serialize hundreds of 100-byte requests per super-block,
 *           and a CTA-wide barrier per super-block cost ~1 us);
 *   decode  8 warps turn raw rows into int8 A tiles (q sc, 128 rows x 128 K,
 *           128-byte swizzle), stage the tokens' q8 values as the B tile
 *           and the per-(row, super-block) scales / per-(token,
 *           super-block) bsums for the epilogue;
 *   mma     one thread issues 4 MMAs (K = 32) per matrix per 128-wide K
 *           chunk into a per-super-block tensor-memory slot (4 slots);
 *   epilog  4 warps read the slot (32 lanes each), form the f32 terms and
 *           add them in super-block order; at the task's last super-block
 *           they write mid = glu(g + gb, u + ub) w (gate/up) or the partial
 *           row (down).
 * Every wait is bounded; on a timeout the kernel records it in the layer's
 * error word, lets the copies and MMAs in flight land and returns.
 */
#pragma once
#include "pm_tc.cuh"

#define PM_I8_N 32u      /* tokens per tile (MMA N: 16 or 32) */
#define PM_I8_RS 2u      /* raw ring depth (super-blocks) */
#define PM_I8_AC 4u      /* tensor-memory / side-data slots (super-blocks) */
#define PM_I8_PITCH 112u /* raw bytes per row per matrix per super-block (84 + alignment) */
#define PM_I8_THREADS 416u /* 8 decode warps, 4 epilogue warps, 1 MMA warp */

/* kind::i8 instruction descriptor: A, B signed 8-bit, D s32, K-major */
__host__ __device__ __forceinline__ uint32_t pm_idesc_i8(uint32_t M, uint32_t N) {
    return (2u << 4)               /* D format: s32 */
           | (1u << 7)             /* A format: s8 */
           | (1u << 10)            /* B format: s8 */
           | ((N >> 3) << 17)      /* N / 8 */
           | ((M >> 4) << 24);     /* M / 16 */
}

__device__ __forceinline__ void pm_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* 16 consecutive s32 columns of this thread's lane */
__device__ __forceinline__ void pm_tmem_ld16i(uint32_t taddr, int32_t *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = (int32_t)r[i];
}

/* close this thread's group of asynchronous copies / wait until at most N
 * of its groups are still in flight */
__device__ __forceinline__ void pm_cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pm_cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

/* 16-byte asynchronous copy global -> shared (L2 only), both 16-byte aligned */
__device__ __forceinline__ void pm_cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pm_smem_addr(dst)), "l"(src) : "memory");
}

/* one arrival on bar once every cp.async this thread issued so far has landed
 * (the barrier's count includes it) */
__device__ __forceinline__ void pm_cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(pm_smem_addr(bar)) : "memory");
}

/* arrive on bar (count 1) after this thread's bulk copies of `bytes` */
__device__ __forceinline__ void pm_mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(pm_smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ int pm_dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

/* shared-memory layout of the kernel (bytes; 1024-aligned tiles first) */
template <int NM>
struct pm_i8_smem {
    static constexpr uint32_t A = 16384u;                      /* one 128 x 128 int8 tile */
    static constexpr uint32_t OFF_A = 0;                        /* [2 buffers][NM] */
    static constexpr uint32_t OFF_B = OFF_A + 2u * NM * A;      /* [2 buffers] 32 x 128 */
    static constexpr uint32_t OFF_RAW = OFF_B + 2u * 4096u;     /* [RS][2 parts][128][PITCH] */
    static constexpr uint32_t RAW_STAGE = 2u * 128u * PM_I8_PITCH;
    static constexpr uint32_t OFF_ARAW = OFF_RAW + PM_I8_RS * RAW_STAGE; /* [RS][2][32 tokens][4] 48 B */
    static constexpr uint32_t ARAW_STAGE = 2u * PM_I8_N * 4u * 48u;
    static constexpr uint32_t OFF_ASRAW = OFF_ARAW + PM_I8_RS * ARAW_STAGE; /* [RS][32 tokens] 64 B */
    static constexpr uint32_t OFF_SIDE = OFF_ASRAW + PM_I8_RS * PM_I8_N * 64u; /* [AC][NM][128] 2 x uint4 */
    static constexpr uint32_t OFF_ASIDE = OFF_SIDE + PM_I8_AC * NM * 128u * 32u; /* [AC][32] 9 words */
    static constexpr uint32_t ASIDE_T = 40u;                    /* yd, lo[4], hi[4] (+ pad) */
    static constexpr uint32_t TOTAL = OFF_ASIDE + PM_I8_AC * PM_I8_N * ASIDE_T;
    static_assert(TOTAL + 1024u <= 227u * 1024u, "integer tensor-core pass exceeds shared memory");
};

/* one task = (tile, 128-row block) */
struct pm_i8_task {
    const uint8_t *w[2]; /* row 0 of the block, per matrix */
    uint64_t rb;         /* row bytes */
    uint32_t s0, nt, row0, e;
};

template <int NM>
__device__ __forceinline__ bool pm_i8_task_get(const pm_layer_args &a, uint32_t j, uint32_t nrb, uint32_t n_tiles,
                                               pm_i8_task &t) {
    const uint32_t tile = j / nrb, rbk = j % nrb;
    if (tile >= n_tiles) return false;
    const uint2 tt = __ldcg(a.i8_tile + tile);
    const uint32_t e = __ldcg(a.item_expert + tt.x);
    const uint32_t s0 = __ldcg(a.item_start + tt.x), cnt = __ldcg(a.item_start + tt.x + 1) - s0;
    t.e = e;
    t.s0 = s0 + tt.y;
    t.nt = cnt - tt.y < PM_I8_N ? cnt - tt.y : PM_I8_N;
    t.row0 = rbk * 128u;
    if (NM == 2) {
        t.rb = a.rb_gu_r;
        t.w[0] = a.gate + (uint64_t)e * a.st_gu_r + (uint64_t)t.row0 * t.rb;
        t.w[1] = a.up + (uint64_t)e * a.st_gu_r + (uint64_t)t.row0 * t.rb;
    } else {
        t.rb = a.rb_dn_r;
        t.w[0] = a.down + (uint64_t)e * a.st_dn_r + (uint64_t)t.row0 * t.rb;
        t.w[1] = nullptr;
    }
    return true;
}

/* the q8_K row a tile token reads: x (gate/up) or q8_K(mid) (down) */
template <int NM>
__device__ __forceinline__ const pm_block_q8K *pm_i8_xrow(const pm_layer_args &a, uint32_t pair) {
    return NM == 2 ? a.xq + (uint64_t)(pair / a.n_slot) * a.hb : a.midq + (uint64_t)pair * a.fb;
}

/* 4-byte words w0..w(N-1) of shared memory starting at byte offset `off`
 * (a multiple of 4) of `base`, read with aligned 16-byte loads */
template <int N>
__device__ __forceinline__ void pm_i8_lds(const uint8_t *base, uint32_t off, uint32_t *w) {
    const uint32_t a0 = off & ~15u, sh = (off & 15u) >> 2; /* words to skip in the first vector */
    uint32_t v[N + 4];
#pragma unroll
    for (int i = 0; i < (N + 4 + 3) / 4; i++) {
        if (4 * i < N + 4) {
            const uint4 q = *(const uint4 *)(base + a0 + 16u * i);
            v[4 * i] = q.x;
            if (4 * i + 1 < N + 4) v[4 * i + 1] = q.y;
            if (4 * i + 2 < N + 4) v[4 * i + 2] = q.z;
            if (4 * i + 3 < N + 4) v[4 * i + 3] = q.w;
        }
    }
#pragma unroll
    for (int i = 0; i < N; i++) w[i] = sh == 0 ? v[i] : (sh == 1 ? v[i + 1] : (sh == 2 ? v[i + 2] : v[i + 3]));
}

template <int Q, int NM>
__global__ void __launch_bounds__(PM_I8_THREADS, 1) pm_tci8_kernel(const __grid_constant__ pm_layer_args a) {
    using SM = pm_i8_smem<NM>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023u) & ~(uintptr_t)1023u);
    __shared__ uint64_t a_full[2], a_empty[2], acc_full[PM_I8_AC], acc_empty[PM_I8_AC], fin;
    __shared__ uint32_t tslot, s_fail;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t n_tiles = __ldcg(a.n_items + 7);
    const uint32_t rows = NM == 2 ? a.Fr : a.H, nrb = rows / 128u;
    const uint32_t nsb = (NM == 2 ? a.H : a.Fr) / 256u;
    const uint32_t n_tasks = n_tiles * nrb;
    if (blockIdx.x >= n_tasks) return;
    if (warp == 12) pm_tmem_alloc(&tslot, 256);
    if (tid == 0) {
        for (uint32_t i = 0; i < 2; i++) {
            pm_mbar_init(&a_full[i], 256);
            pm_mbar_init(&a_empty[i], 1);
        }
        for (uint32_t i = 0; i < PM_I8_AC; i++) {
            pm_mbar_init(&acc_full[i], 1);
            pm_mbar_init(&acc_empty[i], 4);
        }
        pm_mbar_init(&fin, 1);
        s_fail = 0;
        pm_fence_barrier_init();
    }
    pm_tc_fence_before();
    __syncthreads();
    pm_tc_fence_after();
    const uint32_t tmem = tslot;
    /* this CTA's tasks j = blockIdx.x + i gridDim.x; the super-block stream
     * runs across them: global index g -> (i = g / nsb, sb = g % nsb) */
    const uint32_t my_tasks = (n_tasks - blockIdx.x + gridDim.x - 1) / gridDim.x;
    const uint32_t G = my_tasks * nsb;

    if (warp < 8) {
        /* ===== decode warps: thread (r, p) = weight row r, part p.  NM 2: part p takes
         * matrix p; NM 1: part p takes K chunk p of the one matrix.  As token (tk, q) a thread
         * also stages quarter q of token tk's chunk-p q8 values (B), and (p, q) = (0, 0) the
         * token's scale and bsums.  Every thread copies exactly the bytes it later reads, with
         * its own asynchronous-copy groups (one per super-block): no cross-thread hand-off. ===== */
        const uint32_t r = tid & 127u, p = tid >> 7, tk = r >> 2, q = r & 3u;
        const uint32_t m = NM == 2 ? p : 0u; /* the matrix this thread decodes */
        uint32_t iss_task = ~0u;             /* the task of the last request and this thread's token block */
        pm_i8_task ti;
        uintptr_t iss_blk = 0;
        auto issue = [&](uint32_t g) {
            const uint32_t task = g / nsb, sb = g % nsb, slot = g % PM_I8_RS;
            if (task != iss_task) {
                pm_i8_task_get<NM>(a, blockIdx.x + task * gridDim.x, nrb, n_tiles, ti);
                iss_blk = tk < ti.nt ? (uintptr_t)pm_i8_xrow<NM>(a, __ldcg(a.pairs + ti.s0 + tk)) : 0;
                iss_task = task;
            }
            { /* the row's 84 bytes of matrix m, rounded out to 16-byte pieces */
                uint8_t *dst = sm + SM::OFF_RAW + slot * SM::RAW_STAGE + (p * 128u + r) * PM_I8_PITCH;
                const uintptr_t src = (uintptr_t)(ti.w[m] + (uint64_t)r * ti.rb + (uint64_t)sb * PM_Q2_K_BYTES);
                const uintptr_t s0 = src & ~(uintptr_t)15;
                const uint32_t n16 = (uint32_t)((((src + PM_Q2_K_BYTES + 15u) & ~(uintptr_t)15) - s0) >> 4);
#pragma unroll
                for (uint32_t k = 0; k < 7; k++)
                    if (k < n16) pm_cp_async16(dst + 16u * k, (const void *)(s0 + 16u * k));
            }
            if (tk < ti.nt) {
                const uintptr_t blk = iss_blk + (uintptr_t)sb * PM_Q8_K_BYTES;
                { /* quarter q of chunk p's q8 values: 32 bytes from 4 + 128 p + 32 q */
                    const uintptr_t src = blk + 4u + 128u * p + 32u * q, s0 = src & ~(uintptr_t)15;
                    const uint32_t n16 = (uint32_t)((((src + 32u + 15u) & ~(uintptr_t)15) - s0) >> 4);
                    uint8_t *dst = sm + SM::OFF_ARAW + slot * SM::ARAW_STAGE + ((p * PM_I8_N + tk) * 4u + q) * 48u;
#pragma unroll
                    for (uint32_t k = 0; k < 3; k++)
                        if (k < n16) pm_cp_async16(dst + 16u * k, (const void *)(s0 + 16u * k));
                }
                if (p == 0u && q == 0u) { /* the scale d (bytes 0-3) and bsums (260-291) */
                    uint8_t *dst = sm + SM::OFF_ASRAW + (slot * PM_I8_N + tk) * 64u;
                    pm_cp_async16(dst, (const void *)(blk & ~(uintptr_t)15));
                    const uintptr_t src = blk + 260u, s0 = src & ~(uintptr_t)15;
                    const uint32_t n16 = (uint32_t)((((src + 32u + 15u) & ~(uintptr_t)15) - s0) >> 4);
#pragma unroll
                    for (uint32_t k = 0; k < 3; k++)
                        if (k < n16) pm_cp_async16(dst + 16u + 16u * k, (const void *)(s0 + 16u * k));
                }
            }
        };
#pragma unroll
        for (uint32_t g = 0; g < PM_I8_RS; g++) {
            if (g < G) issue(g);
            pm_cp_async_commit(); /* one group per super-block (empty past the end) */
        }
        bool fail = false;
        pm_i8_task t;
        uintptr_t my_blk = 0; /* token tk's q8_K row (block 0) */
        for (uint32_t g = 0; g < G && !fail; g++) {
            const uint32_t sb = g % nsb;
            if (sb == 0) {
                pm_i8_task_get<NM>(a, blockIdx.x + (g / nsb) * gridDim.x, nrb, n_tiles, t);
                my_blk = tk < t.nt ? (uintptr_t)pm_i8_xrow<NM>(a, __ldcg(a.pairs + t.s0 + tk)) : 0;
            }
            const uint32_t slot = g % PM_I8_RS, x = g % PM_I8_AC;
            pm_cp_async_wait<PM_I8_RS - 1>(); /* this thread's copies of super-block g have landed */
            /* side slot x is free once the epilogue finished super-block g - AC */
            if (g >= PM_I8_AC && !pm_mbar_wait(&acc_empty[x], ((g / PM_I8_AC) - 1u) & 1u, a.err, a.wait)) {
                fail = true;
                break;
            }
            const uint8_t *raw = sm + SM::OFF_RAW + slot * SM::RAW_STAGE + (p * 128u + r) * PM_I8_PITCH;
            const uint32_t off = (uint32_t)((uintptr_t)(t.w[m] + (uint64_t)r * t.rb + (uint64_t)sb * PM_Q2_K_BYTES) & 15u);
            const uintptr_t blk = my_blk + (uintptr_t)sb * PM_Q8_K_BYTES;
            /* the row's 16 scale bytes (low nibble: scale, high nibble: min) */
            uint32_t scw[4];
            pm_i8_lds<4>(raw, off, scw);
            if (NM == 2 || p == 0u) { /* side data of (row, super-block, matrix m): d, dmin, 16 mins as bytes */
                uint32_t dd[1];
                pm_i8_lds<1>(raw, off + 80u, dd);
                uint4 sd;
                sd.x = __float_as_uint(pm_h2f(dd[0] & 0xffffu));
                sd.y = __float_as_uint(pm_h2f(dd[0] >> 16));
                sd.z = ((scw[0] >> 4) & 0x0f0f0f0fu); /* mins 0-3 */
                sd.w = ((scw[1] >> 4) & 0x0f0f0f0fu); /* mins 4-7 */
                uint4 *side = (uint4 *)(sm + SM::OFF_SIDE) + (x * NM + m) * 256u + 2u * r;
                side[0] = sd;
                side[1] = make_uint4((scw[2] >> 4) & 0x0f0f0f0fu, (scw[3] >> 4) & 0x0f0f0f0fu, 0u, 0u);
            }
            /* per (token, super-block): yd and the bsums split in low / high bytes */
            if (p == 0u && q == 0u && tk < t.nt) {
                const uint8_t *as_raw = sm + SM::OFF_ASRAW + (slot * PM_I8_N + tk) * 64u;
                uint32_t bw[9];
                pm_i8_lds<1>(as_raw, (uint32_t)(blk & 15u), bw);                      /* d */
                pm_i8_lds<8>(as_raw + 16, (uint32_t)((blk + 260u) & 15u), bw + 1);  /* bsums[16] */
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int qq = 0; qq < 4; qq++) {
                    const uint32_t b01 = bw[1 + 2 * qq], b23 = bw[2 + 2 * qq];
                    /* bsums j = 4qq .. 4qq + 3 as int16; low bytes unsigned, high bytes signed */
                    lo[qq] = (b01 & 0xffu) | ((b01 >> 8) & 0xff00u) | ((b23 & 0xffu) << 16) | ((b23 << 8) & 0xff000000u);
                    hi[qq] = ((b01 >> 8) & 0xffu) | ((b01 >> 16) & 0xff00u) | (((b23 >> 8) & 0xffu) << 16) |
                             (b23 & 0xff000000u);
                }
                uint32_t *as = (uint32_t *)(sm + SM::OFF_ASIDE + (x * PM_I8_N + tk) * SM::ASIDE_T);
                as[0] = bw[0];
#pragma unroll
                for (int qq = 0; qq < 4; qq++) as[1 + qq] = lo[qq], as[5 + qq] = hi[qq];
            }
            /* B quarter of this thread's chunk p */
            uint32_t bv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (tk < t.nt)
                pm_i8_lds<8>(sm + SM::OFF_ARAW + slot * SM::ARAW_STAGE + ((p * PM_I8_N + tk) * 4u + q) * 48u,
                             (uint32_t)((blk + 4u + 128u * p + 32u * q) & 15u), bv);
            /* the two 128-wide K chunks of the super-block */
#pragma unroll 1
            for (uint32_t h = 0; h < 2; h++) {
                const uint32_t c = 2u * g + h, ab = c & 1u;
                if (c >= 2 && !pm_mbar_wait(&a_empty[ab], ((c >> 1) - 1u) & 1u, a.err, a.wait)) {
                    fail = true;
                    break;
                }
                if (NM == 2 || p == h) { /* A: this thread's row of matrix m, chunk h */
                    uint32_t qw[8];
                    pm_i8_lds<8>(raw, off + 16u + 32u * h, qw);
                    const uint32_t sc4[2] = {scw[2 * h] & 0x0f0f0f0fu, scw[2 * h + 1] & 0x0f0f0f0fu};
                    uint8_t *A = sm + SM::OFF_A + (ab * NM + m) * SM::A + (r >> 3) * 1024u + (r & 7u) * 128u;
#pragma unroll
                    for (uint32_t j = 0; j < 8; j++) { /* 16-byte unit j: shift 2 (j / 2), qs words 4 (j % 2) .. + 3 */
                        const uint32_t sc = (sc4[j >> 2] >> (8u * (j & 3u))) & 0xffu;
                        const uint32_t s = 2u * (j >> 1);
                        uint4 o;
                        o.x = ((qw[4 * (j & 1) + 0] >> s) & 0x03030303u) * sc;
                        o.y = ((qw[4 * (j & 1) + 1] >> s) & 0x03030303u) * sc;
                        o.z = ((qw[4 * (j & 1) + 2] >> s) & 0x03030303u) * sc;
                        o.w = ((qw[4 * (j & 1) + 3] >> s) & 0x03030303u) * sc;
                        *(uint4 *)(A + ((j ^ (r & 7u)) << 4)) = o;
                    }
                }
                if (p == h) { /* B of chunk h: 4 threads per token row, 32 q8 bytes each; rows past nt zero */
                    uint8_t *B = sm + SM::OFF_B + ab * 4096u + (tk >> 3) * 1024u + (tk & 7u) * 128u;
                    *(uint4 *)(B + (((2u * q) ^ (tk & 7u)) << 4)) = make_uint4(bv[0], bv[1], bv[2], bv[3]);
                    *(uint4 *)(B + (((2u * q + 1u) ^ (tk & 7u)) << 4)) = make_uint4(bv[4], bv[5], bv[6], bv[7]);
                }
                pm_fence_proxy_async(); /* generic-proxy writes before the MMA reads them */
                pm_mbar_arrive(&a_full[ab]);
            }
            if (fail) break;
            /* this thread's pieces of super-block g are consumed: request g + RS into the slot */
            if (g + PM_I8_RS < G) issue(g + PM_I8_RS);
            pm_cp_async_commit();
        }
        if (fail) atomicOr(&s_fail, 1u);
        pm_cp_async_wait<0>(); /* every copy of this thread has landed before the CTA leaves */
    } else if (warp == 12) {
        /* ===== MMA issue ===== */
        if (lane == 0) {
            bool ok = true;
            pm_i8_task t;
            uint32_t N = 16;
            for (uint32_t g = 0; g < G && ok; g++) {
                const uint32_t sb = g % nsb, x = g % PM_I8_AC;
                if (sb == 0) {
                    pm_i8_task_get<NM>(a, blockIdx.x + (g / nsb) * gridDim.x, nrb, n_tiles, t);
                    N = t.nt > 16u ? 32u : 16u;
                }
                if (g >= PM_I8_AC && !pm_mbar_wait(&acc_empty[x], ((g / PM_I8_AC) - 1u) & 1u, a.err, a.wait)) {
                    ok = false;
                    break;
                }
                pm_tc_fence_after();
                const uint32_t idesc = pm_idesc_i8(128, N);
                for (uint32_t h = 0; h < 2; h++) {
                    const uint32_t c = 2u * g + h, ab = c & 1u;
                    if (!pm_mbar_wait(&a_full[ab], (c >> 1) & 1u, a.err, a.wait)) {
                        ok = false;
                        break;
                    }
                    pm_tc_fence_after();
                    const uint64_t bd = pm_desc_sw128(sm + SM::OFF_B + ab * 4096u);
#pragma unroll
                    for (int m = 0; m < NM; m++) {
                        const uint64_t ad = pm_desc_sw128(sm + SM::OFF_A + (ab * NM + (uint32_t)m) * SM::A);
                        const uint32_t d = tmem + x * (NM * 32u) + (uint32_t)m * 32u;
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; kk++)
                            pm_mma_i8(d, ad + 2 * kk, bd + 2 * kk, idesc, (h > 0 || kk > 0) ? 1u : 0u);
                    }
                    pm_mma_commit(&a_empty[ab]);
                }
                if (ok) pm_mma_commit(&acc_full[x]);
            }
            pm_mma_commit(&fin);
            pm_mbar_wait(&fin, 0, nullptr);
            if (!ok) atomicOr(&s_fail, 1u);
        }
    } else {
        /* ===== epilogue: warps 8-11 read tensor-memory lanes 32 (warp % 4) .. + 31 ===== */
        const uint32_t lq = warp & 3u, row = lq * 32u + lane;
        float acc[NM][PM_I8_N];
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
            for (uint32_t k = 0; k < PM_I8_N; k++) acc[m][k] = 0.0f;
        pm_i8_task t;
        for (uint32_t g = 0; g < G; g++) {
            const uint32_t sb = g % nsb, x = g % PM_I8_AC;
            if (sb == 0) pm_i8_task_get<NM>(a, blockIdx.x + (g / nsb) * gridDim.x, nrb, n_tiles, t);
            if (!pm_mbar_wait(&acc_full[x], (g / PM_I8_AC) & 1u, a.err, a.wait)) {
                atomicOr(&s_fail, 1u);
                break;
            }
            pm_tc_fence_after();
            const uint32_t ncol = t.nt > 16u ? 32u : 16u;
#pragma unroll
            for (int m = 0; m < NM; m++) {
                int32_t v[PM_I8_N];
                const uint32_t base = tmem + ((lq * 32u) << 16) + x * (NM * 32u) + (uint32_t)m * 32u;
                pm_tmem_ld16i(base, v);
                if (ncol > 16u) pm_tmem_ld16i(base + 16u, v + 16);
                const uint4 *side = (const uint4 *)(sm + SM::OFF_SIDE) + (x * NM + (uint32_t)m) * 256u + 2u * row;
                const uint4 s0 = side[0], s1 = side[1];
                const float d = __uint_as_float(s0.x), dm = __uint_as_float(s0.y);
                const uint32_t mw[4] = {s0.z, s0.w, s1.x, s1.y};
#pragma unroll
                for (uint32_t k = 0; k < PM_I8_N; k++) {
                    if (k >= t.nt) break; /* uniform: only the tile's tokens */
                    {
                        const uint32_t *as = (const uint32_t *)(sm + SM::OFF_ASIDE + (x * PM_I8_N + k) * SM::ASIDE_T);
                        const float yd = __uint_as_float(as[0]);
                        int lo = 0, hi = 0;
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            lo = pm_dp4a_uu(mw[q], as[1 + q], lo);
                            hi = pm_dp4a_us(mw[q], (int)as[5 + q], hi);
                        }
                        const int msum = lo + 256 * hi;
                        /* total += yd xd isum - yd xmin msum (cpu_dot.rs:732-767, q2_K) */
                        const float term = __fsub_rn(__fmul_rn(__fmul_rn(yd, d), (float)v[k]),
                                                     __fmul_rn(__fmul_rn(yd, dm), (float)msum));
                        acc[m][k] = __fadd_rn(acc[m][k], term);
                    }
                }
            }
            pm_tc_fence_before();
            __syncwarp();
            if (lane == 0) pm_mbar_arrive(&acc_empty[x]);
            if (sb == nsb - 1u) { /* the task's rows are complete: outputs, in the CPU lane's order */
                const uint32_t grow = t.row0 + row;
#pragma unroll
                for (uint32_t k = 0; k < PM_I8_N; k++) {
                    if (k < t.nt) {
                        const uint32_t pr = __ldcg(a.pairs + t.s0 + k);
                        if (NM == 2) {
                            float gg = acc[0][k], uu = acc[NM - 1][k];
                            if (a.gate_b) gg = __fadd_rn(gg, a.gate_b[(uint64_t)t.e * a.Fr + grow]);
                            if (a.up_b) uu = __fadd_rn(uu, a.up_b[(uint64_t)t.e * a.Fr + grow]);
                            a.mid[(uint64_t)pr * a.Fmax + grow] = __fmul_rn(pm_glu(gg, uu, a.act), __ldcg(a.w + pr));
                        } else {
                            a.partial[(uint64_t)pr * a.H + grow] = acc[0][k];
                        }
                    }
#pragma unroll
                    for (int m = 0; m < NM; m++) acc[m][k] = 0.0f;
                }
            }
        }
    }
    pm_tc_fence_before();
    __syncthreads();
    pm_tc_fence_after();
    if (warp == 12) {
        __syncwarp();
        pm_tmem_free(tmem, 256);
    }
    if (tid == 0 && s_fail) atomicOr(a.err, PM_ERR_TIMEOUT);
}

/* q8_K of the mid rows of every tile pair (the down pass's B operand), the
 * CPU lane's quantizer (cpu_dot.rs:26-50); block = tile, warp per (token,
 * 256-block) */
static __global__ void __launch_bounds__(256) pm_i8_midq_kernel(const __grid_constant__ pm_layer_args a) {
    const uint32_t tile = blockIdx.x;
    if (tile >= __ldcg(a.n_items + 7)) return;
    const uint2 tt = __ldcg(a.i8_tile + tile);
    const uint32_t s0 = __ldcg(a.item_start + tt.x), cnt = __ldcg(a.item_start + tt.x + 1) - s0;
    const uint32_t nt = cnt - tt.y < PM_I8_N ? cnt - tt.y : PM_I8_N;
    const uint32_t nb = (a.Fr + 255u) / 256u;
    for (uint32_t job = threadIdx.x >> 5; job < nt * nb; job += blockDim.x >> 5) {
        const uint32_t k = job / nb, b = job % nb;
        const uint32_t pr = __ldcg(a.pairs + s0 + tt.y + k);
        const uint32_t valid = a.Fr - b * 256u < 256u ? a.Fr - b * 256u : 256u;
        pm_q8k_warp(a.mid + (uint64_t)pr * a.Fmax + b * 256u, valid, a.midq + (uint64_t)pr * a.fb + b);
    }
}

/* one integer tensor-core pass (NM 2: gate/up -> mid, 1: down -> partial
 * rows), one persistent CTA per SM */
template <int Q, int NM>
static int pm_i8_launch(const pm_layer_args &a, cudaStream_t st) {
    static uint64_t done = 0;
    auto k = pm_tci8_kernel<Q, NM>;
    const uint32_t smem = pm_i8_smem<NM>::TOTAL + 1024u;
    if (!pm_smem_attr(k, smem, &done)) return 0;
    k<<<a.n_sm, PM_I8_THREADS, smem, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer integer tensor-core launch");
}

static int pm_i8_midq_launch(const pm_layer_args &a, cudaStream_t st) {
    pm_i8_midq_kernel<<<a.max_i8, 256, 0, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer integer tensor-core mid q8_K launch");
}
