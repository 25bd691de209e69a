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
 * kernel lists them); a task is (tile, two 128-row A matrices: gate and
 * up of one block, or two consecutive blocks of down).  Persistent CTAs take tasks round-robin and stream their
 * super-blocks through four pipelines:
 *   load    one producer warp fills a ring of super-block stages: per
 *           matrix one bulk copy of the 10.5 KB tile-plane chunk (the
 *           load-time image below: 128 rows of one super-block, contiguous
 *           in HBM) and per lane one token's q8_K block in 16-byte
 *           asynchronous copies, all landing on the stage's mbarrier;
 *   decode  8 warps turn a stage into int8 A tiles (q sc, 128 rows x 128 K,
 *           128-byte swizzle), stage the tokens' q8 values as the B tile
 *           and the per-(row, super-block) scales / per-(token,
 *           super-block) bsums for the epilogue, and free the stage as soon
 *           as its bytes are in registers;
 *   mma     one thread issues 4 MMAs (K = 32) per matrix per 128-wide K
 *           chunk into a per-super-block tensor-memory slot (4 slots), and
 *           per matrix one more u8 MMA (K = 32) for the mins sum below;
 *   epilog  8 warps (two per 32-lane quarter of tensor memory, 16 tokens
 *           each) read the slot, form the f32 terms and add them in
 *           super-block order; at the task's last super-block they write
 *           mid = glu(g + gb, u + ub) w (gate/up) or the partial row (down).
 *
 * The mins sum on the tensor cores.  msum = sum_j m_j bsum_j (16 sub-blocks,
 * m_j in 0..15, |bsum_j| <= 16 * 127) is exact as one unsigned 8-bit MMA:
 * write bsum_j + 2048 = l_j + 16 h_j with l_j in 0..15 and h_j in 1..255;
 * the A row is [m_0..m_15 | 16 m_0..16 m_15] (the mins as bytes, and the
 * scale bytes' high nibbles in place), the B row [l_0..l_15 | h_0..h_15],
 * so the s32 result is msum + 2048 sum_j m_j, and the epilogue subtracts
 * the row's 2048 sum_j m_j.  Both 32-byte-wide tiles use the 32-byte
 * swizzle.  Barriers the decode warps signal take one arrival per warp.
 * Every wait is bounded; on a timeout the kernel records it in the layer's
 * error word, lets the copies and MMAs in flight land and returns.
 */
#pragma once
#include "pm_tc.cuh"

#define PM_I8_N 32u      /* tokens per tile (MMA N: 16 or 32) */
#define PM_I8_AC 4u      /* tensor-memory / side-data slots (super-blocks) */
#define PM_I8_EPI_WARPS 8u
#define PM_I8_MMA_WARP 16u
#define PM_I8_PROD_WARP 17u
#define PM_I8_THREADS 576u /* 8 decode warps, 8 epilogue warps, 1 MMA warp, 1 producer warp */

/* kind::i8 instruction descriptor: A, B signed 8-bit (u8: unsigned), D s32, K-major */
__host__ __device__ __forceinline__ uint32_t pm_idesc_i8(uint32_t M, uint32_t N) {
    return (2u << 4)               /* D format: s32 */
           | (1u << 7)             /* A format: s8 */
           | (1u << 10)            /* B format: s8 */
           | ((N >> 3) << 17)      /* N / 8 */
           | ((M >> 4) << 24);     /* M / 16 */
}
__host__ __device__ __forceinline__ uint32_t pm_idesc_u8(uint32_t M, uint32_t N) {
    return (2u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24); /* s32 = u8 x u8 */
}

/* shared-memory descriptor of a K-major tile 32 bytes wide (one K = 32 MMA
 * slice) in the 32-byte swizzle: 8-row groups of 256 bytes, row r at
 * 32 (r % 8), its 16-byte unit u at (u ^ ((r >> 2) & 1)) 16 */
__device__ __forceinline__ uint64_t pm_desc_sw32(const void *tile) {
    const uint64_t a = pm_smem_addr(tile);
    uint64_t d = (a >> 4) & 0x3fffull;
    d |= (uint64_t)1 << 16;           /* leading byte offset (unused for swizzled K-major) */
    d |= (uint64_t)(256 >> 4) << 32;  /* stride byte offset: next 8-row group */
    d |= (uint64_t)1 << 46;           /* descriptor version (sm_100) */
    d |= (uint64_t)6 << 61;           /* layout: 32-byte swizzle */
    return d;
}
__device__ __forceinline__ uint32_t pm_sw32_off(uint32_t r, uint32_t u) {
    return (r >> 3) * 256u + (r & 7u) * 32u + ((u ^ ((r >> 2) & 1u)) << 4);
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

/* 16 consecutive s32 columns of this thread's lane, at ta and at tb, one wait */
__device__ __forceinline__ void pm_tmem_ld16i2(uint32_t ta, uint32_t tb, int32_t *va, int32_t *vb) {
    uint32_t r[16], q[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(ta));
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]), "=r"(q[6]), "=r"(q[7]),
          "=r"(q[8]), "=r"(q[9]), "=r"(q[10]), "=r"(q[11]), "=r"(q[12]), "=r"(q[13]), "=r"(q[14]), "=r"(q[15])
        : "r"(tb));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) va[i] = (int32_t)r[i], vb[i] = (int32_t)q[i];
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

__device__ __forceinline__ int pm_dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

/* Q2_K tile planes: the load-time image of an expert matrix the integer
 * passes stream.  Per (expert, 128-row block, super-block) one contiguous
 * chunk of 128 x 84 bytes (the same bytes as the GGUF blocks, regrouped):
 *     [0, 8192)      qs: [4 units][128 rows] x 16 bytes (unit j = qs bytes 16j..16j+15)
 *     [8192, 10240)  scales: [128 rows] x 16 bytes
 *     [10240, 10752) d, dmin: [128 rows] x 2 f16
 * so one bulk copy brings a super-block of 128 rows, and every decode
 * thread's reads of it are bank-conflict free.  Chunk (e, b, sb) sits at
 * ((e nrb + b) nsb + sb) x 10752: an expert's image has the size of its
 * GGUF rows. */
#define PM_I8_CHUNK 10752u
#define PM_I8_TOKB 304u /* per-token slot of a ring stage: a q8_K block rounded out to 16 bytes */

/* shared-memory layout of the kernel (bytes; 1024-aligned tiles first) */
template <int NM>
struct pm_i8_smem {
    static constexpr uint32_t RS = NM == 2 ? 3u : 8u;         /* ring stages (super-blocks) */
    static constexpr uint32_t A = 16384u;                      /* one 128 x 128 int8 tile */
    static constexpr uint32_t NAB = 2u;                         /* A / B tile buffers (128-wide K chunks) */
    static constexpr uint32_t OFF_A = 0;                        /* [NAB buffers][NM] */
    static constexpr uint32_t OFF_B = OFF_A + NAB * NM * A;     /* [NAB buffers] 32 x 128 */
    static constexpr uint32_t OFF_RING = OFF_B + NAB * 4096u;   /* [RS] stages */
    static constexpr uint32_t STAGE = NM * PM_I8_CHUNK + PM_I8_N * PM_I8_TOKB; /* chunks, then token blocks */
    static constexpr uint32_t OFF_AM = OFF_RING + RS * STAGE;  /* [2 (super-block parity)][NM] 128 x 32 mins tiles */
    static constexpr uint32_t OFF_BM = OFF_AM + 2u * NM * 4096u; /* [2] 32 x 32 bsum split tiles */
    static constexpr uint32_t OFF_SIDE = OFF_BM + 2u * 1024u;   /* [AC][NM][128] uint4: d, dmin, 2048 sum m */
    static constexpr uint32_t OFF_ASIDE = OFF_SIDE + PM_I8_AC * NM * 128u * 16u; /* [AC][32] yd */
    static constexpr uint32_t TMEM_COLS = NM * 64u * PM_I8_AC;  /* per slot and matrix: 32 isum + 32 msum */
    static constexpr uint32_t TOTAL = OFF_ASIDE + PM_I8_AC * PM_I8_N * 4u;
    static_assert(STAGE % 16u == 0 && OFF_RING % 16u == 0, "bulk copies need 16-byte alignment");
    static_assert(OFF_AM % 256u == 0 && OFF_BM % 256u == 0, "32-byte swizzle tiles need 256-byte alignment");
    static_assert(TOTAL + 1024u <= 227u * 1024u, "integer tensor-core pass exceeds shared memory");
};

/* one task = (tile, 128-row block of gate and up, or 256 rows of down) */
struct pm_i8_task {
    const uint8_t *w[2]; /* the block's first chunk (super-block 0), per matrix */
    uint32_t s0, nt, row0, e;
};

template <int NM>
__device__ __forceinline__ bool pm_i8_task_get(const pm_layer_args &a, uint32_t j, uint32_t nrb, uint32_t nsb,
                                               uint32_t n_tiles, pm_i8_task &t) {
    const uint32_t tile = j / nrb, rbk = j % nrb;
    if (tile >= n_tiles) return false;
    const uint2 tt = __ldcg(a.i8_tile + tile);
    const uint32_t e = __ldcg(a.item_expert + tt.x);
    const uint32_t s0 = __ldcg(a.item_start + tt.x), cnt = __ldcg(a.item_start + tt.x + 1) - s0;
    t.e = e;
    t.s0 = s0 + tt.y;
    t.nt = cnt - tt.y < PM_I8_N ? cnt - tt.y : PM_I8_N;
    if (NM == 2) { /* gate and up rows of one 128-row block */
        const uint64_t chunk0 = ((uint64_t)e * nrb + rbk) * nsb * PM_I8_CHUNK;
        t.row0 = rbk * 128u;
        t.w[0] = a.gate_t + chunk0;
        t.w[1] = a.up_t + chunk0;
    } else { /* down: two consecutive 128-row blocks (nrb counts block pairs) */
        const uint64_t chunk0 = ((uint64_t)e * 2u * nrb + 2u * rbk) * nsb * PM_I8_CHUNK;
        t.row0 = rbk * 256u;
        t.w[0] = a.down_t + chunk0;
        t.w[1] = t.w[0] + (uint64_t)nsb * PM_I8_CHUNK;
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
    /* NM: the pass (2 gate/up, 1 down); every task streams NMA = 2 matrices - gate and up
     * of one 128-row block, or two consecutive 128-row blocks of down */
    constexpr int NMA = 2;
    using SM = pm_i8_smem<NMA>;
    constexpr uint32_t RS = SM::RS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023u) & ~(uintptr_t)1023u);
    __shared__ uint64_t full[RS], empty[RS], a_full[SM::NAB], a_empty[SM::NAB], acc_full[PM_I8_AC], acc_empty[PM_I8_AC], fin;
    __shared__ uint32_t tslot, s_fail;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t n_tiles = __ldcg(a.n_items + 7);
    const uint32_t nrb = NM == 2 ? a.Fr / 128u : a.H / 256u; /* tasks per tile */
    const uint32_t nsb = (NM == 2 ? a.H : a.Fr) / 256u;
    const uint32_t n_tasks = n_tiles * nrb;
    if (blockIdx.x >= n_tasks) return;
    if (warp == PM_I8_MMA_WARP) pm_tmem_alloc(&tslot, SM::TMEM_COLS);
    if (tid == 0) {
        for (uint32_t i = 0; i < RS; i++) {
            pm_mbar_init(&full[i], 33);  /* the producer's 32 lanes (token copies) + its expect_tx arrive */
            pm_mbar_init(&empty[i], 8); /* every decode warp */
        }
        for (uint32_t i = 0; i < SM::NAB; i++) {
            pm_mbar_init(&a_full[i], 8);
            pm_mbar_init(&a_empty[i], 1);
        }
        for (uint32_t i = 0; i < PM_I8_AC; i++) {
            pm_mbar_init(&acc_full[i], 1);
            pm_mbar_init(&acc_empty[i], PM_I8_EPI_WARPS);
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
    const uint32_t task0 = blockIdx.x;

    if (warp == PM_I8_PROD_WARP) {
        /* ===== producer: per super-block one bulk copy per matrix (the tile-plane chunk) and,
         * per lane, its token's q8_K block in 16-byte asynchronous copies ===== */
        pm_i8_task t;
        uintptr_t blk0 = 0;
        bool ok = true;
        uint32_t g = 0;
        for (; g < G; g++) {
            const uint32_t sb = g % nsb, s = g % RS;
            if (sb == 0) {
                pm_i8_task_get<NM>(a, task0 + (g / nsb) * gridDim.x, nrb, nsb, n_tiles, t);
                blk0 = lane < t.nt ? (uintptr_t)pm_i8_xrow<NM>(a, __ldcg(a.pairs + t.s0 + lane)) : 0;
            }
            if (g >= RS && !pm_mbar_wait(&empty[s], ((g / RS) - 1u) & 1u, a.err, a.wait)) {
                ok = false;
                break;
            }
            uint8_t *stage = sm + SM::OFF_RING + s * SM::STAGE;
            if (lane == 0) {
                pm_mbar_expect_tx(&full[s], NMA * PM_I8_CHUNK);
#pragma unroll
                for (int m = 0; m < NMA; m++)
                    pm_bulk_g2s(stage + m * PM_I8_CHUNK, t.w[m] + (uint64_t)sb * PM_I8_CHUNK, PM_I8_CHUNK, &full[s]);
            }
            if (lane < t.nt) { /* a q8_K block (292 bytes at a 4-byte boundary) is 19 16-byte pieces */
                const uintptr_t src = (blk0 + (uintptr_t)sb * PM_Q8_K_BYTES) & ~(uintptr_t)15;
                uint8_t *dst = stage + NMA * PM_I8_CHUNK + lane * PM_I8_TOKB;
#pragma unroll
                for (uint32_t k = 0; k < PM_I8_TOKB / 16u; k++) pm_cp_async16(dst + 16u * k, (const void *)(src + 16u * k));
            }
            pm_cp_async_arrive(&full[s]);
        }
        if (!ok) atomicOr(&s_fail, 1u);
        /* the copies of the last stages issued have landed before the CTA leaves */
        for (uint32_t h = g > RS ? g - RS : 0u; h < g; h++) pm_mbar_wait(&full[h % RS], (h / RS) & 1u, nullptr);
        pm_cp_async_wait<0>();
    } else if (warp < 8) {
        /* ===== decode warps: thread (r, p) = row r of the task's matrix p (gate / up, or the
         * first / second 128-row block of down).  As token (tk, q) a thread also stages
         * quarter q of token tk's chunk-p q8 values (B), and p = 0 threads the token's scale
         * and bsums for the epilogue. ===== */
        const uint32_t r = tid & 127u, p = tid >> 7, tk = r >> 2, q = r & 3u;
        const uint32_t m = NMA == 2 ? p : 0u; /* the matrix this thread decodes */
        bool fail = false;
        pm_i8_task t;
        uintptr_t my_blk = 0; /* token tk's q8_K row (block 0) */
        for (uint32_t g = 0; g < G && !fail; g++) {
            const uint32_t sb = g % nsb, s = g % RS, x = g % PM_I8_AC;
            if (sb == 0) {
                pm_i8_task_get<NM>(a, task0 + (g / nsb) * gridDim.x, nrb, nsb, n_tiles, t);
                my_blk = tk < t.nt ? (uintptr_t)pm_i8_xrow<NM>(a, __ldcg(a.pairs + t.s0 + tk)) : 0;
            }
            /* waits decide per warp (one arrival per warp on the barriers below) */
            if (__any_sync(0xffffffffu, !pm_mbar_wait(&full[s], (g / RS) & 1u, a.err, a.wait))) {
                fail = true;
                break;
            }
            /* everything this thread needs of the stage, into registers */
            const uint8_t *W = sm + SM::OFF_RING + s * SM::STAGE + m * PM_I8_CHUNK;
            const uint4 scv = *(const uint4 *)(W + 8192u + 16u * r);
            const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
            const uint32_t dd = *(const uint32_t *)(W + 10240u + 4u * r);
            uint32_t qw[2][8];
#pragma unroll
            for (uint32_t h = 0; h < 2; h++) {
                if (NMA == 2 || p == h) {
                    const uint4 u0 = *(const uint4 *)(W + (2u * h * 128u + r) * 16u);
                    const uint4 u1 = *(const uint4 *)(W + ((2u * h + 1u) * 128u + r) * 16u);
                    qw[h][0] = u0.x, qw[h][1] = u0.y, qw[h][2] = u0.z, qw[h][3] = u0.w;
                    qw[h][4] = u1.x, qw[h][5] = u1.y, qw[h][6] = u1.z, qw[h][7] = u1.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) qw[h][i] = 0u;
                }
            }
            const uintptr_t blk = my_blk + (uintptr_t)sb * PM_Q8_K_BYTES;
            const uint8_t *tok = sm + SM::OFF_RING + s * SM::STAGE + NMA * PM_I8_CHUNK + tk * PM_I8_TOKB;
            const uint32_t tb = (uint32_t)(blk & 15u); /* the block's offset in its slot */
            uint32_t bv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, bw[2] = {0u, 0u}, ydw = 0u;
            if (tk < t.nt) {
                pm_i8_lds<8>(tok, tb + 4u + 128u * p + 32u * q, bv);
                if (p == 0u) {
                    pm_i8_lds<2>(tok, tb + 260u + 8u * q, bw); /* bsums 4q .. 4q + 3 */
                    if (q == 0u) pm_i8_lds<1>(tok, tb, &ydw);  /* d */
                }
            }
            /* the stage is consumed: the producer may refill it */
            __syncwarp();
            if (lane == 0) pm_mbar_arrive(&empty[s]);
            /* side slot x is free once the epilogue finished super-block g - AC */
            if (g >= PM_I8_AC &&
                __any_sync(0xffffffffu, !pm_mbar_wait(&acc_empty[x], ((g / PM_I8_AC) - 1u) & 1u, a.err, a.wait))) {
                fail = true;
                break;
            }
            /* the row's mins (bytes) and 16 x mins (the scale bytes' high nibbles in place) */
            uint32_t mn[4], m16[4];
#pragma unroll
            for (int i = 0; i < 4; i++) mn[i] = (scw[i] >> 4) & 0x0f0f0f0fu, m16[i] = scw[i] & 0xf0f0f0f0u;
            if (NMA == 2 || p == 0u) { /* side data of (row, super-block, matrix m): d, dmin, 2048 sum m */
                int msum = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) msum = pm_dp4a_uu(mn[i], 0x01010101u, msum);
                uint4 *side = (uint4 *)(sm + SM::OFF_SIDE) + (x * NMA + m) * 128u + r;
                *side = make_uint4(__float_as_uint(pm_h2f(dd & 0xffffu)), __float_as_uint(pm_h2f(dd >> 16)),
                                   (uint32_t)(2048 * msum), 0u);
            }
            /* per (token, super-block): yd, and the token's bsums as l + 16 h (bsum + 2048, l 0..15,
             * h 1..255), four per quarter q; rows past nt stay zero */
            uint32_t bl = 0u, bh = 0u;
            if (p == 0u && tk < t.nt) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t w = bw[j >> 1];
                    const int b = (j & 1) ? ((int)w >> 16) : (int)(int16_t)(w & 0xffffu);
                    const uint32_t v = (uint32_t)(b + 2048);
                    bl |= (v & 15u) << (8 * j);
                    bh |= (v >> 4) << (8 * j);
                }
                if (q == 0u) ((float *)(sm + SM::OFF_ASIDE))[x * PM_I8_N + tk] = __uint_as_float(ydw);
            }
            /* the two 128-wide K chunks of the super-block */
#pragma unroll
            for (uint32_t h = 0; h < 2; h++) {
                const uint32_t c = 2u * g + h, ab = c % SM::NAB;
                if (c >= SM::NAB &&
                    __any_sync(0xffffffffu, !pm_mbar_wait(&a_empty[ab], ((c / SM::NAB) - 1u) & 1u, a.err, a.wait))) {
                    fail = true;
                    break;
                }
                if (NMA == 2 || p == h) { /* A: this thread's row of matrix m, chunk h */
                    const uint32_t sc4[2] = {scw[2 * h] & 0x0f0f0f0fu, scw[2 * h + 1] & 0x0f0f0f0fu};
                    uint8_t *A = sm + SM::OFF_A + (ab * NMA + m) * SM::A + (r >> 3) * 1024u + (r & 7u) * 128u;
#pragma unroll
                    for (uint32_t j = 0; j < 8; j++) { /* 16-byte unit j: shift 2 (j / 2), qs words 4 (j % 2) .. + 3 */
                        const uint32_t sc = (sc4[j >> 2] >> (8u * (j & 3u))) & 0xffu;
                        const uint32_t sh = 2u * (j >> 1);
                        uint4 o;
                        o.x = ((qw[h][4 * (j & 1) + 0] >> sh) & 0x03030303u) * sc;
                        o.y = ((qw[h][4 * (j & 1) + 1] >> sh) & 0x03030303u) * sc;
                        o.z = ((qw[h][4 * (j & 1) + 2] >> sh) & 0x03030303u) * sc;
                        o.w = ((qw[h][4 * (j & 1) + 3] >> sh) & 0x03030303u) * sc;
                        *(uint4 *)(A + ((j ^ (r & 7u)) << 4)) = o;
                    }
                }
                if (p == h) { /* B of chunk h: 4 threads per token row, 32 q8 bytes each; rows past nt zero */
                    uint8_t *B = sm + SM::OFF_B + ab * 4096u + (tk >> 3) * 1024u + (tk & 7u) * 128u;
                    *(uint4 *)(B + (((2u * q) ^ (tk & 7u)) << 4)) = make_uint4(bv[0], bv[1], bv[2], bv[3]);
                    *(uint4 *)(B + (((2u * q + 1u) ^ (tk & 7u)) << 4)) = make_uint4(bv[4], bv[5], bv[6], bv[7]);
                }
                if (h == 0u) { /* the mins-sum operands ride with K chunk 0: buffer g % 2, free once the
                                * MMAs of chunk 2g - NAB (issued after super-block g - 2's) are done */
                    if (NMA == 2 || p == 0u) {
                        uint8_t *AM = sm + SM::OFF_AM + ((g & 1u) * NMA + m) * 4096u;
                        *(uint4 *)(AM + pm_sw32_off(r, 0)) = make_uint4(mn[0], mn[1], mn[2], mn[3]);
                        *(uint4 *)(AM + pm_sw32_off(r, 1)) = make_uint4(m16[0], m16[1], m16[2], m16[3]);
                    }
                    if (p == 0u) { /* word q of the token's l and h units */
                        uint8_t *BM = sm + SM::OFF_BM + (g & 1u) * 1024u;
                        *(uint32_t *)(BM + pm_sw32_off(tk, 0) + 4u * q) = bl;
                        *(uint32_t *)(BM + pm_sw32_off(tk, 1) + 4u * q) = bh;
                    }
                }
                pm_fence_proxy_async(); /* generic-proxy writes before the MMA reads them */
                __syncwarp();
                if (lane == 0) pm_mbar_arrive(&a_full[ab]);
            }
        }
        if (fail) atomicOr(&s_fail, 1u);
    } else if (warp == PM_I8_MMA_WARP) {
        /* ===== MMA issue ===== */
        if (lane == 0) {
            bool ok = true;
            pm_i8_task t;
            uint32_t N = 16;
            for (uint32_t g = 0; g < G && ok; g++) {
                const uint32_t sb = g % nsb, x = g % PM_I8_AC;
                if (sb == 0) {
                    pm_i8_task_get<NM>(a, task0 + (g / nsb) * gridDim.x, nrb, nsb, n_tiles, t);
                    N = t.nt > 16u ? 32u : 16u;
                }
                if (g >= PM_I8_AC && !pm_mbar_wait(&acc_empty[x], ((g / PM_I8_AC) - 1u) & 1u, a.err, a.wait)) {
                    ok = false;
                    break;
                }
                pm_tc_fence_after();
                const uint32_t idesc = pm_idesc_i8(128, N), udesc = pm_idesc_u8(128, N);
                for (uint32_t h = 0; h < 2; h++) {
                    const uint32_t c = 2u * g + h, ab = c % SM::NAB;
                    if (!pm_mbar_wait(&a_full[ab], (c / SM::NAB) & 1u, a.err, a.wait)) {
                        ok = false;
                        break;
                    }
                    pm_tc_fence_after();
                    const uint64_t bd = pm_desc_sw128(sm + SM::OFF_B + ab * 4096u);
#pragma unroll
                    for (int mm = 0; mm < NMA; mm++) {
                        const uint64_t ad = pm_desc_sw128(sm + SM::OFF_A + (ab * NMA + (uint32_t)mm) * SM::A);
                        const uint32_t d = tmem + x * (NMA * 64u) + (uint32_t)mm * 64u;
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; kk++)
                            pm_mma_i8(d, ad + 2 * kk, bd + 2 * kk, idesc, (h > 0 || kk > 0) ? 1u : 0u);
                        if (h == 0u) /* msum + 2048 sum m into the slot's second 32 columns */
                            pm_mma_i8(d + 32u, pm_desc_sw32(sm + SM::OFF_AM + ((g & 1u) * NMA + (uint32_t)mm) * 4096u),
                                      pm_desc_sw32(sm + SM::OFF_BM + (g & 1u) * 1024u), udesc, 0u);
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
        /* ===== epilogue: warps 8-15; warp w reads tensor-memory lanes 32 (w % 4) .. + 31 and
         * tokens 16 ((w - 8) / 4) .. + 15 of the tile ===== */
        const uint32_t lq = warp & 3u, row = lq * 32u + lane, k0 = 16u * ((warp - 8u) >> 2);
        float acc[NMA][16];
#pragma unroll
        for (int mm = 0; mm < NMA; mm++)
#pragma unroll
            for (uint32_t k = 0; k < 16; k++) acc[mm][k] = 0.0f;
        pm_i8_task t;
        for (uint32_t g = 0; g < G; g++) {
            const uint32_t sb = g % nsb, x = g % PM_I8_AC;
            if (sb == 0) pm_i8_task_get<NM>(a, task0 + (g / nsb) * gridDim.x, nrb, nsb, n_tiles, t);
            if (__any_sync(0xffffffffu, !pm_mbar_wait(&acc_full[x], (g / PM_I8_AC) & 1u, a.err, a.wait))) {
                atomicOr(&s_fail, 1u);
                break;
            }
            pm_tc_fence_after();
            const bool active = k0 < t.nt; /* warp-uniform */
            if (active) {
#pragma unroll
                for (int mm = 0; mm < NMA; mm++) {
                    int32_t v[16], mv[16];
                    const uint32_t tc = tmem + ((lq * 32u) << 16) + x * (NMA * 64u) + (uint32_t)mm * 64u + k0;
                    pm_tmem_ld16i2(tc, tc + 32u, v, mv);
                    const uint4 s0 = ((const uint4 *)(sm + SM::OFF_SIDE))[(x * NMA + (uint32_t)mm) * 128u + row];
                    const float d = __uint_as_float(s0.x), dm = __uint_as_float(s0.y);
                    const int corr = (int)s0.z;
                    const float4 *yq = (const float4 *)(sm + SM::OFF_ASIDE) + (x * PM_I8_N + k0) / 4u;
                    float yds[16];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 f = yq[i];
                        yds[4 * i] = f.x, yds[4 * i + 1] = f.y, yds[4 * i + 2] = f.z, yds[4 * i + 3] = f.w;
                    }
                    /* all 16 columns, branch-free (independent chains): the terms of tokens past
                     * nt are never written out */
#pragma unroll
                    for (uint32_t k = 0; k < 16; k++) {
                        const float yd = yds[k];
                        const int msum = mv[k] - corr;
                        /* total += yd xd isum - yd xmin msum (cpu_dot.rs:732-767, q2_K) */
                        const float term = __fsub_rn(__fmul_rn(__fmul_rn(yd, d), (float)v[k]),
                                                     __fmul_rn(__fmul_rn(yd, dm), (float)msum));
                        acc[mm][k] = __fadd_rn(acc[mm][k], term);
                    }
                }
            }
            pm_tc_fence_before();
            __syncwarp();
            if (lane == 0) pm_mbar_arrive(&acc_empty[x]);
            if (sb == nsb - 1u && active) { /* the task's rows are complete: outputs, in the CPU lane's order */
                const uint32_t grow = t.row0 + row; /* gate/up; down rows are grow + 128 mm */
#pragma unroll
                for (uint32_t k = 0; k < 16; k++) {
                    if (k0 + k < t.nt) {
                        const uint32_t pr = __ldcg(a.pairs + t.s0 + k0 + k);
                        if (NM == 2) {
                            float gg = acc[0][k], uu = acc[1][k];
                            if (a.gate_b) gg = __fadd_rn(gg, a.gate_b[(uint64_t)t.e * a.Fr + grow]);
                            if (a.up_b) uu = __fadd_rn(uu, a.up_b[(uint64_t)t.e * a.Fr + grow]);
                            a.mid[(uint64_t)pr * a.Fmax + grow] = __fmul_rn(pm_glu(gg, uu, a.act), __ldcg(a.w + pr));
                        } else {
#pragma unroll
                            for (int mm = 0; mm < NMA; mm++) a.partial[(uint64_t)pr * a.H + grow + 128u * mm] = acc[mm][k];
                        }
                    }
#pragma unroll
                    for (int mm = 0; mm < NMA; mm++) acc[mm][k] = 0.0f;
                }
            }
        }
    }
    pm_tc_fence_before();
    __syncthreads();
    pm_tc_fence_after();
    if (warp == PM_I8_MMA_WARP) {
        __syncwarp();
        pm_tmem_free(tmem, SM::TMEM_COLS);
    }
    if (tid == 0 && s_fail) atomicOr(a.err, PM_ERR_TIMEOUT);
}

/* q8_K of the mid rows of every tile pair (the down pass's B operand), the
 * CPU lane's quantizer (cpu_dot.rs:26-50); blocks (tile, y), warp per (token,
 * 256-block) */
static __global__ void __launch_bounds__(256) pm_i8_midq_kernel(const __grid_constant__ pm_layer_args a) {
    const uint32_t tile = blockIdx.x;
    if (tile >= __ldcg(a.n_items + 7)) return;
    const uint2 tt = __ldcg(a.i8_tile + tile);
    const uint32_t s0 = __ldcg(a.item_start + tt.x), cnt = __ldcg(a.item_start + tt.x + 1) - s0;
    const uint32_t nt = cnt - tt.y < PM_I8_N ? cnt - tt.y : PM_I8_N;
    const uint32_t nb = (a.Fr + 255u) / 256u;
    const uint32_t nw = (blockDim.x >> 5) * gridDim.y; /* the tile's jobs spread over gridDim.y blocks */
    for (uint32_t job = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5); job < nt * nb; job += nw) {
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
    const uint32_t smem = pm_i8_smem<2>::TOTAL + 1024u;
    if (!pm_smem_attr(k, smem, &done)) return 0;
    k<<<a.n_sm, PM_I8_THREADS, smem, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer integer tensor-core launch");
}

static int pm_i8_midq_launch(const pm_layer_args &a, cudaStream_t st) {
    pm_i8_midq_kernel<<<dim3(a.max_i8, 8), 256, 0, st>>>(a);
    return pm_ok(cudaGetLastError(), "moe layer integer tensor-core mid q8_K launch");
}
