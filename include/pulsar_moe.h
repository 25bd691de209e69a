/* pulsar_moe.h - C ABI of the B200 (sm_100a) routed-expert FFN library
 * libpulsar_moe.so.
 *
 * Part 1 replaces, symbol for symbol, the MoE entries of pulsar's kernel
 * library crates/kernels/cuda/pulsar_kernels.cu (bound from Rust in
 * crates/kernels/src/lib.rs:78-200).  Same C signatures, same argument
 * meaning, same convention: every call returns 1 on success and 0 on
 * failure (invalid arguments or a launch error), launches are
 * asynchronous on the calling thread's default stream (per-thread default
 * stream, as crates/kernels/build.rs:42-48 builds it), nothing allocates,
 * so the calls are graph-capturable.
 *
 * All pointers are device pointers owned by the caller.  Expert slabs keep
 * the crates/quant block layouts (gguf/src/lib.rs:145-170); slab e of a
 * tensor sits at base + e * rows * row_bytes (crates/engine/src/lib.rs:
 * 576-592).  q8_K activation buffers use the 292-byte block of the
 * reference (cu:1492), ceil(dim / 256) blocks per row.
 *
 * Supported expert formats (quant codes of crates/kernels/src/lib.rs:
 * 55-73): Q2_K = 0, IQ2_XXS = 1, Q4_K = 2, Q8_0 = 10, MXFP4 = 12.  Any
 * other code returns 0.
 *
 * Part 2 adds entry points with no single-call counterpart in the
 * reference: the fused router, the fused whole-layer call with a caller
 * workspace, and the GPU block encoders.
 */
#ifndef PULSAR_MOE_H
#define PULSAR_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PULSAR_QUANT_Q2_K 0u
#define PULSAR_QUANT_IQ2_XXS 1u
#define PULSAR_QUANT_Q4_K 2u
#define PULSAR_QUANT_Q8_0 10u
#define PULSAR_QUANT_MXFP4 12u

/* One (token, slot) of an MoE call: explicit device pointers to the
 * expert's slabs; NULL gate/up writes a zero mid row, NULL down skips the
 * slot.  48 bytes, identical to pulsar_expert_ptrs (cu:2555-2563) and
 * ExpertPtrs (crates/kernels/src/lib.rs:21-48). */
typedef struct pulsar_expert_ptrs {
    const void *gate;
    const void *up;
    const void *down;
    const float *gate_b; /* [mid_dim] or NULL */
    const float *up_b;   /* [mid_dim] or NULL */
    const float *down_b; /* [out_dim] or NULL */
} pulsar_expert_ptrs;

/* ======================================================================
 * Part 1 - reference entry points (crates/kernels/cuda/pulsar_kernels.cu)
 * ====================================================================== */

/* replaces cu:1052 pulsar_router_select (klib:118).  selected int32
 * [n_tok][k_used(+n_shexp)], weights f32 likewise, logits f32
 * [n_tok][n_expert(+n_shexp)], bias f32 [n_expert] (NULL = zeros).
 * softmax_mode 0 sigmoid + bias, 1 softmax over the selected logits,
 * 2 sink.  Ties go to the lower expert index.  n_expert <= 4096. */
int pulsar_router_select(void *selected, void *weights, const void *logits, const void *bias, uint32_t n_expert,
                         uint32_t k_used, float weight_scale, uint32_t n_tok, uint32_t softmax_mode,
                         uint32_t n_shexp);

/* replaces cu:1552 pulsar_quantize_q8_K (klib:119): f32 [n_rows][in_dim]
 * -> q8_K [n_rows][ceil(in_dim/256)], quantized like the CPU expert lane
 * (crates/quant/src/cpu_dot.rs:26: d = amax/127, round half away). */
int pulsar_quantize_q8_K(void *out, const void *x, uint32_t in_dim, uint32_t n_rows);

/* replaces cu:5149 pulsar_moe_pair_swiglu (klib:124):
 * mid[t][s][r] = glu(gate_r . xq[t] + gate_b, up_r . xq[t] + up_b) * weights[t][s] */
int pulsar_moe_pair_swiglu(void *mid, const void *ptrs, const void *weights, const void *xq, uint32_t in_dim,
                           uint32_t mid_dim, uint32_t n_used, uint32_t n_tok, uint64_t row_bytes, uint32_t quant,
                           uint32_t act_op);

/* replaces cu:5289 pulsar_moe_down (klib:125):
 * out[t][r] = sum over slots s (in order) of down_r(s) . midq[t][s] */
int pulsar_moe_down(void *out, const void *ptrs, const void *midq, uint32_t mid_dim, uint32_t out_dim,
                    uint32_t n_used, uint32_t n_tok, uint64_t row_bytes, uint32_t quant);

/* replaces cu:3483 pulsar_moe_pair_swiglu_grouped (klib:126): gptrs
 * [n_group], starts u32 [n_group+1], pairs u32 (token << 4 | slot) */
int pulsar_moe_pair_swiglu_grouped(void *mid, const void *gptrs, const void *starts, const void *pairs,
                                   const void *weights, const void *xq, uint32_t in_dim, uint32_t mid_dim,
                                   uint32_t n_used, uint32_t n_group, uint64_t row_bytes, uint32_t quant,
                                   uint32_t act_op);

/* replaces cu:3537 pulsar_moe_down_grouped (klib:127): partial f32
 * [n_tok][n_used][out_dim], written for the grouped pairs only */
int pulsar_moe_down_grouped(void *partial, const void *gptrs, const void *starts, const void *pairs,
                            const void *midq, uint32_t mid_dim, uint32_t out_dim, uint32_t n_used, uint32_t n_group,
                            uint64_t row_bytes, uint32_t quant);

/* replaces cu:3651 pulsar_moe_slot_sum (klib:128) */
int pulsar_moe_slot_sum(void *out, const void *partial, uint32_t out_dim, uint32_t n_used, uint32_t n_tok);

/* replaces cu:3640 pulsar_moe_down_bias (klib:129): out += sum_s w_s * down_b_s */
int pulsar_moe_down_bias(void *out, const void *ptrs, const void *weights, uint32_t out_dim, uint32_t n_used,
                         uint32_t n_tok);

/* replaces cu:3631 pulsar_add_bias_rows: x[r][i] += bias[i] */
int pulsar_add_bias_rows(void *x, const void *bias, uint32_t dim, uint32_t rows);

/* replaces cu:6526 pulsar_matmul_f32 (klib:93), the router logits GEMV:
 * out[t][r] = W[r] . x[t] accumulated in f32 fused multiply-adds in a fixed order */
int pulsar_matmul_f32(void *out, const void *w, const void *x, uint32_t in_dim, uint32_t out_dim, uint32_t n_tok);

/* replaces cu:6494 pulsar_rms_norm (klib:88): out = x / rms(x) * w per
 * row (w may be NULL = ones); the normalisation ahead of an FFN layer */
int pulsar_rms_norm(void *out, const void *x, const void *w, uint32_t n, uint32_t rows, float eps);

/* replaces cu:6551 pulsar_swiglu (klib:111) */
int pulsar_swiglu(void *out, const void *gate, const void *up, uint32_t n, float clamp, float weight,
                  uint32_t act_op);

/* replaces cu:6754 pulsar_add (klib:114) */
int pulsar_add(void *out, const void *a, const void *b, uint32_t n);

/* replace cu:1271 / cu:6421 (klib:145-146, run by tests/selftests.rs):
 * device results against this library's host mirrors; 1 = pass */
int pulsar_router_selftest(void);
int pulsar_moe_selftest(void);

/* ======================================================================
 * Part 2 - additions
 * ====================================================================== */

/* Router GEMV fused with top-k: logits = W x (+ logit_bias), then
 * selection as pulsar_router_select modes 0/1, optionally group-limited
 * (n_group > 1: keep the topk_group groups whose two best scores sum
 * highest).  logits [n_tok][n_expert] is an output.  stream: a
 * cudaStream_t, NULL = per-thread default stream.  No reference
 * counterpart as a single call (it is matmul_f32 + add_bias_rows +
 * router_select, cu:6526 + cu:3631 + cu:1052). */
int pulsar_router_logits_select(void *selected, void *weights, void *logits, const void *x, const void *w,
                                const void *logit_bias, const void *select_bias, uint32_t in_dim, uint32_t n_expert,
                                uint32_t k_used, float weight_scale, uint32_t n_tok, uint32_t mode, uint32_t n_group,
                                uint32_t topk_group, void *stream);

/* One MoE layer (the Ffn::Moe arm of crates/engine/src/lib.rs:7537-8705:
 * router -> q8_K -> gate/up + glu -> q8_K -> down -> combine) as one call,
 * with the expert resolve done on the device: no host round trip. */
typedef struct pulsar_moe_layer_desc {
    uint32_t n_embd;      /* H */
    uint32_t n_ff;        /* F, routed expert intermediate */
    uint32_t n_expert;    /* E */
    uint32_t n_used;      /* k */
    uint32_t quant;       /* routed expert format (gate, up, down) */
    uint32_t act_op;      /* glu op (cu:124) */
    uint32_t router_mode; /* 0 sigmoid + selection bias, 1 softmax */
    uint32_t n_group;     /* group-limited routing: groups (0/1 = off) */
    uint32_t topk_group;  /* groups kept */
    float weight_scale;   /* expert_weight_scale */
    uint64_t row_bytes_gu, row_bytes_down;     /* routed row bytes */
    uint64_t expert_stride_gu, expert_stride_down; /* bytes between experts; 0 = rows * row_bytes */
    const void *gate, *up, *down;              /* routed slabs [E] */
    const float *gate_b, *up_b, *down_b;       /* [E][F], [E][F], [E][H] or NULL */
    const float *router_w;                     /* [E][H] f32 */
    const float *router_logit_b;               /* [E] added to the logits, or NULL */
    const float *router_select_b;              /* [E] added to the selection score, or NULL */
    /* always-on shared expert (weight 1.0), n_shared 0 or 1 */
    uint32_t n_shared;
    uint32_t shared_quant;
    uint32_t shared_n_ff;
    uint32_t expert_lo, expert_hi; /* experts computed here: [lo, hi); hi = 0 -> all */
    uint64_t shared_row_bytes_gu, shared_row_bytes_down;
    const void *shared_gate, *shared_up, *shared_down;
    /* limit of each device wait on a copy or MMA stage, in SM cycles; 0 =
     * the default (2^31, about one second).  A wait that runs out sets bit 0
     * of the call's error word, the kernel drains what it has in flight and
     * returns; the output of that call is then invalid. */
    uint64_t wait_cycles;
    /* qwen35 shared-expert gate (crates/engine/src/real/qwen35.rs:2167-2169):
     * [n_embd] f32 or NULL.  With it, the shared expert's output row of
     * token t is scaled by sigmoid(shared_gate_w . x[t]) before it joins the
     * routed sum (the dot in the router's fixed f32 order). */
    const float *shared_gate_w;
    /* PULSAR_LAYER_* path flags (0 = the default paths) */
    uint32_t path_flags;
    /* Q2_K tile-plane images of gate, up and down (pulsar_repack_q2k_tiles;
     * based like gate/up/down: expert e's image at base + e x its GGUF
     * bytes), or NULL.  The integer tensor-core passes read these; without
     * them a Q2_K layer keeps to the dp4a and fp16 tensor-core paths. */
    const void *gate_tiles, *up_tiles, *down_tiles;
} pulsar_moe_layer_desc;

/* Load-time repack of Q2_K expert matrices into tile planes (the GGUF
 * bytes stay the interchange format; this is the device image the integer
 * tensor-core passes stream).  src: n_mat matrices of `rows` GGUF Q2_K rows
 * of `cols` values (row_bytes apart, mat_stride bytes between matrices);
 * dst: n_mat x rows x row_bytes(cols) bytes, 16-byte aligned.  Per
 * (matrix, 128-row block, 256-value super-block) one contiguous chunk of
 * 10752 bytes: qs as [4 x 16-byte units][128 rows], then the 16 scale
 * bytes of each row, then each row's d and dmin (f16).  rows % 128 == 0
 * and cols % 256 == 0.  Returns 1 (launched on `stream`) or 0. */
int pulsar_repack_q2k_tiles(void *dst, const void *src, uint32_t n_mat, uint32_t rows, uint32_t cols,
                            uint64_t row_bytes, uint64_t mat_stride, void *stream);

/* path_flags: keep routed Q2_K experts off the integer tensor-core passes
 * (dp4a engine / fp16 tensor-core tiles instead), or put them there even
 * below the default threshold of one routed token per expert on average; for
 * comparisons and tests */
#define PULSAR_LAYER_NO_I8 1u
#define PULSAR_LAYER_FORCE_I8 2u

/* pulsar_rms_norm on an explicit stream (cudaStream_t, NULL = per-thread default) */
int pulsar_rms_norm_stream(void *out, const void *x, const void *w, uint32_t n, uint32_t rows, float eps,
                           void *stream);

/* bytes of workspace pulsar_moe_layer needs for up to max_tok tokens */
size_t pulsar_moe_layer_workspace(const pulsar_moe_layer_desc *d, uint32_t max_tok);

/* out[t] = (residual ? residual[t] : 0) + moe(x[t]) for n_tok tokens.
 * x, out, residual f32 [n_tok][n_embd] (out may alias residual).  ws is
 * caller device memory of pulsar_moe_layer_workspace bytes; it carries
 * state between the layer's kernels only (the call's first kernel clears
 * its control words), so one ws serves any number of sequential calls on
 * one stream, of any n_tok and descriptor that fit it.  stream:
 * cudaStream_t or NULL. */
int pulsar_moe_layer(const pulsar_moe_layer_desc *d, float *out, const float *x, const float *residual,
                     uint32_t n_tok, void *ws, size_t ws_bytes, void *stream);

/* pulsar_moe_layer for callers that cannot allocate device memory (a
 * plugin inside a host that owns all device memory through its own pool,
 * or code that must not call cudaMalloc while it runs).  No counterpart in
 * the reference.  The workspace is a fixed 32 MiB array inside the library,
 * held by every GPU that loads it until the process exits; a call whose
 * workspace (pulsar_moe_layer_workspace) exceeds 32 MiB returns 0 with a
 * message.  Every call looks up the array's address on the current device;
 * the first call on a device also loads the library's module there, so make
 * that first call before any stream capture.  Every call shares the one
 * array: calls that overlap on the GPU (other streams, other threads) race
 * and must be serialised by the caller.  The call's error word is read with
 * pulsar_moe_layer_ws_view(d, n_tok, NULL, &view).  Allocates nothing. */
int pulsar_moe_layer_noalloc(const pulsar_moe_layer_desc *d, float *out, const float *x, const float *residual,
                             uint32_t n_tok, void *stream);

/* Expert parallel over `world` GPUs, one process (or thread) per GPU, one
 * call per rank with the same descriptor shapes and n_tok (north star:
 * experts sharded over the box, NCCL dispatch / combine over NVLink; the
 * reference's tier launches crates/engine/src/lib.rs:8395-8450 and their
 * gather :8620-8638 do the same job across its CPU / GPU / NVMe tiers).
 * d->expert_lo, expert_hi name this rank's experts (the ranks' ranges
 * partition [0, n_expert)); its routed slabs need hold only those.  Each
 * rank routes its own n_tok tokens, the (q8_K rows, expert ids, route
 * weights) of every rank's tokens are all-gathered, every rank runs its
 * experts for all tokens that chose them plus its shared expert for its own
 * tokens, and the per-token sums are reduce-scattered back to the token
 * owners: out[t] = residual[t] + moe(x[t]) for this rank's tokens.
 * nccl_comm: an ncclComm_t of the world (pulsar_ep_comm_init, or the
 * caller's own, from the same NCCL library); all collectives run on
 * `stream`, so the call stays capturable into a CUDA graph.  world 1 is a
 * plain pulsar_moe_layer call.  Workspace: pulsar_moe_layer_ep_workspace;
 * pulsar_moe_layer_ws_view describes it for n_tok * world tokens. */
size_t pulsar_moe_layer_ep_workspace(const pulsar_moe_layer_desc *d, uint32_t world, uint32_t max_tok);
int pulsar_moe_layer_ep(const pulsar_moe_layer_desc *d, void *nccl_comm, uint32_t rank, uint32_t world,
                        float *out, const float *x, const float *residual, uint32_t n_tok, void *ws, size_t ws_bytes,
                        void *stream);
/* NCCL communicator helpers for pulsar_moe_layer_ep: rank 0 makes the
 * 128-byte id, the caller hands it to every rank, each rank (with its GPU
 * current) creates its communicator */
int pulsar_ep_unique_id(void *id);
int pulsar_ep_comm_init(void **comm, const void *id, uint32_t world, uint32_t rank);
int pulsar_ep_comm_destroy(void *comm);

/* device pointers into a layer workspace after a call, for inspection.
 * ws NULL describes the built-in array of pulsar_moe_layer_noalloc on the
 * current device (so its callers can read the call's error word). */
typedef struct pulsar_moe_ws_view {
    float *logits;        /* [n_tok][E] */
    int32_t *selected;    /* [n_tok][n_slot] (routed slots, then shared ids E + s) */
    float *weights;       /* [n_tok][n_slot] */
    void *xq;             /* q8_K [n_tok][ceil(H/256)] */
    float *mid;           /* [n_tok * n_slot][F_max] */
    uint32_t *err;        /* error word: bit 0 wait timeout */
    uint32_t *n_items;    /* [0] expert work items, [1] routed ones (distinct experts), [2] work units,
                           * [3] routed work units, [4] tensor-core tiles, [5] their gate/up K splits */
    uint32_t *item_expert, *item_start, *pairs; /* CSR of (token, slot) pairs by expert */
    uint32_t *work_item, *work_t0;              /* work units: (item, first token of its chunk) */
    float *partial;                             /* [n_tok * n_slot][H] down rows before the combine */
    uint32_t *tc_tile;                          /* tensor-core tiles: (item, first token) pairs of u32 */
    uint32_t n_slot, f_max;
    uint8_t *tc_img;        /* expanded tensor-core weight images of the last pass's last wave */
    uint8_t *tc_lo;         /* per image pair: 1 if its lo image was written */
    uint64_t tc_slot_bytes; /* bytes of one expert's images in tc_img */
    uint32_t tc_slots;      /* experts per wave */
    uint32_t max_tc;        /* tensor-core tile capacity */
} pulsar_moe_ws_view;
/* pulsar_moe_layer that also records events[0..5] (cudaEvent_t, NULL
 * entries skipped) around its kernels: before the router, after the
 * logits, after q8_K(x), after selection, after the gate/up weight passes,
 * after the mid q8_K (large batches), down and combine.  For per-kernel
 * timing; otherwise identical to pulsar_moe_layer. */
int pulsar_moe_layer_profiled(const pulsar_moe_layer_desc *d, float *out, const float *x, const float *residual,
                              uint32_t n_tok, void *ws, size_t ws_bytes, void *stream, void *const *events);

int pulsar_moe_layer_ws_view(const pulsar_moe_layer_desc *d, uint32_t max_tok, void *ws, pulsar_moe_ws_view *v);

/* GPU block encoders (crates/quant/src/lib.rs:251 q8_0, :271 q2_K,
 * :570 q4_K; iq.rs:227 iq2_xxs with importance qw or NULL = 1.0;
 * MXFP4 per the OCP MX rules): x f32 [rows][n] -> out [rows][row_bytes].
 * Byte-identical to the CPU encoders. */
int pulsar_quantize_rows(void *out, const void *x, const void *qw, uint32_t quant, uint64_t rows, uint32_t n,
                         void *stream);
uint64_t pulsar_row_bytes(uint32_t quant, uint32_t n);

/* Failure-detection check of the kernels' bounded device wait: one thread
 * waits on an mbarrier phase that nothing completes, with a limit of
 * `cycles` SM cycles (1 .. 2^31); the wait runs out, the kernel records the
 * timeout and returns.  Returns the error word (1 = timeout recorded, the
 * expected result), 0xffffffff on a launch error.  Synchronous; allocates
 * 4 bytes of device memory for the word. */
uint32_t pulsar_wait_selftest(uint64_t cycles);

/* reads and clears the error word of the Part-1 kernels (synchronous) */
uint32_t pulsar_b200_abi_error(void);

#ifdef __cplusplus
}
#endif
#endif
