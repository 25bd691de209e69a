/* oracle.h - CPU restatement of pulsar's routed-expert FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA implementation in pulsar_b200/: only tests/, __graft_entry__.smoke()
 * and the CPU-baseline leg of bench.py load it.  Nothing in the product
 * links or calls it.
 *
 * What it restates (reference paths are relative to the pulsar repo):
 *   encoders      crates/quant/src/lib.rs (q8_0 :251, q2_K :271, q4_K :570),
 *                 crates/quant/src/iq.rs:227 (iq2_xxs with imatrix), and an
 *                 MXFP4 encoder defined from the OCP MX rules (no encoder
 *                 exists in the reference; its decode is pinned by
 *                 crates/kernels/cuda/pulsar_kernels.cu:2053).
 *   q8_K          crates/quant/src/cpu_dot.rs:26 quantize_row_q8_k
 *   dots          cpu_dot.rs:92 (iq2_xxs), :250 (q4_K), :732 (q2_K); MXFP4 and
 *                 Q8_0 follow the reference GPU math (cu:2053, cu:2174)
 *   router        cu:939-1050 router_select_kernel semantics, logits from a
 *                 fixed-order binary64 dot (the contract the CUDA router keeps)
 *   expert FFN    crates/engine/src/lib.rs:1994-2101 (cpu_tier::Lane) plus
 *                 biases (cu:2604-2609, cu:3601) and shared experts as
 *                 always-on slots of weight 1.0
 */
#ifndef PM_ORACLE_H
#define PM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- encoders: n values -> row bytes; return bytes written ---- */
size_t orc_quantize_row_q8_0(const float *x, size_t n, uint8_t *out);
size_t orc_quantize_row_q2_k(const float *x, size_t n, uint8_t *out);
size_t orc_quantize_row_q4_k(const float *x, size_t n, uint8_t *out);
size_t orc_quantize_row_iq2_xxs(const float *x, const float *qw, size_t n, uint8_t *out);
size_t orc_quantize_row_mxfp4(const float *x, size_t n, uint8_t *out);
/* rows x n matrix, one call; quant = ORF_* code (the reference quant codes); qw may be NULL
 * (iq2_xxs then uses a uniform importance of 1.0) */
int orc_quantize_rows(int quant, const float *x, size_t rows, size_t n, const float *qw, uint8_t *out);
uint64_t orc_row_bytes(int quant, uint64_t n);

/* ---- decoders (f32 values, for the f64 known-answer tests) ---- */
int orc_dequant_row(int quant, const uint8_t *row, size_t n, float *out);

/* ---- q8_K activations (292-byte blocks, tail zero-padded) ---- */
void orc_quantize_q8k(const float *x, size_t n, void *out_blocks);
void orc_quantize_q8k_rows(const float *x, size_t n, size_t rows, void *out_blocks);

/* ---- one weight row . one q8_K row ---- */
float orc_vec_dot(int quant, const uint8_t *row, const void *xq_blocks, size_t n);

/* ---- glu (elib:2134 / cu:124) ---- */
float orc_glu(float g, float u, uint32_t act_op);

/* ---- router ---- */
void orc_router_logits(float *logits, const float *w, const float *x, const float *logit_bias,
                       uint32_t n_expert, uint32_t in_dim, uint32_t n_tok);
int orc_router_select(int32_t *selected, float *weights, const float *logits, const float *bias,
                      uint32_t n_expert, uint32_t k_used, float weight_scale, uint32_t n_tok,
                      uint32_t softmax_mode, uint32_t n_shexp, uint32_t n_group, uint32_t topk_group);

/* ---- expert FFN ---- */
typedef struct {
    const uint8_t *gate, *up, *down;         /* host rows; NULL gate/up -> mid 0, NULL down -> skip */
    const float *gate_b, *up_b, *down_b;      /* optional biases */
} orc_expert_ptrs;

/* The full FFN of the routed (and shared) slots for n_tok tokens.
 *   ptrs   [n_tok][n_slot] slot pointers (routed slots first, then shared)
 *   w      [n_tok][n_slot] slot weights (shared slots carry 1.0)
 *   quant  per-slot format code, row bytes per slot class:
 *          slots < n_routed use (quant_r, rb_gu_r, rb_down_r), the rest the
 *          shared triple
 *   out    [n_tok][H]
 *   mid_out (optional) [n_tok][n_slot][F_slot_max] f32 mids before q8_K
 * Threads: n_threads workers (0 = all cores), job split as the reference
 * lane (256-row gate/up jobs, 512-row down jobs). */
int orc_moe_ffn(float *out, float *mid_out, const orc_expert_ptrs *ptrs, const float *w,
                const float *x, uint32_t H, uint32_t n_tok, uint32_t n_slot, uint32_t n_routed,
                uint32_t F_r, uint32_t quant_r, uint64_t rb_gu_r, uint64_t rb_down_r,
                uint32_t F_s, uint32_t quant_s, uint64_t rb_gu_s, uint64_t rb_down_s,
                uint32_t act_op, int n_threads);

/* orf_expf / orf_sigmoid exported for the math tests */
float orc_expf(float x);
float orc_sigmoid(float x);
uint64_t orc_iq2xxs_grid(int i);

#ifdef __cplusplus
}
#endif
#endif
