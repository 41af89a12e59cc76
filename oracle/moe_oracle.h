/*
 * moe_oracle.h -- CPU restatement of tt-lab's gpt-oss MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This header and moe_oracle.c are the checker that
 * the parity tests, the smoke check and the CPU-baseline leg of the benchmark
 * compare the CUDA path against.  Nothing in the product library links or calls
 * this code.
 *
 * Every function restates one piece of the reference (tenstorrent/tt-lab) and
 * cites the file:line it follows.  Floating-point order is kept exactly:
 * products are rounded before the add unless the reference uses an explicit
 * fused multiply-add (the reference builds with -ffp-contract=off).  The
 * reference's MXFP4 kernels exist as two ISA clones with different rounding
 * (src/tensor.cpp:239-304 and :319-495); both are restated and selected with
 * `isa` (OREF_ISA_V4 = AVX-512 clone, OREF_ISA_DEFAULT = scalar clone).
 *
 * Parity of this restatement is pinned two ways (tests/test_oracle.py):
 *   - the reference's own known-answer vectors (tests/host_dispatch.cpp:92-127,
 *     src/tests.cpp:42);
 *   - bit-exact agreement with the reference compiled from its own sources
 *     (oracle/_ref, built by oracle/Makefile) on seeded inputs.
 */
#ifndef TTL_MOE_ORACLE_H
#define TTL_MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OREF_ISA_DEFAULT = 0, OREF_ISA_V4 = 1 };

enum {
    OREF_DIM = 2880,                /* src/model.h:34, :43 */
    OREF_BLOCKS = 90,               /* src/tensor.cpp:78 */
    OREF_ROW_BYTES = 1530,          /* src/tensor.cpp:79 (90 blocks x 17 B) */
    OREF_TOPK = 4,                  /* src/model.h:42 */
    OREF_MATVEC_SELECTED_MAX = 4    /* src/model.cpp:22 */
};

/* One MoE layer, all arrays in GGUF order (src/model.cpp:157-169). */
typedef struct {
    size_t experts;            /* E: 32 (20b) or 128 (120b) */
    const float *router_w;     /* [E][2880] f32, ffn_gate_inp.weight */
    const float *router_b;     /* [E] f32, ffn_gate_inp.bias */
    const uint8_t *gate_w;     /* [E][2880 rows][90 blocks][17 B] MXFP4 */
    const uint8_t *up_w;
    const uint8_t *down_w;
    const float *gate_b;       /* [E][2880] f32 */
    const float *up_b;
    const float *down_b;
} oref_layer;

float oref_mxfp4_scale(uint8_t exponent);
void oref_matvec_add_f32(const float *w, const float *bias, const float *x, float *y, size_t rows, size_t cols);
void oref_matvec_add_mxfp4(const uint8_t *w_expert, const float *bias_expert, const float *x, float *y, int isa);
void oref_matmul_add_mxfp4_selected(const uint8_t *w_expert, const float *bias_expert, const float *xt,
                                    const size_t *tokens, size_t n, float *out, int isa);
void oref_select_top4(const float *logits, size_t experts, int32_t idx[4]);
void oref_softmax4(const float *logits, const int32_t idx[4], float w[4]);
float oref_swiglu(float gate, float up);
void oref_rms_norm(const float *x, const float *g, float eps, float *out, size_t n);

/* Decode MoE for one token (src/model.cpp:292-338).  idx/w may be NULL. */
void oref_moe_decode(const oref_layer *layer, const float *x, float *out, int32_t *idx, float *w, int isa);
/* Prefill MoE for T tokens (src/model.cpp:340-461).  Returns 0, or -1 on
 * allocation failure.  idx/w ([T][4]) may be NULL. */
int oref_moe_prefill(const oref_layer *layer, const float *x, size_t tokens, float *out, int32_t *idx, float *w,
                     int isa);

/* Output head (src/model.cpp:598-612): y = matvec_q8_0(w, x) over `rows`
 * rows of 2880 columns (src/tensor.cpp:202-218), greedy argmax, and the exact
 * half -> float conversion the Q8_0 scales use (src/tensor.cpp:163-165). */
void oref_matvec_q8_0(const uint8_t *w, const float *x, float *y, size_t rows);
int32_t oref_greedy(const float *logits, size_t n);
float oref_half_to_float(uint16_t h);

/* Attention block (oracle/attn_oracle.c; src/model.cpp:578-590 with the
 * constants of src/model.h:36-50). */
enum {
    OREF_HEAD_SIZE = 64,
    OREF_QUERY_HEADS = 64,
    OREF_KV_HEADS = 8,
    OREF_QUERY_WIDTH = 4096,
    OREF_KV_WIDTH = 512,
    OREF_SLIDING_WINDOW = 128
};
typedef struct {
    const float *attn_norm;                 /* [2880] attn_norm.weight */
    const uint8_t *q_w; const float *q_b;   /* Q8_0 [4096 rows][90 blocks][34 B]; [4096] */
    const uint8_t *k_w; const float *k_b;   /* [512 rows]; [512] */
    const uint8_t *v_w; const float *v_b;   /* [512 rows]; [512] */
    const uint8_t *o_w; const float *o_b;   /* Q8_0 [2880 rows][128 blocks][34 B]; [2880] */
    const float *sinks;                     /* [64] attn_sinks.weight */
} oref_attn_layer;

void oref_matvec_add_q8_0(const uint8_t *w, const float *bias, const float *x, float *y, size_t rows,
                          size_t cols);
void oref_rope_frequencies(float freq[OREF_HEAD_SIZE / 2]);
void oref_apply_rope(float *v, size_t heads, size_t position, const float freq[OREF_HEAD_SIZE / 2]);
void oref_attention(size_t layer_index, size_t position, const float *q, const float *k_cache, const float *v_cache,
                    const float *sinks, float *scores, float *out);
int oref_attention_step(const oref_attn_layer *layer, size_t layer_index, size_t position, float *k_cache,
                        float *v_cache, size_t capacity, const float *x, float *residual, float *attended);

#ifdef __cplusplus
}
#endif
#endif
