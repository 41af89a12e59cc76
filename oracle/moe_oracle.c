/*
 * moe_oracle.c -- CPU restatement of tt-lab's gpt-oss MoE path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Build with -ffp-contract=off so every `a * b + c` below rounds the product
 * before the add, as the reference does (rules.py:6-7).  Fused operations are
 * written as explicit fmaf() where the reference uses _mm512_fmadd_ps.
 *
 * Citations are paths inside tenstorrent/tt-lab.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* 2 x E2M1 as small integers: src/tensor.cpp:34. */
static const int8_t kMxfp4Doubled[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* E8M0 byte -> 2^(e-128) as an f32 bit pattern, denormal for e < 2:
 * src/tensor.cpp:36-44.  Together with the doubled table this gives
 * value = E2M1(code) * 2^(e-127) for every byte, 255 included (2^127). */
float oref_mxfp4_scale(uint8_t exponent) {
    uint32_t bits;
    float out;
    if (exponent < 2) {
        bits = 0x00200000u << exponent;
    } else {
        bits = (uint32_t)(exponent - 1) << 23;
    }
    memcpy(&out, &bits, sizeof(out));
    return out;
}

/* Router matvec: src/tensor.cpp:186-200.  Sequential in the column, product
 * rounded before the add, bias first. */
void oref_matvec_add_f32(const float *w, const float *bias, const float *x, float *y, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) {
        float sum = bias[r];
        for (size_t c = 0; c < cols; ++c) {
            float p = w[r * cols + c] * x[c];
            sum = sum + p;
        }
        y[r] = sum;
    }
}

/* GCC's _mm512_reduce_add_ps (avx512fintrin.h __MM512_REDUCE_OP): halves,
 * then quarters, then pairs (0,2)(1,3), then the two survivors. */
static float reduce16(const float a[16]) {
    float t3[8], t6[4];
    for (int i = 0; i < 8; ++i) {
        t3[i] = a[8 + i] + a[i];
    }
    for (int i = 0; i < 4; ++i) {
        t6[i] = t3[4 + i] + t3[i];
    }
    float t8_0 = t6[0] + t6[2];
    float t8_1 = t6[1] + t6[3];
    return t8_0 + t8_1;
}

/* Expert matvec, one 2880x2880 slice.
 * v4 clone: src/tensor.cpp:239-256 with the block FMA :116-131 -- sixteen
 * lanes, x pre-multiplied by the block scale, fused multiply-add with the
 * doubled integer value, then the lane reduction and the bias added last.
 * default clone: src/tensor.cpp:258-304 -- one running sum per row seeded
 * with the bias, product (scale*value table entry, :58-71) rounded then added,
 * element i then element i+16 for each byte i of the block. */
void oref_matvec_add_mxfp4(const uint8_t *w_expert, const float *bias_expert, const float *x, float *y, int isa) {
    if (isa == OREF_ISA_V4) {
        for (size_t row = 0; row < OREF_DIM; ++row) {
            const uint8_t *data = w_expert + row * OREF_ROW_BYTES;
            float acc[16] = {0};
            for (size_t block = 0; block < OREF_BLOCKS; ++block) {
                const uint8_t *src = data + block * 17;
                const float scale = oref_mxfp4_scale(src[0]);
                const float *in = x + block * 32;
                for (int i = 0; i < 16; ++i) {
                    const float lo = (float)kMxfp4Doubled[src[1 + i] & 0x0f];
                    const float x0 = in[i] * scale;
                    acc[i] = fmaf(lo, x0, acc[i]);
                }
                for (int i = 0; i < 16; ++i) {
                    const float hi = (float)kMxfp4Doubled[src[1 + i] >> 4];
                    const float x1 = in[16 + i] * scale;
                    acc[i] = fmaf(hi, x1, acc[i]);
                }
            }
            y[row] = bias_expert[row] + reduce16(acc);
        }
        return;
    }
    for (size_t row = 0; row < OREF_DIM; ++row) {
        const uint8_t *data = w_expert + row * OREF_ROW_BYTES;
        float sum = bias_expert[row];
        for (size_t block = 0; block < OREF_BLOCKS; ++block) {
            const uint8_t *src = data + block * 17;
            const float multiplier = oref_mxfp4_scale(src[0]);
            const float *in = x + block * 32;
            for (int i = 0; i < 16; ++i) {
                const uint8_t packed = src[1 + i];
                const float w0 = multiplier * (float)kMxfp4Doubled[packed & 0x0f];
                const float w1 = multiplier * (float)kMxfp4Doubled[packed >> 4];
                float p0 = w0 * in[i];
                sum = sum + p0;
                float p1 = w1 * in[16 + i];
                sum = sum + p1;
            }
        }
        y[row] = sum;
    }
}

/* Selected-token expert matmul on a K-major gathered input xt[k * n + s].
 * v4: src/tensor.cpp:319-420 -- per token a fused multiply-add chain seeded
 * with the bias, weight = scale * value rounded first.  default:
 * src/tensor.cpp:422-495 -- same chain with the product rounded.  Row r of
 * token tokens[s] is written to out[tokens[s] * 2880 + r] (:413-418). */
void oref_matmul_add_mxfp4_selected(const uint8_t *w_expert, const float *bias_expert, const float *xt,
                                    const size_t *tokens, size_t n, float *out, int isa) {
    for (size_t row = 0; row < OREF_DIM; ++row) {
        const uint8_t *data = w_expert + row * OREF_ROW_BYTES;
        for (size_t s = 0; s < n; ++s) {
            float acc = bias_expert[row];
            for (size_t block = 0; block < OREF_BLOCKS; ++block) {
                const uint8_t *src = data + block * 17;
                const float scale = oref_mxfp4_scale(src[0]);
                for (int i = 0; i < 16; ++i) {
                    const uint8_t packed = src[1 + i];
                    const float w0 = scale * (float)kMxfp4Doubled[packed & 0x0f];
                    const float w1 = scale * (float)kMxfp4Doubled[packed >> 4];
                    const float x0 = xt[(block * 32 + (size_t)i) * n + s];
                    const float x1 = xt[(block * 32 + 16 + (size_t)i) * n + s];
                    if (isa == OREF_ISA_V4) {
                        acc = fmaf(w0, x0, acc);
                        acc = fmaf(w1, x1, acc);
                    } else {
                        float p0 = w0 * x0;
                        acc = acc + p0;
                        float p1 = w1 * x1;
                        acc = acc + p1;
                    }
                }
            }
            out[tokens[s] * OREF_DIM + row] = acc;
        }
    }
}

/* Top-4 by selection sort over a permuted index array: src/model.cpp:296-309
 * (prefill :350-364).  Strict '>' keeps the earlier *current* position on a
 * tie, so ties resolve by the permuted order the swaps leave behind. */
void oref_select_top4(const float *logits, size_t experts, int32_t idx[4]) {
    size_t order[128];
    for (size_t i = 0; i < experts; ++i) {
        order[i] = i;
    }
    for (size_t i = 0; i < OREF_TOPK; ++i) {
        size_t best = i;
        for (size_t j = i + 1; j < experts; ++j) {
            if (logits[order[j]] > logits[order[best]]) {
                best = j;
            }
        }
        size_t tmp = order[i];
        order[i] = order[best];
        order[best] = tmp;
        idx[i] = (int32_t)order[i];
    }
}

/* Softmax over the four selected logits: src/model.cpp:310-321.  std::max is
 * (a < b) ? b : a; the sum runs in rank order, then each weight is divided. */
void oref_softmax4(const float *logits, const int32_t idx[4], float w[4]) {
    float maximum = -INFINITY;
    for (int i = 0; i < OREF_TOPK; ++i) {
        const float v = logits[idx[i]];
        maximum = (maximum < v) ? v : maximum;
    }
    float sum = 0.0f;
    for (int i = 0; i < OREF_TOPK; ++i) {
        w[i] = expf(logits[idx[i]] - maximum);
        sum = sum + w[i];
    }
    for (int i = 0; i < OREF_TOPK; ++i) {
        w[i] = w[i] / sum;
    }
}

/* Clamped SwiGLU: src/model.cpp:328-332.  std::min(gate, 7) is
 * (7 < gate) ? 7 : gate (gate clamped above only); std::clamp(up, -7, 7). */
float oref_swiglu(float gate, float up) {
    const float x = (7.0f < gate) ? 7.0f : gate;
    const float y = (up < -7.0f) ? -7.0f : ((7.0f < up) ? 7.0f : up);
    const float t = -1.702f * x;
    const float e = expf(t);
    const float d = 1.0f + e;
    const float q = x / d;
    const float y1 = y + 1.0f;
    return q * y1;
}

/* RMSNorm: src/tensor.cpp:568-580.  Sequential sum of squares; the output is
 * (x * scale) * weight. */
void oref_rms_norm(const float *x, const float *g, float eps, float *out, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float p = x[i] * x[i];
        sum = sum + p;
    }
    const float scale = 1.0f / sqrtf(sum / (float)n + eps);
    for (size_t i = 0; i < n; ++i) {
        float t = x[i] * scale;
        out[i] = t * g[i];
    }
}

static const uint8_t *expert_slice(const uint8_t *w, size_t expert) {
    return w + expert * (size_t)OREF_DIM * OREF_ROW_BYTES;
}

/* Decode MoE: src/model.cpp:292-338. */
void oref_moe_decode(const oref_layer *L, const float *x, float *out, int32_t *idx_out, float *w_out, int isa) {
    float router[128];
    int32_t idx[4];
    float w[4];
    float gate[OREF_DIM], up[OREF_DIM], hidden[OREF_DIM], down[OREF_DIM];

    oref_matvec_add_f32(L->router_w, L->router_b, x, router, L->experts, OREF_DIM);
    oref_select_top4(router, L->experts, idx);
    oref_softmax4(router, idx, w);

    for (size_t i = 0; i < OREF_DIM; ++i) {
        out[i] = 0.0f;
    }
    for (int sel = 0; sel < OREF_TOPK; ++sel) {
        const size_t e = (size_t)idx[sel];
        oref_matvec_add_mxfp4(expert_slice(L->gate_w, e), L->gate_b + e * OREF_DIM, x, gate, isa);
        oref_matvec_add_mxfp4(expert_slice(L->up_w, e), L->up_b + e * OREF_DIM, x, up, isa);
        for (size_t i = 0; i < OREF_DIM; ++i) {
            hidden[i] = oref_swiglu(gate[i], up[i]);
        }
        oref_matvec_add_mxfp4(expert_slice(L->down_w, e), L->down_b + e * OREF_DIM, hidden, down, isa);
        for (size_t i = 0; i < OREF_DIM; ++i) {
            float p = w[sel] * down[i];
            out[i] = out[i] + p;
        }
    }
    if (idx_out) {
        memcpy(idx_out, idx, sizeof(idx));
    }
    if (w_out) {
        memcpy(w_out, w, sizeof(w));
    }
}

/* Prefill MoE: src/model.cpp:340-461.  Router per token (matmul_add_f32,
 * src/tensor.cpp:497-527, same per-token order as the matvec), per-token
 * top-4 and softmax, stable per-expert buckets in token order (:380-394),
 * then experts in ascending id: <= 4 tokens use the matvec, more use the
 * gathered matmul; SwiGLU; down; weighted scatter-add (:450-459). */
int oref_moe_prefill(const oref_layer *L, const float *x, size_t T, float *out, int32_t *idx_out, float *w_out,
                     int isa) {
    const size_t E = L->experts;
    const size_t D = OREF_DIM;
    int rc = -1;
    float *router = malloc(E * sizeof(float));
    int32_t *idx = malloc(T * 4 * sizeof(int32_t));
    float *wts = malloc(T * 4 * sizeof(float));
    size_t *counts = calloc(E, sizeof(size_t));
    size_t *buckets = malloc(E * T * sizeof(size_t));
    float *bucket_w = malloc(E * T * sizeof(float));
    float *gate = malloc(T * D * sizeof(float));
    float *up = malloc(T * D * sizeof(float));
    float *hidden = malloc(T * D * sizeof(float));
    float *down = malloc(T * D * sizeof(float));
    float *xt = malloc(T * D * sizeof(float));
    if (!router || !idx || !wts || !counts || !buckets || !bucket_w || !gate || !up || !hidden || !down || !xt) {
        goto done;
    }

    for (size_t t = 0; t < T; ++t) {
        oref_matvec_add_f32(L->router_w, L->router_b, x + t * D, router, E, D);
        oref_select_top4(router, E, idx + t * 4);
        oref_softmax4(router, idx + t * 4, wts + t * 4);
    }
    for (size_t i = 0; i < T * D; ++i) {
        out[i] = 0.0f;
    }
    for (size_t t = 0; t < T; ++t) {
        for (int r = 0; r < 4; ++r) {
            const size_t e = (size_t)idx[t * 4 + r];
            buckets[e * T + counts[e]] = t;
            bucket_w[e * T + counts[e]] = wts[t * 4 + r];
            ++counts[e];
        }
    }
    for (size_t e = 0; e < E; ++e) {
        const size_t n = counts[e];
        if (n == 0) {
            continue;
        }
        const size_t *sel = buckets + e * T;
        const float *selw = bucket_w + e * T;
        if (n <= OREF_MATVEC_SELECTED_MAX) {
            for (size_t s = 0; s < n; ++s) {
                const size_t t = sel[s];
                oref_matvec_add_mxfp4(expert_slice(L->gate_w, e), L->gate_b + e * D, x + t * D, gate + t * D, isa);
                oref_matvec_add_mxfp4(expert_slice(L->up_w, e), L->up_b + e * D, x + t * D, up + t * D, isa);
            }
        } else {
            for (size_t s = 0; s < n; ++s) {
                for (size_t k = 0; k < D; ++k) {
                    xt[k * n + s] = x[sel[s] * D + k];
                }
            }
            oref_matmul_add_mxfp4_selected(expert_slice(L->gate_w, e), L->gate_b + e * D, xt, sel, n, gate, isa);
            oref_matmul_add_mxfp4_selected(expert_slice(L->up_w, e), L->up_b + e * D, xt, sel, n, up, isa);
        }
        for (size_t s = 0; s < n; ++s) {
            const size_t t = sel[s];
            for (size_t i = 0; i < D; ++i) {
                hidden[t * D + i] = oref_swiglu(gate[t * D + i], up[t * D + i]);
            }
        }
        if (n <= OREF_MATVEC_SELECTED_MAX) {
            for (size_t s = 0; s < n; ++s) {
                const size_t t = sel[s];
                oref_matvec_add_mxfp4(expert_slice(L->down_w, e), L->down_b + e * D, hidden + t * D, down + t * D,
                                      isa);
            }
        } else {
            for (size_t s = 0; s < n; ++s) {
                for (size_t k = 0; k < D; ++k) {
                    xt[k * n + s] = hidden[sel[s] * D + k];
                }
            }
            oref_matmul_add_mxfp4_selected(expert_slice(L->down_w, e), L->down_b + e * D, xt, sel, n, down, isa);
        }
        for (size_t s = 0; s < n; ++s) {
            const size_t t = sel[s];
            const float ew = selw[s];
            for (size_t i = 0; i < D; ++i) {
                float p = ew * down[t * D + i];
                out[t * D + i] = out[t * D + i] + p;
            }
        }
    }
    if (idx_out) {
        memcpy(idx_out, idx, T * 4 * sizeof(int32_t));
    }
    if (w_out) {
        memcpy(w_out, wts, T * 4 * sizeof(float));
    }
    rc = 0;
done:
    free(router);
    free(idx);
    free(wts);
    free(counts);
    free(buckets);
    free(bucket_w);
    free(gate);
    free(up);
    free(hidden);
    free(down);
    free(xt);
    return rc;
}

/* ---- output head: rms_norm -> matvec_q8_0 -> greedy ----------------------- */

/* IEEE half -> float, exact (src/tensor.cpp:163-165 converts through
 * _Float16).  Subnormal halves are normalised; inf and NaN keep their class. */
static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 31u;
    uint32_t mant = h & 1023u;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                ++e;
                mant <<= 1;
            } while ((mant & 1024u) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 1023u) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

float oref_half_to_float(uint16_t h) {
    return half_to_float(h);
}

/* matvec_q8_0 (src/tensor.cpp:202-218 with q8_0_vector_fma_block :90-114):
 * a Q8_0 block is a half scale and 32 int8 quants (34 B).  Two 16-lane
 * accumulators take elements 0..15 and 16..31 of every block in block order,
 * each term rounded as (q * scale) * x, then lane-wise acc0 + acc1, then the
 * 16 lanes summed in order from 0.  rows x 2880 columns. */
void oref_matvec_q8_0(const uint8_t *w, const float *x, float *y, size_t rows) {
    const size_t blocks = OREF_DIM / 32;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *row = w + r * blocks * 34;
        float acc0[16] = {0}, acc1[16] = {0};
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *src = row + b * 34;
            const float scale = half_to_float((uint16_t)(src[0] | (src[1] << 8)));
            for (int i = 0; i < 16; ++i) {
                const float q0 = (float)(int8_t)src[2 + i] * scale;
                const float q1 = (float)(int8_t)src[18 + i] * scale;
                const float p0 = q0 * x[b * 32 + i];
                const float p1 = q1 * x[b * 32 + 16 + i];
                acc0[i] = acc0[i] + p0;
                acc1[i] = acc1[i] + p1;
            }
        }
        float sum = 0.0f;
        for (int i = 0; i < 16; ++i) {
            const float a = acc0[i] + acc1[i];
            sum = sum + a;
        }
        y[r] = sum;
    }
}

/* GptOssModel::greedy (src/model.cpp:604-612): the first index whose logit
 * is greater than every earlier one's, starting from index 0 (a NaN is never
 * greater, so NaNs are passed over, and a NaN at index 0 is never replaced). */
int32_t oref_greedy(const float *logits, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; ++i) {
        if (logits[i] > logits[best]) {
            best = i;
        }
    }
    return (int32_t)best;
}
