/*
 * attn_oracle.c -- CPU restatement of the attention block of tt-lab's
 * GptOssModel::forward (src/model.cpp:578-590).  TEST INFRASTRUCTURE ONLY:
 * the checker the attention parity tests compare the CUDA path against;
 * nothing in the product library links or calls it.
 *
 * Floating-point order follows the reference (built with -ffp-contract=off):
 * products rounded before adds, sequential sums, std::cos / std::sin /
 * std::exp as the float functions of the C library.  The Q8_0 matvec
 * restates the AVX-512 clone's lane order (two 16-lane accumulators, src/
 * tensor.cpp:220-237 with the block kernel it calls).  Pinned bit for bit
 * against the reference compiled from its own sources (tests/test_attn_oracle.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "moe_oracle.h"

static float h2f(uint16_t h) {
    return oref_half_to_float(h);
}

/* matvec_add_q8_0 (src/tensor.cpp:220-237): y[r] = bias[r] + the row's dot
 * product, accumulated in two 16-lane f32 accumulators (elements i and i+16
 * of each 32-element block) and reduced lane by lane. */
void oref_matvec_add_q8_0(const uint8_t *w, const float *bias, const float *x, float *y, size_t rows,
                          size_t cols) {
    const size_t blocks = cols / 32;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *row = w + r * blocks * 34;
        float acc0[16] = {0}, acc1[16] = {0};
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *src = row + b * 34;
            const float scale = h2f((uint16_t)(src[0] | (src[1] << 8)));
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
        y[r] = bias[r] + sum;
    }
}

/* The YaRN frequency table of the GptOssModel constructor
 * (src/model.cpp:123-138), with the constants of src/model.h:38-50. */
void oref_rope_frequencies(float freq[OREF_HEAD_SIZE / 2]) {
    const float head = (float)OREF_HEAD_SIZE;
    const float base = 150000.0f, scale = 1.0f / 32.0f, original = 4096.0f, fast = 32.0f, slow = 1.0f;
    const float pi = 3.14159265358979323846f;
    const float corr = head * logf(original / (fast * 2.0f * pi)) / (2.0f * logf(base));
    const float corr_slow = head * logf(original / (slow * 2.0f * pi)) / (2.0f * logf(base));
    const float low = fmaxf(0.0f, floorf(corr));
    const float high = fminf(head - 1.0f, ceilf(corr_slow));
    for (size_t pair = 0; pair < OREF_HEAD_SIZE / 2; ++pair) {
        const float dimension = (float)(pair * 2);
        const float theta_extrap = powf(base, -dimension / head);
        const float y = ((float)pair - low) / fmaxf(0.001f, high - low);
        float clamped = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
        const float ramp = 1.0f - clamped;
        const float a = scale * theta_extrap;
        const float b = a * (1.0f - ramp);
        const float c = theta_extrap * ramp;
        freq[pair] = b + c;
    }
}

/* apply_rope (src/model.cpp:230-245): each head's pairs (i, i + 32) rotated
 * by position * freq[i], both factors scaled by 1 + 0.1 ln(1 / rope_scale). */
void oref_apply_rope(float *v, size_t heads, size_t position, const float freq[OREF_HEAD_SIZE / 2]) {
    const float magnitude = 1.0f + 0.1f * logf(1.0f / (1.0f / 32.0f));
    for (size_t h = 0; h < heads; ++h) {
        float *values = v + h * OREF_HEAD_SIZE;
        for (size_t pair = 0; pair < OREF_HEAD_SIZE / 2; ++pair) {
            const float theta = (float)position * freq[pair];
            const float cosine = cosf(theta) * magnitude;
            const float sine = sinf(theta) * magnitude;
            const float x = values[pair];
            const float yv = values[pair + OREF_HEAD_SIZE / 2];
            const float xc = x * cosine, ys = yv * sine, xs = x * sine, yc = yv * cosine;
            values[pair] = xc - ys;
            values[pair + OREF_HEAD_SIZE / 2] = xs + yc;
        }
    }
}

/* attention_from_cache (src/model.cpp:255-290): per query head, scores
 * q.k / 8 over the layer's window (even layers: the last 128 positions), the
 * head's sink in the max and the denominator, weights = score / denominator
 * applied to V in position order.  dot (src/model.cpp:36-42) is sequential. */
void oref_attention(size_t layer_index, size_t position, const float *q, const float *k_cache, const float *v_cache,
                    const float *sinks, float *scores, float *out) {
    const size_t first =
        (layer_index % 2 == 0 && position + 1 > OREF_SLIDING_WINDOW) ? position + 1 - OREF_SLIDING_WINDOW : 0;
    const size_t count = position + 1 - first;
    const float scale = 1.0f / sqrtf((float)OREF_HEAD_SIZE);
    for (size_t head = 0; head < OREF_QUERY_HEADS; ++head) {
        const size_t kv = head / (OREF_QUERY_HEADS / OREF_KV_HEADS);
        const float *qh = q + head * OREF_HEAD_SIZE;
        float maximum = sinks[head];
        for (size_t i = 0; i < count; ++i) {
            const float *k = k_cache + ((first + i) * OREF_KV_HEADS + kv) * OREF_HEAD_SIZE;
            float d = 0.0f;
            for (size_t j = 0; j < OREF_HEAD_SIZE; ++j) {
                const float p = qh[j] * k[j];
                d = d + p;
            }
            scores[i] = d * scale;
            maximum = (maximum < scores[i]) ? scores[i] : maximum;  /* std::max */
        }
        float denominator = expf(sinks[head] - maximum);
        for (size_t i = 0; i < count; ++i) {
            scores[i] = expf(scores[i] - maximum);
            denominator = denominator + scores[i];
        }
        float *result = out + head * OREF_HEAD_SIZE;
        for (size_t d = 0; d < OREF_HEAD_SIZE; ++d) {
            result[d] = 0.0f;
        }
        for (size_t i = 0; i < count; ++i) {
            const float weight = scores[i] / denominator;
            const float *v = v_cache + ((first + i) * OREF_KV_HEADS + kv) * OREF_HEAD_SIZE;
            for (size_t d = 0; d < OREF_HEAD_SIZE; ++d) {
                const float p = weight * v[d];
                result[d] = result[d] + p;
            }
        }
    }
}

/* One token through the attention block of layer `layer_index` at
 * `position` (src/model.cpp:578-590): rms_norm with attn_norm, the Q / K / V
 * projections, RoPE on Q and K, K and V stored at `position` of the layer's
 * caches ([capacity][8 heads][64]), attention, the output projection, and
 * residual = x + projection.  attended (optional) receives the attention
 * output [4096].  Returns -1 when position >= capacity (src/model.cpp:250-252). */
int oref_attention_step(const oref_attn_layer *L, size_t layer_index, size_t position, float *k_cache,
                        float *v_cache, size_t capacity, const float *x, float *residual, float *attended) {
    static float normalized[OREF_DIM], q[OREF_QUERY_WIDTH], k[OREF_KV_WIDTH], v[OREF_KV_WIDTH];
    static float att[OREF_QUERY_WIDTH], proj[OREF_DIM], freq[OREF_HEAD_SIZE / 2];
    static float scores[1 << 20];
    if (position >= capacity || position + 1 > (size_t)(1 << 20)) {
        return -1;
    }
    oref_rope_frequencies(freq);
    oref_rms_norm(x, L->attn_norm, 1.0e-5f, normalized, OREF_DIM);
    oref_matvec_add_q8_0(L->q_w, L->q_b, normalized, q, OREF_QUERY_WIDTH, OREF_DIM);
    oref_matvec_add_q8_0(L->k_w, L->k_b, normalized, k, OREF_KV_WIDTH, OREF_DIM);
    oref_matvec_add_q8_0(L->v_w, L->v_b, normalized, v, OREF_KV_WIDTH, OREF_DIM);
    oref_apply_rope(q, OREF_QUERY_HEADS, position, freq);
    oref_apply_rope(k, OREF_KV_HEADS, position, freq);
    memcpy(k_cache + position * OREF_KV_WIDTH, k, sizeof(k));
    memcpy(v_cache + position * OREF_KV_WIDTH, v, sizeof(v));
    oref_attention(layer_index, position, q, k_cache, v_cache, L->sinks, scores, att);
    oref_matvec_add_q8_0(L->o_w, L->o_b, att, proj, OREF_DIM, OREF_QUERY_WIDTH);
    for (size_t j = 0; j < OREF_DIM; ++j) {
        residual[j] = x[j] + proj[j];
    }
    if (attended) {
        memcpy(attended, att, sizeof(att));
    }
    return 0;
}
