/*
 * ttl_attn.h -- C ABI of the attention block of a gpt-oss decode layer on the
 * B200 (the part of GptOssModel::forward before the MoE).
 *
 * Reference interface replaced (tenstorrent/tt-lab): per layer and token,
 *   rms_norm(x, attn_norm) -> matvec_add_q8_0 Q / K / V -> apply_rope ->
 *   store_kv -> attention_from_cache -> matvec_add_q8_0 output -> residual
 *   = x + projection                      src/model.cpp:578-590
 * with apply_rope :230-245, store_kv :247-253, attention_from_cache :255-290
 * (sinks; even layers attend to the last 128 positions) and
 * matvec_add_q8_0 src/tensor.cpp:220-237.  The MoE half of the layer
 * (rms_norm(post_attention_norm) -> moe -> residual) is ttl_moe_forward
 * (ttl_moe.h): attention's `residual` output is its input.
 *
 * Conventions as in ttl_moe.h: TTL_OK or a negative status, messages from
 * ttl_attn_last_error; buffers are allocated in create / upload only.
 */
#ifndef TTL_ATTN_H
#define TTL_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ttl_attn ttl_attn;

typedef struct {
    uint32_t layers;         /* 1..36; a layer's index decides its window (even: sliding) */
    uint32_t token_capacity; /* positions per layer's KV cache (the reference's token_capacity) */
    int32_t device;          /* CUDA device ordinal, -1 = the calling thread's current device */
    void *stream;            /* cudaStream_t to enqueue on (e.g. ttl_moe_stream of a MoE handle), NULL = own */
} ttl_attn_config;

int ttl_attn_create(const ttl_attn_config *config, ttl_attn **handle_out);
void ttl_attn_destroy(ttl_attn *handle);
const char *ttl_attn_last_error(const ttl_attn *handle);

/* One layer's attention tensors, in GGUF order (src/model.cpp:140-156):
 *   attn_norm f32 [2880]; attn_q Q8_0 [4096 rows][90 blocks][34 B] + f32 [4096];
 *   attn_k, attn_v Q8_0 [512][90][34] + f32 [512];
 *   attn_output Q8_0 [2880][128][34] + f32 [2880]; attn_sinks f32 [64].
 * Host or device pointers.  Synchronous. */
int ttl_attn_upload_layer(ttl_attn *handle, int layer, const float *attn_norm, const void *q_w, const float *q_b,
                          const void *k_w, const float *k_b, const void *v_w, const float *v_b, const void *o_w,
                          const float *o_b, const float *sinks);

/* The attention block for one token at `position` of layer `layer`:
 * residual = x + O(attention(RoPE(Q x'), cache)), x' = rms_norm(x), with K
 * and V of this position stored in the layer's cache first.  Positions of a
 * layer must come in order (the cache holds every earlier one).  Device
 * pointers [2880]; enqueued on the handle's stream. */
int ttl_attn_forward_async(ttl_attn *handle, int layer, size_t position, const float *x, float *residual);
/* The same with host (or device) buffers, blocking; `attended` (optional,
 * [4096]) receives the attention output before the projection. */
int ttl_attn_forward(ttl_attn *handle, int layer, size_t position, const float *x, float *residual, float *attended);
int ttl_attn_sync(ttl_attn *handle);
void *ttl_attn_stream(ttl_attn *handle);

#ifdef __cplusplus
}
#endif

#endif
