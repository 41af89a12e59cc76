/*
 * ttl_moe.h -- C ABI of the B200 gpt-oss MoE backend for tt-lab.
 *
 * This is the whole boundary between tt-lab's host code and the CUDA kernels:
 * plain C, scalars and pointers only (the rule tt-lab states for its own native
 * kernels at src/tt_matvec.h:9).  Every entry point returns TTL_OK (0) or a
 * negative status; ttl_moe_last_error() gives the message.  A C++ caller turns a
 * failure into std::runtime_error (tt-lab's error style, src/main.cpp:414-417);
 * tt-lab_b200/host/cuda_moe.hpp does exactly that.
 *
 * Reference interfaces replaced (paths inside tenstorrent/tt-lab):
 *   ttl_moe_decode        GptOssModel::moe          src/model.cpp:292-338
 *   ttl_moe_prefill       GptOssModel::moe_batch    src/model.cpp:340-461
 *   ttl_moe_forward       the per-layer RMSNorm -> moe -> residual sequence of
 *                         GptOssModel::forward      src/model.cpp:586-595
 *   ttl_moe_upload_layer  the weight binding of the GptOssModel constructor
 *                         (require_tensor)          src/model.cpp:157-169
 *   ttl_moe_create        backend start-up, as run_tt_firmware_inference's
 *                         runtime open              src/tt_backend.h:38-41
 *   ttl_pack_mxfp4        the requant payload packer write_bfp8_strip_payload
 *                                                   src/requant.cpp:258-277
 *   ttl_ttq_*             the TTQ container writer  src/requant.cpp:23-68,
 *                                                   :415-504; src/requant.h:31-52
 *   ttl_head_*            the output head of GptOssModel::forward: rms_norm,
 *                         matvec_q8_0 and greedy    src/model.cpp:598-612
 *
 * Memory: device buffers, pinned host staging and the blocking decode's
 * captured graphs are made in ttl_moe_create and ttl_moe_upload_layer and freed
 * in ttl_moe_destroy ("allocate dynamic memory at startup only", tt-lab
 * AGENTS.md).  The compute calls allocate nothing, with one exception: the
 * first ttl_moe_forward / ttl_moe_forward_async call for a new (buffers, token
 * count, layer range) captures and instantiates a CUDA graph for it (at most 64
 * are kept, least recently used dropped).  The diagnostic calls
 * (ttl_moe_profile, ttl_moe_trace, ttl_moe_record) recapture graphs.
 * Threading: one host thread per handle; calls on one handle are serialised on
 * the handle's CUDA stream.
 */
#ifndef TTL_MOE_H
#define TTL_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTL_MOE_ABI_VERSION 1
#define TTL_MOE_DIM 2880          /* hidden = expert intermediate (src/model.h:34, :43) */
#define TTL_MOE_TOPK 4            /* experts per token (src/model.h:42) */
#define TTL_MOE_BLOCK_BYTES 17    /* GGUF MXFP4 block: E8M0 scale + 16 quant bytes */
#define TTL_MOE_NCCL_ID_BYTES 128 /* sizeof(ncclUniqueId) */

enum {
    TTL_OK = 0,
    TTL_ERR_ARGUMENT = -1,    /* bad argument; nothing was enqueued */
    TTL_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    TTL_ERR_STATE = -3,       /* layer not uploaded, capacity exceeded, ... */
    TTL_ERR_NCCL = -4,        /* a NCCL call failed or its communicator broke */
    TTL_ERR_DEVICE = -5,      /* a kernel reported an error in the device status word */
    TTL_ERR_UNSUPPORTED = -6, /* no sm_100 device, or a feature not built */
    TTL_ERR_IO = -7           /* TTQ file I/O */
};

typedef struct ttl_moe ttl_moe;

typedef struct {
    uint32_t experts;    /* 32 (gpt-oss-20b) or 128 (gpt-oss-120b) */
    uint32_t layers;     /* MoE layers the handle holds, 1..36 */
    uint32_t max_tokens; /* prefill capacity per call; 0 = decode only */
    int32_t device;      /* CUDA device ordinal, -1 = the calling thread's current device */
    uint32_t rank;       /* expert-parallel rank in [0, world) */
    uint32_t world;      /* 1, 2, 4 or 8 ranks, one process (and one GPU) each */
    const void *nccl_id; /* world > 1: the TTL_MOE_NCCL_ID_BYTES id from ttl_moe_nccl_id() on rank 0 */
    uint32_t flags;      /* reserved, 0 */
} ttl_moe_config;

int ttl_moe_abi_version(void);

/* Message of the last failed call on `handle`, or of the calling thread's last
 * failed ttl_moe_create / ttl_pack / ttl_ttq call when `handle` is NULL. */
const char *ttl_moe_last_error(const ttl_moe *handle);

/* Writes a fresh NCCL unique id (TTL_MOE_NCCL_ID_BYTES) for a multi-rank handle. */
int ttl_moe_nccl_id(void *id_out);

int ttl_moe_create(const ttl_moe_config *config, ttl_moe **handle_out);
void ttl_moe_destroy(ttl_moe *handle);

/* Copies one layer's MoE tensors to the device and packs the experts this rank
 * owns (experts [rank*E/world, (rank+1)*E/world)).  The arrays are the GGUF
 * tensors bound at src/model.cpp:157-169, for all E experts:
 *   router_w  f32 [E][2880]            ffn_gate_inp.weight
 *   router_b  f32 [E]                  ffn_gate_inp.bias
 *   gate_w    MXFP4 [E][2880][90][17]  ffn_gate_exps.weight   (GGUF blocks)
 *   gate_b    f32 [E][2880]            ffn_gate_exps.bias
 *   up_w/up_b, down_w/down_b           ffn_up_exps.*, ffn_down_exps.*
 * Host or device pointers.  Synchronous. */
int ttl_moe_upload_layer(ttl_moe *handle, int layer, const float *router_w, const float *router_b,
                         const void *gate_w, const float *gate_b, const void *up_w, const float *up_b,
                         const void *down_w, const float *down_b);

/* ttl_moe_upload_layer with the expert matrices already in the GPU layout:
 * gate/up/down_packed are TTL_TTQ_FORMAT_MXFP4_GPU payloads of all E experts
 * (ttl_packed_bytes(E) bytes each, as ttl_requant_gpu writes them); the rest
 * as for ttl_moe_upload_layer.  A scale byte of 255 is refused the same way.
 * Counterpart: the expert-weight binding from tt-lab's TtqFile
 * (src/tt_backend.cpp:315-445).  Synchronous. */
int ttl_moe_upload_layer_packed(ttl_moe *handle, int layer, const float *router_w, const float *router_b,
                                const void *gate_packed, const float *gate_b, const void *up_packed,
                                const float *up_b, const void *down_packed, const float *down_b);

/* Post-attention RMSNorm weights (blk.N.post_attention_norm.weight, f32 [2880])
 * applied by ttl_moe_forward before layer `layer`'s MoE.  Default: all ones. */
int ttl_moe_upload_norm(ttl_moe *handle, int layer, const float *norm_w);

/* Decode MoE of one token on layer `layer`: GptOssModel::moe.
 * x, out: HOST f32 [2880]; top4_idx/top4_w: optional host [4] (rank order).
 * Blocking: returns after `out` is written. */
int ttl_moe_decode(ttl_moe *handle, int layer, const float *x, float *out, int32_t *top4_idx, float *top4_w);

/* Prefill MoE of `tokens` tokens: GptOssModel::moe_batch.
 * x, out: HOST f32 [tokens][2880]; idx/w: optional host [tokens][4].
 * tokens <= max_tokens.  With world > 1 each rank passes its own tokens (its
 * share of the batch) and receives their outputs: the token rows go to the
 * ranks owning their experts and the weighted expert outputs come back
 * (NCCL send/recv), then the owner combines them in ascending expert id.
 * Every rank must call it (with at least one token).  Blocking. */
int ttl_moe_prefill(ttl_moe *handle, int layer, const float *x, size_t tokens, float *out, int32_t *top4_idx,
                    float *top4_w);

/* Decode `tokens` independent tokens, one after another, each through layers
 * [layer_begin, layer_end): per layer h = RMSNorm(x) * norm_w, x = x + MoE(h)
 * (src/model.cpp:590-594 with the attention block left out).
 * x: HOST f32 [tokens][2880] residual inputs; y: HOST f32 [tokens][2880]
 * outputs (may alias x).  The tokens pass through device staging made at
 * create (max(max_tokens, 256) rows) in chunks of that size.  Blocking. */
int ttl_moe_forward(ttl_moe *handle, int layer_begin, int layer_end, const float *x, float *y, size_t tokens);

/* Device-pointer forms of the three calls above: all pointers are device
 * memory of the handle's GPU; the work is enqueued on the handle's stream and
 * the call returns without waiting.  ttl_moe_sync() waits and reports.
 * Prefill's x must be 16-byte aligned (TTL_ERR_ARGUMENT otherwise); with
 * world > 1 prefill waits once inside the call, for the ranks' send counts. */
int ttl_moe_decode_async(ttl_moe *handle, int layer, const float *x, float *out, int32_t *top4_idx,
                         float *top4_w);
int ttl_moe_prefill_async(ttl_moe *handle, int layer, const float *x, size_t tokens, float *out,
                          int32_t *top4_idx, float *top4_w);
int ttl_moe_forward_async(ttl_moe *handle, int layer_begin, int layer_end, const float *x, float *y,
                          size_t tokens);

/* Waits for the handle's stream, then checks the device status word that the
 * kernels set on a bounds or bounded-wait failure (TTL_ERR_DEVICE). */
int ttl_moe_sync(ttl_moe *handle);

/* Expert parallelism (world > 1): failures and recovery.
 * Every compute call is collective: each rank makes the same calls in the
 * same order.  After any call on a multi-rank handle returns an error (on
 * this rank: a rejected argument, a failed launch, a device timeout waiting
 * for a peer), the handle refuses compute calls with TTL_ERR_STATE until
 * every rank has called ttl_moe_resync, which brings the ranks' kernel tag
 * bases and peer-memory flags back into agreement (two NCCL collectives).
 * The kernels' waits on peers are bounded on the device (2 s, then
 * TTL_ERR_DEVICE).  The communicator is nonblocking and every host wait on it
 * or on the handle's stream is bounded by the handle's timeout (default
 * 60000 ms); past it the communicator is aborted (TTL_ERR_NCCL), after which
 * the handle refuses everything but ttl_moe_destroy.  World 1:
 * ttl_moe_resync waits for the stream and clears the status word. */
int ttl_moe_resync(ttl_moe *handle);

/* Decode server (single-GPU handles): with idle_us > 0, blocking
 * ttl_moe_decode calls are answered by a resident launch of the decode kernel
 * fed through a mailbox in mapped pinned memory -- no kernel launch, copy or
 * stream synchronisation per call.  This is for callers that make one
 * blocking MoE call per (token, layer) with the rest of the model elsewhere
 * (tt-lab's GptOssModel::moe hook).  While the launch is resident it holds
 * every SM, so no other kernel runs on the GPU: it leaves after idle_us
 * microseconds without a request (at most 1 s) and is started again by the
 * next call, and every other call on the handle stops it first.  Requires
 * every layer uploaded.  idle_us = 0 turns it off.  Results equal those of
 * the ordinary blocking call bit for bit.  Allocates its mailbox on first use. */
int ttl_moe_serve(ttl_moe *handle, uint32_t idle_us);
int ttl_moe_set_timeout(ttl_moe *handle, uint32_t milliseconds);

/* The handle's cudaStream_t, as void *. */
void *ttl_moe_stream(ttl_moe *handle);

/* Diagnostic counters: [0] decode router exact re-evaluations at near-ties,
 * [1] prefill tokens re-evaluated, [2] kernels launched by this handle,
 * [3] 1 when decode runs in the persistent kernel (with world > 1: the ranks
 * exchange their partial outputs inside it), 0 when it runs per layer.
 * Returns the number written (<= n). */
int ttl_moe_counters(const ttl_moe *handle, uint64_t *out, size_t n);

/* Kernel timing for benchmarks: with `enable` set, forward graphs captured
 * afterwards record CUDA events around their main decode kernel.
 * ttl_moe_kernel_ms() then writes, for the last completed replay:
 *   [0] duration in ms of one launch of the dominant decode kernel (the
 *       persistent kernel, or for expert-parallel handles the gate/up kernel),
 *   [1] (token, layer) steps that launch covered,
 *   [2] 1 for the persistent kernel, 0 for the per-layer kernels.
 * No counterpart in tt-lab (it profiles with device cycle stamps,
 * src/tt_backend.cpp:2338-2380). */
int ttl_moe_profile(ttl_moe *handle, int enable);

/* Phase timeline of the persistent decode kernel, the counterpart of tt-lab's
 * firmware stage stamps (src/tt_backend.cpp:2338-2380): with steps > 0, later
 * launches record %globaltimer (ns) at 10 points of each of the first `steps`
 * (token, layer) steps: 0 layer start, 1 selection done, 2 gate/up operands
 * ready, 3 CTA 0 gate/up done, 4 after the barrier, 5 down operands ready,
 * 6 CTA 0 down done, 7 after the barrier, 8/9 latest gate/up and down end
 * over all CTAs.  With out != NULL, waits and copies steps*10 stamps. */
int ttl_moe_trace(ttl_moe *handle, int steps, uint64_t *out);
int ttl_moe_kernel_ms(ttl_moe *handle, float *ms, size_t n);

/* Step log of the persistent decode kernel, for parity checks at full size:
 * with steps > 0, later ttl_moe_forward* / ttl_moe_decode* calls write, for
 * each (token, layer) step s = token * (layer_end - layer_begin) +
 * (layer - layer_begin) below `steps`, the step's output row -- the layer
 * output x + MoE(RMSNorm(x)) for forward, the MoE output for decode -- to
 * y_log + 2880 s, and its top-4 experts (rank order) and their weights to
 * idx_log + 4 s and w_log + 4 s.  Device memory of the handle's GPU, owned by
 * the caller until the log is turned off (steps = 0).  Per-layer decode (an
 * expert-parallel handle whose ranks could not map each other's buffers)
 * writes no log.  Counterpart: tt-lab's --dump-tensors files "output" and
 * "router" (src/model.cpp:294, :595, :614-645). */
int ttl_moe_record(ttl_moe *handle, size_t steps, float *y_log, int32_t *idx_log, float *w_log);

/* One expert matrix on the tensor cores: y = bias + W x, tt-lab's
 * matvec_add_mxfp4_2880 (src/tensor.cpp:239-304).  packed: one 2880 x 2880
 * matrix in the GPU layout (ttl_pack_mxfp4); bias, x, y: f32 [2880].  Device
 * pointers on `device`; synchronous. */
int ttl_matvec_mxfp4(const void *packed, const float *bias, const float *x, float *y, int device);

/* ttl_matvec_mxfp4 for `matrices` consecutive problems (matrix m at
 * packed + m * ttl_packed_bytes(1), its bias, x and y at + m * 2880 floats)
 * that allocates no device memory: its per-matrix status words live in a
 * fixed 1 KB static device array, so matrices must be 1..256 (more is refused
 * with TTL_ERR_ARGUMENT before any GPU work).  For callers that cannot
 * allocate (a fixed memory budget, a pool-owning host).  The first call on a
 * device looks the array up (cudaGetSymbolAddress) with that device current;
 * make it before any stream capture.  The array is shared by all calls on a
 * device, so overlapping calls from several threads or streams race.  The
 * looked-up address is kept for the life of the process: resetting the device
 * (cudaDeviceReset) while using this entry is not supported.
 * Synchronous, on the device's legacy default stream.  No counterpart in
 * tt-lab. */
int ttl_matvec_mxfp4_noalloc(const void *packed, const float *bias, const float *x, float *y, size_t matrices,
                             int device);

/* ---- GPU weight-layout packer (requant) -------------------------------- */

/* Bytes of the packed layout (TTQ format TTL_TTQ_FORMAT_MXFP4_GPU) of
 * `matrices` MXFP4 matrices of 2880 rows x 2880 columns. */
size_t ttl_packed_bytes(size_t matrices);

/* Packs `matrices` GGUF MXFP4 matrices (2880 x 2880 each, 17-byte blocks) into
 * the GPU layout on device `device`.  src/dst host or device.  Lossless:
 * ttl_unpack_mxfp4 restores the GGUF bytes exactly. */
int ttl_pack_mxfp4(const void *gguf, size_t matrices, void *packed, int device);
int ttl_unpack_mxfp4(const void *packed, size_t matrices, void *gguf, int device);

/* ---- TTQ container (TTLBQNT1, src/requant.h:31-52) ----------------------- */

#define TTL_TTQ_FORMAT_MXFP4_GPU 6 /* new format id next to tt-lab's 1..5 */
#define TTL_TTQ_FORMAT_F32 7       /* an f32 tensor exactly as the GGUF stores it */

typedef struct ttl_ttq_writer ttl_ttq_writer;

/* Opens `path` for an atomic write: data goes to a temporary file beside it and
 * ttl_ttq_finish renames it over `path` (src/requant.cpp:23-68).  model is 20
 * or 120; layers/experts as in the GGUF. */
int ttl_ttq_open(const char *path, uint32_t model, uint32_t layers, uint32_t experts, uint32_t tensor_count,
                 ttl_ttq_writer **writer_out);
/* Appends one tensor record and its payload (64-byte aligned). */
int ttl_ttq_add(ttl_ttq_writer *writer, const char *name, uint32_t format, uint32_t rank, const uint64_t *shape,
                const void *payload, uint64_t size);
int ttl_ttq_finish(ttl_ttq_writer *writer);
/* Frees the writer; an unfinished file is removed. */
void ttl_ttq_close(ttl_ttq_writer *writer);

/* requant --cuda: reads a gpt-oss GGUF (v3) and writes, atomically, a TTQ
 * file with the MoE tensors of layers [layer_begin, layer_end) (layer_end -1:
 * all): per layer ffn_gate_inp.{weight,bias} and ffn_{gate,up,down}_exps.bias
 * as TTL_TTQ_FORMAT_F32 records under their GGUF names, and the three expert
 * matrices packed on `device` as TTL_TTQ_FORMAT_MXFP4_GPU records named
 * "<GGUF name>.mxfp4gpu".  The header carries the model (20 / 120), layer and
 * expert counts, dim and vocab, so tt-lab's TtqFile reads the file.
 * Counterpart: write_requant (src/requant.cpp:415-504). */
int ttl_requant_gpu(const char *gguf_path, const char *ttq_path, int layer_begin, int layer_end, int device);

/* ---- output head (logits) ---------------------------------------------- */

/* The last step of GptOssModel::forward / prefill (src/model.cpp:598-612):
 * normalized = rms_norm(x, output_norm.weight), logits = matvec_q8_0(
 * output.weight, normalized), token = greedy(logits) (src/tensor.cpp:202-218,
 * :568-580), computed on the GPU with tt-lab's exact arithmetic, so logits and
 * token equal the reference's bit for bit.  One handle holds one output
 * matrix of `vocab` rows x 2880 columns (201088 rows for gpt-oss). */
typedef struct ttl_head ttl_head;

int ttl_head_create(int device, uint32_t vocab, ttl_head **handle_out);
void ttl_head_destroy(ttl_head *handle);
/* Message of the last failed call on `handle` (NULL: of the calling thread). */
const char *ttl_head_last_error(const ttl_head *handle);
/* q8_0: output.weight in GGUF Q8_0 blocks [vocab][90][34 B] (half scale, 32
 * int8); norm_w: output_norm.weight f32 [2880].  Host or device pointers;
 * repacked on the device to aligned rows.  Synchronous. */
int ttl_head_upload(ttl_head *handle, const void *q8_0, const float *norm_w);
/* The uploaded matrix back in GGUF bytes (host or device), for checks. */
int ttl_head_unpack(ttl_head *handle, void *gguf_out);
/* x: HOST f32 [2880] (the residual stream after the last layer); logits:
 * optional HOST f32 [vocab]; token: optional HOST int32 (at least one of
 * the two).  Blocking. */
int ttl_head_forward(ttl_head *handle, const float *x, float *logits, int32_t *token);
/* Device-pointer form on the handle's stream (logits, token optional). */
int ttl_head_forward_async(ttl_head *handle, const float *x, float *logits, int32_t *token);
int ttl_head_sync(ttl_head *handle);
void *ttl_head_stream(ttl_head *handle);

/* ---- synthetic inputs (benchmarks and tests) ---------------------------- */

/* Fills GGUF-layout MXFP4 blocks from (seed, stream): quant bytes uniform,
 * scale bytes uniform over [scale_lo, scale_lo + scale_count).  dst host or
 * device. */
int ttl_synth_mxfp4(void *dst, size_t blocks, uint64_t seed, uint64_t stream, uint32_t scale_lo,
                    uint32_t scale_count);
/* Fills GGUF-layout Q8_0 blocks from (seed, stream): half scales in
 * [2^-11, 2^-9), int8 quants uniform.  dst host or device. */
int ttl_synth_q8_0(void *dst, size_t blocks, uint64_t seed, uint64_t stream);
/* Fills n f32 values sigma * IrwinHall12(seed, stream) + mean.  dst host or device. */
int ttl_synth_normal(float *dst, size_t n, uint64_t seed, uint64_t stream, float sigma, float mean);

#ifdef __cplusplus
}
#endif
#endif
