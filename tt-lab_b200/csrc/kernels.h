// kernels.h -- launchers of the MoE kernels (internal to libttl_moe).
#pragma once

#include <cstddef>

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ttl {

// Device view of one layer's weights on this rank.
struct LayerDev {
    const float *router_w;  // [E][2880]
    const float *router_b;  // [E]
    const float *norm_w;    // [2880]
    const uint8_t *gate;    // packed [E_local] matrices
    const uint8_t *up;
    const uint8_t *down;
    const float *gate_b;    // [E_local][2880]
    const float *up_b;
    const float *down_b;
};

// Decode scratch, allocated once per handle.
struct DecodeWork {
    float *h;               // [2880] router / expert input of the current layer
    float *logits;          // [E] fast logits
    float *bounds;          // [E] error bounds of the fast logits
    int32_t *top_idx;       // [4]
    float *top_w;           // [4]
    float *hidden;          // [4][2880]
    float *partial;         // [2880] combined output of this rank's experts
    unsigned int *arrive;   // last-CTA arrival counter (self-resetting)
    unsigned long long *counters;  // [4] device counters
    uint32_t *status;       // device status word
};

struct DecodeShape {
    int experts;       // E
    int expert_begin;  // first expert owned by this rank
    int expert_count;  // experts owned by this rank
    int sms;           // multiprocessors of the device
};

// Router + top-4 + softmax.  mode 0: h = x (x already normalized);
// mode 1: h = RMSNorm(x) * norm_w (eps 1e-5).
void launch_decode_router(const LayerDev &L, const DecodeWork &w, const DecodeShape &s, const float *x, int mode,
                          cudaStream_t stream);
// gate/up matvecs of the selected experts with the SwiGLU epilogue.
void launch_decode_gateup(const LayerDev &L, const DecodeWork &w, const DecodeShape &s, cudaStream_t stream);
// down matvecs + weighted combine in rank order.  residual: if non-null,
// out = residual + moe, else out = moe (this rank's partial when EP).
void launch_decode_down(const LayerDev &L, const DecodeWork &w, const DecodeShape &s, const float *residual,
                        float *out, cudaStream_t stream);
// out[i] = residual[i] + moe[i]
void launch_add(const float *residual, const float *moe, float *out, int n, cudaStream_t stream);

// GGUF -> packed layout on the device; bit 0 of *flags (optional) is set when
// a scale byte is 255.
void launch_pack(const uint8_t *gguf_dev, uint8_t *packed_dev, size_t matrices, cudaStream_t stream,
                 uint32_t *flags = nullptr);
// Sets bit 0 of *flags when a scale byte of `matrices` packed matrices is 255.
void launch_scan_scales(const uint8_t *packed_dev, size_t matrices, cudaStream_t stream, uint32_t *flags);

// ---- persistent decode (decode_tc.cu) ----
// A CUtensorMap, kept opaque here (128 bytes, 64-byte aligned).
struct alignas(64) TmaDesc {
    unsigned long long w[16];
};

// Tensor maps of one layer's packed expert matrices: the nibble rows as bytes
// (all local experts; box coordinates (byte of the row, row, expert); boxes
// of 128 bytes x 128 rows, 128-byte swizzle; bytes past 1440 read as zero).
// kTmaRouter (handles of more than 32 experts only): the router weights f32
// [experts][2880], box (128 rows of the hidden dimension, experts 32..E-1),
// no swizzle, rows past 2880 read as zero -- the decode kernel's staging of
// one down tile's next-layer router weights in a single copy.
enum TmaIndex {
    kTmaGate,
    kTmaUp,
    kTmaDown,
    kTmaRouter,
    kTmaCount
};
constexpr int kRouterMapFirstExpert = 32;

struct StackLayer {
    const float *router_w;
    const float *router_b;
    const float *norm_w;
    const uint8_t *gate;
    const uint8_t *up;
    const uint8_t *down;
    const float *gate_b;
    const float *up_b;
    const float *down_b;
    const TmaDesc *tma;  // [kTmaCount] in device memory (tensor-core decode)
};

// The decode server's mailbox (mode 2): pinned host memory mapped into the
// device's address space.  The host writes x, then the request word (number
// and layer).  The answer comes as tagged 8-byte words (the request's number
// in the high half, the value's bits in the low half): the down reducers
// store y, CTA 0 the top-4, so a word carrying the current number is the
// data -- no fence, no completion count.  `resp` / `status` report a failed
// step; `alive` drops to 0 once the kernel takes no more requests.
struct DecodeMailbox {
    unsigned long long reqw;  // (number of the last request << 32) | its layer (host, one store)
    uint32_t stop;    // nonzero: the kernel leaves after the request in hand (host)
    uint32_t alive;   // 1 while the kernel takes requests (kernel clears it)
    uint32_t resp;    // number of a request whose step failed (kernel)
    uint32_t status;  // the device status word of that step (kernel)
    uint32_t pad[2];
    unsigned long long top[8];   // tagged: the 4 expert ids, then the 4 weights (kernel)
    float x[2880];               // 16-byte aligned: the kernel reads it as float4 (host)
    unsigned long long y[2880];  // tagged output row (kernel)
};
static_assert(offsetof(DecodeMailbox, reqw) % 8 == 0, "mailbox request word");
static_assert(offsetof(DecodeMailbox, x) % 16 == 0 && offsetof(DecodeMailbox, y) % 8 == 0, "mailbox rows");

struct StackArgs {
    const StackLayer *layers;  // device array indexed by layer
    int layer_begin;
    int layer_end;
    const float *x;            // [tokens][2880] input (h in mode 0, residual x in mode 1)
    float *y;                  // [tokens][2880] output
    int tokens;
    int mode;                  // 0: one plain MoE per token (h given); 1: RMSNorm + MoE + residual;
                               // 2: decode server (mode 0 steps on requests from `mbox`)
    int row_mask;              // token row of x / y = token & row_mask (0 in mode 2: one row)
    DecodeMailbox *mbox;       // mode 2: the mailbox (device address of mapped host memory)
    float *srv_x;              // mode 2: [2880] the request's input, copied from the mailbox
    unsigned long long *go;    // mode 2: [1] (step tag << 32) | layer, published by CTA 0
    uint32_t mbox_base;        // mode 2: requests answered before this launch
    unsigned long long idle_ns;  // mode 2: the kernel leaves after this long without a request
    int experts;
    int expert_begin;
    int expert_count;
    double *acc;               // [2][129] router sums (f64), zeroed by the host before a launch
    unsigned long long *rlog;  // [2][128][2] modes 0 and 2: each expert's fast logit and its error
                               // bound as two tagged words (16 bytes), steps of even and odd index in turn
    float *hidden;             // [4][2880]
    int32_t *top_idx;          // [4] selection of the last (token, layer)
    float *top_w;              // [4]
    unsigned *barrier;         // [2] arrival count (zeroed by the host before a launch), generation
    uint32_t *status;
    unsigned long long *counters;
    // tensor-core decode workspace.  Buffers marked [2] are used by steps of
    // even and odd index in turn; "tagged" words hold an f32 in the low half
    // and, in the high half, the tag seq + step + 1 of the step that wrote it.
    uint32_t *seq_state;           // [0] tag base of the next launch, [1] CTAs finished (the last one
                                   //     advances [0] by the launch's steps and clears [1])
    unsigned long long *part_gu;   // [2][4 * 23 tiles][16 slots][256] gate/up tile partials, tagged
    unsigned long long *part_dn;   // [2][23 tiles][16 slots][128] down tile partials, tagged
    unsigned long long *rpt;       // [2][23 tiles][129][2] next step's router sums per down tile (the sum of
                                   // squares at index E), each f64 as two tagged f32 words (hi, then lo)
    unsigned *cnt_b;               // [4] gate/up tiles reduced per expert slot (zeroed by the host)
    unsigned *cnt_y;               // down tiles whose output rows and next B operand are written (zeroed
                                   // by the host)
    uint8_t *bdown;                // [2][4][90 K-blocks][2][8][16] down B operand: digit terms of w * hidden
    uint8_t *sfb_down;             // [2][4][96] their block codes (90 + padding, 127)
    uint8_t *bnext;                // [2][90 K-blocks][2][8][16] next step's gate/up B operand: digit terms of x * g
    uint8_t *bnext_code;           // [2][96] their block codes (90 + padding, 127)
    unsigned long long *trace; // optional: [steps][kTracePoints] %globaltimer stamps of CTA 0 (+ CTA-max phase ends)
    int trace_steps;
    // optional step log: step s < log_steps writes its output row (the layer
    // output in mode 1, the MoE output in mode 0) to ylog[s][2880] and its
    // top-4 (rank order) to ilog[s][4] / wlog[s][4]
    float *ylog;
    int32_t *ilog;
    float *wlog;
    int log_steps;
    // Expert parallelism inside the launch (world > 1): a device array of
    // every rank's exchange buffer as this GPU addresses it (its own, and the
    // peers' mapped over NVLink), each [2 step parities][world][kXchRow]
    // tagged partial output rows.
    int rank;
    int world;
    unsigned long long *const *xch;
};
constexpr int kMaxWorld = 8;
constexpr int kXchRow = 23 * 128;  // rows of one rank's partial output (2880, padded to whole tiles)
constexpr size_t xch_words(int world) {
    return size_t(2) * size_t(world) * kXchRow;
}

constexpr int kTracePoints = 10;

// Sizes of the tensor-core decode workspace (StackArgs), in elements.
constexpr size_t kPartGuWords = size_t(2) * 4 * 23 * 16 * 256;
constexpr size_t kPartDnWords = size_t(2) * 23 * 16 * 128;
constexpr size_t kRptWords = size_t(2) * 23 * 129 * 2;
constexpr size_t kRlogWords = size_t(2) * 128 * 2;
constexpr size_t kBdownBytes = size_t(2) * 4 * 90 * 256;
constexpr size_t kSfbDownBytes = size_t(2) * 4 * 96;
constexpr size_t kBnextBytes = size_t(2) * 90 * 256;
constexpr size_t kBnextCodeBytes = size_t(2) * 96;

size_t decode_tc_smem_bytes();
void configure_decode_tc();
cudaError_t launch_decode_tc(const StackArgs &args, int sms, cudaStream_t stream);


// ---- prefill ----
struct PrefillWork {
    float *logits;            // [T][E]
    int32_t *top_idx;         // [T][4]
    float *top_w;             // [T][4]
    int32_t *counts;          // [E] routed pairs per local expert
    int32_t *offsets;         // [E + 1] first slot of each expert (its pairs padded to a multiple of 16)
    int32_t *pair_token;      // [slots] token of each slot, -1 for padding
    int32_t *pair_slot;       // [T][4] slot of (token, rank), -1 if not local
    int32_t *tiles;           // [groups] work list: (expert << 20) | first slot of a 16-slot group
    int32_t *tile_count;      // [1] groups
    int32_t *units;           // [groups] expert-product work list: first group | (groups - 1) << 24, a
    int32_t *unit_count;      //   unit being one or two consecutive groups of one expert; [1] its length
    float *down;              // [slots][2880] down output per slot
    uint8_t *bdig;            // [units][96 K-blocks][192 rows][16 B] gate/up B operand (digit rows of x)
    uint8_t *bsfb;            // [units][24 chunks][2][512] its scale blocks (tcgen05.cp 32x128b order)
    uint8_t *bdig_dn;         // the down B operand (SwiGLU output per slot), same layout, written by
    uint8_t *bsfb_dn;         //   the gate/up epilogue, and its scale blocks
    uint32_t *status;
    // expert parallelism: the rows are [world][seg_rows] (one region per
    // source rank), row t live iff t % seg_rows < seg_count[t / seg_rows];
    // seg_count == nullptr: every row is live
    const int32_t *seg_count;
    int seg_rows;
};

struct PrefillShape {
    int experts;
    int expert_begin;
    int expert_count;
    int tokens;
    int sms;
};

void launch_prefill_router(const LayerDev &L, const PrefillWork &w, const PrefillShape &s, const float *x,
                           cudaStream_t stream);
void launch_prefill_route(const PrefillWork &w, const PrefillShape &s, cudaStream_t stream);
void launch_prefill_gateup(const LayerDev &L, const TmaDesc *tma, const PrefillWork &w, const PrefillShape &s,
                           const float *x, cudaStream_t stream);
void launch_prefill_down(const LayerDev &L, const TmaDesc *tma, const PrefillWork &w, const PrefillShape &s,
                         cudaStream_t stream);
// Groups and units of a prefill of `tokens` tokens over `experts` local
// experts (capacity): groups <= 4T/16 + E, units <= 4T/32 + E.
constexpr size_t prefill_groups(size_t tokens, size_t experts) {
    return (4 * tokens) / 16 + experts + 1;
}
constexpr size_t prefill_units(size_t tokens, size_t experts) {
    return tokens / 8 + experts + 1;
}
// Per unit: [96 K-blocks][2 groups x 16 slots x 6 digit rows][16 B] and
// [24 chunks][2 blocks (rows 0-127, 128-191)][512 B].
constexpr size_t kPrefillUnitBytes = size_t(96) * 192 * 16;
constexpr size_t kPrefillUnitScaleBytes = size_t(24) * 2 * 512;
void launch_prefill_combine(const PrefillWork &w, const PrefillShape &s, float *out, cudaStream_t stream);

// Expert-parallel prefill over peer memory (prefill_ep.cu).  Every rank
// holds one receive block (an IPC allocation mapped by every peer), laid out
// identically on all ranks for a given (world, cap):
struct EpInbox {
    float *x;                  // [world][cap][2880] token rows, by source rank
    int32_t *idx;              // [world][cap][4] their top-4 expert ids
    float *w;                  // [world][cap][4] and weights
    int32_t *src;              // [world][cap] each row's token index on its source rank
    float *back;               // [cap][4][2880] w * down of this rank's own tokens, by (token, rank q)
    unsigned long long *cnt;   // [world] tagged (call tag, rows sent) from each source rank
    unsigned long long *done;  // [world] tagged (call tag, 0): each rank has written its rows back
};
__host__ __device__ constexpr size_t ep_align256(size_t v) {
    return (v + 255) & ~size_t(255);
}
inline size_t ep_inbox_bytes(int world, int cap) {
    const size_t rows = size_t(world) * size_t(cap);
    return ep_align256(rows * kDim * 4) + ep_align256(rows * 16) + ep_align256(rows * 16) + ep_align256(rows * 4) +
           ep_align256(size_t(cap) * 4 * kDim * 4) + ep_align256(size_t(world) * 8) + ep_align256(size_t(world) * 8);
}
__host__ __device__ inline EpInbox ep_inbox_at(void *base, int world, int cap) {
    const size_t rows = size_t(world) * size_t(cap);
    uint8_t *p = static_cast<uint8_t *>(base);
    EpInbox in{};
    in.x = reinterpret_cast<float *>(p);
    p += ep_align256(rows * kDim * 4);
    in.idx = reinterpret_cast<int32_t *>(p);
    p += ep_align256(rows * 16);
    in.w = reinterpret_cast<float *>(p);
    p += ep_align256(rows * 16);
    in.src = reinterpret_cast<int32_t *>(p);
    p += ep_align256(rows * 4);
    in.back = reinterpret_cast<float *>(p);
    p += ep_align256(size_t(cap) * 4 * kDim * 4);
    in.cnt = reinterpret_cast<unsigned long long *>(p);
    p += ep_align256(size_t(world) * 8);
    in.done = reinterpret_cast<unsigned long long *>(p);
    return in;
}

struct EpPeers {
    void *base[kMaxWorld];  // every rank's receive block as this GPU addresses it (own included)
};

void configure_prefill_ep();
void launch_ep_plan(const int32_t *idx, int tokens, int world, int per_rank, int32_t *tok_off, int32_t *cnt,
                    cudaStream_t stream);
void launch_ep_send(const float *x, const int32_t *idx, const float *wts, int tokens, int world, int rank, int cap,
                    const int32_t *tok_off, const int32_t *cnt, const EpPeers &peers, uint32_t tag,
                    unsigned *arrive, int sms, cudaStream_t stream);
void launch_ep_wait(const unsigned long long *flags, int world, uint32_t tag, int cap, int32_t *counts,
                    uint32_t *status, cudaStream_t stream);
void launch_ep_back(const PrefillWork &w, const EpInbox &in, int world, int rank, int per_rank, int cap,
                    const EpPeers &peers, uint32_t tag, unsigned *arrive, int sms, cudaStream_t stream);
void launch_ep_combine(const int32_t *idx, int tokens, const float *back, float *out, cudaStream_t stream);

} // namespace ttl
