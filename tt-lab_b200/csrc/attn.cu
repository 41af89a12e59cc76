// attn.cu -- the attention block of a gpt-oss decode layer on the GPU.
//
// Reference: GptOssModel::forward, tt-lab src/model.cpp:578-590 (rms_norm
// with attn_norm; matvec_add_q8_0 for Q, K and V, src/tensor.cpp:220-237;
// apply_rope, :230-245, with the YaRN table of the constructor, :123-138;
// store_kv, :247-253; attention_from_cache with sinks and the sliding window
// of even layers, :255-290; matvec_add_q8_0 for the output; residual add).
// Constants: 64 query heads, 8 KV heads, head size 64, window 128
// (src/model.h:36-50).
//
// Three launches per (layer, position), on the handle's stream:
//   attn_qkv_kernel   every CTA first reduces x to its RMS (a block tree,
//                     identical in every CTA) and keeps the normalized x in
//                     shared memory; then one warp per row pair: Q / K rows
//                     (r, r + 32) of one head, which RoPE rotates together,
//                     or two V rows.  A row's dot product runs in 32 lane
//                     chains, lane c taking byte 2 + c of every 34-byte Q8_0
//                     block (the reference's two 16-lane accumulators, one
//                     coalesced 32-byte load per block and warp), products
//                     rounded before the add.  Rotated Q goes to scratch, K and
//                     V into the layer's cache at `position`.
//   attn_decode_kernel  grid (KV head, split of the window): the 8 query heads
//                     of the KV head (one warp each) run an online softmax over
//                     the split's positions, K / V tiles staged in shared
//                     memory once for all 8; partials (max, sum, 64 values)
//                     go to scratch, and the last CTA of the KV head merges
//                     them with the heads' sinks.
//   attn_out_kernel   the output projection (4096 columns) with the same
//                     lane chains, plus bias and the residual x.
// The matrices are HBM-bound streams (Q/K/V 15.7 MB, output 12.5 MB per
// layer); the KV cache adds 4 KB per attended position.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"
#include "ttl_attn.h"

namespace {

using ttl::kDim;
constexpr int kHeads = 64;
constexpr int kKvHeads = 8;
constexpr int kHead = 64;
constexpr int kQWidth = kHeads * kHead;    // 4096
constexpr int kKvWidth = kKvHeads * kHead; // 512
constexpr int kWindow = 128;
constexpr int kMaxSplits = 32;
constexpr int kQkvThreads = 512;
constexpr int kOutThreads = 256;
constexpr int kQkvRowBytes = 90 * 34;                     // 3060: a row of 2880 Q8_0 columns
constexpr int kOutRowBytes = 128 * 34;                    // 4352: a row of 4096
// staging pitches: 8 banks apart, so the four rows a warp reads at once hit
// different banks
constexpr int kQkvRowPitch = 3104;
constexpr int kOutRowPitch = 4384;
constexpr int kRowsPerWarp = 4;                           // 8 lanes per row
constexpr size_t kRowPad = 64;                            // bytes after each matrix (rounded row copies)
constexpr int kQkvSmem = (kQkvThreads / 32) * kRowsPerWarp * kQkvRowPitch + kDim * 4;
constexpr int kOutSmem = (kOutThreads / 32) * kRowsPerWarp * kOutRowPitch + 4096 * 4;
constexpr int kTile = 32;  // positions per staged K / V tile

struct AttnLayer {
    float *norm = nullptr;           // [2880]
    uint8_t *q = nullptr;            // Q8_0 [4096][90][34]
    float *qb = nullptr;
    uint8_t *k = nullptr;            // [512][90][34]
    float *kb = nullptr;
    uint8_t *v = nullptr;
    float *vb = nullptr;
    uint8_t *o = nullptr;            // Q8_0 [2880][128][34]
    float *ob = nullptr;
    float *sinks = nullptr;          // [64]
    float *kc = nullptr;             // KV cache [capacity][8][64]
    float *vc = nullptr;
    bool uploaded = false;
};

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t su32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Bulk copies of a warp's four rows into its shared-memory slots, completed
// on the warp's mbarrier (lane 0 issues them; one instruction per row).  A
// row that does not start on 16 bytes is copied from the 16-byte boundary
// below it to the one above its end, so `lead` (0, 4, 8 or 12 bytes) is where
// the row starts in its slot; the weight buffers carry 64 bytes of padding,
// so the rounded end stays inside them.
__device__ __forceinline__ void stage_rows(uint64_t *bar, uint8_t *slots, int pitch, const uint8_t *const rows[4],
                                           int bytes, int lane) {
    if (lane == 0) {
        // the slots' earlier contents were read through the generic proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        uint32_t total = 0;
        uint32_t size[4];
        const uint8_t *src[4];
        for (int k = 0; k < 4; ++k) {
            const uintptr_t a = reinterpret_cast<uintptr_t>(rows[k]);
            const uintptr_t lo = a & ~uintptr_t(15), hi = (a + bytes + 15) & ~uintptr_t(15);
            src[k] = reinterpret_cast<const uint8_t *>(lo);
            size[k] = uint32_t(hi - lo);
            total += size[k];
        }
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(total) : "memory");
        for (int k = 0; k < 4; ++k) {
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                             su32(slots + k * pitch)),
                         "l"(src[k]), "r"(size[k]), "r"(su32(bar))
                         : "memory");
        }
    }
}

__device__ __forceinline__ int row_lead(const uint8_t *row) {
    return int(reinterpret_cast<uintptr_t>(row) & 15);
}

// Waits (bounded, 2 s) for the warp's staged rows; on a timeout it records
// kStatusWaitTimeout, waits once more for the copies in flight and returns
// false.
__device__ __forceinline__ bool wait_rows(uint64_t *bar, uint32_t &phase, uint32_t *status) {
    const uint32_t p = phase;
    phase ^= 1u;
    // every lane observes the phase (so the copied bytes are visible to it);
    // the warp decides together, so no lane leaves a later shuffle
    const bool ok = __all_sync(0xffffffffu, ttl::tc::mbar_wait(bar, p));
    if (!ok) {
        if ((threadIdx.x & 31) == 0) {
            ttl::set_status(status, ttl::kStatusWaitTimeout);
        }
        ttl::tc::mbar_wait(bar, p);  // the copies in flight, bounded again
    }
    return ok;
}

// The dot product of one staged Q8_0 row with x (cols = 32 * blocks) by the
// 8 lanes of a row group: lane j takes elements 4j .. 4j + 3 of every block
// (two 16-bit loads of its quants, the block's scale, four x values in one
// 16-byte load).  Returns the row's value on all 8 lanes.
__device__ __forceinline__ float q8_dot8(const uint8_t *row, const float *xs, int blocks, int j) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 4
    for (int b = 0; b < blocks; ++b) {
        const uint8_t *blk = row + b * 34;
        const float sc = h2f(*reinterpret_cast<const uint16_t *>(blk));
        const uint32_t q4 = uint32_t(*reinterpret_cast<const uint16_t *>(blk + 2 + 4 * j)) |
                            (uint32_t(*reinterpret_cast<const uint16_t *>(blk + 4 + 4 * j)) << 16);
        const float4 xv = *reinterpret_cast<const float4 *>(xs + b * 32 + 4 * j);
        a0 = fmaf(float(int8_t(q4)) * sc, xv.x, a0);
        a1 = fmaf(float(int8_t(q4 >> 8)) * sc, xv.y, a1);
        a2 = fmaf(float(int8_t(q4 >> 16)) * sc, xv.z, a2);
        a3 = fmaf(float(int8_t(q4 >> 24)) * sc, xv.w, a3);
    }
    float v = (a0 + a1) + (a2 + a3);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    return v;
}

struct QkvArgs {
    const float *x;
    const float *norm;
    const uint8_t *q, *k, *v;
    const float *qb, *kb, *vb;
    const float *freq;   // [32]
    float magnitude;
    int position;
    float *qout;         // [4096] rotated
    float *kc, *vc;      // this layer's caches
    uint32_t *status;
};

// Work items, four rows each (one per 8-lane row group): 1024 Q items and
// 128 K items -- rows (r, r + 32, r + 1, r + 33) of a head, two RoPE pairs --
// and 128 V items of four consecutive rows.
constexpr int kQItems = kQWidth / 4;
constexpr int kKItems = kKvWidth / 4;
constexpr int kQkvItems = kQItems + kKItems + kKvWidth / 4;

// Rows of QKV item `item` (see above); returns the matrix they are rows of.
__device__ __forceinline__ const uint8_t *qkv_item_rows(const QkvArgs &a, int item, int rows4[4]) {
    if (item < kQItems + kKItems) {
        const bool is_q = item < kQItems;
        const int local = is_q ? item : item - kQItems;
        const int r0 = (local / 16) * kHead + (local % 16) * 2;
        rows4[0] = r0;
        rows4[1] = r0 + kHead / 2;
        rows4[2] = r0 + 1;
        rows4[3] = r0 + 1 + kHead / 2;
        return is_q ? a.q : a.k;
    }
    const int r0 = 4 * (item - kQItems - kKItems);
    for (int k = 0; k < 4; ++k) {
        rows4[k] = r0 + k;
    }
    return a.v;
}

__global__ void __launch_bounds__(kQkvThreads) attn_qkv_kernel(QkvArgs a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    uint8_t *rows = dyn;                                                    // [warps][4][3104]
    float *xs = reinterpret_cast<float *>(dyn + (kQkvThreads / 32) * kRowsPerWarp * kQkvRowPitch);
    __shared__ float red[kQkvThreads / 32];
    __shared__ __align__(8) uint64_t wbar[kQkvThreads / 32];
    const int lane = threadIdx.x & 31;
    uint8_t *slots = rows + size_t(threadIdx.x >> 5) * kRowsPerWarp * kQkvRowPitch;
    uint64_t *bar = &wbar[threadIdx.x >> 5];
    if (lane == 0) {
        ttl::tc::mbar_init(bar, 1);
        ttl::tc::fence_mbar_init();
    }
    __syncwarp();
    uint32_t phase = 0;
    // items spread over the CTAs first (warp w of every CTA, then w + 1); the
    // first item's rows are requested before the norm, so the weight stream
    // overlaps it
    const int stride = gridDim.x * (blockDim.x >> 5);
    const int first = (threadIdx.x >> 5) * gridDim.x + blockIdx.x;
    if (first < kQkvItems) {
        int r4[4];
        const uint8_t *base = qkv_item_rows(a, first, r4);
        const uint8_t *src[4];
        for (int k = 0; k < 4; ++k) {
            src[k] = base + size_t(r4[k]) * kQkvRowBytes;
        }
        stage_rows(bar, slots, kQkvRowPitch, src, kQkvRowBytes, lane);
    }
    // rms_norm (src/tensor.cpp:568-580) of x: a tree over the block, the
    // same in every CTA
    float ss = 0.0f;
    for (int i = threadIdx.x; i < kDim; i += blockDim.x) {
        const float v = a.x[i];
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = ss;
    }
    __syncthreads();
    float total = 0.0f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) {
        total += red[w];
    }
    const float scale = 1.0f / sqrtf(total / float(kDim) + 1.0e-5f);
    for (int i = threadIdx.x; i < kDim; i += blockDim.x) {
        xs[i] = a.x[i] * scale * a.norm[i];
    }
    __syncthreads();
    const int g = lane >> 3;   // row group
    const int j = lane & 7;
    for (int item = first; item < kQkvItems; item += stride) {
        int rows4[4];
        const uint8_t *base = qkv_item_rows(a, item, rows4);
        const bool rope = item < kQItems + kKItems;
        const bool is_q = item < kQItems;
        const uint8_t *src[4];
        for (int k = 0; k < 4; ++k) {
            src[k] = base + size_t(rows4[k]) * kQkvRowBytes;
        }
        if (item != first) {
            __syncwarp();  // the slots' previous rows are consumed
            stage_rows(bar, slots, kQkvRowPitch, src, kQkvRowBytes, lane);
        }
        if (!wait_rows(bar, phase, a.status)) {
            break;
        }
        const int row = rows4[g];
        const float d = q8_dot8(slots + g * kQkvRowPitch + row_lead(src[g]), xs, 90, j);
        if (rope) {
            // groups (0, 1) and (2, 3) hold rows (r, r + 32): lane 0 of
            // groups 0 and 2 rotates its pair
            const float other = __shfl_xor_sync(0xffffffffu, d, 8);
            if (j == 0 && (g & 1) == 0) {
                const float *bias = is_q ? a.qb : a.kb;
                const int r1 = rows4[g + 1];
                const int pair = row % kHead;
                const float x0 = __fadd_rn(bias[row], d);
                const float x1 = __fadd_rn(bias[r1], other);
                const float theta = __fmul_rn(float(a.position), a.freq[pair]);
                const float c = __fmul_rn(cosf(theta), a.magnitude);
                const float sn = __fmul_rn(sinf(theta), a.magnitude);
                const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
                const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
                if (is_q) {
                    a.qout[row] = y0;
                    a.qout[r1] = y1;
                } else {
                    a.kc[size_t(a.position) * kKvWidth + row] = y0;
                    a.kc[size_t(a.position) * kKvWidth + r1] = y1;
                }
            }
        } else if (j == 0) {
            a.vc[size_t(a.position) * kKvWidth + row] = __fadd_rn(a.vb[row], d);
        }
    }
}

struct DecodeArgs {
    const float *q;      // [4096] rotated
    const float *kc, *vc;
    const float *sinks;
    int first, count;    // window [first, first + count)
    int per_split;
    float *part;         // [64 heads][kMaxSplits][66]: max, sum, 64 values
    unsigned *arrive;    // [8] per KV head
    float *out;          // [4096]
};

// grid (8 KV heads, splits), 8 warps: warp w = query head kv * 8 + w.
__global__ void __launch_bounds__(256) attn_decode_kernel(DecodeArgs a) {
    __shared__ float qs[8][kHead];
    __shared__ float ks[kTile][kHead + 1];
    __shared__ float vs[kTile][kHead];
    __shared__ unsigned last;
    const int kv = blockIdx.x;
    const int split = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const int head = kv * 8 + w;
    for (int i = threadIdx.x; i < 8 * kHead; i += blockDim.x) {
        qs[i / kHead][i % kHead] = a.q[(kv * 8) * kHead + i];
    }
    const int begin = a.first + split * a.per_split;
    const int end = min(a.first + a.count, begin + a.per_split);
    float m = -INFINITY, l = 0.0f, acc0 = 0.0f, acc1 = 0.0f;
    const float scale = 0.125f;  // 1 / sqrt(64)
    for (int t0 = begin; t0 < end; t0 += kTile) {
        __syncthreads();
        const int n = min(kTile, end - t0);
        for (int i = threadIdx.x; i < n * kHead; i += blockDim.x) {
            const int t = i / kHead, d = i % kHead;
            const size_t off = (size_t(t0 + t) * kKvHeads + kv) * kHead + d;
            ks[t][d] = a.kc[off];
            vs[t][d] = a.vc[off];
        }
        __syncthreads();
        float s = -INFINITY;
        if (lane < n) {
            float d = 0.0f;
#pragma unroll 8
            for (int j = 0; j < kHead; ++j) {
                d = __fadd_rn(d, __fmul_rn(qs[w][j], ks[lane][j]));
            }
            s = __fmul_rn(d, scale);
        }
        float mt = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
        }
        const float mn = fmaxf(m, mt);
        const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
        const float p = (lane < n) ? expf(s - mn) : 0.0f;
        float ps = p;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ps += __shfl_xor_sync(0xffffffffu, ps, o);
        }
        l = l * corr + ps;
        acc0 *= corr;
        acc1 *= corr;
        for (int t = 0; t < n; ++t) {
            const float pt = __shfl_sync(0xffffffffu, p, t);
            acc0 = fmaf(pt, vs[t][2 * lane], acc0);
            acc1 = fmaf(pt, vs[t][2 * lane + 1], acc1);
        }
        m = mn;
    }
    float *part = a.part + (size_t(head) * kMaxSplits + split) * 66;
    if (lane == 0) {
        part[0] = m;
        part[1] = l;
    }
    part[2 + 2 * lane] = acc0;
    part[3 + 2 * lane] = acc1;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = (atomicAdd(&a.arrive[kv], 1u) == gridDim.y - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!last) {
        return;
    }
    __threadfence();
    // merge the splits of this warp's head with its sink (src/model.cpp:270-288):
    // lane s holds split s's max and sum (all loads in flight together)
    const float sink = a.sinks[head];
    const float *ph = a.part + size_t(head) * kMaxSplits * 66;
    const int ns = int(gridDim.y);
    const float ms = (lane < ns) ? __ldcg(ph + lane * 66) : -INFINITY;
    const float ls = (lane < ns) ? __ldcg(ph + lane * 66 + 1) : 0.0f;
    float mx = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    mx = fmaxf(mx, sink);
    const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
    float den = ls * f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        den += __shfl_xor_sync(0xffffffffu, den, o);
    }
    den += expf(sink - mx);
    float o0 = 0.0f, o1 = 0.0f;
#pragma unroll 8
    for (int sp = 0; sp < ns; ++sp) {
        const float fs = __shfl_sync(0xffffffffu, f, sp);
        const float2 v = __ldcg(reinterpret_cast<const float2 *>(ph + sp * 66 + 2) + lane);
        o0 = fmaf(v.x, fs, o0);
        o1 = fmaf(v.y, fs, o1);
    }
    a.out[head * kHead + 2 * lane] = o0 / den;
    a.out[head * kHead + 2 * lane + 1] = o1 / den;
    if (threadIdx.x == 0) {
        a.arrive[kv] = 0u;  // re-armed for the next launch
    }
}

// residual[r] = x[r] + (bias[r] + the row's dot product with the attention
// output), four rows per warp (8 lanes each) of the 2880 x 4096 output
// projection; rows arrive by bulk copies, the next item's while the current
// one is summed.
__global__ void __launch_bounds__(kOutThreads) attn_out_kernel(const uint8_t *__restrict__ o, const float *__restrict__ ob,
                                                              const float *__restrict__ att, const float *__restrict__ x,
                                                              float *__restrict__ residual, uint32_t *status) {
    extern __shared__ __align__(16) uint8_t dyn[];
    __shared__ __align__(8) uint64_t wbar[kOutThreads / 32];
    float *as = reinterpret_cast<float *>(dyn);                              // [4096]
    uint8_t *slots = dyn + kQWidth * 4 + size_t(threadIdx.x >> 5) * kRowsPerWarp * kOutRowPitch;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 3, j = lane & 7;
    uint64_t *bar = &wbar[threadIdx.x >> 5];
    if (lane == 0) {
        ttl::tc::mbar_init(bar, 1);
        ttl::tc::fence_mbar_init();
    }
    __syncwarp();
    uint32_t phase = 0;
    constexpr int kItems = kDim / kRowsPerWarp;  // 720
    const int stride = gridDim.x * (blockDim.x >> 5);
    auto issue = [&](int it) {
        const uint8_t *src[4];
        for (int k = 0; k < kRowsPerWarp; ++k) {
            src[k] = o + size_t(it * kRowsPerWarp + k) * kOutRowBytes;
        }
        stage_rows(bar, slots, kOutRowPitch, src, kOutRowBytes, lane);
    };
    int item = (threadIdx.x >> 5) * gridDim.x + blockIdx.x;
    if (item < kItems) {  // the first rows' copies go out before the attention output is staged
        issue(item);
    }
    for (int i = threadIdx.x; i < kQWidth; i += blockDim.x) {
        as[i] = att[i];
    }
    __syncthreads();
    for (; item < kItems; item += stride) {
        if (!wait_rows(bar, phase, status)) {
            break;
        }
        const int r = item * kRowsPerWarp + g;
        const float d = q8_dot8(slots + g * kOutRowPitch, as, 128, j);  // rows of 4352 B start on 16 B
        __syncwarp();
        if (item + stride < kItems) {
            issue(item + stride);
        }
        if (j == 0) {
            residual[r] = __fadd_rn(x[r], __fadd_rn(ob[r], d));
        }
    }
}

}  // namespace

struct ttl_attn {
    int device = 0;
    int sms = 148;
    uint32_t layers = 0;
    uint32_t capacity = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::vector<AttnLayer> L;
    std::vector<void *> allocations;
    float *freq = nullptr;       // [32] YaRN frequencies
    float magnitude = 1.0f;
    float *q = nullptr;          // [4096] rotated query
    float *att = nullptr;        // [4096] attention output
    float *part = nullptr;       // [64][kMaxSplits][66]
    unsigned *arrive = nullptr;  // [8]
    float *d_x = nullptr;        // host-call staging [2880] x, [2880] residual
    float *d_res = nullptr;
    uint32_t *status = nullptr;  // device status word (kStatusWaitTimeout)
    std::string error;
};

namespace {

int attn_fail(ttl_attn *h, int code, const std::string &msg) {
    if (h) {
        h->error = msg;
    }
    return ttl::fail(nullptr, code, msg);
}

#define TTL_ATTN_CUDA(h, expr)                                                                         \
    do {                                                                                               \
        const cudaError_t e_ = (expr);                                                                 \
        if (e_ != cudaSuccess) {                                                                       \
            return attn_fail((h), TTL_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));   \
        }                                                                                              \
    } while (0)

template <class T> int attn_alloc(ttl_attn *h, T **p, size_t count) {
    void *q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return attn_fail(h, TTL_ERR_CUDA, "device allocation of " + std::to_string(count * sizeof(T)) + " bytes failed");
    }
    h->allocations.push_back(q);
    *p = static_cast<T *>(q);
    return TTL_OK;
}

// The YaRN table and magnitude of the GptOssModel constructor and apply_rope
// (src/model.cpp:123-138, :231), in the same f32 operations.
void rope_table(float freq[kHead / 2], float *magnitude) {
    const float head = float(kHead);
    const float base = 150000.0f, scale = 1.0f / 32.0f, original = 4096.0f, fast = 32.0f, slow = 1.0f;
    const float pi = 3.14159265358979323846f;  // std::numbers::pi_v<float>
    const float corr = head * std::log(original / (fast * 2.0f * pi)) / (2.0f * std::log(base));
    const float corr_slow = head * std::log(original / (slow * 2.0f * pi)) / (2.0f * std::log(base));
    const float low = std::max(0.0f, std::floor(corr));
    const float high = std::min(head - 1.0f, std::ceil(corr_slow));
    for (int pair = 0; pair < kHead / 2; ++pair) {
        const float theta_extrap = std::pow(base, -float(pair * 2) / head);
        const float y = (float(pair) - low) / std::max(0.001f, high - low);
        const float ramp = 1.0f - std::clamp(y, 0.0f, 1.0f);
        freq[pair] = scale * theta_extrap * (1.0f - ramp) + theta_extrap * ramp;
    }
    *magnitude = 1.0f + 0.1f * std::log(1.0f / scale);
}

// Reads and clears the device status word; a set bit is TTL_ERR_DEVICE.
int check_status(ttl_attn *h) {
    uint32_t st = 0;
    TTL_ATTN_CUDA(h, cudaMemcpy(&st, h->status, sizeof(st), cudaMemcpyDeviceToHost));
    if (st) {
        cudaMemset(h->status, 0, sizeof(uint32_t));
        return attn_fail(h, TTL_ERR_DEVICE, "device status: bounded-wait-timeout");
    }
    return TTL_OK;
}

int check_layer(ttl_attn *h, int layer) {
    if (layer < 0 || layer >= int(h->layers)) {
        return attn_fail(h, TTL_ERR_ARGUMENT, "layer " + std::to_string(layer) + " out of range");
    }
    if (!h->L[size_t(layer)].uploaded) {
        return attn_fail(h, TTL_ERR_STATE, "layer " + std::to_string(layer) + " was not uploaded");
    }
    return TTL_OK;
}

}  // namespace

extern "C" {

int ttl_attn_create(const ttl_attn_config *c, ttl_attn **out) {
    if (!c || !out) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "null argument");
    }
    *out = nullptr;
    if (c->layers == 0 || c->layers > 36 || c->token_capacity == 0 || c->token_capacity > (1u << 20)) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "layers must be 1..36 and token_capacity 1..2^20");
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return attn_fail(nullptr, TTL_ERR_UNSUPPORTED, "no CUDA device");
    }
    int device = c->device;
    if (device < 0 && cudaGetDevice(&device) != cudaSuccess) {
        return attn_fail(nullptr, TTL_ERR_CUDA, "cudaGetDevice failed");
    }
    if (device >= count) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "device ordinal out of range");
    }
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
        return attn_fail(nullptr, TTL_ERR_UNSUPPORTED, "the kernels are built for sm_100a (B200)");
    }
    ttl_attn *h = new ttl_attn();
    h->device = device;
    h->sms = prop.multiProcessorCount;
    h->layers = c->layers;
    h->capacity = c->token_capacity;
    h->L.resize(c->layers);
    auto bail = [&](int rc) {
        ttl_attn_destroy(h);
        return rc;
    };
    if (cudaSetDevice(device) != cudaSuccess) {
        return bail(attn_fail(nullptr, TTL_ERR_CUDA, "cudaSetDevice failed"));
    }
    if (c->stream) {
        h->stream = static_cast<cudaStream_t>(c->stream);
    } else {
        if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
            return bail(attn_fail(nullptr, TTL_ERR_CUDA, "cannot create a stream"));
        }
        h->own_stream = true;
    }
    int rc = attn_alloc(h, &h->freq, kHead / 2);
    rc = rc ? rc : attn_alloc(h, &h->q, kQWidth);
    rc = rc ? rc : attn_alloc(h, &h->att, kQWidth);
    rc = rc ? rc : attn_alloc(h, &h->part, size_t(kHeads) * kMaxSplits * 66);
    rc = rc ? rc : attn_alloc(h, &h->arrive, kKvHeads);
    rc = rc ? rc : attn_alloc(h, &h->d_x, kDim);
    rc = rc ? rc : attn_alloc(h, &h->d_res, kDim);
    rc = rc ? rc : attn_alloc(h, &h->status, 1);
    if (rc) {
        return bail(attn_fail(nullptr, rc, h->error));
    }
    // all three kernels ask for the largest shared-memory carveout (as the
    // MoE kernels on the same stream need), so consecutive launches never
    // wait for the SMs to repartition L1 and shared memory
    if (cudaFuncSetAttribute(attn_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQkvSmem) != cudaSuccess ||
        cudaFuncSetAttribute(attn_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kOutSmem) != cudaSuccess ||
        cudaFuncSetAttribute(attn_qkv_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_out_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared)) != cudaSuccess) {
        return bail(attn_fail(nullptr, TTL_ERR_CUDA, "cannot configure the attention kernels"));
    }
    float freq[kHead / 2];
    rope_table(freq, &h->magnitude);
    if (cudaMemcpy(h->freq, freq, sizeof(freq), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(h->arrive, 0, kKvHeads * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(h->status, 0, sizeof(uint32_t)) != cudaSuccess) {
        return bail(attn_fail(nullptr, TTL_ERR_CUDA, "device initialisation failed"));
    }
    *out = h;
    return TTL_OK;
}

void ttl_attn_destroy(ttl_attn *h) {
    if (!h) {
        return;
    }
    cudaSetDevice(h->device);
    if (h->stream) {
        cudaStreamSynchronize(h->stream);
    }
    for (void *p : h->allocations) {
        cudaFree(p);
    }
    if (h->own_stream && h->stream) {
        cudaStreamDestroy(h->stream);
    }
    delete h;
}

const char *ttl_attn_last_error(const ttl_attn *h) {
    return h ? h->error.c_str() : ttl::thread_error().c_str();
}

int ttl_attn_upload_layer(ttl_attn *h, int layer, const float *attn_norm, const void *q_w, const float *q_b,
                          const void *k_w, const float *k_b, const void *v_w, const float *v_b, const void *o_w,
                          const float *o_b, const float *sinks) {
    if (!h) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (layer < 0 || layer >= int(h->layers)) {
        return attn_fail(h, TTL_ERR_ARGUMENT, "layer out of range");
    }
    if (!attn_norm || !q_w || !q_b || !k_w || !k_b || !v_w || !v_b || !o_w || !o_b || !sinks) {
        return attn_fail(h, TTL_ERR_ARGUMENT, "null tensor pointer");
    }
    TTL_ATTN_CUDA(h, cudaSetDevice(h->device));
    AttnLayer &s = h->L[size_t(layer)];
    const size_t qbytes = size_t(kQWidth) * 90 * 34, kbytes = size_t(kKvWidth) * 90 * 34;
    const size_t obytes = size_t(kDim) * 128 * 34;
    if (!s.norm) {
        int rc = attn_alloc(h, &s.norm, kDim);
        rc = rc ? rc : attn_alloc(h, &s.q, qbytes + kRowPad);
        rc = rc ? rc : attn_alloc(h, &s.qb, kQWidth);
        rc = rc ? rc : attn_alloc(h, &s.k, kbytes + kRowPad);
        rc = rc ? rc : attn_alloc(h, &s.kb, kKvWidth);
        rc = rc ? rc : attn_alloc(h, &s.v, kbytes + kRowPad);
        rc = rc ? rc : attn_alloc(h, &s.vb, kKvWidth);
        rc = rc ? rc : attn_alloc(h, &s.o, obytes + kRowPad);
        rc = rc ? rc : attn_alloc(h, &s.ob, kDim);
        rc = rc ? rc : attn_alloc(h, &s.sinks, kHeads);
        rc = rc ? rc : attn_alloc(h, &s.kc, size_t(h->capacity) * kKvWidth);
        rc = rc ? rc : attn_alloc(h, &s.vc, size_t(h->capacity) * kKvWidth);
        if (rc) {
            return rc;
        }
    }
    TTL_ATTN_CUDA(h, cudaMemcpy(s.norm, attn_norm, kDim * sizeof(float), cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.q, q_w, qbytes, cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.qb, q_b, kQWidth * sizeof(float), cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.k, k_w, kbytes, cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.kb, k_b, kKvWidth * sizeof(float), cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.v, v_w, kbytes, cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.vb, v_b, kKvWidth * sizeof(float), cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.o, o_w, obytes, cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.ob, o_b, kDim * sizeof(float), cudaMemcpyDefault));
    TTL_ATTN_CUDA(h, cudaMemcpy(s.sinks, sinks, kHeads * sizeof(float), cudaMemcpyDefault));
    s.uploaded = true;
    return TTL_OK;
}

int ttl_attn_forward_async(ttl_attn *h, int layer, size_t position, const float *x, float *residual) {
    if (!h) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (!x || !residual) {
        return attn_fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    int rc = check_layer(h, layer);
    if (rc) {
        return rc;
    }
    if (position >= h->capacity) {
        return attn_fail(h, TTL_ERR_STATE, "position exceeds startup token capacity");  // src/model.cpp:250-252
    }
    TTL_ATTN_CUDA(h, cudaSetDevice(h->device));
    const AttnLayer &s = h->L[size_t(layer)];
    QkvArgs qa{x,  s.norm, s.q, s.k, s.v, s.qb, s.kb, s.vb, h->freq, h->magnitude, int(position), h->q, s.kc, s.vc,
               h->status};
    // every SM: items are spread over the CTAs first, so each CTA gets about
    // 1280 / 148 of them
    attn_qkv_kernel<<<h->sms, kQkvThreads, kQkvSmem, h->stream>>>(qa);
    // window (src/model.cpp:261-262): even layers attend to the last 128 positions
    const size_t first = (layer % 2 == 0 && position + 1 > size_t(kWindow)) ? position + 1 - kWindow : 0;
    const int count = int(position + 1 - first);
    const int splits = std::clamp((count + 31) / 32, 1, std::min(kMaxSplits, std::max(1, h->sms / kKvHeads)));
    const int per_split = (count + splits - 1) / splits;
    DecodeArgs da{h->q, s.kc, s.vc, s.sinks, int(first), count, per_split, h->part, h->arrive, h->att};
    attn_decode_kernel<<<dim3(kKvHeads, splits), 256, 0, h->stream>>>(da);
    attn_out_kernel<<<h->sms, kOutThreads, kOutSmem, h->stream>>>(s.o, s.ob, h->att, x, residual, h->status);
    TTL_ATTN_CUDA(h, cudaGetLastError());
    return TTL_OK;
}

int ttl_attn_forward(ttl_attn *h, int layer, size_t position, const float *x, float *residual, float *attended) {
    if (!h) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (!x || !residual) {
        return attn_fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    TTL_ATTN_CUDA(h, cudaSetDevice(h->device));
    TTL_ATTN_CUDA(h, cudaMemcpyAsync(h->d_x, x, kDim * sizeof(float), cudaMemcpyDefault, h->stream));
    int rc = ttl_attn_forward_async(h, layer, position, h->d_x, h->d_res);
    if (rc) {
        return rc;
    }
    TTL_ATTN_CUDA(h, cudaMemcpyAsync(residual, h->d_res, kDim * sizeof(float), cudaMemcpyDefault, h->stream));
    if (attended) {
        TTL_ATTN_CUDA(h, cudaMemcpyAsync(attended, h->att, kQWidth * sizeof(float), cudaMemcpyDefault, h->stream));
    }
    TTL_ATTN_CUDA(h, cudaStreamSynchronize(h->stream));
    return check_status(h);
}

int ttl_attn_sync(ttl_attn *h) {
    if (!h) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    TTL_ATTN_CUDA(h, cudaSetDevice(h->device));
    TTL_ATTN_CUDA(h, cudaStreamSynchronize(h->stream));
    return check_status(h);
}

void *ttl_attn_stream(ttl_attn *h) {
    return h ? static_cast<void *>(h->stream) : nullptr;
}

}  // extern "C"
