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

// y = the dot product of one Q8_0 row with x (cols = 32 * blocks), as the
// reference's AVX-512 clone orders it: lane c accumulates element (c & 15)
// + 16 (c >> 4) of every block, product of the dequantized weight and x
// rounded before the add; then acc0[i] + acc1[i] and a sequential sum over
// i.  Returns the value on every lane.
__device__ __forceinline__ float q8_row_dot(const uint8_t *__restrict__ row, const float *__restrict__ xs, int blocks,
                                            int lane) {
    float acc = 0.0f;
#pragma unroll 4
    for (int b = 0; b < blocks; ++b) {
        const uint8_t *blk = row + size_t(b) * 34;
        const uint16_t sbits = uint16_t(__ldg(blk)) | uint16_t(uint16_t(__ldg(blk + 1)) << 8);
        const int8_t q = int8_t(__ldg(blk + 2 + lane));
        const float w = __fmul_rn(float(q), h2f(sbits));
        acc = __fadd_rn(acc, __fmul_rn(w, xs[b * 32 + lane]));
    }
    const float pair = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 16));  // acc0[i] + acc1[i]
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, pair, i));
    }
    return sum;
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
};

// Work items: 2048 Q pairs, 256 K pairs (rows r, r + 32 of a head), 256 V
// row pairs.
constexpr int kQPairs = kQWidth / 2;
constexpr int kKPairs = kKvWidth / 2;
constexpr int kQkvItems = kQPairs + 2 * kKPairs;

__global__ void __launch_bounds__(kQkvThreads) attn_qkv_kernel(QkvArgs a) {
    __shared__ float xs[kDim];
    __shared__ float red[kQkvThreads / 32];
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
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < kQkvItems; item += warps) {
        if (item < kQPairs + kKPairs) {
            // a Q or K pair of one head: rows r and r + 32, rotated together
            const bool is_q = item < kQPairs;
            const int local = is_q ? item : item - kQPairs;
            const int head = local / 32, pair = local % 32;
            const int r0 = head * kHead + pair, r1 = r0 + kHead / 2;
            const uint8_t *w = is_q ? a.q : a.k;
            const float *bias = is_q ? a.qb : a.kb;
            const float d0 = q8_row_dot(w + size_t(r0) * 90 * 34, xs, 90, lane);
            const float d1 = q8_row_dot(w + size_t(r1) * 90 * 34, xs, 90, lane);
            if (lane == 0) {
                const float x0 = __fadd_rn(bias[r0], d0);
                const float x1 = __fadd_rn(bias[r1], d1);
                const float theta = __fmul_rn(float(a.position), a.freq[pair]);
                const float c = __fmul_rn(cosf(theta), a.magnitude);
                const float s = __fmul_rn(sinf(theta), a.magnitude);
                const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
                const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
                if (is_q) {
                    a.qout[r0] = y0;
                    a.qout[r1] = y1;
                } else {
                    a.kc[size_t(a.position) * kKvWidth + r0] = y0;
                    a.kc[size_t(a.position) * kKvWidth + r1] = y1;
                }
            }
        } else {
            const int r0 = 2 * (item - kQPairs - kKPairs);
            const float d0 = q8_row_dot(a.v + size_t(r0) * 90 * 34, xs, 90, lane);
            const float d1 = q8_row_dot(a.v + size_t(r0 + 1) * 90 * 34, xs, 90, lane);
            if (lane == 0) {
                a.vc[size_t(a.position) * kKvWidth + r0] = __fadd_rn(a.vb[r0], d0);
                a.vc[size_t(a.position) * kKvWidth + r0 + 1] = __fadd_rn(a.vb[r0 + 1], d1);
            }
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
    // merge the splits of this warp's head with its sink (src/model.cpp:270-288)
    const float sink = a.sinks[head];
    const float *ph = a.part + size_t(head) * kMaxSplits * 66;
    float mx = sink;
    for (int sp = 0; sp < int(gridDim.y); ++sp) {
        mx = fmaxf(mx, __ldcg(ph + sp * 66));
    }
    float den = expf(sink - mx);
    float o0 = 0.0f, o1 = 0.0f;
    for (int sp = 0; sp < int(gridDim.y); ++sp) {
        const float ms = __ldcg(ph + sp * 66);
        if (ms == -INFINITY) {
            continue;
        }
        const float f = expf(ms - mx);
        den = fmaf(__ldcg(ph + sp * 66 + 1), f, den);
        o0 = fmaf(__ldcg(ph + sp * 66 + 2 + 2 * lane), f, o0);
        o1 = fmaf(__ldcg(ph + sp * 66 + 3 + 2 * lane), f, o1);
    }
    a.out[head * kHead + 2 * lane] = o0 / den;
    a.out[head * kHead + 2 * lane + 1] = o1 / den;
    if (threadIdx.x == 0) {
        a.arrive[kv] = 0u;  // re-armed for the next launch
    }
}

// residual[r] = x[r] + (bias[r] + the row's dot product with the attention
// output), one warp per row of the 2880 x 4096 output projection.
__global__ void __launch_bounds__(kOutThreads) attn_out_kernel(const uint8_t *__restrict__ o, const float *__restrict__ ob,
                                                              const float *__restrict__ att, const float *__restrict__ x,
                                                              float *__restrict__ residual) {
    __shared__ float as[kQWidth];
    for (int i = threadIdx.x; i < kQWidth; i += blockDim.x) {
        as[i] = att[i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < kDim; r += warps) {
        const float d = q8_row_dot(o + size_t(r) * 128 * 34, as, 128, lane);
        if (lane == 0) {
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
    if (rc) {
        return bail(attn_fail(nullptr, rc, h->error));
    }
    float freq[kHead / 2];
    rope_table(freq, &h->magnitude);
    if (cudaMemcpy(h->freq, freq, sizeof(freq), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(h->arrive, 0, kKvHeads * sizeof(unsigned)) != cudaSuccess) {
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
        rc = rc ? rc : attn_alloc(h, &s.q, qbytes);
        rc = rc ? rc : attn_alloc(h, &s.qb, kQWidth);
        rc = rc ? rc : attn_alloc(h, &s.k, kbytes);
        rc = rc ? rc : attn_alloc(h, &s.kb, kKvWidth);
        rc = rc ? rc : attn_alloc(h, &s.v, kbytes);
        rc = rc ? rc : attn_alloc(h, &s.vb, kKvWidth);
        rc = rc ? rc : attn_alloc(h, &s.o, obytes);
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
    QkvArgs qa{x, s.norm, s.q, s.k, s.v, s.qb, s.kb, s.vb, h->freq, h->magnitude, int(position), h->q, s.kc, s.vc};
    const int qkv_ctas = std::min(h->sms, (kQkvItems + kQkvThreads / 32 - 1) / (kQkvThreads / 32));
    attn_qkv_kernel<<<qkv_ctas, kQkvThreads, 0, h->stream>>>(qa);
    // window (src/model.cpp:261-262): even layers attend to the last 128 positions
    const size_t first = (layer % 2 == 0 && position + 1 > size_t(kWindow)) ? position + 1 - kWindow : 0;
    const int count = int(position + 1 - first);
    const int splits = std::clamp((count + 31) / 32, 1, std::min(kMaxSplits, std::max(1, h->sms / kKvHeads)));
    const int per_split = (count + splits - 1) / splits;
    DecodeArgs da{h->q, s.kc, s.vc, s.sinks, int(first), count, per_split, h->part, h->arrive, h->att};
    attn_decode_kernel<<<dim3(kKvHeads, splits), 256, 0, h->stream>>>(da);
    attn_out_kernel<<<h->sms, kOutThreads, 0, h->stream>>>(s.o, s.ob, h->att, x, residual);
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
    return TTL_OK;
}

int ttl_attn_sync(ttl_attn *h) {
    if (!h) {
        return attn_fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    TTL_ATTN_CUDA(h, cudaSetDevice(h->device));
    TTL_ATTN_CUDA(h, cudaStreamSynchronize(h->stream));
    return TTL_OK;
}

void *ttl_attn_stream(ttl_attn *h) {
    return h ? static_cast<void *>(h->stream) : nullptr;
}

}  // extern "C"
