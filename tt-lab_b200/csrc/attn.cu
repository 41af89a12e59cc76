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
// Weights.  The upload re-lays each Q8_0 matrix (34-byte blocks: an f16 scale
// and 32 int8) as 16-byte-aligned int8 rows plus a separate table of f16
// scales per row, so a row moves with one bulk copy and is read with 16-byte
// loads.  The Q, K and V rows form one matrix in unit order: unit u is a
// RoPE pair (rows r and r + 32 of one head; Q heads, then K heads) or two
// consecutive V rows, stored as packed rows 2u and 2u + 1.
//
// Three launches per (layer, position), on the handle's stream, each with
// programmatic dependent launch: a kernel requests its weight rows first,
// then waits for the previous kernel's results (griddepcontrol.wait), so the
// weight stream overlaps the previous kernel and the launch gap.
//   attn_qkv_kernel   CTA c takes a contiguous range of units (about 17 of
//                     the 2560) and bulk-copies their rows into shared
//                     memory, one mbarrier per unit; every CTA reduces x to
//                     its RMS (a block tree, identical in every CTA) and keeps
//                     the normalized x in shared memory; warp w sums unit w
//                     (lane l: 16-column chunks l, l + 32, ...), rotates
//                     Q / K pairs and writes Q to scratch, K and V into the
//                     layer's cache at `position`.
//   attn_decode_kernel  grid (KV head, 8 splits of the window), one cluster of
//                     8 CTAs per KV head: the 8 query heads of the KV head (one
//                     warp each) run an online softmax over the split's
//                     positions, in K / V tiles of 64 positions bulk-copied
//                     into shared memory (two in flight; the earlier
//                     positions' copies go out before the wait); CTA r of the
//                     cluster then merges head r's partials (max, sum, 64
//                     values) over the cluster's shared memory with the sink.
//   attn_out_kernel   the output projection (4096 columns): CTA c takes rows
//                     [c * 2880 / G, (c + 1) * 2880 / G), warp w sums row pair
//                     w, adds bias and the residual x.
// The matrices are HBM-bound streams (Q/K/V 15.7 MB, output 12.6 MB per
// layer); the KV cache adds 4 KB per attended position.
#include <cooperative_groups.h>
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

// Packed Q/K/V: 5120 rows in unit order (see above).
constexpr int kQkvRows = kQWidth + 2 * kKvWidth;  // 5120
constexpr int kQkvUnits = kQkvRows / 2;           // 2560
constexpr int kQUnits = kQWidth / 2;              // 2048
constexpr int kKUnits = kKvWidth / 2;             // 256
constexpr int kQkvBlocks = kDim / 32;             // 90
constexpr int kOutBlocks = kQWidth / 32;          // 128
constexpr int kQkvScalePitch = 192;               // bytes of f16 scales per packed row (90 used)
constexpr int kOutScalePitch = 256;
constexpr int kQkvMaxUnits = 18;                  // units of one CTA (2560 over >= 148 CTAs)
constexpr int kOutMaxRows = 20;                   // output rows of one CTA (2880 over >= 148 CTAs)
constexpr int kQkvThreads = 32 * kQkvMaxUnits;      // a warp per unit
constexpr int kOutThreads = 512;
constexpr int kMinCtas = 148;                     // the grids are the SM count, at least this many
constexpr size_t kQkvSmem = size_t(kQkvMaxUnits) * 2 * (kDim + kQkvScalePitch) + kDim * 4;
constexpr size_t kOutSmem = size_t(kOutMaxRows) * (kQWidth + kOutScalePitch) + kQWidth * 4;
static_assert((kQkvUnits + kMinCtas - 1) / kMinCtas <= kQkvMaxUnits, "units per CTA");
static_assert((kDim + kMinCtas - 1) / kMinCtas <= kOutMaxRows, "rows per CTA");
static_assert(kQkvSmem <= 227 * 1024 && kOutSmem <= 227 * 1024, "shared memory per CTA");

struct AttnLayer {
    float *norm = nullptr;           // [2880]
    uint8_t *wq = nullptr;           // packed Q/K/V int8 [5120][2880]
    uint8_t *ws = nullptr;           // their f16 scales [5120][192 bytes]
    float *wb = nullptr;             // their biases [5120], packed order
    uint8_t *oq = nullptr;           // output int8 [2880][4096]
    uint8_t *os = nullptr;           // its f16 scales [2880][256 bytes]
    float *ob = nullptr;             // [2880]
    float *sinks = nullptr;          // [64]
    float *kc = nullptr;             // KV cache, head-major: [8][capacity][64]
    float *vc = nullptr;
    bool uploaded = false;
};

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t su32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch: let the next kernel on the stream start
// (its CTAs only request weights until they wait), and wait for the previous
// kernel's results.  No-ops for a launch without the attribute.
__device__ __forceinline__ void launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_previous() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// One bulk copy global -> shared completed on `bar` (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ void expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}

// Waits (bounded, 2 s) for phase 0 of `bar` by the whole warp; on a timeout
// it records kStatusWaitTimeout, waits once more for the copies in flight
// and returns false.  Warp-uniform result.
__device__ __forceinline__ bool wait_rows(uint64_t *bar, uint32_t *status) {
    const bool ok = __all_sync(0xffffffffu, ttl::tc::mbar_wait(bar, 0));
    if (!ok) {
        if ((threadIdx.x & 31) == 0) {
            ttl::set_status(status, ttl::kStatusWaitTimeout);
        }
        ttl::tc::mbar_wait(bar, 0);  // the copies in flight, bounded again
    }
    return ok;
}

// Byte k of w (w with every byte's top bit flipped: the int8 q as q + 128)
// as an f32: the bytes 0x4B00_00{q+128} are the float 2^23 + 128 + q, so one
// byte permute and one subtraction give q exactly.
__device__ __forceinline__ float q8f(uint32_t w, uint32_t k) {
    return __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7540u + k))) - 8388736.0f;
}

// Dot product of 16 int8 (one 16-byte load) with 16 f32 of x.
__device__ __forceinline__ float dot16(uint4 q, const float4 (&x)[4]) {
    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        a0 = fmaf(q8f(w[i], 0), x[i].x, a0);
        a1 = fmaf(q8f(w[i], 1), x[i].y, a1);
        a0 = fmaf(q8f(w[i], 2), x[i].z, a0);
        a1 = fmaf(q8f(w[i], 3), x[i].w, a1);
    }
    return a0 + a1;
}

// x in shared memory is laid out in 16-column chunks of four float4, float4 i
// of chunk c stored at slot i ^ ((c >> 1) & 3): the eight lanes of a quarter
// warp, reading float4 i of chunks c .. c + 7 (64 bytes apart), then hit
// eight different bank groups.
__device__ __forceinline__ int xswz(int k) {  // float index of column k
    const int c = k >> 4, i = (k >> 2) & 3;
    return 16 * c + 4 * (i ^ ((c >> 1) & 3)) + (k & 3);
}

// Two staged rows (int8 at q0 / q1, f16 scales at s0 / s1) times x (shared,
// swizzled as above), kChunks 16-column chunks, lane l taking chunks l,
// l + 32, ...; the sums land on every lane.
template <int kChunks>
__device__ __forceinline__ void dot_pair(const uint8_t *q0, const uint8_t *q1, const uint16_t *s0, const uint16_t *s1,
                                         const float *xs, int lane, float &r0, float &r1) {
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
    for (int m = 0; m < (kChunks + 31) / 32; ++m) {
        const int c = lane + 32 * m;
        if (kChunks % 32 == 0 || c < kChunks) {
            float4 x[4];
            const int f = (c >> 1) & 3;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                x[i] = reinterpret_cast<const float4 *>(xs)[4 * c + (i ^ f)];
            }
            const uint4 w0 = reinterpret_cast<const uint4 *>(q0)[c];
            const uint4 w1 = reinterpret_cast<const uint4 *>(q1)[c];
            acc0 = fmaf(h2f(s0[c >> 1]), dot16(w0, x), acc0);
            acc1 = fmaf(h2f(s1[c >> 1]), dot16(w1, x), acc1);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, o);
    }
    r0 = acc0;
    r1 = acc1;
}

// Source of packed Q/K/V row p: matrix (0 Q, 1 K, 2 V) and its row.
__host__ __device__ __forceinline__ void qkv_source(int p, int &mat, int &row) {
    const int u = p >> 1, h = p & 1;
    if (u < kQUnits + kKUnits) {
        const int v = (u < kQUnits) ? u : u - kQUnits;
        mat = (u < kQUnits) ? 0 : 1;
        row = (v / 32) * kHead + (v % 32) + 32 * h;
    } else {
        mat = 2;
        row = 2 * (u - kQUnits - kKUnits) + h;
    }
}

// Upload-time re-layout of one Q8_0 matrix (rows of `blocks` 34-byte blocks)
// into int8 rows and an f16 scale table: packed row p is row p of mats[0],
// or with `qkv` set the row qkv_source names (and its bias goes to b[p]).
// One CTA per packed row.
struct RepackArgs {
    const uint8_t *mats[3];
    const float *bias[3];
    int blocks;
    int scale_pitch;
    int qkv;  // rows in unit order from the three matrices
    uint8_t *q;
    uint8_t *s;
    float *b;
};

__global__ void attn_repack_kernel(RepackArgs a) {
    const int p = blockIdx.x;
    int mat = 0, row = p;
    if (a.qkv) {
        qkv_source(p, mat, row);
    }
    const uint8_t *src = a.mats[mat] + size_t(row) * size_t(a.blocks) * 34;
    uint8_t *dq = a.q + size_t(p) * size_t(a.blocks) * 32;
    uint8_t *ds = a.s + size_t(p) * size_t(a.scale_pitch);
    for (int b = threadIdx.x; b < a.blocks; b += blockDim.x) {
        const uint8_t *blk = src + size_t(b) * 34;
        ds[2 * b] = blk[0];
        ds[2 * b + 1] = blk[1];
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            dq[32 * b + k] = blk[2 + k];
        }
    }
    for (int b = a.blocks * 2 + threadIdx.x; b < a.scale_pitch; b += blockDim.x) {
        ds[b] = 0;
    }
    if (threadIdx.x == 0 && a.b) {
        a.b[p] = a.bias[mat][row];
    }
}

struct QkvArgs {
    const float *x;
    const float *norm;
    const uint8_t *wq;   // packed int8 rows
    const uint8_t *ws;   // packed f16 scales
    const float *wb;     // packed biases
    const float *freq;   // [32]
    float magnitude;
    int position;
    float *qout;         // [4096] rotated
    float *kc, *vc;      // this layer's caches, [8][capacity][64]
    int capacity;
    uint32_t *status;
};

// Units [u0, u1) of CTA c: contiguous, as even as the grid allows.
__device__ __forceinline__ int unit_lo(int c, int g, int n) {
    return int((long long)c * n / g);
}

__global__ void __launch_bounds__(kQkvThreads, 1) attn_qkv_kernel(QkvArgs a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    uint8_t *sq = dyn;                                                        // [36][2880] int8
    uint8_t *ss = sq + size_t(kQkvMaxUnits) * 2 * kDim;                      // [36][192] f16 scales
    float *xs = reinterpret_cast<float *>(ss + size_t(kQkvMaxUnits) * 2 * kQkvScalePitch);  // [2880]
    __shared__ float red[kQkvThreads / 32];
    __shared__ __align__(8) uint64_t bar[kQkvMaxUnits];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int u0 = unit_lo(blockIdx.x, gridDim.x, kQkvUnits);
    const int n = unit_lo(blockIdx.x + 1, gridDim.x, kQkvUnits) - u0;
    // lane k of warp 0 requests unit k's two rows and their scales (weights
    // only: nothing the previous kernel writes)
    if (warp == 0 && lane < n) {
        uint64_t *b = &bar[lane];
        ttl::tc::mbar_init(b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        expect_tx(b, 2u * (kDim + kQkvScalePitch));
        const size_t p = 2 * size_t(u0 + lane);
        bulk_copy(sq + size_t(lane) * 2 * kDim, a.wq + p * kDim, 2u * kDim, b);
        bulk_copy(ss + size_t(lane) * 2 * kQkvScalePitch, a.ws + p * kQkvScalePitch, 2u * kQkvScalePitch, b);
    }
    launch_dependents();
    wait_previous();  // x is the previous kernel's output
    // rms_norm (src/tensor.cpp:568-580) of x: a tree over the block, the
    // same in every CTA
    float ssum = 0.0f;
    for (int i = threadIdx.x; i < kDim; i += blockDim.x) {
        const float v = a.x[i];
        ssum = fmaf(v, v, ssum);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    }
    if (lane == 0) {
        red[warp] = ssum;
    }
    __syncthreads();  // also: the mbarrier initialisations are visible
    float total = 0.0f;
    for (int w = 0; w < kQkvThreads / 32; ++w) {
        total += red[w];
    }
    const float scale = 1.0f / sqrtf(total / float(kDim) + 1.0e-5f);
    for (int i = threadIdx.x; i < kDim; i += blockDim.x) {
        xs[xswz(i)] = a.x[i] * scale * a.norm[i];
    }
    __syncthreads();
    for (int k = warp; k < n; k += kQkvThreads / 32) {
        if (!wait_rows(&bar[k], a.status)) {
            break;
        }
        const uint8_t *q0 = sq + size_t(k) * 2 * kDim;
        const uint16_t *s0 = reinterpret_cast<const uint16_t *>(ss + size_t(k) * 2 * kQkvScalePitch);
        float d0, d1;
        dot_pair<kDim / 16>(q0, q0 + kDim, s0, s0 + kQkvScalePitch / 2, xs, lane, d0, d1);
        if (lane == 0) {
            const int p = 2 * (u0 + k);
            int mat, r0;
            qkv_source(p, mat, r0);
            const float x0 = __fadd_rn(a.wb[p], d0);
            const float x1 = __fadd_rn(a.wb[p + 1], d1);
            if (mat < 2) {
                // rows (r0, r0 + 32) of a head: one RoPE pair
                const int pair = r0 % kHead;
                const float theta = __fmul_rn(float(a.position), a.freq[pair]);
                const float c = __fmul_rn(cosf(theta), a.magnitude);
                const float sn = __fmul_rn(sinf(theta), a.magnitude);
                const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
                const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
                float *dst = (mat == 0) ? a.qout + r0
                                        : a.kc + (size_t(r0 / kHead) * a.capacity + a.position) * kHead + r0 % kHead;
                dst[0] = y0;
                dst[kHead / 2] = y1;
            } else {
                float *dst = a.vc + (size_t(r0 / kHead) * a.capacity + a.position) * kHead + r0 % kHead;
                dst[0] = x0;
                dst[1] = x1;
            }
        }
    }
    // a unit whose wait gave up leaves its copies to this bounded drain
    if (warp == 0 && lane < n) {
        ttl::tc::mbar_wait(&bar[lane], 0);
    }
}

struct DecodeArgs {
    const float *q;      // [4096] rotated
    const float *kc, *vc;  // [8][capacity][64]
    int capacity;
    const float *sinks;
    int first, count;    // window [first, first + count); its last position is `position`
    int position;        // written by the QKV kernel of this launch: read after the wait
    int per_split;       // positions per split (ceil(count / kSplits))
    float *out;          // [4096]
    uint32_t *status;
};

constexpr int kSplits = 8;     // CTAs per KV head: one cluster, merged in distributed shared memory
constexpr int kTileP = 64;     // positions per staged tile (two tiles in flight)
constexpr int kPartPitch = 68; // max, sum, 64 values (+ padding)
struct DecodeSmem {
    float k[2][kTileP][kHead];
    float v[2][kTileP][kHead];
    float q[8][kHead];
    float p[8][kTileP];
    float part[8][kPartPitch];
    float cur_k[kHead];
    float cur_v[kHead];
    alignas(8) uint64_t bar[2];
};
constexpr size_t kDecodeSmem = sizeof(DecodeSmem) + 16;

// Stages positions [t0, t1) of KV head kv into buffer b: one bulk copy for
// the K rows and one for the V rows (contiguous in the head-major cache).
// `position`'s rows are being written by the QKV kernel while these copies
// run; the slot is overwritten from cur_k / cur_v once the tile has landed.
__device__ __forceinline__ void stage_tile(DecodeSmem &s, const DecodeArgs &a, int kv, int t0, int t1, int b) {
    const size_t off = (size_t(kv) * a.capacity + t0) * kHead;
    const uint32_t bytes = uint32_t(t1 - t0) * kHead * 4u;
    expect_tx(&s.bar[b], 2u * bytes);
    bulk_copy(&s.k[b][0][0], a.kc + off, bytes, &s.bar[b]);
    bulk_copy(&s.v[b][0][0], a.vc + off, bytes, &s.bar[b]);
}

// grid (8 KV heads, kSplits), clusters of kSplits along y, 8 warps: warp w is
// query head kv * 8 + w.  Each CTA runs the online softmax of its split of the
// window; then CTA r of the cluster merges head kv * 8 + r over the splits
// with the head's sink (src/model.cpp:270-288).
__global__ void __launch_bounds__(256, 2) attn_decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) uint8_t dyn_raw[];
    DecodeSmem &s = *reinterpret_cast<DecodeSmem *>((reinterpret_cast<uintptr_t>(dyn_raw) + 15) & ~uintptr_t(15));
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int kv = blockIdx.x;
    const int split = int(cluster.block_rank());
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const int begin = a.first + split * a.per_split;
    const int end = min(a.first + a.count, begin + a.per_split);
    const int ntiles = (end > begin) ? (end - begin + kTileP - 1) / kTileP : 0;
    // the cache rows of earlier positions were written by earlier launches:
    // their copies go out before the wait for the QKV kernel
    if (threadIdx.x == 0) {
        ttl::tc::mbar_init(&s.bar[0], 1);
        ttl::tc::mbar_init(&s.bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int t = 0; t < 2 && t < ntiles; ++t) {
            const int t0 = begin + t * kTileP;
            stage_tile(s, a, kv, t0, min(end, t0 + kTileP), t);
        }
    }
    launch_dependents();
    wait_previous();  // the rotated query and this position's K / V
    for (int i = threadIdx.x; i < 8 * kHead; i += blockDim.x) {
        s.q[i / kHead][i % kHead] = a.q[(kv * 8) * kHead + i];
    }
    const bool has_cur = (a.position >= begin && a.position < end);
    if (has_cur && threadIdx.x < 2 * kHead) {
        const size_t off = (size_t(kv) * a.capacity + a.position) * kHead;
        const int d = threadIdx.x & (kHead - 1);
        if (threadIdx.x < kHead) {
            s.cur_k[d] = __ldcg(a.kc + off + d);
        } else {
            s.cur_v[d] = __ldcg(a.vc + off + d);
        }
    }
    __syncthreads();
    const float scale = 0.125f;  // 1 / sqrt(64)
    float m = -INFINITY, l = 0.0f, acc0 = 0.0f, acc1 = 0.0f;
    bool ok = true;
    int staged = min(2, ntiles);  // tiles whose copies were issued
    int t = 0;
    for (; t < ntiles; ++t) {
        const int b = t & 1;
        const int t0 = begin + t * kTileP;
        const int t1 = min(end, t0 + kTileP);
        const int n = t1 - t0;
        if (!__syncthreads_and(ttl::tc::mbar_wait(&s.bar[b], uint32_t(t >> 1) & 1u))) {
            if (threadIdx.x == 0) {
                ttl::set_status(a.status, ttl::kStatusWaitTimeout);
            }
            ok = false;
            break;
        }
        if (a.position >= t0 && a.position < t1 && threadIdx.x < 2 * kHead) {
            const int d = threadIdx.x & (kHead - 1);
            if (threadIdx.x < kHead) {
                s.k[b][a.position - t0][d] = s.cur_k[d];
            } else {
                s.v[b][a.position - t0][d] = s.cur_v[d];
            }
        }
        __syncthreads();
        // scores of positions lane and lane + 32
        float sc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = lane + 32 * h;
            float d = 0.0f;
            if (j < n) {
                // float4 (c + lane) % 16 at step c: the rows are 256 bytes
                // apart, so the eight lanes of a quarter warp hit eight bank
                // groups
#pragma unroll 4
                for (int c = 0; c < kHead / 4; ++c) {
                    const int cc = (c + lane) & (kHead / 4 - 1);
                    const float4 kk = *reinterpret_cast<const float4 *>(&s.k[b][j][4 * cc]);
                    const float4 qq = *reinterpret_cast<const float4 *>(&s.q[w][4 * cc]);
                    d = fmaf(qq.x, kk.x, d);
                    d = fmaf(qq.y, kk.y, d);
                    d = fmaf(qq.z, kk.z, d);
                    d = fmaf(qq.w, kk.w, d);
                }
            }
            sc[h] = (j < n) ? __fmul_rn(d, scale) : -INFINITY;
        }
        float mt = fmaxf(sc[0], sc[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
        }
        const float mn = fmaxf(m, mt);
        const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
        const float p0 = (lane < n) ? expf(sc[0] - mn) : 0.0f;
        const float p1 = (lane + 32 < n) ? expf(sc[1] - mn) : 0.0f;
        s.p[w][lane] = p0;
        s.p[w][lane + 32] = p1;
        float ps = p0 + p1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ps += __shfl_xor_sync(0xffffffffu, ps, o);
        }
        l = l * corr + ps;
        acc0 *= corr;
        acc1 *= corr;
        __syncwarp();
        for (int j = 0; j < n; ++j) {
            const float pj = s.p[w][j];
            const float2 vv = *reinterpret_cast<const float2 *>(&s.v[b][j][2 * lane]);
            acc0 = fmaf(pj, vv.x, acc0);
            acc1 = fmaf(pj, vv.y, acc1);
        }
        m = mn;
        // buffer b is read (generic proxy): it may be refilled (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (t + 2 < ntiles) {
            const int u0 = begin + (t + 2) * kTileP;
            if (threadIdx.x == 0) {
                stage_tile(s, a, kv, u0, min(end, u0 + kTileP), b);
            }
            ++staged;
        }
    }
    if (!ok) {
        // copies still in flight (tiles t .. staged - 1) land before the
        // shared memory goes (bounded)
        if (threadIdx.x == 0) {
            for (int u = t; u < staged; ++u) {
                ttl::tc::mbar_wait(&s.bar[u & 1], uint32_t(u >> 1) & 1u);
            }
        }
        m = -INFINITY;
        l = acc0 = acc1 = 0.0f;
    }
    if (lane == 0) {
        s.part[w][0] = m;
        s.part[w][1] = l;
    }
    s.part[w][2 + 2 * lane] = acc0;
    s.part[w][3 + 2 * lane] = acc1;
    cluster.sync();
    // merge head kv * 8 + split over the cluster's CTAs (warp 0): lane l
    // holds dimensions 2l, 2l + 1
    if (w == 0) {
        const int hm = kv * 8 + split;
        const float sink = a.sinks[hm];
        float ms[kSplits], ls[kSplits];
        float mx = sink;
#pragma unroll
        for (int r = 0; r < kSplits; ++r) {
            const float *rp = cluster.map_shared_rank(&s.part[split][0], r);
            ms[r] = rp[0];
            ls[r] = rp[1];
            mx = fmaxf(mx, ms[r]);
        }
        float den = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int r = 0; r < kSplits; ++r) {
            const float f = (ms[r] == -INFINITY) ? 0.0f : expf(ms[r] - mx);
            const float *rp = cluster.map_shared_rank(&s.part[split][0], r);
            den = fmaf(ls[r], f, den);
            o0 = fmaf(rp[2 + 2 * lane], f, o0);
            o1 = fmaf(rp[3 + 2 * lane], f, o1);
        }
        den += expf(sink - mx);
        a.out[hm * kHead + 2 * lane] = o0 / den;
        a.out[hm * kHead + 2 * lane + 1] = o1 / den;
    }
    cluster.sync();  // no CTA leaves while another reads its partials
}

// residual[r] = x[r] + (bias[r] + the row's dot product with the attention
// output) for the 2880 x 4096 output projection: CTA c takes rows
// [c * 2880 / G, (c + 1) * 2880 / G) (at most 20), requested as bulk copies
// before it waits for the attention output; warp w sums rows (2w, 2w + 1).
__global__ void __launch_bounds__(kOutThreads, 1) attn_out_kernel(const uint8_t *__restrict__ oq,
                                                                 const uint8_t *__restrict__ os,
                                                                 const float *__restrict__ ob,
                                                                 const float *__restrict__ att,
                                                                 const float *__restrict__ x,
                                                                 float *__restrict__ residual, uint32_t *status) {
    extern __shared__ __align__(16) uint8_t dyn[];
    uint8_t *sq = dyn;                                                 // [20][4096] int8
    uint8_t *ss = sq + size_t(kOutMaxRows) * kQWidth;                  // [20][256] f16 scales
    float *as = reinterpret_cast<float *>(ss + size_t(kOutMaxRows) * kOutScalePitch);  // [4096]
    __shared__ __align__(8) uint64_t bar[kOutMaxRows / 2];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int r0 = unit_lo(blockIdx.x, gridDim.x, kDim);
    const int n = unit_lo(blockIdx.x + 1, gridDim.x, kDim) - r0;
    const int pairs = (n + 1) / 2;
    if (warp == 0 && lane < pairs) {
        uint64_t *b = &bar[lane];
        ttl::tc::mbar_init(b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t rows = uint32_t(min(2, n - 2 * lane));
        expect_tx(b, rows * (kQWidth + kOutScalePitch));
        const size_t r = size_t(r0 + 2 * lane);
        bulk_copy(sq + size_t(2 * lane) * kQWidth, oq + r * kQWidth, rows * kQWidth, b);
        bulk_copy(ss + size_t(2 * lane) * kOutScalePitch, os + r * kOutScalePitch, rows * kOutScalePitch, b);
    }
    launch_dependents();
    wait_previous();  // the attention output is the previous kernel's
    for (int i = threadIdx.x; i < kQWidth / 4; i += blockDim.x) {
        reinterpret_cast<float4 *>(as)[xswz(4 * i) >> 2] = __ldcg(reinterpret_cast<const float4 *>(att) + i);
    }
    __syncthreads();
    for (int k = warp; k < pairs; k += kOutThreads / 32) {
        if (!wait_rows(&bar[k], status)) {
            break;
        }
        const int two = min(2, n - 2 * k);
        const uint8_t *q0 = sq + size_t(2 * k) * kQWidth;
        const uint16_t *s0 = reinterpret_cast<const uint16_t *>(ss + size_t(2 * k) * kOutScalePitch);
        // a lone last row reads its own row twice
        const size_t second = (two == 2) ? 1 : 0;
        float d0, d1;
        dot_pair<kQWidth / 16>(q0, q0 + second * kQWidth, s0, s0 + second * (kOutScalePitch / 2), as, lane, d0, d1);
        if (lane == 0) {
            const int r = r0 + 2 * k;
            residual[r] = __fadd_rn(x[r], __fadd_rn(ob[r], d0));
            if (two == 2) {
                residual[r + 1] = __fadd_rn(x[r + 1], __fadd_rn(ob[r + 1], d1));
            }
        }
    }
    if (warp == 0 && lane < pairs) {
        ttl::tc::mbar_wait(&bar[lane], 0);
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
    // the grids cover at least kMinCtas CTAs (the per-CTA row shares are
    // sized for that)
    h->sms = std::max(prop.multiProcessorCount, kMinCtas);
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
    rc = rc ? rc : attn_alloc(h, &h->d_x, kDim);
    rc = rc ? rc : attn_alloc(h, &h->d_res, kDim);
    rc = rc ? rc : attn_alloc(h, &h->status, 1);
    if (rc) {
        return bail(attn_fail(nullptr, rc, h->error));
    }
    // all three kernels ask for the largest shared-memory carveout (as the
    // MoE kernels on the same stream need), so consecutive launches never
    // wait for the SMs to repartition L1 and shared memory
    if (cudaFuncSetAttribute(attn_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kQkvSmem)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kOutSmem)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_qkv_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDecodeSmem)) !=
            cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_out_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared)) != cudaSuccess) {
        return bail(attn_fail(nullptr, TTL_ERR_CUDA, "cannot configure the attention kernels"));
    }
    float freq[kHead / 2];
    rope_table(freq, &h->magnitude);
    if (cudaMemcpy(h->freq, freq, sizeof(freq), cudaMemcpyHostToDevice) != cudaSuccess ||
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
    const size_t qbytes = size_t(kQWidth) * kQkvBlocks * 34, kbytes = size_t(kKvWidth) * kQkvBlocks * 34;
    const size_t obytes = size_t(kDim) * kOutBlocks * 34;
    if (!s.norm) {
        int rc = attn_alloc(h, &s.norm, kDim);
        rc = rc ? rc : attn_alloc(h, &s.wq, size_t(kQkvRows) * kDim);
        rc = rc ? rc : attn_alloc(h, &s.ws, size_t(kQkvRows) * kQkvScalePitch);
        rc = rc ? rc : attn_alloc(h, &s.wb, kQkvRows);
        rc = rc ? rc : attn_alloc(h, &s.oq, size_t(kDim) * kQWidth);
        rc = rc ? rc : attn_alloc(h, &s.os, size_t(kDim) * kOutScalePitch);
        rc = rc ? rc : attn_alloc(h, &s.ob, kDim);
        rc = rc ? rc : attn_alloc(h, &s.sinks, kHeads);
        rc = rc ? rc : attn_alloc(h, &s.kc, size_t(h->capacity) * kKvWidth);
        rc = rc ? rc : attn_alloc(h, &s.vc, size_t(h->capacity) * kKvWidth);
        if (rc) {
            return rc;
        }
    }
    // the GGUF tensors go to a scratch area, from which the re-layout kernel
    // writes the packed rows (upload is not a compute call: it may allocate)
    const size_t raw = qbytes + 2 * kbytes + obytes;
    const size_t braw = size_t(kQWidth + 2 * kKvWidth) * sizeof(float);
    uint8_t *tmp = nullptr;
    if (cudaMalloc(&tmp, raw + braw) != cudaSuccess) {
        cudaGetLastError();
        return attn_fail(h, TTL_ERR_CUDA, "device allocation of the upload scratch failed");
    }
    uint8_t *tq = tmp, *tk = tq + qbytes, *tv = tk + kbytes, *to = tv + kbytes;
    float *tb = reinterpret_cast<float *>(to + obytes);
    const cudaStream_t st = h->stream;
    cudaError_t e = cudaMemcpyAsync(tq, q_w, qbytes, cudaMemcpyDefault, st);
    e = (e == cudaSuccess) ? cudaMemcpyAsync(tk, k_w, kbytes, cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess) ? cudaMemcpyAsync(tv, v_w, kbytes, cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess) ? cudaMemcpyAsync(to, o_w, obytes, cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess) ? cudaMemcpyAsync(tb, q_b, kQWidth * sizeof(float), cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess) ? cudaMemcpyAsync(tb + kQWidth, k_b, kKvWidth * sizeof(float), cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess)
            ? cudaMemcpyAsync(tb + kQWidth + kKvWidth, v_b, kKvWidth * sizeof(float), cudaMemcpyDefault, st)
            : e;
    if (e == cudaSuccess) {
        RepackArgs qa{{tq, tk, tv}, {tb, tb + kQWidth, tb + kQWidth + kKvWidth}, kQkvBlocks, kQkvScalePitch, 1,
                      s.wq, s.ws, s.wb};
        attn_repack_kernel<<<kQkvRows, 128, 0, st>>>(qa);
        RepackArgs oa{{to, to, to}, {nullptr, nullptr, nullptr}, kOutBlocks, kOutScalePitch, 0, s.oq, s.os, nullptr};
        attn_repack_kernel<<<kDim, 128, 0, st>>>(oa);
        e = cudaGetLastError();
    }
    e = (e == cudaSuccess) ? cudaMemcpyAsync(s.norm, attn_norm, kDim * sizeof(float), cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess) ? cudaMemcpyAsync(s.ob, o_b, kDim * sizeof(float), cudaMemcpyDefault, st) : e;
    e = (e == cudaSuccess) ? cudaMemcpyAsync(s.sinks, sinks, kHeads * sizeof(float), cudaMemcpyDefault, st) : e;
    const cudaError_t es = cudaStreamSynchronize(st);
    cudaFree(tmp);
    e = (e == cudaSuccess) ? es : e;
    if (e != cudaSuccess) {
        cudaGetLastError();
        return attn_fail(h, TTL_ERR_CUDA, std::string("attention weight upload: ") + cudaGetErrorString(e));
    }
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
    // programmatic dependent launch for all three: each may start while its
    // predecessor runs and requests its weights before it waits
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.stream = h->stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    QkvArgs qa{x,    s.norm, s.wq, s.ws, s.wb, h->freq, h->magnitude, int(position), h->q, s.kc, s.vc,
               int(h->capacity), h->status};
    cfg.gridDim = dim3(unsigned(h->sms));
    cfg.blockDim = dim3(kQkvThreads);
    cfg.dynamicSmemBytes = kQkvSmem;
    TTL_ATTN_CUDA(h, cudaLaunchKernelEx(&cfg, attn_qkv_kernel, qa));
    // window (src/model.cpp:261-262): even layers attend to the last 128 positions
    const size_t first = (layer % 2 == 0 && position + 1 > size_t(kWindow)) ? position + 1 - kWindow : 0;
    const int count = int(position + 1 - first);
    const int per_split = (count + kSplits - 1) / kSplits;
    DecodeArgs da{h->q,         s.kc,      s.vc,   int(h->capacity), s.sinks, int(first), count, int(position),
                  per_split, h->att, h->status};
    cudaLaunchAttribute dattr[2];
    dattr[0] = pdl[0];
    dattr[1].id = cudaLaunchAttributeClusterDimension;
    dattr[1].val.clusterDim.x = 1;
    dattr[1].val.clusterDim.y = kSplits;
    dattr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t dcfg = cfg;
    dcfg.attrs = dattr;
    dcfg.numAttrs = 2;
    dcfg.gridDim = dim3(kKvHeads, kSplits);
    dcfg.blockDim = dim3(256);
    dcfg.dynamicSmemBytes = kDecodeSmem;
    TTL_ATTN_CUDA(h, cudaLaunchKernelEx(&dcfg, attn_decode_kernel, da));
    cfg.gridDim = dim3(unsigned(h->sms));
    cfg.blockDim = dim3(kOutThreads);
    cfg.dynamicSmemBytes = kOutSmem;
    const uint8_t *oq = s.oq, *os = s.os;
    const float *ob = s.ob, *att = h->att;
    TTL_ATTN_CUDA(h, cudaLaunchKernelEx(&cfg, attn_out_kernel, oq, os, ob, att, x, residual, h->status));
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
