// prefill.cu -- batched (prefill) MoE: router, routing histogram and stable
// permute, grouped expert products, un-permute combine.
//
// Reference: GptOssModel::moe_batch, tt-lab src/model.cpp:340-461.
//   router      matmul_add_f32 (src/tensor.cpp:497-527): here one thread per
//               (token, expert) runs the reference's own sequential chain
//               (bias first, f32 products rounded, added in column order), so
//               logits -- and therefore top-4 indices -- equal the reference's
//               bit for bit.  Throughput-bound, so the exact order costs little.
//   top-4       selection sort + softmax per token (src/model.cpp:344-378).
//   histogram   per-expert counts, prefix offsets and buckets that are stable in
//               token order (src/model.cpp:380-394).
//   experts     grouped products over each expert's tokens (src/model.cpp:396-448)
//               with the SwiGLU epilogue (:423-433).
//   combine     per token, experts in ascending id order, out += w * down with
//               the product rounded first (src/model.cpp:450-459).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ttl {
namespace {

constexpr int kRouterTokens = 8;          // tokens per router CTA
constexpr int kXRowStride = kDim + 4;     // padded shared row (bank spread)
constexpr int kTile = 8;                  // routed pairs per expert-product tile
constexpr int kXStride = 36;              // padded floats per K-block
constexpr int kTileFloats = kBlocks * kXStride;  // one padded row
constexpr int kProductThreads = 512;

__global__ void prefill_router_kernel(LayerDev L, PrefillWork w, int experts, int tokens,
                                      const float *__restrict__ x) {
    extern __shared__ float xs[];  // [kRouterTokens][kXRowStride]
    const int t0 = blockIdx.x * kRouterTokens;
    const int nt = min(kRouterTokens, tokens - t0);
    for (int i = threadIdx.x; i < nt * kDim; i += blockDim.x) {
        const int t = i / kDim;
        const int c = i - t * kDim;
        xs[t * kXRowStride + c] = x[size_t(t0 + t) * kDim + c];
    }
    __syncthreads();
    const int e = threadIdx.x / kRouterTokens;
    const int t = threadIdx.x % kRouterTokens;
    if (e >= experts || t >= nt) {
        return;
    }
    const float *wr = L.router_w + size_t(e) * kDim;
    const float *xr = xs + t * kXRowStride;
    float s = L.router_b[e];
    for (int c = 0; c < kDim; c += 8) {
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            p[j] = __fmul_rn(__ldg(wr + c + j), xr[c + j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s = __fadd_rn(s, p[j]);
        }
    }
    w.logits[size_t(t0 + t) * experts + e] = s;
}

__global__ void prefill_select_kernel(PrefillWork w, int experts, int tokens) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= tokens) {
        return;
    }
    const float *r = w.logits + size_t(t) * experts;
    uint8_t order[kMaxExperts];
    for (int i = 0; i < experts; ++i) {
        order[i] = uint8_t(i);
    }
    float sel[4];
    for (int i = 0; i < kTopK; ++i) {
        int best = i;
        for (int j = i + 1; j < experts; ++j) {
            if (r[order[j]] > r[order[best]]) {
                best = j;
            }
        }
        const uint8_t tmp = order[i];
        order[i] = order[best];
        order[best] = tmp;
        w.top_idx[t * 4 + i] = order[i];
        sel[i] = r[order[i]];
    }
    float maximum = -INFINITY;
    for (int i = 0; i < kTopK; ++i) {
        maximum = (maximum < sel[i]) ? sel[i] : maximum;
    }
    float wt[4];
    float sum = 0.0f;
    for (int i = 0; i < kTopK; ++i) {
        wt[i] = expf(__fsub_rn(sel[i], maximum));
        sum = __fadd_rn(sum, wt[i]);
    }
    for (int i = 0; i < kTopK; ++i) {
        w.top_w[t * 4 + i] = __fdiv_rn(wt[i], sum);
    }
}

// One CTA: histogram, offsets, stable buckets and the tile work list.
__global__ void __launch_bounds__(1024) prefill_route_kernel(PrefillWork w, int experts, int expert_begin,
                                                             int expert_count, int tokens) {
    __shared__ int counts[kMaxExperts];
    __shared__ int offsets[kMaxExperts + 1];
    for (int e = threadIdx.x; e < experts; e += blockDim.x) {
        counts[e] = 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tokens * kTopK; i += blockDim.x) {
        w.pair_slot[i] = -1;
        const int e = w.top_idx[i];
        if (e < 0 || e >= experts) {
            set_status(w.status, kStatusBadExpert);
            continue;
        }
        const int le = e - expert_begin;
        if (le >= 0 && le < expert_count) {
            atomicAdd(&counts[le], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        int tiles = 0;
        for (int le = 0; le < expert_count; ++le) {
            offsets[le] = run;
            w.counts[le] = counts[le];
            w.offsets[le] = run;
            for (int k = 0; k < counts[le]; k += kTile) {
                w.tiles[tiles++] = (le << 20) | (run + k);
            }
            run += counts[le];
        }
        offsets[expert_count] = run;
        w.offsets[expert_count] = run;
        *w.tile_count = tiles;
    }
    __syncthreads();
    // Stable placement: each warp owns experts; tokens are scanned in order.
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    for (int le = warp; le < expert_count; le += nwarps) {
        const int e = le + expert_begin;
        int base = offsets[le];
        for (int t0 = 0; t0 < tokens; t0 += 32) {
            const int t = t0 + lane;
            int rank = -1;
            if (t < tokens) {
#pragma unroll
                for (int r = 0; r < kTopK; ++r) {
                    if (w.top_idx[t * 4 + r] == e) {
                        rank = r;
                    }
                }
            }
            const unsigned ballot = __ballot_sync(0xffffffffu, rank >= 0);
            if (rank >= 0) {
                const int pos = base + __popc(ballot & ((1u << lane) - 1u));
                w.pair_token[pos] = t;
                w.pair_slot[t * 4 + rank] = pos;
            }
            base += __popc(ballot);
        }
    }
}

__device__ __forceinline__ void load_row_padded(float *dst, const float *__restrict__ src) {
    for (int i = threadIdx.x; i < kDim / 4; i += blockDim.x) {
        const float4 q = *reinterpret_cast<const float4 *>(src + 4 * i);
        const int kb = (4 * i) >> 5;
        *reinterpret_cast<float4 *>(dst + kb * kXStride + ((4 * i) & 31)) = q;
    }
}

// Decodes 16 packed bytes into 32 f32 E2M1 values (exact).
__device__ __forceinline__ void decode_block(const uint4 q, float v[32]) {
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float2 f = __half22float2(e2m1x2_to_half2((words[wd] >> (8 * b)) & 0xffu));
            v[wd * 8 + b * 2] = f.x;
            v[wd * 8 + b * 2 + 1] = f.y;
        }
    }
}

__device__ __forceinline__ float dot32(const float v[32], const float *xb) {
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const float4 p = *reinterpret_cast<const float4 *>(xb + i);
        const float4 q = *reinterpret_cast<const float4 *>(xb + i + 4);
        a0 = fmaf(v[i], p.x, a0);
        a1 = fmaf(v[i + 1], p.y, a1);
        a0 = fmaf(v[i + 2], p.z, a0);
        a1 = fmaf(v[i + 3], p.w, a1);
        a0 = fmaf(v[i + 4], q.x, a0);
        a1 = fmaf(v[i + 5], q.y, a1);
        a0 = fmaf(v[i + 6], q.z, a0);
        a1 = fmaf(v[i + 7], q.w, a1);
    }
    return a0 + a1;
}

// Grouped gate/up products: one tile = up to kTile routed pairs of one expert.
// The tile's activations sit in shared memory; each warp takes output rows,
// lanes split K, and the decoded weights of a block are reused for every pair.
__global__ void __launch_bounds__(kProductThreads, 1)
    prefill_gateup_kernel(LayerDev L, PrefillWork w, const float *__restrict__ x) {
    extern __shared__ __align__(16) float xs[];  // [kTile][kTileFloats]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = kProductThreads / 32;
    const int tiles = *w.tile_count;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int code = w.tiles[tile];
        const int le = code >> 20;
        const int first = code & 0xfffff;
        const int n = min(kTile, w.offsets[le + 1] - first);
        __syncthreads();
        for (int p = 0; p < n; ++p) {
            load_row_padded(xs + p * kTileFloats, x + size_t(w.pair_token[first + p]) * kDim);
        }
        __syncthreads();
        const uint8_t *gm = L.gate + size_t(le) * kPackedMatrixBytes;
        const uint8_t *um = L.up + size_t(le) * kPackedMatrixBytes;
        for (int row = warp; row < kDim; row += nwarps) {
            float ag[kTile], au[kTile];
#pragma unroll
            for (int p = 0; p < kTile; ++p) {
                ag[p] = 0.0f;
                au[p] = 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int kb = lane + 32 * j;
                if (kb < kBlocks) {
                    const uint4 gq = *reinterpret_cast<const uint4 *>(gm + size_t(row) * kNibbleRowBytes + kb * 16);
                    const uint4 uq = *reinterpret_cast<const uint4 *>(um + size_t(row) * kNibbleRowBytes + kb * 16);
                    const float gs = e8m0_ref_scale(gm[scale_offset(row, kb)]);
                    const float us = e8m0_ref_scale(um[scale_offset(row, kb)]);
                    float v[32];
                    decode_block(gq, v);
#pragma unroll
                    for (int p = 0; p < kTile; ++p) {
                        if (p < n) {
                            ag[p] = fmaf(gs, 2.0f * dot32(v, xs + p * kTileFloats + kb * kXStride), ag[p]);
                        }
                    }
                    decode_block(uq, v);
#pragma unroll
                    for (int p = 0; p < kTile; ++p) {
                        if (p < n) {
                            au[p] = fmaf(us, 2.0f * dot32(v, xs + p * kTileFloats + kb * kXStride), au[p]);
                        }
                    }
                }
            }
#pragma unroll
            for (int p = 0; p < kTile; ++p) {
                ag[p] = warp_sum(ag[p]);
                au[p] = warp_sum(au[p]);
            }
            if (lane == 0) {
                const float gb = L.gate_b[size_t(le) * kDim + row];
                const float ub = L.up_b[size_t(le) * kDim + row];
#pragma unroll
                for (int p = 0; p < kTile; ++p) {
                    if (p < n) {
                        w.hidden[size_t(first + p) * kDim + row] =
                            swiglu_ref(__fadd_rn(gb, ag[p]), __fadd_rn(ub, au[p]));
                    }
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kProductThreads, 1) prefill_down_kernel(LayerDev L, PrefillWork w) {
    extern __shared__ __align__(16) float hs[];  // [kTile][kTileFloats]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = kProductThreads / 32;
    const int tiles = *w.tile_count;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int code = w.tiles[tile];
        const int le = code >> 20;
        const int first = code & 0xfffff;
        const int n = min(kTile, w.offsets[le + 1] - first);
        __syncthreads();
        for (int p = 0; p < n; ++p) {
            load_row_padded(hs + p * kTileFloats, w.hidden + size_t(first + p) * kDim);
        }
        __syncthreads();
        const uint8_t *dm = L.down + size_t(le) * kPackedMatrixBytes;
        for (int row = warp; row < kDim; row += nwarps) {
            float acc[kTile];
#pragma unroll
            for (int p = 0; p < kTile; ++p) {
                acc[p] = 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int kb = lane + 32 * j;
                if (kb < kBlocks) {
                    const uint4 q = *reinterpret_cast<const uint4 *>(dm + size_t(row) * kNibbleRowBytes + kb * 16);
                    const float sc = e8m0_ref_scale(dm[scale_offset(row, kb)]);
                    float v[32];
                    decode_block(q, v);
#pragma unroll
                    for (int p = 0; p < kTile; ++p) {
                        if (p < n) {
                            acc[p] = fmaf(sc, 2.0f * dot32(v, hs + p * kTileFloats + kb * kXStride), acc[p]);
                        }
                    }
                }
            }
#pragma unroll
            for (int p = 0; p < kTile; ++p) {
                acc[p] = warp_sum(acc[p]);
            }
            if (lane == 0) {
                const float db = L.down_b[size_t(le) * kDim + row];
#pragma unroll
                for (int p = 0; p < kTile; ++p) {
                    if (p < n) {
                        w.down[size_t(first + p) * kDim + row] = __fadd_rn(db, acc[p]);
                    }
                }
            }
        }
    }
}

// out[t] = sum over the token's experts in ascending id of w * down.
__global__ void prefill_combine_kernel(PrefillWork w, int tokens, float *__restrict__ out) {
    const int t = blockIdx.x;
    if (t >= tokens) {
        return;
    }
    int e[4], r[4];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        e[i] = w.top_idx[t * 4 + i];
        r[i] = i;
    }
    // Sort the four (expert, rank) pairs by expert id (distinct ids).
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
#pragma unroll
        for (int j = 0; j + 1 < kTopK - i; ++j) {
            if (e[j] > e[j + 1]) {
                const int te = e[j], tr = r[j];
                e[j] = e[j + 1];
                r[j] = r[j + 1];
                e[j + 1] = te;
                r[j + 1] = tr;
            }
        }
    }
    int slot[4];
    float wt[4];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        slot[i] = w.pair_slot[t * 4 + r[i]];
        wt[i] = w.top_w[t * 4 + r[i]];
    }
    for (int c = threadIdx.x; c < kDim; c += blockDim.x) {
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < kTopK; ++i) {
            if (slot[i] >= 0) {
                o = __fadd_rn(o, __fmul_rn(wt[i], w.down[size_t(slot[i]) * kDim + c]));
            }
        }
        out[size_t(t) * kDim + c] = o;
    }
}

} // namespace

void configure_prefill_kernels() {
    cudaFuncSetAttribute(prefill_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kRouterTokens * kXRowStride * int(sizeof(float)));
    cudaFuncSetAttribute(prefill_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kTile * kTileFloats * int(sizeof(float)));
    cudaFuncSetAttribute(prefill_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kTile * kTileFloats * int(sizeof(float)));
}

void launch_prefill_router(const LayerDev &L, const PrefillWork &w, const PrefillShape &s, const float *x,
                           cudaStream_t stream) {
    const int grid = (s.tokens + kRouterTokens - 1) / kRouterTokens;
    const int threads = s.experts * kRouterTokens;
    prefill_router_kernel<<<grid, threads, kRouterTokens * kXRowStride * sizeof(float), stream>>>(
        L, w, s.experts, s.tokens, x);
    prefill_select_kernel<<<(s.tokens + 127) / 128, 128, 0, stream>>>(w, s.experts, s.tokens);
}

void launch_prefill_route(const PrefillWork &w, const PrefillShape &s, cudaStream_t stream) {
    prefill_route_kernel<<<1, 1024, 0, stream>>>(w, s.experts, s.expert_begin, s.expert_count, s.tokens);
}

void launch_prefill_gateup(const LayerDev &L, const PrefillWork &w, const PrefillShape &s, const float *x,
                           cudaStream_t stream) {
    prefill_gateup_kernel<<<s.sms, kProductThreads, kTile * kTileFloats * sizeof(float), stream>>>(L, w, x);
}

void launch_prefill_down(const LayerDev &L, const PrefillWork &w, const PrefillShape &s, cudaStream_t stream) {
    prefill_down_kernel<<<s.sms, kProductThreads, kTile * kTileFloats * sizeof(float), stream>>>(L, w);
}

void launch_prefill_combine(const PrefillWork &w, const PrefillShape &s, float *out, cudaStream_t stream) {
    prefill_combine_kernel<<<s.tokens, 256, 0, stream>>>(w, s.tokens, out);
}

} // namespace ttl
